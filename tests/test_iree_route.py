"""The IREE substitution route (compile.sh:47-66, kernels/cuda/dispatch_N.mlir):
six hal.executable wrappers in qwen3-iree_b200/iree/ name one sm_100a object
built by `make iree` from the kernels of csrc/q3_iree.cuh.  On the CPU: each
wrapper's export, push-constant count, workgroup count and size agree with
the kernel declared under that name; the object builds.  On a GPU (marked
gpu): the cubin loads through the CUDA driver the way the IREE HAL loads an
executable object, every export resolves by name, and a launch with the
wrapper's geometry writes the same bytes as the library's own launcher."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest
from conftest import ROOT, bits

PKG = os.path.join(ROOT, "qwen3-iree_b200")
IREE_DIR = os.path.join(PKG, "iree")
DISPATCHES = (3, 4, 12, 18, 20, 24)


def _kernels():
    """export name -> number of u32 push constants, from csrc/q3_iree.cuh"""
    src = open(os.path.join(PKG, "csrc", "q3_iree.cuh")).read()
    out = {}
    for m in re.finditer(r'extern "C" __global__ void __launch_bounds__\(256\)\s*(\w+)\(([^)]*)\)', src):
        out[m.group(1)] = m.group(2).count("uint32_t")
    return out


def _wrapper(n):
    text = open(os.path.join(IREE_DIR, f"dispatch_{n}.mlir")).read()
    return {
        "executable": re.search(r"hal\.executable public @(\w+)", text).group(1),
        "target": re.search(r'target\(<"cuda", "([\w-]+)">\)', text).group(1),
        "object": re.search(r'#hal\.executable\.object<\{path = "([^"]+)"\}>', text).group(1),
        "export": re.search(r"hal\.executable\.export public @(\w+)", text).group(1),
        "constants": int(re.search(r"constants = (\d+)", text).group(1)),
        "bindings": len(re.findall(r"#hal\.pipeline\.binding<", text)),
        "count": int(re.search(r"hal\.return %c(\d+)", text).group(1)),
        "wg": [int(v) for v in re.search(r"workgroup_size = \[(\d+) : index, (\d+) : index, (\d+) : index\]", text).groups()],
    }


@pytest.mark.parametrize("n", DISPATCHES)
def test_wrapper_matches_the_kernel(n):
    w, k = _wrapper(n), _kernels()
    assert w["executable"] == f"decode_dispatch_{n}"
    assert w["target"] == "cuda-nvptx-fb" and w["object"] == "q3_dispatch.ptx"
    assert w["export"] in k, w["export"]
    assert w["constants"] == k[w["export"]]
    assert w["bindings"] == 3 and w["wg"] == [256, 1, 1]
    rows = int(re.search(r"matmul_(\d+)x1x", w["export"]).group(1))
    assert w["count"] == rows // 8  # 8 output rows per workgroup


def test_iree_object_builds():
    subprocess.run(["make", "-s", "-C", PKG, "iree"], check=True)
    for f in ("q3_dispatch.ptx", "q3_dispatch.cubin"):
        assert os.path.getsize(os.path.join(IREE_DIR, f)) > 0


# ------------------------------------------------------------------ GPU
def _cu_ok(r):
    from cuda.bindings import driver as cu

    err = r[0] if isinstance(r, tuple) else r
    assert err == cu.CUresult.CUDA_SUCCESS, err
    return r[1] if isinstance(r, tuple) and len(r) == 2 else r


@pytest.fixture(scope="module")
def iree_module(gpu):
    from cuda.bindings import driver as cu

    subprocess.run(["make", "-s", "-C", PKG, "iree"], check=True)
    _cu_ok(cu.cuInit(0))
    dev = _cu_ok(cu.cuDeviceGet(0))
    ctx = _cu_ok(cu.cuDevicePrimaryCtxRetain(dev))  # the runtime's (libq3b200's) context
    _cu_ok(cu.cuCtxPushCurrent(ctx))
    data = open(os.path.join(IREE_DIR, "q3_dispatch.cubin"), "rb").read()
    mod = _cu_ok(cu.cuModuleLoadData(data))
    yield mod
    _cu_ok(cu.cuModuleUnload(mod))
    _cu_ok(cu.cuCtxPopCurrent())
    _cu_ok(cu.cuDevicePrimaryCtxRelease(dev))


CASES = [  # (dispatch, N, K, in_off, out_off)
    (3, 2048, 1024, 2112, 4160), (4, 1024, 1024, 2112, 8192), (12, 1024, 2048, 12352, 2048),
    (18, 6144, 1024, 64, 6144), (20, 1024, 3072, 18432, 0), (24, 151936, 1024, 64, 256),
]


@pytest.mark.gpu
@pytest.mark.parametrize("n,N,K,in_off,out_off", CASES)
def test_object_exports_load_and_match_the_library(gpu, O, iree_module, n, N, K, in_off, out_off):
    from cuda.bindings import driver as cu

    wr = _wrapper(n)
    fn = _cu_ok(cu.cuModuleGetFunction(iree_module, wr["export"].encode()))
    rng = np.random.default_rng(n)
    if n == 24:
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    else:
        w = np.stack([O.quantize_q8_0_c((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
                      for _ in range(2)])
    x = rng.standard_normal(K).astype(np.float16)
    b1 = np.zeros(in_off + 2 * K + 64, np.uint8)
    b1[in_off:in_off + 2 * K] = x.view(np.uint8)
    dw, db1 = gpu.DeviceArray.from_host(w), gpu.DeviceArray.from_host(b1)
    layer = 0 if n == 24 else 1
    outs = []
    for how in ("object", "library"):
        db2 = gpu.DeviceArray((out_off + 2 * N + 64,), np.uint8)
        db2.fill_bytes(0xAB)
        consts = {24: [out_off], 4: [out_off, layer, 0]}.get(n, [layer, 0])
        if how == "object":
            vals = (dw.ptr, db1.ptr, db2.ptr, *consts)
            types = (ctypes.c_void_p,) * 3 + (ctypes.c_uint32,) * len(consts)
            _cu_ok(cu.cuLaunchKernel(fn, wr["count"], 1, 1, 256, 1, 1, 0, 0, (vals, types), 0))
            _cu_ok(cu.cuCtxSynchronize())
        else:
            L = gpu.lib()
            assert getattr(L, f"q3_iree_dispatch_{n}")(dw.ptr, db1.ptr, db2.ptr, *consts, None) == 0
            assert L.q3_stream_synchronize(None) == 0
        outs.append(db2.download())
    assert np.array_equal(outs[0], outs[1])
    y = outs[0][out_off:out_off + 2 * N].view(np.float16)
    want = O.gemv_f16(w, x) if n == 24 else O.gemv_q8(w[layer], x, N, K, "cuda")
    assert np.array_equal(bits(y), bits(want))
