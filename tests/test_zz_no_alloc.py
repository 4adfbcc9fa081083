"""q3_decode_attention_noalloc: the decode attention for callers that cannot
allocate device memory where they launch -- a kernel substituted into an IREE
executable only receives its bindings, and code running under a fixed memory
plan may not call cudaMalloc.  It keeps the kernel's scratch in a static
device array of the library instead of a caller workspace.

Checked through the C ABI against q3_decode_attention (same kernel, caller
workspace), bit for bit, on two consecutive calls: the second call attends
over the K/V row the first one wrote, and reuses the static scratch the first
one left behind.  This file is collected last so that a failing run has
already exercised every other test."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

S, LAYER = 1024, 1


def _up(q3, a):
    return q3.DeviceArray.from_host(np.ascontiguousarray(a))


def _setup(q3, seed):
    rng = np.random.default_rng(seed)
    kc = rng.standard_normal(((LAYER + 1) * S, 8, 128)).astype(np.float16)
    vc = rng.standard_normal(((LAYER + 1) * S, 8, 128)).astype(np.float16)
    c = np.empty((S, 64), np.float32)
    s = np.empty((S, 64), np.float32)
    assert q3.lib().q3_rope_table(S, c.ctypes.data, s.ctypes.data) == 0
    gq = (1 + 0.1 * rng.standard_normal(128)).astype(np.float16)
    gk = (1 + 0.1 * rng.standard_normal(128)).astype(np.float16)
    qkv = [rng.standard_normal(4096).astype(np.float16) for _ in range(2)]
    return dict(kc=kc, vc=vc, c=c, s=s, gq=gq, gk=gk, qkv=qkv)


def _run(q3, d, positions, noalloc, stream=None):
    L = q3.lib()
    kc, vc = _up(q3, d["kc"]), _up(q3, d["vc"])
    c, s, gq, gk = _up(q3, d["c"]), _up(q3, d["s"]), _up(q3, d["gq"]), _up(q3, d["gk"])
    ws = q3.DeviceArray((L.q3_attention_workspace_bytes(S),), np.uint8, zero=True)
    outs = []
    for qkv_h, pos in zip(d["qkv"], positions):
        qkv = _up(q3, qkv_h)
        p = _up(q3, np.array([pos], np.int64))
        out = q3.DeviceArray((2048,), np.float16)
        out.fill_bytes(0xFF)
        if noalloc:
            rc = L.q3_decode_attention_noalloc(qkv.ptr, gq.ptr, gk.ptr, c.ptr, s.ptr, S, kc.ptr,
                                               vc.ptr, LAYER * S, S, p.ptr, out.ptr, stream)
        else:
            rc = L.q3_decode_attention(qkv.ptr, gq.ptr, gk.ptr, c.ptr, s.ptr, S, kc.ptr, vc.ptr,
                                       LAYER * S, S, p.ptr, out.ptr, ws.ptr, stream)
        assert rc == 0, L.q3_last_error()
        if stream is not None:
            assert L.q3_stream_synchronize(stream) == 0
        outs.append(out.download())
    return outs, kc.download(), vc.download()


@pytest.mark.parametrize("positions", [(299, 300), (5, 6), (1023, 1023)])
def test_noalloc_attention_matches_workspace_version(gpu, positions):
    d = _setup(gpu, sum(positions))
    want, wk, wv = _run(gpu, d, positions, noalloc=False)
    got, gk, gv = _run(gpu, d, positions, noalloc=True)
    for w, g in zip(want, got):
        assert np.array_equal(w.view(np.uint16), g.view(np.uint16))
    assert np.array_equal(wk.view(np.uint16), gk.view(np.uint16))
    assert np.array_equal(wv.view(np.uint16), gv.view(np.uint16))


def test_noalloc_attention_rejects_contexts_beyond_its_scratch(gpu):
    L = gpu.lib()
    buf = gpu.DeviceArray((64,), np.uint8, zero=True)
    p = buf.ptr
    rc = L.q3_decode_attention_noalloc(p, p, p, p, p, 8192, p, p, 0, 8192, p, p, None)
    assert rc == 1
    assert b"4096" in L.q3_last_error()


def test_noalloc_attention_on_a_created_stream(gpu):
    """Two calls in a row on a non-default stream: the counter clear of each
    call is ordered on that stream before its kernel."""
    L = gpu.lib()
    st = ctypes.c_void_p()
    assert L.q3_stream_create(ctypes.byref(st)) == 0
    try:
        d = _setup(gpu, 77)
        want, wk, wv = _run(gpu, d, (700, 701), noalloc=False, stream=st)
        got, gk, gv = _run(gpu, d, (700, 701), noalloc=True, stream=st)
    finally:
        L.q3_stream_destroy(st)
    for w, g in zip(want, got):
        assert np.array_equal(w.view(np.uint16), g.view(np.uint16))
    assert np.array_equal(wk.view(np.uint16), gk.view(np.uint16))


def test_noalloc_attention_rejects_a_misaligned_output(gpu):
    """out is stored 4 f16 at a time: a buffer off an 8-byte boundary is
    refused on the host before anything is launched."""
    L = gpu.lib()
    buf = gpu.DeviceArray((64,), np.uint8, zero=True)
    p = buf.ptr
    rc = L.q3_decode_attention_noalloc(p, p, p, p, p, 16, p, p, 0, 16, p, p + 2, None)
    assert rc == 1
    assert b"8-byte" in L.q3_last_error()
