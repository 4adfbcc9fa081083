"""The C ABI library without a GPU: it loads, exports every declared symbol,
its host-side functions match the oracle, and argument errors are reported
as status codes before anything touches a device."""
import ctypes
import os
import re

import numpy as np
import pytest
from conftest import GOLDEN, ROOT

HEADER = os.path.join(ROOT, "include", "q3b200.h")
IREE_KERNELS = [
    "decode_dispatch_3_matmul_2048x1x1024_f16", "decode_dispatch_4_matmul_1024x1x1024_f16",
    "decode_dispatch_12_matmul_1024x1x2048_f16", "decode_dispatch_18_matmul_6144x1x1024_f16",
    "decode_dispatch_20_matmul_1024x1x3072_f16", "decode_dispatch_24_matmul_151936x1x1024_f16",
]


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(q3_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_api():
    names = declared_functions()
    for must in ("q3_gemv_q8", "q3_vocab_argmax", "q3_decode_attention", "q3_run", "q3_decode",
                 "q3_chat_turn", "q3_iree_dispatch_3", "q3_iree_dispatch_24", "q3_model_create"):
        assert must in names


def test_library_exports_every_declared_symbol(q3):
    L = q3.lib()
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert missing == []
    for k in IREE_KERNELS:  # extern "C" kernels keep the reference's export names
        assert hasattr(L, k), k
    assert L.q3_abi_version() == 1


def test_python_binding_covers_header(q3):
    from q3b200._lib import SIGNATURES

    assert sorted(set(declared_functions()) - set(SIGNATURES)) == []


def test_rope_table_bit_exact_vs_oracle(q3, O):
    n = 4096
    c = np.empty((n, 64), np.float32)
    s = np.empty((n, 64), np.float32)
    assert q3.lib().q3_rope_table(n, c.ctypes.data, s.ctypes.data) == 0
    oc, os_ = O.rope_table(n)
    assert np.array_equal(c.view(np.uint32), oc.view(np.uint32))
    assert np.array_equal(s.view(np.uint32), os_.view(np.uint32))


def test_host_quantizer_matches_reference_golden(q3):
    from q3b200.weights import quantize_q8_0

    g = np.load(os.path.join(GOLDEN, "q8_golden.npz"))
    for case in ("small", "edge"):
        assert np.array_equal(quantize_q8_0(g[f"{case}_w"]), g[f"{case}_q8"])


def test_device_count_without_gpu_is_not_an_error(q3):
    assert q3.device_count() >= 0


def test_argument_errors_are_statuses(q3):
    L = q3.lib()
    buf = ctypes.create_string_buffer(4096 + 16)
    p = (ctypes.addressof(buf) + 15) & ~15
    assert L.q3_gemv_q8(p, p, p, 8, 100, None) == 1          # K not a multiple of 256
    assert b"multiple of 256" in L.q3_last_error()
    assert L.q3_gemv_q8(p, p, p, 7, 256, None) == 1          # N not a multiple of 8
    assert L.q3_gemv_q8(p + 2, p, p, 8, 256, None) == 1      # misaligned weights
    assert L.q3_gemv_q8(None, p, p, 8, 256, None) == 1
    assert L.q3_gemv_q8(p, p, p, 8, 4096, None) == 1         # above 3072
    assert L.q3_vocab_argmax(p, p, None, None, p, p, 16, 512, None) == 1
    assert L.q3_run(None, p, 1, 1, 0, p, None) == 1
    assert L.q3_gemv_q8_layers(p, 16, p, p, 8, 256, 0, None) == 1
    assert L.q3_quantize_q8_0(p, 33, p) == 1
    assert L.q3_bvocab_argmax(p, 128, p, 1, None, p, p + 4, None) == 1  # workspace below 8 bytes
    assert b"8-byte aligned" in L.q3_last_error()
    assert L.q3_strerror(3).startswith(b"kernel reported")


def test_workspace_sizes(q3):
    L = q3.lib()
    assert L.q3_vocab_argmax_workspace_bytes() >= 16 * 148
    assert L.q3_attention_workspace_bytes(4096) > L.q3_attention_workspace_bytes(256)


def test_synthetic_weights_layout(q3):
    from q3b200 import weights as W

    w = W.synthetic_weights(seed=3, layers=1)
    assert w["token_embd.weight"] is w["output_T.weight"]
    assert w["stacked.q8.attn_q.weight"].shape == (28, 2228224)
    assert w["stacked.q8.ffn_gate_up.weight"].shape == (28, 6684672)
    assert w["stacked.q8.ffn_down.weight"].shape == (28, 3342336)
    assert w["stacked.attn_q_norm.weight"].dtype == np.float16
    assert not w["stacked.q8.attn_q.weight"][1].any()   # layers beyond `layers` stay zero
    total = sum(W.bytes_per_layer(N, K) for _, N, K in W.Q8_MATRICES) * 28
    assert total == 467_927_040
