"""One decoder layer through the C ABI vs the CPU oracle, bit for bit.

one Qwen3-0.6B layer, batch 1, at position 511 over an
f16 KV cache of 512 positions (511 cached N(0,1) rows + the new one),
residual x ~ N(0,1), the synthetic N(0,0.02) Q8_0 weights and 1+N(0,0.1)
gammas (model/qwen3_full.mlir:751-864).  Two implementations:

* the fused engine's layer (q3_fused_layer: the attention-block and
  feed-forward-block cluster kernels) against the oracle in its fused orders;
* the exact engine's layer as the chain of stateless entry points
  (q3_gemv_q8_norm x3, q3_decode_attention, q3_gemv_q8_resid,
  q3_gemv_q8_swiglu, q3_gemv_q8_resid) against the oracle in the reference
  kernels' orders.

Further positions cover every attention shape of the fused kernel: one
partial chunk, a rank with one chunk, ranks with several chunks (a K/V slot
refilled after the dependency wait), and a full 4096-position cache.
"""
import ctypes

import numpy as np
import pytest
from conftest import bits

pytestmark = pytest.mark.gpu

LAYER = 2


@pytest.fixture(scope="module")
def layer_models(gpu, O, model_weights):
    from q3b200.weights import to_oracle_dict

    dw = gpu.DeviceWeights(model_weights)
    od = to_oracle_dict(model_weights)
    return dw, O.Model(od, order=O.ORDER_EXACT), O.Model(od, order=O.ORDER_FUSED)


def _case(S, pos, seed):
    rng = np.random.default_rng(seed)
    n = (LAYER + 1) * S
    kc = np.zeros((n, 8, 128), np.float16)
    vc = np.zeros((n, 8, 128), np.float16)
    kc[LAYER * S:LAYER * S + pos] = rng.standard_normal((pos, 8, 128)).astype(np.float16)
    vc[LAYER * S:LAYER * S + pos] = rng.standard_normal((pos, 8, 128)).astype(np.float16)
    x = rng.standard_normal(1024).astype(np.float16)
    return x, kc, vc


def _rope(q3, S):
    c = np.empty((S, 64), np.float32)
    s = np.empty((S, 64), np.float32)
    assert q3.lib().q3_rope_table(S, c.ctypes.data, s.ctypes.data) == 0
    return q3.DeviceArray.from_host(c), q3.DeviceArray.from_host(s)


def _fused_layer(q3, dw, x, kc, vc, S, pos):
    L = q3.lib()
    dx, dy = q3.DeviceArray.from_host(x), q3.DeviceArray((1024,), np.float16)
    dkc, dvc = q3.DeviceArray.from_host(kc), q3.DeviceArray.from_host(vc)
    dpos = q3.DeviceArray.from_host(np.array([pos], np.int64))
    c, s = _rope(q3, S)
    ws = q3.DeviceArray((L.q3_fused_layer_workspace_bytes(),), np.uint8, zero=True)
    rc = L.q3_fused_layer(ctypes.byref(dw.struct), LAYER, dx.ptr, dy.ptr, dkc.ptr, dvc.ptr, S,
                          dpos.ptr, c.ptr, s.ptr, ws.ptr, 0, None)
    assert rc == 0, L.q3_last_error()
    assert L.q3_stream_synchronize(None) == 0
    return dy.download(), dkc.download(), dvc.download()


def _exact_layer_chain(q3, dw, w, x, kc, vc, S, pos):
    """The exact engine's five launches of a layer, through the stateless API."""
    L = q3.lib()
    up = lambda a: q3.DeviceArray.from_host(np.ascontiguousarray(a))
    ptr = lambda name: dw.buffers[name].ptr
    bpl = lambda name: w[name].shape[1]
    q8 = lambda name: ptr(name) + LAYER * bpl(name)
    g = lambda name, n: ptr(name) + LAYER * n * 2
    dx = up(x)
    qkv = q3.DeviceArray((4096,), np.float16)
    att = q3.DeviceArray((2048,), np.float16)
    h1 = q3.DeviceArray((1024,), np.float16)
    act = q3.DeviceArray((3072,), np.float16)
    out = q3.DeviceArray((1024,), np.float16)
    dkc, dvc = up(kc), up(vc)
    dpos = up(np.array([pos], np.int64))
    c, s = _rope(q3, S)
    ws = q3.DeviceArray((L.q3_attention_workspace_bytes(S),), np.uint8, zero=True)
    an = g("stacked.attn_norm.weight", 1024)
    calls = [
        ("q3_gemv_q8_norm", q8("stacked.q8.attn_q.weight"), dx.ptr, an, qkv.ptr, 2048, 1024, None),
        ("q3_gemv_q8_norm", q8("stacked.q8.attn_k.weight"), dx.ptr, an, qkv.ptr + 4096, 1024, 1024,
         None),
        ("q3_gemv_q8_norm", q8("stacked.q8.attn_v.weight"), dx.ptr, an, qkv.ptr + 6144, 1024, 1024,
         None),
        ("q3_decode_attention", qkv.ptr, g("stacked.attn_q_norm.weight", 128),
         g("stacked.attn_k_norm.weight", 128), c.ptr, s.ptr, S, dkc.ptr, dvc.ptr, LAYER * S, S,
         dpos.ptr, att.ptr, ws.ptr, None),
        ("q3_gemv_q8_resid", q8("stacked.q8.attn_output.weight"), att.ptr, dx.ptr, h1.ptr, 1024,
         2048, None),
        ("q3_gemv_q8_swiglu", q8("stacked.q8.ffn_gate_up.weight"), h1.ptr,
         g("stacked.ffn_norm.weight", 1024), act.ptr, 3072, 1024, None),
        ("q3_gemv_q8_resid", q8("stacked.q8.ffn_down.weight"), act.ptr, h1.ptr, out.ptr, 1024,
         3072, None),
    ]
    for name, *args in calls:
        assert getattr(L, name)(*args) == 0, (name, L.q3_last_error())
    assert L.q3_stream_synchronize(None) == 0
    return out.download(), dkc.download(), dvc.download()


def _check(got, want):
    y, kc, vc = got
    wy, wkc, wvc = want
    assert np.array_equal(bits(kc), bits(wkc)), "K cache"
    assert np.array_equal(bits(vc), bits(wvc)), "V cache"
    assert np.array_equal(bits(y), bits(wy)), "layer output"


def test_fused_layer_configs1_bit_exact(gpu, layer_models, model_weights):
    """position 511 over a 512-position cache, fused orders."""
    dw, _, om = layer_models
    S, pos = 512, 511
    x, kc, vc = _case(S, pos, 11)
    want_kc, want_vc = kc.copy(), vc.copy()
    want = om.layer(LAYER, x, pos, want_kc, want_vc, S)
    _check(_fused_layer(gpu, dw, x, kc, vc, S, pos), (want, want_kc, want_vc))


def test_exact_layer_configs1_bit_exact(gpu, layer_models, model_weights):
    """configs[1] through the exact engine's stateless kernels, reference orders."""
    dw, om, _ = layer_models
    S, pos = 512, 511
    x, kc, vc = _case(S, pos, 11)
    want_kc, want_vc = kc.copy(), vc.copy()
    want = om.layer(LAYER, x, pos, want_kc, want_vc, S)
    _check(_exact_layer_chain(gpu, dw, model_weights, x, kc, vc, S, pos), (want, want_kc, want_vc))


@pytest.mark.parametrize("S,pos", [(64, 0), (64, 31), (64, 32), (1024, 300), (2048, 1055),
                                   (2048, 2047), (4096, 4095)])
def test_fused_layer_positions_bit_exact(gpu, layer_models, S, pos):
    dw, _, om = layer_models
    x, kc, vc = _case(S, pos, pos + 5)
    want_kc, want_vc = kc.copy(), vc.copy()
    want = om.layer(LAYER, x, pos, want_kc, want_vc, S)
    _check(_fused_layer(gpu, dw, x, kc, vc, S, pos), (want, want_kc, want_vc))


def test_fused_layer_rejects_long_caches(gpu, layer_models):
    dw, _, _ = layer_models
    L = gpu.lib()
    buf = gpu.DeviceArray((64,), np.uint8, zero=True)
    p = buf.ptr
    rc = L.q3_fused_layer(ctypes.byref(dw.struct), 0, p, p, p, p, 8192, p, p, p, p, 0, None)
    assert rc == 1 and b"4096" in L.q3_last_error()
