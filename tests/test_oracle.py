"""CPU oracle: pinned against the reference's golden vectors, then checked
against float64 restatements of the reference math (no GPU needed)."""
import hashlib
import math
import os

import numpy as np
import pytest
from conftest import GOLDEN, bits, rel_l2


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLDEN, "q8_golden.npz"))


# ---------------------------------------------------------------- Q8_0 format
@pytest.mark.parametrize("case", ["small", "edge"])
def test_quantize_matches_reference_golden(O, golden, case):
    w = golden[f"{case}_w"]
    assert np.array_equal(O.quantize_q8_0(w), golden[f"{case}_q8"])
    assert np.array_equal(O.quantize_q8_0_c(w), golden[f"{case}_q8"])


@pytest.mark.parametrize("case", ["small", "edge"])
def test_dequant_bit_exact_vs_reference_golden(O, golden, case):
    n = golden[f"{case}_w"].size
    want = golden[f"{case}_deq"].reshape(-1).view(np.uint32)
    assert np.array_equal(O.dequant_q8_0(golden[f"{case}_q8"], n).view(np.uint32), want)
    assert np.array_equal(O.dequant_q8_0_c(golden[f"{case}_q8"], n).view(np.uint32), want)


def test_config1_quantized_digest(O, golden):
    rng = np.random.default_rng(0)
    w = rng.standard_normal((2048, 1024), dtype=np.float32) * np.float32(0.02)
    q = O.quantize_q8_0_c(w)
    assert q.size == int(golden["cfg1_nbytes"][0])
    assert hashlib.sha256(q.tobytes()).digest() == golden["cfg1_sha256"].tobytes()


def test_q8_block_layout(O):
    # scale f16 little-endian in bytes 0-1, then 32 int8 (create_q8_irpa.py:115-117)
    w = np.zeros(32, np.float32)
    w[3] = 1.27
    q = O.quantize_q8_0(w)
    assert q.size == 34
    assert q[:2].copy().view(np.float16)[0] == np.float16(np.float32(1.27) / np.float32(127.0))
    assert q[2 + 3].view(np.int8) == 127 and np.all(np.delete(q[2:], 3) == 0)


# ---------------------------------------------------------------- numerics
def test_expf_within_2ulp(O):
    xs = np.concatenate([np.linspace(-103.9, 88.7, 40001, dtype=np.float32),
                         -np.random.default_rng(1).exponential(4, 20000).astype(np.float32)])
    worst = 0
    for x in xs:
        t = math.exp(float(x))
        if t < 1.2e-38:
            continue
        v = np.float32(O.expf(float(x)))
        worst = max(worst, abs(int(v.view(np.int32)) - int(np.float32(t).view(np.int32))))
    assert worst <= 2
    assert O.expf(-200.0) == 0.0 and math.isinf(O.expf(100.0)) and O.expf(0.0) == 1.0


def test_f16_conversion_matches_numpy(O):
    L = O.lib()
    rng = np.random.default_rng(3)
    xs = np.concatenate([rng.standard_normal(5000).astype(np.float32) * 1000,
                         rng.standard_normal(5000).astype(np.float32) * 1e-5,
                         np.array([65504, 65520, -65520, 6e-8, 3e-8], np.float32)])
    got = np.array([L.q3o_f2h(float(x)) for x in xs], np.uint16)
    with np.errstate(over="ignore"):
        want = xs.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)


# ---------------------------------------------------------------- GEMVs
def _q8_problem(O, N, K, seed):
    rng = np.random.default_rng(seed)
    w = O.quantize_q8_0((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    x = rng.standard_normal(K).astype(np.float16)
    wd = O.dequant_q8_0(w, N * K).reshape(N, K).astype(np.float64)
    return w, x, wd @ x.astype(np.float64)


@pytest.mark.parametrize("N,K", [(64, 256), (128, 1024), (64, 2048), (32, 3072)])
def test_gemv_q8_orders_vs_float64(O, N, K):
    w, x, ref = _q8_problem(O, N, K, N + K)
    for order in ("mlir", "cuda"):
        y = O.gemv_q8(w, x, N, K, order)
        assert rel_l2(y, ref) < 1e-3
        # f16 output: every element within one f16 rounding of the exact value
        assert np.all(np.abs(y.astype(np.float64) - ref) <= np.abs(ref) * 2 ** -10 + 1e-6)


def test_gemv_q8_two_orders_agree_closely(O):
    w, x, _ = _q8_problem(O, 256, 2048, 5)
    a, b = O.gemv_q8(w, x, 256, 2048, "mlir"), O.gemv_q8(w, x, 256, 2048, "cuda")
    assert rel_l2(a, b) < 1e-3
    assert np.mean(bits(a) == bits(b)) > 0.9


def test_gemv_f16_vs_float64(O):
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((300 * 8, 1024)) * 0.02).astype(np.float16)
    x = rng.standard_normal(1024).astype(np.float16)
    ref = w.astype(np.float64) @ x.astype(np.float64)
    assert rel_l2(O.gemv_f16(w, x), ref) < 1e-3


# ---------------------------------------------------------------- argmax
def test_argmax_rules(O):
    inf = np.inf
    assert O.argmax_f16(np.array([1, 3, 3, 2], np.float16)) == 1          # lowest index on ties
    assert O.argmax_f16(np.array([-inf, -inf], np.float16)) == -1         # nothing above -inf
    assert O.argmax_f16(np.array([np.nan, 1, np.nan, 5, 5], np.float16)) == 3  # NaN never chosen
    assert O.argmax_f16(np.array([-inf, -65504], np.float16)) == 1
    assert O.argmax_f16(np.array([inf, inf, 1], np.float16)) == 0
    v = np.full(151936, -1, np.float16)
    v[151935] = 0
    v[77] = 0
    assert O.argmax_f16(v) == 77


# ---------------------------------------------------------------- small ops
def _rms_ref(x, g, eps=9.99999997e-7):
    x = x.astype(np.float64)
    return x / np.sqrt(np.mean(x * x) + eps) * g.astype(np.float64)


def test_rmsnorm_vs_float64(O):
    rng = np.random.default_rng(4)
    x = rng.standard_normal(1024).astype(np.float16)
    g = (1 + 0.1 * rng.standard_normal(1024)).astype(np.float16)
    assert rel_l2(O.rmsnorm(x, g), _rms_ref(x, g)) < 1e-3


def test_rope_table_formula(O):
    c, s = O.rope_table(600)
    i = np.arange(64)
    theta = np.power(np.float32(1e6), -((2.0 * i) / 128.0)).astype(np.float64)
    ang = np.arange(600)[:, None] * theta[None, :]
    assert np.max(np.abs(c - np.cos(ang))) < 2e-4 and np.max(np.abs(s - np.sin(ang))) < 2e-4


def _qk_ref(x, g, pos):
    heads = x.size // 128
    xh = x.reshape(heads, 128)
    n = np.stack([_rms_ref(h, g) for h in xh]).astype(np.float16).astype(np.float64)
    i = np.arange(64)
    th = np.power(1e6, -(2.0 * i) / 128.0) * pos
    c, s = np.cos(th), np.sin(th)
    out = np.empty_like(n)
    out[:, :64] = n[:, :64] * c - n[:, 64:] * s
    out[:, 64:] = n[:, 64:] * c + n[:, :64] * s
    return out.reshape(-1)


@pytest.mark.parametrize("pos", [0, 1, 511, 4000])
def test_qk_norm_rope_vs_float64(O, pos):
    rng = np.random.default_rng(pos)
    x = rng.standard_normal(16 * 128).astype(np.float16)
    g = (1 + 0.1 * rng.standard_normal(128)).astype(np.float16)
    assert rel_l2(O.qk_norm_rope(x, g, pos), _qk_ref(x, g, pos)) < 2e-3


def test_swiglu_vs_float64(O):
    rng = np.random.default_rng(6)
    gu = (rng.standard_normal(6144) * 2).astype(np.float16)
    g, u = gu[:3072].astype(np.float64), gu[3072:].astype(np.float64)
    ref = g / (1 + np.exp(-g)) * u
    assert rel_l2(O.swiglu(gu), ref) < 2e-3
    # saturation ends: large |gate| behave like relu(gate)*up
    big = np.array([-30000, 30000] + [0] * 2 + [2, 3] + [0] * 2, np.float16)
    out = O.swiglu(big)  # gate [-3e4, 3e4, 0, 0], up [2, 3, 0, 0]
    assert out[0] == 0 and np.isinf(out[1]) and out[2] == 0


def _attn_ref(q, kc, vc, slot0, T):
    out = np.empty((16, 128))
    for h in range(16):
        k = kc[slot0:slot0 + T, h // 2].astype(np.float64)
        v = vc[slot0:slot0 + T, h // 2].astype(np.float64)
        s = k @ q[h * 128:(h + 1) * 128].astype(np.float64) / math.sqrt(128)
        p = np.exp(s - s.max())
        out[h] = p @ v / p.sum()
    return out.reshape(-1)


@pytest.mark.parametrize("T", [1, 5, 32, 33, 256, 257, 700])
def test_attention_vs_float64(O, T):
    rng = np.random.default_rng(T)
    slot0 = 3
    kc = rng.standard_normal((slot0 + T + 2, 8, 128)).astype(np.float16)
    vc = rng.standard_normal((slot0 + T + 2, 8, 128)).astype(np.float16)
    q = rng.standard_normal(2048).astype(np.float16)
    got = O.attention(q, kc, vc, slot0, T)
    assert rel_l2(got, _attn_ref(q, kc, vc, slot0, T)) < 1e-3


def test_oracle_weight_generator_matches_library(O, q3):
    """bench.py's CPU legs build their weights with the oracle's generator and
    quantizer (never the product library); both generators must give the same
    bytes for the same seed."""
    from q3b200.weights import synthetic_weights, to_oracle_dict

    a = O.synthetic_weights(seed=5, layers=2)
    b = to_oracle_dict(synthetic_weights(seed=5, layers=2))
    assert set(a) == set(b)
    for k in a:
        assert a[k].shape == b[k].shape, k
        assert np.array_equal(a[k].view(np.uint8), b[k].view(np.uint8)), k
