"""CPU oracle for the Qwen3-0.6B Q8_0 decode hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module.  It is the checker the CUDA library is compared against; the
product never imports it.

Two layers:
  * numpy restatements of the reference's Q8_0 quantizer and dequantizer
    (tools/create_q8_irpa.py:103-129), used to cross-check the C oracle;
  * ctypes bindings of liboracle.so (q3_oracle.c), the C restatement of the
    decode path (model/qwen3_full.mlir, kernels/cuda, kernels/mlir).

All f16 tensors are numpy float16 arrays (passed to C as their bit patterns).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libref_dispatch.so")

LAYERS, DIM, NQ, NKV, HD, FFN, VOCAB = 28, 1024, 16, 8, 128, 3072, 151936
QBLK, QBYTES = 32, 34


# --------------------------------------------------------------------------
# numpy restatement of tools/create_q8_irpa.py:103-129
# --------------------------------------------------------------------------
def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    """tools/create_q8_irpa.py:103-118: blocks of 32, scale = amax/127 (f32,
    0 -> 1.0), q = round-half-even(w/scale) clipped to [-128,127], 34-byte
    blocks [f16 scale | 32 x int8].  Returns uint8 bytes."""
    flat = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    assert flat.size % QBLK == 0
    blocks = flat.reshape(-1, QBLK)
    amax = np.max(np.abs(blocks), axis=1, keepdims=True)
    scales = (amax / np.float32(127.0)).astype(np.float32)
    scales = np.where(scales == 0, np.float32(1.0), scales).astype(np.float32)
    q = np.round(blocks / scales).clip(-128, 127).astype(np.int8)
    raw = np.concatenate([scales.astype(np.float16).view(np.uint8), q.view(np.uint8)], axis=1)
    return raw.reshape(-1)


def dequant_q8_0(raw: np.ndarray, n: int) -> np.ndarray:
    """tools/create_q8_irpa.py:121-129: f32(scale_f16) * f32(q)."""
    r = np.frombuffer(np.ascontiguousarray(raw, dtype=np.uint8).tobytes(), dtype=np.uint8)
    r = r[: (n // QBLK) * QBYTES].reshape(-1, QBYTES)
    scales = r[:, :2].copy().view(np.float16).astype(np.float32)
    q = r[:, 2:].view(np.int8).astype(np.float32)
    return (scales * q).reshape(-1)


# --------------------------------------------------------------------------
# C oracle
# --------------------------------------------------------------------------
_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


class Weights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "token_embd", "output_norm", "output_T", "attn_norm", "ffn_norm", "q_norm", "k_norm",
        "q8_q", "q8_k", "q8_v", "q8_o", "q8_gate_up", "q8_down")] + [("n_layers", ctypes.c_int),
                                                                    ("order", ctypes.c_int)]

# summation orders of the C oracle (q3_oracle.h): the exact engine's, or the
# fused engine's (split O / down projections, cluster attention fold)
ORDER_EXACT, ORDER_FUSED = 0, 1


def _declare(L: ctypes.CDLL) -> None:
    P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    sig = {
        "q3o_h2f": (F, [ctypes.c_uint16]),
        "q3o_f2h": (ctypes.c_uint16, [F]),
        "q3o_expf": (F, [F]),
        "q3o_quantize_q8_0": (None, [P, I64, P]),
        "q3o_dequant_q8_0": (None, [P, I64, P]),
        "q3o_gemv_q8_mlir": (None, [P, P, P, I, I]),
        "q3o_gemv_q8_cuda": (None, [P, P, P, I, I]),
        "q3o_gemv_f16": (None, [P, P, P, I, I]),
        "q3o_argmax_f16": (I64, [P, I64]),
        "q3o_rmsnorm": (None, [P, P, P, I]),
        "q3o_rope_table": (None, [I64, P, P]),
        "q3o_qk_norm_rope": (None, [P, P, I, I64, P]),
        "q3o_swiglu": (None, [P, P, I]),
        "q3o_add_f16": (None, [P, P, P, I]),
        "q3o_attention": (None, [P, P, P, I64, I64, P]),
        "q3o_attention_fused": (None, [P, P, P, I64, I64, P]),
        "q3o_gemv_q8_split": (None, [P, P, P, I, I, I]),
        "q3o_layer": (None, [ctypes.POINTER(Weights), I, P, I64, P, P, I64]),
        "q3o_decode_step": (I64, [ctypes.POINTER(Weights), I64, I64, P, P, I64, P, I]),
        "q3o_generate": (I64, [ctypes.POINTER(Weights), P, I64, I64, I64, P, P, I64, P, P]),
        "q3o_num_threads": (I, []),
        "q3o_set_num_threads": (None, [I]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _p(a: np.ndarray | None) -> ctypes.c_void_p | None:
    if a is None:
        return None
    assert a.flags.c_contiguous
    return ctypes.c_void_p(a.ctypes.data)


def _h(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float16)


def expf(x: float) -> float:
    return lib().q3o_expf(x)


def quantize_q8_0_c(w: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    out = np.empty((w.size // QBLK) * QBYTES, dtype=np.uint8)
    lib().q3o_quantize_q8_0(_p(w), w.size, _p(out))
    return out


def dequant_q8_0_c(raw: np.ndarray, n: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty(n, dtype=np.float32)
    lib().q3o_dequant_q8_0(_p(raw), n, _p(out))
    return out


def gemv_q8(w: np.ndarray, x: np.ndarray, N: int, K: int, order: str = "mlir") -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    assert w.size >= N * (K // QBLK) * QBYTES
    x = _h(x)
    y = np.empty(N, dtype=np.float16)
    fn = lib().q3o_gemv_q8_mlir if order == "mlir" else lib().q3o_gemv_q8_cuda
    fn(_p(w), _p(x), _p(y), N, K)
    return y


def gemv_f16(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    w = _h(w)
    N, K = w.shape
    x = _h(x)
    y = np.empty(N, dtype=np.float16)
    lib().q3o_gemv_f16(_p(w), _p(x), _p(y), N, K)
    return y


def argmax_f16(v: np.ndarray) -> int:
    v = _h(v)
    return int(lib().q3o_argmax_f16(_p(v), v.size))


def rmsnorm(x: np.ndarray, g: np.ndarray) -> np.ndarray:
    x, g = _h(x), _h(g)
    y = np.empty_like(x)
    lib().q3o_rmsnorm(_p(x), _p(g), _p(y), x.size)
    return y


def rope_table(n_pos: int) -> tuple[np.ndarray, np.ndarray]:
    c = np.empty((n_pos, 64), dtype=np.float32)
    s = np.empty((n_pos, 64), dtype=np.float32)
    lib().q3o_rope_table(n_pos, _p(c), _p(s))
    return c, s


def qk_norm_rope(x: np.ndarray, g: np.ndarray, pos: int) -> np.ndarray:
    x, g = _h(x), _h(g)
    heads = x.size // HD
    y = np.empty_like(x)
    lib().q3o_qk_norm_rope(_p(x), _p(g), heads, pos, _p(y))
    return y


def swiglu(gate_up: np.ndarray) -> np.ndarray:
    gu = _h(gate_up)
    n = gu.size // 2
    y = np.empty(n, dtype=np.float16)
    lib().q3o_swiglu(_p(gu), _p(y), n)
    return y


def add_f16(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a, b = _h(a), _h(b)
    y = np.empty_like(a)
    lib().q3o_add_f16(_p(a), _p(b), _p(y), a.size)
    return y


def attention(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, slot0: int, T: int,
              order: int = ORDER_EXACT) -> np.ndarray:
    """q: f16[16*128] (normed+roped); kc/vc: f16 [slots, 8, 128]."""
    q, kc, vc = _h(q), _h(kc), _h(vc)
    out = np.empty(NQ * HD, dtype=np.float16)
    fn = lib().q3o_attention_fused if order == ORDER_FUSED else lib().q3o_attention
    fn(_p(q), _p(kc), _p(vc), slot0, T, _p(out))
    return out


def gemv_q8_split(w: np.ndarray, x: np.ndarray, N: int, K: int, nparts: int = 8) -> np.ndarray:
    """The fused engine's K-split Q8_0 GEMV (O and down projections)."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    assert w.size >= N * (K // QBLK) * QBYTES
    x = _h(x)
    y = np.empty(N, dtype=np.float16)
    lib().q3o_gemv_q8_split(_p(w), _p(x), _p(y), N, K, nparts)
    return y


class Model:
    """Keeps numpy weight arrays alive and exposes the C layer/step/generate."""

    def __init__(self, w: dict[str, np.ndarray], n_layers: int = LAYERS, order: int = ORDER_EXACT):
        self.arrays = {k: np.ascontiguousarray(v) for k, v in w.items()}
        a = self.arrays
        self.c = Weights(
            token_embd=a["token_embd"].ctypes.data, output_norm=a["output_norm"].ctypes.data,
            output_T=a["output_T"].ctypes.data, attn_norm=a["attn_norm"].ctypes.data,
            ffn_norm=a["ffn_norm"].ctypes.data, q_norm=a["q_norm"].ctypes.data,
            k_norm=a["k_norm"].ctypes.data, q8_q=a["q8_q"].ctypes.data,
            q8_k=a["q8_k"].ctypes.data, q8_v=a["q8_v"].ctypes.data, q8_o=a["q8_o"].ctypes.data,
            q8_gate_up=a["q8_gate_up"].ctypes.data, q8_down=a["q8_down"].ctypes.data,
            n_layers=n_layers, order=order)
        self.n_layers = n_layers
        self.order = order

    def new_cache(self, S: int) -> tuple[np.ndarray, np.ndarray]:
        return (np.zeros((LAYERS * S, NKV, HD), np.float16),
                np.zeros((LAYERS * S, NKV, HD), np.float16))

    def layer(self, layer: int, x: np.ndarray, pos: int, kc, vc, S: int) -> np.ndarray:
        x = _h(x).copy()
        lib().q3o_layer(ctypes.byref(self.c), layer, _p(x), pos, _p(kc), _p(vc), S)
        return x

    def decode_step(self, token: int, pos: int, kc, vc, S: int) -> tuple[int, np.ndarray]:
        logits = np.empty(VOCAB, dtype=np.float16)
        t = lib().q3o_decode_step(ctypes.byref(self.c), token, pos, _p(kc), _p(vc), S,
                                  _p(logits), 1)
        return int(t), logits

    def generate(self, prompt, max_gen: int, eos: int, S: int, force=None):
        kc, vc = self.new_cache(S)
        prompt = np.ascontiguousarray(prompt, dtype=np.int64)
        out = np.zeros(max(max_gen, 1), dtype=np.int64)
        f = None if force is None else np.ascontiguousarray(force, dtype=np.int64)
        n = lib().q3o_generate(ctypes.byref(self.c), _p(prompt), prompt.size, max_gen, eos,
                               _p(kc), _p(vc), S, _p(out), _p(f))
        return out[:n].copy(), kc, vc


def num_threads() -> int:
    return int(lib().q3o_num_threads())


def set_num_threads(n: int) -> None:
    lib().q3o_set_num_threads(n)


# --------------------------------------------------------------------------
# Seeded synthetic weights for the CPU legs (the oracle's own quantizer)
# --------------------------------------------------------------------------
# The benchmark configurations' weights: every matrix f32 N(0, 0.02)
# quantised Q8_0, gammas 1 + N(0, 0.1) as f16, a tied f16 embedding / vocab
# N(0, 0.02).  Each tensor draws from its own PCG64 stream spawned from
# SeedSequence(seed) in a fixed order -- the same streams, in the same order,
# as the library's host generator, so both produce the same bytes (a test
# checks that) while bench.py's CPU legs never load the product library.
Q8_SHAPES = [("q8_q", 2048, 1024), ("q8_k", 1024, 1024), ("q8_v", 1024, 1024),
             ("q8_o", 1024, 2048), ("q8_gate_up", 6144, 1024), ("q8_down", 1024, 3072)]
EMB_CHUNKS = 16


def _normal_f32(rng: np.random.Generator, shape, std: float) -> np.ndarray:
    out = np.empty(shape, dtype=np.float32)
    rng.standard_normal(out=out, dtype=np.float32)
    out *= np.float32(std)
    return out


def _gamma_f16(rng: np.random.Generator, shape) -> np.ndarray:
    return (np.float32(1.0) + _normal_f32(rng, shape, 0.1)).astype(np.float16)


def synthetic_weights(seed: int = 0, layers: int = LAYERS, threads: int | None = None
                      ) -> dict[str, np.ndarray]:
    """The decode path's parameters under the oracle's field names (Model()).
    Layers beyond `layers` stay zero."""
    from concurrent.futures import ThreadPoolExecutor

    streams = iter(np.random.SeedSequence(seed).spawn(16 + EMB_CHUNKS + len(Q8_SHAPES) * LAYERS))
    gen = lambda: np.random.Generator(np.random.PCG64(next(streams)))
    w: dict[str, np.ndarray] = {}
    jobs = []
    emb = np.empty((VOCAB, DIM), dtype=np.float16)
    rows = VOCAB // EMB_CHUNKS

    def emb_chunk(c, g):
        emb[c * rows:(c + 1) * rows] = _normal_f32(g, (rows, DIM), 0.02).astype(np.float16)

    for c in range(EMB_CHUNKS):
        jobs.append((emb_chunk, c, gen()))
    w["token_embd"] = emb
    w["output_T"] = emb
    w["output_norm"] = _gamma_f16(gen(), (DIM,))
    w["attn_norm"] = _gamma_f16(gen(), (LAYERS, DIM))
    w["ffn_norm"] = _gamma_f16(gen(), (LAYERS, DIM))
    w["q_norm"] = _gamma_f16(gen(), (LAYERS, HD))
    w["k_norm"] = _gamma_f16(gen(), (LAYERS, HD))
    for name, N, K in Q8_SHAPES:
        st = np.zeros((LAYERS, N * (K // QBLK) * QBYTES), dtype=np.uint8)
        w[name] = st

        def q8_layer(l, g, st=st, N=N, K=K):
            st[l] = quantize_q8_0_c(_normal_f32(g, (N, K), 0.02))

        for l in range(LAYERS):
            g = gen()
            if l < layers:
                jobs.append((q8_layer, l, g))
    nt = threads or min(32, os.cpu_count() or 1)
    with ThreadPoolExecutor(nt) as ex:
        for f in [ex.submit(fn, a, g) for fn, a, g in jobs]:
            f.result()
    return w
