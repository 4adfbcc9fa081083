"""Seeded synthetic Qwen3-0.6B weights in the reference's parameter layout.

Shapes and names follow tools/create_q8_irpa.py:146-224 and
model/qwen3_full.mlir:65-79, :772-777 (stacked [28, bytes_per_layer] Q8_0
matrices in GGUF-native [N, K] block order, gate rows then up rows for
ffn_gate_up, f16 norms).  Values follow the benchmark configurations: every
matrix drawn f32 N(0, 0.02) and quantised Q8_0 (amax/127), norm gammas
1 + N(0, 0.1) as f16, a tied f16 embedding / vocab matrix N(0, 0.02).
There are no real checkpoints in this environment.
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from ._lib import call

LAYERS, DIM, NQ, NKV, HD, FFN, VOCAB = 28, 1024, 16, 8, 128, 3072, 151936
QBLK, QBYTES = 32, 34

# (name, N, K) of the stacked Q8_0 matrices, in generation order
Q8_MATRICES = [
    ("stacked.q8.attn_q.weight", 2048, 1024),
    ("stacked.q8.attn_k.weight", 1024, 1024),
    ("stacked.q8.attn_v.weight", 1024, 1024),
    ("stacked.q8.attn_output.weight", 1024, 2048),
    ("stacked.q8.ffn_gate_up.weight", 6144, 1024),
    ("stacked.q8.ffn_down.weight", 1024, 3072),
]


def bytes_per_layer(N: int, K: int) -> int:
    return N * (K // QBLK) * QBYTES


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    """Q8_0 quantizer of tools/create_q8_irpa.py:103-118 (library host code)."""
    w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    out = np.empty((w.size // QBLK) * QBYTES, dtype=np.uint8)
    call("q3_quantize_q8_0", w.ctypes.data, w.size, out.ctypes.data)
    return out


def normal_f32(rng: np.random.Generator, shape, std: float) -> np.ndarray:
    out = np.empty(shape, dtype=np.float32)
    rng.standard_normal(out=out, dtype=np.float32)
    out *= np.float32(std)
    return out


def gamma_f16(rng: np.random.Generator, shape) -> np.ndarray:
    return (np.float32(1.0) + normal_f32(rng, shape, 0.1)).astype(np.float16)


def make_q8_matrix(rng: np.random.Generator, N: int, K: int, std: float = 0.02) -> np.ndarray:
    return quantize_q8_0(normal_f32(rng, (N, K), std))


EMB_CHUNKS = 16


def synthetic_weights(seed: int = 0, layers: int = LAYERS,
                      threads: int | None = None) -> dict[str, np.ndarray]:
    """All parameters of the decode path as host numpy arrays.

    Every tensor (each layer of each stacked matrix, each embedding chunk)
    draws from its own PCG64 stream spawned from SeedSequence(seed) in a fixed
    order, so the result does not depend on the thread count.  Layers beyond
    `layers` stay zero (only small tests use that)."""
    streams = iter(np.random.SeedSequence(seed).spawn(16 + EMB_CHUNKS + len(Q8_MATRICES) * LAYERS))
    gen = lambda: np.random.Generator(np.random.PCG64(next(streams)))
    w: dict[str, np.ndarray] = {}
    jobs = []
    emb = np.empty((VOCAB, DIM), dtype=np.float16)
    rows = VOCAB // EMB_CHUNKS

    def emb_chunk(c, g):
        emb[c * rows:(c + 1) * rows] = normal_f32(g, (rows, DIM), 0.02).astype(np.float16)

    for c in range(EMB_CHUNKS):
        jobs.append((emb_chunk, c, gen()))
    w["token_embd.weight"] = emb
    w["output_T.weight"] = emb  # tied
    w["output_norm.weight"] = gamma_f16(gen(), (DIM,))
    w["stacked.attn_norm.weight"] = gamma_f16(gen(), (LAYERS, DIM))
    w["stacked.ffn_norm.weight"] = gamma_f16(gen(), (LAYERS, DIM))
    w["stacked.attn_q_norm.weight"] = gamma_f16(gen(), (LAYERS, HD))
    w["stacked.attn_k_norm.weight"] = gamma_f16(gen(), (LAYERS, HD))
    for name, N, K in Q8_MATRICES:
        st = np.zeros((LAYERS, bytes_per_layer(N, K)), dtype=np.uint8)
        w[name] = st

        def q8_layer(l, g, st=st, N=N, K=K):
            st[l] = make_q8_matrix(g, N, K)

        for l in range(LAYERS):
            g = gen()
            if l < layers:
                jobs.append((q8_layer, l, g))
    nt = threads or min(32, os.cpu_count() or 1)
    with ThreadPoolExecutor(nt) as ex:
        for f in [ex.submit(fn, a, g) for fn, a, g in jobs]:
            f.result()
    return w


def to_oracle_dict(w: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    """Rename to the CPU oracle's field names."""
    return {
        "token_embd": w["token_embd.weight"], "output_norm": w["output_norm.weight"],
        "output_T": w["output_T.weight"], "attn_norm": w["stacked.attn_norm.weight"],
        "ffn_norm": w["stacked.ffn_norm.weight"], "q_norm": w["stacked.attn_q_norm.weight"],
        "k_norm": w["stacked.attn_k_norm.weight"], "q8_q": w["stacked.q8.attn_q.weight"],
        "q8_k": w["stacked.q8.attn_k.weight"], "q8_v": w["stacked.q8.attn_v.weight"],
        "q8_o": w["stacked.q8.attn_output.weight"],
        "q8_gate_up": w["stacked.q8.ffn_gate_up.weight"],
        "q8_down": w["stacked.q8.ffn_down.weight"],
    }


def total_bytes(w: dict[str, np.ndarray]) -> int:
    seen, n = set(), 0
    for a in w.values():
        if id(a) not in seen:
            seen.add(id(a))
            n += a.nbytes
    return n
