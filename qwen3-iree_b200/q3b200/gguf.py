"""Qwen3-0.6B Q8_0 weights from a GGUF checkpoint, in the stacked parameter
layout the decoder uses -- the layout tools/create_q8_irpa.py:146-224 builds
for the reference's IRPA archive -- so a real checkpoint can replace the
seeded random init:

  * stacked.q8.{attn_q,attn_k,attn_v,attn_output,ffn_down}.weight:
    [28, bytes per layer] raw Q8_0 blocks, GGUF-native [N, K] order;
  * stacked.q8.ffn_gate_up.weight: each layer's gate blocks then up blocks;
  * stacked.{attn,ffn,attn_q,attn_k}_norm.weight: [28, n] f16;
  * token_embd.weight, output_norm.weight: f16 (Q8_0 embeddings dequantised
    as f16(f32(scale) * q), tools/create_q8_irpa.py:121-129);
  * output_T.weight: the vocab matrix as [vocab, dim] f16 rows -- GGUF's own
    orientation of output.weight, which the vocab kernel reads directly (the
    reference transposes it for its matmul, :157-165); the token embedding
    when the checkpoint ties them.

GGUF container (llama.cpp, versions 2 and 3): little-endian magic "GGUF",
version u32, tensor count u64, metadata count u64, the metadata key/values,
the tensor infos (name, dims innermost first, ggml type, data offset), then
the tensor data from the next multiple of general.alignment (default 32).
ggml types read here: 0 f32, 1 f16, 8 q8_0.
"""
from __future__ import annotations

import struct

import numpy as np

from .weights import DIM, FFN, HD, LAYERS, QBLK, QBYTES, VOCAB, bytes_per_layer

GGUF_MAGIC = 0x46554747
GGML_F32, GGML_F16, GGML_Q8_0 = 0, 1, 8
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q",
           11: "<q", 12: "<d"}


class GGUFError(ValueError):
    pass


def _read_value(buf, off: int, vtype: int):
    if vtype in _SCALAR:
        fmt = _SCALAR[vtype]
        return struct.unpack_from(fmt, buf, off)[0], off + struct.calcsize(fmt)
    if vtype == 8:
        n = struct.unpack_from("<Q", buf, off)[0]
        return bytes(buf[off + 8:off + 8 + n]).decode("utf-8"), off + 8 + n
    if vtype == 9:
        atype, n = struct.unpack_from("<IQ", buf, off)
        off += 12
        vals = []
        for _ in range(n):
            v, off = _read_value(buf, off, atype)
            vals.append(v)
        return vals, off
    raise GGUFError(f"unknown metadata value type {vtype}")


def read_gguf(path: str):
    """(metadata dict, {name: (array view of the raw data, numpy shape, ggml type)})."""
    buf = np.memmap(path, dtype=np.uint8, mode="r")
    if len(buf) < 24 or struct.unpack_from("<I", buf, 0)[0] != GGUF_MAGIC:
        raise GGUFError(f"{path}: not a GGUF file")
    version, n_tensors, n_kv = struct.unpack_from("<IQQ", buf, 4)
    if version not in (2, 3):
        raise GGUFError(f"{path}: GGUF version {version} unsupported")
    off = 24
    meta = {}
    for _ in range(n_kv):
        key, off = _read_value(buf, off, 8)
        vtype = struct.unpack_from("<I", buf, off)[0]
        meta[key], off = _read_value(buf, off + 4, vtype)
    infos = []
    for _ in range(n_tensors):
        name, off = _read_value(buf, off, 8)
        nd = struct.unpack_from("<I", buf, off)[0]
        dims = struct.unpack_from(f"<{nd}Q", buf, off + 4)
        off += 4 + 8 * nd
        ttype, toff = struct.unpack_from("<IQ", buf, off)
        off += 12
        infos.append((name, tuple(reversed(dims)), ttype, toff))
    align = int(meta.get("general.alignment", 32))
    data0 = (off + align - 1) // align * align
    tensors = {}
    for name, shape, ttype, toff in infos:
        n = int(np.prod(shape, dtype=np.int64))
        if ttype == GGML_F32:
            nbytes = 4 * n
        elif ttype == GGML_F16:
            nbytes = 2 * n
        elif ttype == GGML_Q8_0:
            if n % QBLK:
                raise GGUFError(f"{name}: {n} elements is not a whole number of Q8_0 blocks")
            nbytes = n // QBLK * QBYTES
        else:
            tensors[name] = (None, shape, ttype)  # a type the decode path does not read
            continue
        start = data0 + toff
        if start + nbytes > len(buf):
            raise GGUFError(f"{name}: data runs past the end of the file")
        tensors[name] = (buf[start:start + nbytes], shape, ttype)
    return meta, tensors


def dequant_q8_0_f16(raw: np.ndarray, shape) -> np.ndarray:
    """Q8_0 blocks -> f16(f32(scale) * q) (tools/create_q8_irpa.py:121-129)."""
    blocks = np.asarray(raw, dtype=np.uint8).reshape(-1, QBYTES)
    scale = blocks[:, :2].copy().view(np.float16).astype(np.float32)
    q = blocks[:, 2:].view(np.int8).astype(np.float32)
    return (scale * q).astype(np.float16).reshape(shape)


def _f16(tensors, name: str, shape) -> np.ndarray:
    if name not in tensors:
        raise GGUFError(f"tensor {name} missing")
    raw, tshape, ttype = tensors[name]
    if int(np.prod(tshape)) != int(np.prod(shape)):
        raise GGUFError(f"{name}: shape {tshape}, expected {shape}")
    if ttype == GGML_F16:
        return np.array(raw).view(np.float16).reshape(shape)
    if ttype == GGML_F32:
        return np.array(raw).view(np.float32).astype(np.float16).reshape(shape)
    if ttype == GGML_Q8_0:
        return dequant_q8_0_f16(raw, shape)
    raise GGUFError(f"{name}: ggml type {ttype} not readable as f16")


def _q8(tensors, name: str, N: int, K: int) -> np.ndarray:
    if name not in tensors:
        raise GGUFError(f"tensor {name} missing")
    raw, shape, ttype = tensors[name]
    if ttype != GGML_Q8_0 or tuple(shape) != (N, K):
        raise GGUFError(f"{name}: {shape} type {ttype}, expected Q8_0 [{N}, {K}]")
    return np.asarray(raw)


def load_qwen3_q8(path: str, layers: int = LAYERS) -> dict[str, np.ndarray]:
    """The decoder's parameter dict (the keys synthetic_weights returns) from
    a Qwen3-0.6B Q8_0 GGUF.  Layers at or beyond `layers` stay zero (small
    test checkpoints)."""
    _, t = read_gguf(path)
    w: dict[str, np.ndarray] = {}
    emb = _f16(t, "token_embd.weight", (VOCAB, DIM))
    w["token_embd.weight"] = emb
    w["output_T.weight"] = _f16(t, "output.weight", (VOCAB, DIM)) if "output.weight" in t else emb
    w["output_norm.weight"] = _f16(t, "output_norm.weight", (DIM,))
    for key, n in (("attn_norm", DIM), ("ffn_norm", DIM), ("attn_q_norm", HD), ("attn_k_norm", HD)):
        st = np.zeros((LAYERS, n), np.float16)
        for l in range(layers):
            st[l] = _f16(t, f"blk.{l}.{key}.weight", (n,))
        w[f"stacked.{key}.weight"] = st
    plain = (("attn_q", 2048, DIM), ("attn_k", 1024, DIM), ("attn_v", 1024, DIM),
             ("attn_output", DIM, 2048), ("ffn_down", DIM, FFN))
    for key, N, K in plain:
        st = np.zeros((LAYERS, bytes_per_layer(N, K)), np.uint8)
        for l in range(layers):
            st[l] = _q8(t, f"blk.{l}.{key}.weight", N, K)
        w[f"stacked.q8.{key}.weight"] = st
    half = bytes_per_layer(FFN, DIM)
    gu = np.zeros((LAYERS, 2 * half), np.uint8)
    for l in range(layers):
        gu[l, :half] = _q8(t, f"blk.{l}.ffn_gate.weight", FFN, DIM)
        gu[l, half:] = _q8(t, f"blk.{l}.ffn_up.weight", FFN, DIM)
    w["stacked.q8.ffn_gate_up.weight"] = gu
    return w
