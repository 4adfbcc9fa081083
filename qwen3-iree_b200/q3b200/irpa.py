"""Reader (and writer) of IREE parameter archives (.irpa), the container the
reference's hosts load its weights from (scripts/benchmark.py:38-45; written
by tools/create_q8_irpa.py:185-226 through iree.runtime.ParameterIndex).

The archive holds named byte ranges and no type information; the reference's
module knows each parameter's type and shape.  ``load_qwen3_q8_irpa`` does the
same: it reads the names tools/create_q8_irpa.py writes and reinterprets
their bytes in the layout of q3b200.weights (f16 norms and embedding, the
stacked Q8_0 matrices), transposing ``output.weight`` -- stored as
[1024, 151936] for the reference's matmul -- back to the [151936, 1024] rows
of the vocab GEMV.

Layout read (IREE parameter archive, format version 0), all little-endian:

  header   u32 magic 'IRPA' | u16 major | u16 minor | u64 header_size |
           u64 next_header_offset | u64 flags | u64 entry_count |
           3 x (u64 offset, u64 length): entry, metadata, storage segments
  entry    u64 entry_size | u32 type | u32 flags | (u64, u64) name |
           (u64, u64) metadata | u64 minimum_alignment, then
           type 2 (data):  (u64 offset, u64 length) into the storage segment
           type 1 (splat): u64 length | 16-byte pattern | u8 pattern_length
           type 0: skipped
  Segment offsets count from the start of the header, entry ranges from the
  start of their segment.

Only host memory and numpy are involved; no IREE runtime is needed.
"""
from __future__ import annotations

import mmap
import struct

import numpy as np

MAGIC = 0x41505249  # "IRPA"
_HEADER = struct.Struct("<IHHQQQQQQQQQQ")
_ENTRY = struct.Struct("<QII" "QQ" "QQ" "Q")
_DATA = struct.Struct("<QQ")
_SPLAT = struct.Struct("<Q16sB")
TYPE_SKIP, TYPE_SPLAT, TYPE_DATA = 0, 1, 2


class IrpaError(ValueError):
    pass


class IrpaArchive:
    """Named parameters of one archive, read without copying (mmap)."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        self._m = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self.entries: dict[str, tuple] = {}
        self._parse()

    def _parse(self) -> None:
        m = self._m
        if len(m) < _HEADER.size:
            raise IrpaError(f"{self.path}: shorter than an archive header")
        (magic, major, minor, header_size, next_header, flags, count, e_off, e_len, m_off, m_len,
         s_off, s_len) = _HEADER.unpack_from(m, 0)
        if magic != MAGIC:
            raise IrpaError(f"{self.path}: not an IRPA archive (magic 0x{magic:08x})")
        if major != 0:
            raise IrpaError(f"{self.path}: archive format {major}.{minor}; this reader knows 0.x")
        if next_header != 0:
            raise IrpaError(f"{self.path}: multi-part archives are not supported")
        size = len(m)
        for off, ln, what in ((e_off, e_len, "entry"), (m_off, m_len, "metadata"),
                              (s_off, s_len, "storage")):
            if off + ln > size:
                raise IrpaError(f"{self.path}: {what} segment [{off}, {off + ln}) past the end ({size})")
        pos = e_off
        for i in range(count):
            if pos + _ENTRY.size > e_off + e_len:
                raise IrpaError(f"{self.path}: entry {i} runs past the entry segment")
            (esize, etype, eflags, n_off, n_len, md_off, md_len, align) = _ENTRY.unpack_from(m, pos)
            if esize < _ENTRY.size or n_off + n_len > m_len:
                raise IrpaError(f"{self.path}: entry {i} is malformed")
            name = bytes(m[m_off + n_off:m_off + n_off + n_len]).decode("utf-8")
            body = pos + _ENTRY.size
            if etype == TYPE_DATA:
                d_off, d_len = _DATA.unpack_from(m, body)
                if d_off + d_len > s_len:
                    raise IrpaError(f"{self.path}: data of {name!r} past the storage segment")
                self.entries[name] = ("data", s_off + d_off, d_len)
            elif etype == TYPE_SPLAT:
                length, pattern, plen = _SPLAT.unpack_from(m, body)
                self.entries[name] = ("splat", pattern[:plen], length)
            pos += esize

    def names(self) -> list[str]:
        return list(self.entries)

    def raw(self, name: str) -> np.ndarray:
        """The parameter's bytes (a read-only view for data entries)."""
        kind, a, b = self.entries[name]
        if kind == "data":
            return np.frombuffer(self._m, dtype=np.uint8, count=b, offset=a)
        pattern, length = a, b
        reps = length // len(pattern)
        return np.frombuffer(pattern * reps, dtype=np.uint8)

    def close(self) -> None:
        self._m.close()
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def write_irpa(path: str, params: dict[str, np.ndarray], alignment: int = 64) -> None:
    """Write named byte buffers as a version-0 archive (data entries, storage
    aligned to `alignment`): the layout IrpaArchive reads."""
    names = list(params)
    metadata = bytearray()
    name_refs = []
    for n in names:
        b = n.encode("utf-8")
        name_refs.append((len(metadata), len(b)))
        metadata += b
    storage_refs, off = [], 0
    for n in names:
        nbytes = np.ascontiguousarray(params[n]).nbytes
        off = (off + alignment - 1) // alignment * alignment
        storage_refs.append((off, nbytes))
        off += nbytes
    storage_len = off
    entry_size = _ENTRY.size + _DATA.size
    e_off = _HEADER.size
    e_len = entry_size * len(names)
    m_off = e_off + e_len
    m_len = len(metadata)
    s_off = (m_off + m_len + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(_HEADER.pack(MAGIC, 0, 0, _HEADER.size, 0, 0, len(names), e_off, e_len, m_off,
                             m_len, s_off, storage_len))
        for (n_off, n_len), (d_off, d_len) in zip(name_refs, storage_refs):
            f.write(_ENTRY.pack(entry_size, TYPE_DATA, 0, n_off, n_len, 0, 0, alignment))
            f.write(_DATA.pack(d_off, d_len))
        f.write(bytes(metadata))
        f.write(b"\0" * (s_off - (m_off + m_len)))
        for n, (d_off, d_len) in zip(names, storage_refs):
            here = f.tell() - s_off
            f.write(b"\0" * (d_off - here))
            f.write(np.ascontiguousarray(params[n]).tobytes())


# tools/create_q8_irpa.py:146-224 names -> (our name, dtype, shape)
_Q8 = {
    "stacked.q8.attn_q.weight": (2048, 1024), "stacked.q8.attn_k.weight": (1024, 1024),
    "stacked.q8.attn_v.weight": (1024, 1024), "stacked.q8.attn_output.weight": (1024, 2048),
    "stacked.q8.ffn_gate_up.weight": (6144, 1024), "stacked.q8.ffn_down.weight": (1024, 3072),
}
_NORMS = {"stacked.attn_norm.weight": 1024, "stacked.ffn_norm.weight": 1024,
          "stacked.attn_q_norm.weight": 128, "stacked.attn_k_norm.weight": 128}


def load_qwen3_q8_irpa(*paths: str) -> dict[str, np.ndarray]:
    """Qwen3-0.6B Q8_0 weights from the archive(s) tools/create_q8_irpa.py
    writes, as the host dict q3b200.weights produces (tied embedding when
    the archive's output.weight equals the embedding)."""
    from .weights import DIM, LAYERS, VOCAB, bytes_per_layer

    found: dict[str, np.ndarray] = {}
    archives = [IrpaArchive(p) for p in paths]
    for a in archives:
        for n in a.names():
            found.setdefault(n, a.raw(n))

    def need(name: str, nbytes: int) -> np.ndarray:
        if name not in found:
            raise IrpaError(f"parameter {name!r} not in {paths}")
        r = found[name]
        if r.size != nbytes:
            raise IrpaError(f"{name!r}: {r.size} bytes, expected {nbytes}")
        return r

    w: dict[str, np.ndarray] = {}
    w["token_embd.weight"] = need("token_embd.weight", VOCAB * DIM * 2).view(np.float16).reshape(VOCAB, DIM).copy()
    w["output_norm.weight"] = need("output_norm.weight", DIM * 2).view(np.float16).copy()
    out_t = need("output.weight", VOCAB * DIM * 2).view(np.float16).reshape(DIM, VOCAB)
    out = np.ascontiguousarray(out_t.T)
    w["output_T.weight"] = w["token_embd.weight"] if np.array_equal(out.view(np.uint16), w["token_embd.weight"].view(np.uint16)) else out
    for name, k in _NORMS.items():
        w[name] = need(name, LAYERS * k * 2).view(np.float16).reshape(LAYERS, k).copy()
    for name, (N, K) in _Q8.items():
        bpl = bytes_per_layer(N, K)
        w[name] = need(name, LAYERS * bpl).reshape(LAYERS, bpl).copy()
    del found, out_t  # the views into the mapped files go before the files close
    for a in archives:
        a.close()
    return w
