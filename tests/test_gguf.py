"""The GGUF checkpoint loader (q3b200.gguf) against the stacked layout the
decoder reads: a 2-layer checkpoint written from the seeded synthetic
weights (token embedding stored Q8_0, norms stored f32 and f16, tied output)
must load back into exactly the arrays the decoder would get."""
import struct

import numpy as np
import pytest

from q3b200 import gguf
from q3b200.weights import FFN, QBYTES, bytes_per_layer, quantize_q8_0, synthetic_weights


def _write_gguf(path, tensors, align=32, version=3):
    """tensors: list of (name, numpy shape, ggml type, raw bytes)."""
    def s(x):
        b = x.encode()
        return struct.pack("<Q", len(b)) + b

    meta = s("general.architecture") + struct.pack("<I", 8) + s("qwen3")
    meta += s("general.alignment") + struct.pack("<I", 4) + struct.pack("<I", align)
    infos, off, blobs = b"", 0, []
    for name, shape, ttype, raw in tensors:
        dims = list(reversed(shape))
        infos += s(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        infos += struct.pack("<IQ", ttype, off)
        blobs.append((off, raw))
        off = (off + len(raw) + align - 1) // align * align
    head = struct.pack("<IIQQ", gguf.GGUF_MAGIC, version, len(tensors), 2) + meta + infos
    data0 = (len(head) + align - 1) // align * align
    with open(path, "wb") as f:
        f.write(head + b"\0" * (data0 - len(head)))
        for o, raw in blobs:
            f.seek(data0 + o)
            f.write(raw)


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    w = synthetic_weights(seed=3, layers=2)
    emb_q8 = quantize_q8_0(w["token_embd.weight"].astype(np.float32))
    T = [("token_embd.weight", (151936, 1024), gguf.GGML_Q8_0, emb_q8.tobytes()),
         ("output_norm.weight", (1024,), gguf.GGML_F16, w["output_norm.weight"].tobytes())]
    plain = (("attn_q", 2048, 1024), ("attn_k", 1024, 1024), ("attn_v", 1024, 1024),
             ("attn_output", 1024, 2048), ("ffn_down", 1024, 3072))
    half = bytes_per_layer(FFN, 1024)
    for l in range(2):
        T.append((f"blk.{l}.attn_norm.weight", (1024,), gguf.GGML_F32,
                  w["stacked.attn_norm.weight"][l].astype(np.float32).tobytes()))
        T.append((f"blk.{l}.ffn_norm.weight", (1024,), gguf.GGML_F16,
                  w["stacked.ffn_norm.weight"][l].tobytes()))
        T.append((f"blk.{l}.attn_q_norm.weight", (128,), gguf.GGML_F32,
                  w["stacked.attn_q_norm.weight"][l].astype(np.float32).tobytes()))
        T.append((f"blk.{l}.attn_k_norm.weight", (128,), gguf.GGML_F32,
                  w["stacked.attn_k_norm.weight"][l].astype(np.float32).tobytes()))
        for key, N, K in plain:
            T.append((f"blk.{l}.{key}.weight", (N, K), gguf.GGML_Q8_0,
                      w[f"stacked.q8.{key}.weight"][l].tobytes()))
        gu = w["stacked.q8.ffn_gate_up.weight"][l]
        T.append((f"blk.{l}.ffn_gate.weight", (3072, 1024), gguf.GGML_Q8_0, gu[:half].tobytes()))
        T.append((f"blk.{l}.ffn_up.weight", (3072, 1024), gguf.GGML_Q8_0, gu[half:].tobytes()))
    path = tmp_path_factory.mktemp("gguf") / "qwen3-0.6b-q8_0.gguf"
    _write_gguf(str(path), T)
    return str(path), w, emb_q8


def test_loader_reproduces_the_decoder_layout(checkpoint, O):
    path, w, emb_q8 = checkpoint
    got = gguf.load_qwen3_q8(path, layers=2)
    assert set(got) == set(w)
    # Q8_0 embedding dequantised like tools/create_q8_irpa.py:121-129, then f16
    want_emb = O.dequant_q8_0(emb_q8, 151936 * 1024).astype(np.float16).reshape(151936, 1024)
    assert np.array_equal(got["token_embd.weight"].view(np.uint16), want_emb.view(np.uint16))
    assert got["output_T.weight"] is got["token_embd.weight"]  # tied
    for k, a in w.items():
        if k in ("token_embd.weight", "output_T.weight"):
            continue
        assert got[k].dtype == a.dtype and got[k].shape == a.shape, k
        if k.startswith("stacked."):  # two layers in the file; the rest stay zero
            assert np.array_equal(got[k][:2].view(np.uint8), a[:2].view(np.uint8)), k
            assert not got[k][2:].any(), k
        else:
            assert np.array_equal(got[k].view(np.uint8), a.view(np.uint8)), k


def test_loader_rejects_bad_files(tmp_path, checkpoint):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOTGGUF" + b"\0" * 64)
    with pytest.raises(gguf.GGUFError):
        gguf.read_gguf(str(bad))
    # a checkpoint without its layers' tensors
    path, w, emb_q8 = checkpoint
    small = tmp_path / "one_layer.gguf"
    _write_gguf(str(small), [("token_embd.weight", (151936, 1024), gguf.GGML_Q8_0, emb_q8.tobytes()),
                             ("output_norm.weight", (1024,), gguf.GGML_F16,
                              w["output_norm.weight"].tobytes())])
    with pytest.raises(gguf.GGUFError, match="missing"):
        gguf.load_qwen3_q8(str(small), layers=1)
    # a projection stored in the wrong type
    wrong = tmp_path / "wrong.gguf"
    _write_gguf(str(wrong), [("blk.0.attn_q.weight", (2048, 1024), gguf.GGML_F16, b"\0" * 2048 * 1024 * 2)])
    _, t = gguf.read_gguf(str(wrong))
    with pytest.raises(gguf.GGUFError, match="Q8_0"):
        gguf._q8(t, "blk.0.attn_q.weight", 2048, 1024)
    assert QBYTES == 34
