"""The .irpa reader (q3b200/irpa.py): archives round-trip through the writer
of the same version-0 layout, malformed files are refused with a clear error,
and the Qwen3 loader maps the names tools/create_q8_irpa.py:146-224 writes
(output.weight transposed to [1024, 151936]) onto the stacked layout the
decoder uses, byte for byte."""
import os

import numpy as np
import pytest


def test_round_trip(tmp_path):
    from q3b200.irpa import IrpaArchive, write_irpa

    rng = np.random.default_rng(0)
    params = {"a": rng.integers(0, 255, 1000, dtype=np.uint8),
              "b.weight": rng.standard_normal((3, 5)).astype(np.float16),
              "stacked.q8.x": rng.integers(-128, 127, (2, 34), dtype=np.int8),
              "empty": np.zeros(0, np.uint8)}
    p = str(tmp_path / "t.irpa")
    write_irpa(p, params)
    with IrpaArchive(p) as a:
        assert a.names() == list(params)
        for k, v in params.items():
            assert a.raw(k).tobytes() == v.tobytes(), k


def test_malformed_archives_are_refused(tmp_path):
    from q3b200.irpa import IrpaArchive, IrpaError, write_irpa

    p = str(tmp_path / "bad.irpa")
    open(p, "wb").write(b"GGUF" + b"\0" * 200)
    with pytest.raises(IrpaError, match="not an IRPA"):
        IrpaArchive(p)
    write_irpa(p, {"w": np.arange(100, dtype=np.float32)})
    data = open(p, "rb").read()
    open(p, "wb").write(data[:-64])  # storage cut short
    with pytest.raises(IrpaError, match="past the end"):
        IrpaArchive(p)


def test_qwen3_loader_maps_the_reference_names(tmp_path):
    from q3b200.irpa import load_qwen3_q8_irpa, write_irpa
    from q3b200.weights import synthetic_weights

    w = synthetic_weights(seed=7, layers=1)
    ref_names = {  # tools/create_q8_irpa.py:146-224
        "token_embd.weight": w["token_embd.weight"],
        "output_norm.weight": w["output_norm.weight"],
        "output.weight": np.ascontiguousarray(w["output_T.weight"].T),  # [1024, 151936]
    }
    for k in ("stacked.attn_norm.weight", "stacked.ffn_norm.weight", "stacked.attn_q_norm.weight",
              "stacked.attn_k_norm.weight", "stacked.q8.attn_q.weight", "stacked.q8.attn_k.weight",
              "stacked.q8.attn_v.weight", "stacked.q8.attn_output.weight",
              "stacked.q8.ffn_gate_up.weight", "stacked.q8.ffn_down.weight"):
        ref_names[k] = w[k]
    p = str(tmp_path / "qwen3-0.6b-q8-stacked.irpa")
    write_irpa(p, ref_names)
    got = load_qwen3_q8_irpa(p)
    os.remove(p)
    assert set(got) == set(w)
    for k in w:
        assert got[k].shape == w[k].shape, k
        assert np.array_equal(got[k].view(np.uint8), w[k].view(np.uint8)), k
    assert got["output_T.weight"] is got["token_embd.weight"]  # tied, one buffer
