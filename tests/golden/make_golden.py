"""Generate the Q8_0 golden vectors from the reference's OWN functions.

Run in the build container, where the reference checkout exists:

    python tests/golden/make_golden.py [--ref <reference checkout>]

(default: $Q3_REFERENCE, else a checkout named `reference` beside this
repository).

It imports quantize_q8_0 / dequant_q8_0 from the reference's
tools/create_q8_irpa.py (lines 103-129; the module imports only numpy and
struct at top level) and records their outputs on seeded inputs into
tests/golden/q8_golden.npz.  The tests never read the reference tree; they
read this committed fixture.
"""
import argparse
import hashlib
import importlib.util
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(ref_root):
    path = os.path.join(ref_root, "tools", "create_q8_irpa.py")
    spec = importlib.util.spec_from_file_location("ref_create_q8_irpa", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def edge_blocks():
    """Blocks exercising the quantizer's corner cases."""
    rng = np.random.default_rng(7)
    blocks = []
    blocks.append(np.zeros(32, np.float32))                        # amax 0 -> scale 1.0
    b = np.zeros(32, np.float32); b[5] = 0.5; blocks.append(b)      # single nonzero
    b = rng.standard_normal(32).astype(np.float32); b[0] = -4.0; blocks.append(b)  # negative amax
    blocks.append(np.full(32, 1e-9, np.float32))                   # scale underflows in f16
    blocks.append(np.linspace(-1000, 1000, 32).astype(np.float32))  # large magnitudes
    # values whose quotient by the scale lands on .5 (round-half-even)
    b = (np.arange(32, dtype=np.float32) - 16.0) * np.float32(0.5); b[31] = 127.0
    blocks.append(b)
    b = (np.arange(32, dtype=np.float32) + 0.5); b[0] = -127.0; blocks.append(b)
    blocks.append(np.full(32, -3.25, np.float32))                  # all equal, negative
    return np.concatenate(blocks)


def main():
    ap = argparse.ArgumentParser()
    here = os.path.dirname(os.path.abspath(__file__))
    sibling = os.path.normpath(os.path.join(here, "..", "..", "..", "reference"))
    ap.add_argument("--ref", default=os.environ.get("Q3_REFERENCE", sibling))
    args = ap.parse_args()
    ref = load_reference(args.ref)

    out = {}
    # (1) seeded N(0, 0.02) weights, a [64, 256] matrix
    rng = np.random.default_rng(1234)
    w = (rng.standard_normal((64, 256), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    out["small_w"] = w
    out["small_q8"] = ref.quantize_q8_0(w).view(np.uint8)
    out["small_deq"] = ref.dequant_q8_0(out["small_q8"].tobytes(), w.shape).astype(np.float32)
    # (2) edge-case blocks
    e = edge_blocks()
    out["edge_w"] = e
    out["edge_q8"] = ref.quantize_q8_0(e).view(np.uint8)
    out["edge_deq"] = ref.dequant_q8_0(out["edge_q8"].tobytes(), e.shape).astype(np.float32)
    # (3) config 1 (attn_q [2048,1024], N(0,0.02), seed 0) -- digest only
    rng = np.random.default_rng(0)
    wq = rng.standard_normal((2048, 1024), dtype=np.float32) * np.float32(0.02)
    q = ref.quantize_q8_0(wq).view(np.uint8)
    out["cfg1_sha256"] = np.frombuffer(hashlib.sha256(q.tobytes()).digest(), np.uint8)
    out["cfg1_nbytes"] = np.array([q.size], np.int64)
    path = os.path.join(HERE, "q8_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
