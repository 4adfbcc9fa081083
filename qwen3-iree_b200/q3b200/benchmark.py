"""ctypes twin of the reference's scripts/benchmark.py.

The reference times `@run` of an IREE module once per prompt
(scripts/benchmark.py:52-81): chat-formatted prompt tokens in, up to
MAX_TOKENS greedy tokens out, output cut at the first end-of-text token,
tok/s = kept tokens / wall time of the call, then mean +- std over the
prompts (:157-170) and a JSON dump (:203-206).  This twin makes the same
calls through libq3b200.so (`Qwen3Decoder.run` = q3_run), with no IREE and
no PyTorch.

Differences forced by this environment: there is no checkpoint or
tokenizer.json here, so weights are the seeded random-init model of the
benchmark configs unless --irpa (the reference's archives) or --gguf names a
Q8_0 checkpoint, and prompts are
token-id lists -- seeded ones by default, one line of ids per prompt with
--prompts-file, or text with --tokenizer.

  python -m q3b200.benchmark [--max-tokens 128] [--json out.json]
  python -m q3b200.benchmark --batch 32 --context 128 2048 --steps 128
  python -m q3b200.benchmark --num-prompts 1 --prompt-len 1 --max-tokens 3 --no-warmup
      (the smallest whole decode: 4 steps of 141 launches, for profilers)
  python -m q3b200.benchmark --gemv-stream gate_up   (GEMV HBM GB/s, 28 layers a launch)
"""
from __future__ import annotations

import argparse
import json
import sys
import time

import numpy as np

EOS_TOKEN = 151645
MAX_TOKENS = 128
VOCAB = 151936
CHAT_TEMPLATE = "<|im_start|>user\n{}<|im_end|>\n<|im_start|>assistant\n"


def trim_eos(tokens, eos: int = EOS_TOKEN) -> list[int]:
    """Tokens up to (not including) the first end-of-text token
    (scripts/benchmark.py:77-79)."""
    tokens = [int(t) for t in tokens]
    return tokens[:tokens.index(eos)] if eos in tokens else tokens


def synthetic_prompts(n: int = 10, seed: int = 0, length: int = 0) -> list[list[int]]:
    """n seeded token-id prompts: of increasing length (12..48 ids, the range
    of short chat-formatted questions), or all `length` ids long."""
    rng = np.random.default_rng(seed)
    lengths = [length] * n if length > 0 else np.linspace(12, 48, n).astype(int)
    return [rng.integers(0, VOCAB, size=int(L)).tolist() for L in lengths]


def read_prompts_file(path: str) -> list[list[int]]:
    """One prompt per non-empty line: whitespace- or comma-separated token ids."""
    out = []
    for line in open(path):
        ids = [int(t) for t in line.replace(",", " ").split()]
        if ids:
            out.append(ids)
    return out


def load_tokenizer(path: str | None):
    if not path:
        return None
    from tokenizers import Tokenizer  # optional dependency, only with --tokenizer

    return Tokenizer.from_file(path)


def load_weights(args):
    """The checkpoint given with --irpa (the reference's archives) or --gguf,
    else the seeded random-init model."""
    if getattr(args, "irpa", None):
        from .irpa import load_qwen3_q8_irpa

        return load_qwen3_q8_irpa(*args.irpa)
    if getattr(args, "gguf", None):
        from .gguf import load_qwen3_q8

        return load_qwen3_q8(args.gguf)
    from .weights import synthetic_weights

    return synthetic_weights(seed=args.seed)


def bench_one(dec, tokens: list[int], max_tokens: int, eos: int = EOS_TOKEN):
    """One @run call (scripts/benchmark.py:52-81): (n_in, n_out, seconds)."""
    t0 = time.perf_counter()
    out, n = dec.run(np.asarray(tokens, np.int64), max_tokens, eos)
    dt = time.perf_counter() - t0
    return len(tokens), len(trim_eos(out[:n], eos)), dt


def bench_batched(dw, B: int, lo: int, hi: int, steps: int, seed: int = 0) -> dict:
    """B sequences with cached contexts of U[lo, hi] positions, `steps`
    decode steps of all of them on the tensor-core batched path."""
    from . import BatchDecoder, Events

    rng = np.random.default_rng(seed + B)
    ctx = rng.integers(lo, hi + 1, size=B)
    tok = rng.integers(0, VOCAB, size=B)
    bd = BatchDecoder(dw, max_batch=B, max_seq_len=int(hi + steps + 5))
    bd.begin_random(ctx, tok, seed=seed)
    bd.steps(3)
    bd.synchronize()
    ev = Events()
    ev.record_start(bd.stream)
    bd.steps(steps)
    ev.record_end(bd.stream)
    ms = ev.elapsed_ms()
    _, pos = bd.read()
    bd.close()
    assert (pos == ctx + 3 + steps).all()
    return {"batch": B, "context": [lo, hi], "steps": steps, "ms_per_step": ms / steps,
            "tok_s": B * steps / (ms / 1e3)}


GEMV_STREAM_SHAPES = {  # projection: (stacked parameter, N, K)
    "attn_q": ("stacked.q8.attn_q.weight", 2048, 1024),
    "attn_o": ("stacked.q8.attn_output.weight", 1024, 2048),
    "gate_up": ("stacked.q8.ffn_gate_up.weight", 6144, 1024),
    "down": ("stacked.q8.ffn_down.weight", 1024, 3072),
}


def gemv_stream(dw, name: str, reps: int = 20, warmup: int = 3) -> dict:
    """One projection over all 28 layers in ONE launch (q3_gemv_q8_layers):
    the streaming bandwidth of the Q8_0 GEMV without launch gaps.  L2 is
    flushed (a 256 MB write) before every timed launch, so the 62 MB pools
    of attn_q and attn_o are read from HBM like the larger ones."""
    from . import DeviceArray, Events
    from ._lib import lib

    key, N, K = GEMV_STREAM_SHAPES[name]
    L = lib()
    w = dw.buffers[key]
    bpl = N * (K // 32) * 34
    x = DeviceArray.from_host(np.random.default_rng(1).standard_normal((28, K)).astype(np.float16))
    y = DeviceArray((28, N), np.float16)
    flush = DeviceArray((256 << 20,), np.uint8)
    ev = Events()
    for _ in range(warmup):
        assert L.q3_gemv_q8_layers(w.ptr, bpl, x.ptr, y.ptr, N, K, 28, None) == 0
    total_ms = 0.0
    for r in range(reps):
        flush.fill_bytes(r & 0xFF)
        ev.record_start(None)
        assert L.q3_gemv_q8_layers(w.ptr, bpl, x.ptr, y.ptr, N, K, 28, None) == 0
        ev.record_end(None)
        total_ms += ev.elapsed_ms()
    flush.free()
    us = total_ms * 1e3 / reps
    b = 28 * (bpl + 2 * K + 2 * N)
    return {"us_per_launch": us, "bytes": b, "gbs": b / (us * 1e-6) / 1e9, "l2": "flushed"}


class _Graph:
    """A CUDA graph of the calls made inside `with` on a created stream."""

    def __init__(self, stream):
        self.stream, self.exec = stream, None

    def __enter__(self):
        from ._lib import call

        call("q3_graph_capture_begin", self.stream)
        return self

    def __exit__(self, *exc):
        import ctypes

        from ._lib import call

        e = ctypes.c_void_p()
        call("q3_graph_capture_end", self.stream, ctypes.byref(e))
        self.exec = e.value
        return False

    def launch(self):
        from ._lib import call

        call("q3_graph_launch", self.exec, self.stream)

    def close(self):
        from ._lib import lib

        if self.exec:
            lib().q3_graph_destroy(self.exec)
            self.exec = None


def _stream():
    import ctypes

    from ._lib import call

    s = ctypes.c_void_p()
    call("q3_stream_create", ctypes.byref(s))
    return s.value


# one attn_q-shaped Q8_0 GEMV [2048, 1024]
GEMV_POOL = 64            # distinct weight matrices (143 MB, larger than the 126 MB L2)
GEMV_N, GEMV_K = 2048, 1024
GEMV_ALG_BYTES = GEMV_N * (GEMV_K // 32) * 34 + 2 * GEMV_K + 2 * GEMV_N


def gemv_pool(seed: int = 0, reps: int = 20, warmup: int = 3) -> dict:
    """the attn_q GEMV over a rotating pool of 64 seeded matrices
    (W N(0,0.02) quantised Q8_0, x N(0,1) f16), larger than L2, so every call
    reads its weights from HBM.  One CUDA graph holds a call per matrix:
    q3_gemv_q8_overlapped (each call's weight copies start while the previous
    call runs) and, for comparison, q3_gemv_q8 (each call after the previous
    one).  Device time of whole replays / calls."""
    from . import DeviceArray, Events
    from ._lib import call
    from .weights import make_q8_matrix

    rng = np.random.default_rng(seed)
    mats = [make_q8_matrix(rng, GEMV_N, GEMV_K) for _ in range(GEMV_POOL)]
    w = DeviceArray.from_host(np.stack(mats))
    x = DeviceArray.from_host(rng.standard_normal(GEMV_K).astype(np.float16))
    y = DeviceArray((GEMV_POOL, GEMV_N), np.float16)
    bpm = mats[0].nbytes
    st = _stream()
    ev = Events()
    out = {"workload": f"configs[0]: Q8_0 GEMV [{GEMV_N},{GEMV_K}], a rotating pool of "
                       f"{GEMV_POOL} matrices ({GEMV_POOL * bpm / 1e6:.0f} MB > L2)",
           "alg_bytes_per_call": GEMV_ALG_BYTES}
    for name in ("q3_gemv_q8_overlapped", "q3_gemv_q8"):
        g = _Graph(st)
        with g:
            for i in range(GEMV_POOL):
                call(name, w.ptr + i * bpm, x.ptr, y.ptr + i * GEMV_N * 2, GEMV_N, GEMV_K, st)
        for _ in range(warmup):
            g.launch()
        ev.record_start(st)
        for _ in range(reps):
            g.launch()
        ev.record_end(st)
        us = ev.elapsed_ms() * 1e3 / (reps * GEMV_POOL)
        g.close()
        out[name] = {"us_per_call": us, "gbs": GEMV_ALG_BYTES / (us * 1e-6) / 1e9}
    from ._lib import lib

    lib().q3_stream_destroy(st)
    return out


# one decoder layer at position 511 over a 512-position cache
LAYER_S, LAYER_POS = 512, 511
LAYER_ALG_BYTES = (2228224 + 2 * 1114112 + 2228224 + 6684672 + 3342336  # Q8_0 weights
                   + 4 * 1024 * 2 + 2 * 128 * 2                          # gammas
                   + 2 * (LAYER_POS + 1) * 8 * 128 * 2                   # K and V read
                   + 2 * 8 * 128 * 2                                     # new K/V row written
                   + 2 * 1024 * 2)                                       # x in, x out


def layer_bench(dw, seed: int = 0, reps: int = 10, warmup: int = 3) -> dict:
    """q3_fused_layer at position 511 over a cache of 512
    positions (511 cached N(0,1) rows).  One CUDA graph runs the layer once
    for each of the 28 layers' weights (468 MB, larger than L2), each over its
    own cache slice; device time per layer call."""
    import ctypes

    from . import DeviceArray, Events
    from ._lib import call, lib

    rng = np.random.default_rng(seed)
    S, pos = LAYER_S, LAYER_POS
    kv = rng.standard_normal((28 * S, 8, 128)).astype(np.float16)
    kc, vc = DeviceArray.from_host(kv), DeviceArray.from_host(kv[::-1].copy())
    xs = [DeviceArray.from_host(rng.standard_normal(1024).astype(np.float16)) for _ in range(2)]
    dpos = DeviceArray.from_host(np.array([pos], np.int64))
    c = np.empty((S, 64), np.float32)
    sn = np.empty((S, 64), np.float32)
    call("q3_rope_table", S, c.ctypes.data, sn.ctypes.data)
    dc, ds = DeviceArray.from_host(c), DeviceArray.from_host(sn)
    ws = DeviceArray((lib().q3_fused_layer_workspace_bytes(),), np.uint8, zero=True)
    st = _stream()
    g = _Graph(st)
    with g:
        for l in range(28):
            call("q3_fused_layer", ctypes.byref(dw.struct), l, xs[l % 2].ptr, xs[(l + 1) % 2].ptr,
                 kc.ptr, vc.ptr, S, dpos.ptr, dc.ptr, ds.ptr, ws.ptr, 1, st)
    ev = Events()
    for _ in range(warmup):
        g.launch()
    ev.record_start(st)
    for _ in range(reps):
        g.launch()
    ev.record_end(st)
    us = ev.elapsed_ms() * 1e3 / (reps * 28)
    g.close()
    lib().q3_stream_destroy(st)
    return {"workload": "configs[1]: one decoder layer at position 511, cache of 512 positions, "
                        "the 28 layers' weights in turn (468 MB > L2)",
            "call": "q3_fused_layer (attention block, feed-forward block, residual rebuild)",
            "us_per_layer": us, "alg_bytes_per_layer": LAYER_ALG_BYTES,
            "gbs": LAYER_ALG_BYTES / (us * 1e-6) / 1e9}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Benchmark Qwen3-0.6B Q8_0 decode on libq3b200.so")
    ap.add_argument("--max-tokens", type=int, default=MAX_TOKENS)
    ap.add_argument("--prompts-file", default=None, help="one line of token ids per prompt")
    ap.add_argument("--tokenizer", default=None, help="tokenizer.json (text prompts)")
    ap.add_argument("--text", action="append", default=None, help="text prompt (with --tokenizer)")
    ap.add_argument("--seed", type=int, default=0, help="weights and synthetic prompts")
    ap.add_argument("--gguf", default=None, help="Qwen3-0.6B Q8_0 GGUF checkpoint (else random init)")
    ap.add_argument("--irpa", nargs="+", default=None,
                    help="the reference's .irpa archive(s) (tools/create_q8_irpa.py output)")
    ap.add_argument("--engine", default=None, choices=["fused", "graph", "persistent"],
                    help="decode engine (default: the library's, fused where available)")
    ap.add_argument("--max-seq-len", type=int, default=1024)
    ap.add_argument("--json", default=None, help="write results here")
    ap.add_argument("--batch", type=int, default=0, help="batched mode: B sequences")
    ap.add_argument("--context", type=int, nargs=2, default=[128, 2048], metavar=("LO", "HI"))
    ap.add_argument("--steps", type=int, default=128, help="batched mode: decode steps")
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--num-prompts", type=int, default=10, help="synthetic prompts")
    ap.add_argument("--prompt-len", type=int, default=0, help="synthetic prompt length (0: 12..48)")
    ap.add_argument("--no-warmup", action="store_true", help="skip the untimed first call")
    ap.add_argument("--gemv-stream", choices=sorted(GEMV_STREAM_SHAPES), default=None,
                    help="time one projection over all 28 layers per launch")
    ap.add_argument("--reps", type=int, default=20, help="with --gemv-stream: timed launches")
    args = ap.parse_args(argv)

    from . import DeviceWeights, Qwen3Decoder, set_device

    set_device(args.device)
    dw = DeviceWeights(load_weights(args))

    if args.gemv_stream:
        r = gemv_stream(dw, args.gemv_stream, args.reps, 0 if args.no_warmup else 3)
        print(f"  {args.gemv_stream} x 28 layers: {r['us_per_launch']:.1f} us/launch, "
              f"{r['gbs']:.0f} GB/s", flush=True)
        if args.json:
            with open(args.json, "w") as f:
                json.dump(r, f, indent=2)
        return 0

    if args.batch:
        r = bench_batched(dw, args.batch, args.context[0], args.context[1], args.steps, args.seed)
        print(f"  B={r['batch']} context U[{args.context[0]},{args.context[1]}] "
              f"{r['steps']} steps: {r['ms_per_step']:.3f} ms/step, {r['tok_s']:.0f} tok/s",
              flush=True)
        if args.json:
            with open(args.json, "w") as f:
                json.dump(r, f, indent=2)
        return 0

    tok = load_tokenizer(args.tokenizer)
    if tok is not None and args.text:
        prompts = [tok.encode(CHAT_TEMPLATE.format(t)).ids for t in args.text]
        labels = [t[:40] for t in args.text]
    else:
        prompts = (read_prompts_file(args.prompts_file) if args.prompts_file
                   else synthetic_prompts(args.num_prompts, args.seed, args.prompt_len))
        labels = [f"{len(p)} ids" for p in prompts]

    dec = Qwen3Decoder(dw, max_seq_len=args.max_seq_len, engine=args.engine)
    if not args.no_warmup:
        bench_one(dec, prompts[0], 4)  # graph capture and first-call set-up
    tps = []
    for i, (p, label) in enumerate(zip(prompts, labels)):
        n_in, n_out, dt = bench_one(dec, p, args.max_tokens)
        tps.append(n_out / dt if dt > 0 else 0.0)
        print(f"  [{i + 1:2d}/{len(prompts)}] {label:<40s} in={n_in:3d} out={n_out:3d} "
              f"{dt:6.3f}s {tps[-1]:7.1f} tok/s", flush=True)
    mean, std = float(np.mean(tps)), float(np.std(tps))
    print(f"  -> mean={mean:.1f} +- {std:.1f} tok/s", flush=True)
    if args.json:
        with open(args.json, "w") as f:
            json.dump({"libq3b200": {"tps": tps, "mean": mean, "std": std,
                                     "prompts": labels, "engine": dec.engine}}, f, indent=2)
    dec.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
