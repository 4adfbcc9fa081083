#!/usr/bin/env python3
"""Qwen3-0.6B Q8_0 greedy decode on B200 -- the BASELINE metric.

Workload: 28 layers of Q8_0 projections + GQA
attention over the flat KV cache + tied f16 vocab GEMV + argmax, seeded
random-init weights (N(0,0.02) quantised Q8_0, gammas 1+N(0,0.1)), a 32-token
prompt of ids U[0,151936), 256 generated tokens per sequence, KV cache of
1024 positions.  A "step" is one decode step (one token through all 28 layers
and the vocab head).  Timed steps are grouped in sequences of up to 256
generated tokens; every sequence restarts from the same prompt.

  python bench.py [--gpus N --steps K --warmup W]      our sm_100a path
  python bench.py --impl reference [...]               the CPU oracle (reference arm)

value: tokens/s over all ranks, device time (CUDA events on the decoder's
stream) of the K timed steps, max over ranks, on the library's default
engine (fused: two cluster kernels per layer).  e2e: q3_run (the public call
mirroring the reference's @run) with host prompt in / host tokens out, wall
clock, as scripts/benchmark.py measures it.  N>1 (torchrun): independent
replicas, one per GPU, no collective on the data path (replicas only); the
ranks meet only for the start barrier and the max / sum of their timings,
over gloo (host memory), not NCCL.
roofline: the per-step fraction -- algorithmic bytes of a step (weights + the
KV rows read and written) over the measured step time, against the measured
copy bandwidth -- with each kernel kind's share and bandwidth from the live
kernel trace (global-timer stamps inside the kernels; nothing serialised).
Extra legs: "configs0" (the attn_q GEMV over a rotating
pool larger than L2), "configs1" (configs[1]: one layer at position 511),
"batched" (configs[3] B=32 and configs[4] B=64 per replica, tensor-core
path, device time of 128 steps).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "qwen3-iree_b200"))

METRIC = "Qwen3-0.6B Q8_0 decode tok/s (B=1, B=32) and GEMV HBM GB/s vs 8 TB/s peak"
UNIT = "tok/s"
PROMPT_LEN, GEN_PER_SEQ, CACHE = 32, 256, 1024
EOS = 151645
NOMINAL_HBM_GBS = 8000.0
KIND_NAMES = ["qkv", "attn", "o", "gate_up", "down", "vocab"]
# Algorithmic bytes per launch (weights + activations read and written).
Q8_BYTES = {"qkv": 2228224 + 2 * 1114112, "o": 2228224, "gate_up": 6684672, "down": 3342336}
ACT_BYTES = {"qkv": 2048 + 2048 + 8192, "o": 4096 + 2048 + 2048, "gate_up": 2048 + 2048 + 6144,
             "down": 6144 + 2048 + 2048}
VOCAB_BYTES = 151936 * 1024 * 2 + 2048 + 2048 + 151936 * 2
NORM_BYTES = 28 * (1024 + 1024 + 128 + 128) * 2 + 1024 * 2
KV_ROW = 8 * 128 * 2  # one position of K (or V) for one layer


def step_bytes(pos: int) -> int:
    """Algorithmic HBM bytes of one decode step at position pos (attends pos+1 keys)."""
    w = sum(Q8_BYTES.values()) * 28 + VOCAB_BYTES + NORM_BYTES
    kv = 28 * (2 * KV_ROW * (pos + 1) + 2 * KV_ROW)
    return w + kv


def attn_bytes(pos: int) -> int:
    return 2 * KV_ROW * (pos + 1) + 2 * KV_ROW + 8192 + 4096 + 512


def load_peaks() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_traffic() -> dict:
    """ncu DRAM bytes per launch, from profiles/ncu_traffic.txt ("kind bytes" lines)."""
    out = {}
    p = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    if os.path.exists(p):
        for line in open(p):
            parts = line.split()
            if len(parts) >= 2 and not line.startswith("#"):
                try:
                    out[parts[0]] = float(parts[1])
                except ValueError:
                    pass
    return out


# ---------------------------------------------------------------- clocks
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device, self.lines, self.proc = device, [], None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.device)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


# ---------------------------------------------------------------- distributed plumbing
class Dist:
    """torch.distributed for the barrier and the max/sum over ranks of the
    timings only; the decode itself has no collective (replicas).  gloo over
    host tensors: no NCCL is involved, on the GPU box or in the tests."""

    def __init__(self, backend: str = "gloo"):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.torch = None
        self.device = "cpu"
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist

            # a replica that fails ends the others' next collective with an
            # error after this long, instead of holding them
            timeout = datetime.timedelta(seconds=float(os.environ.get("Q3_DIST_TIMEOUT_S", "300")))
            if backend == "nccl":
                torch.cuda.set_device(self.local)
                dist.init_process_group("nccl", timeout=timeout,
                                        device_id=torch.device("cuda", self.local))
                self.device = "cuda"
            else:
                dist.init_process_group(backend, timeout=timeout)
            self.torch, self.dist = torch, dist

    def barrier(self):
        if self.torch:
            self.dist.barrier()

    def _reduce(self, v: float, op) -> float:
        t = self.torch.tensor([v], dtype=self.torch.float64, device=self.device)
        self.dist.all_reduce(t, op=op)
        return float(t.item())

    def max(self, v: float) -> float:
        return self._reduce(v, self.dist.ReduceOp.MAX) if self.torch else v

    def sum(self, v: float) -> float:
        return self._reduce(v, self.dist.ReduceOp.SUM) if self.torch else v

    def close(self):
        if self.torch:
            self.dist.destroy_process_group()


# The JSON line is the only thing on stdout: libraries that print there (NCCL
# announces its version on rank 0) are routed to stderr by main().
_JSON_OUT = sys.stdout


def emit(line: dict) -> None:
    _JSON_OUT.write(json.dumps(line) + "\n")
    _JSON_OUT.flush()


def route_stdout_to_stderr() -> None:
    global _JSON_OUT
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    sys.stdout = sys.stderr


def aggregate(units_per_rank: list[float], times_ms: list[float]) -> tuple[float, float]:
    """Whole-job throughput: all units over the slowest rank's time."""
    t = max(times_ms)
    return sum(units_per_rank) / (t / 1e3), t


# ---------------------------------------------------------------- CPU oracle legs
def cpu_oracle_decode(steps: int, warmup: int, seed: int, budget_s: float) -> dict:
    """The CPU oracle (oracle/q3_oracle.c, all host threads) on the same
    workload: prompt ingestion (timed separately) then up to `steps` decode
    steps, stopping early once `budget_s` of decode time is spent."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    # the oracle's own generator and quantizer: this leg never loads libq3b200.so
    m = O.Model(O.synthetic_weights(seed=seed))
    prompt = np.random.default_rng(seed).integers(0, 151936, PROMPT_LEN, dtype=np.int64)
    kc, vc = m.new_cache(CACHE)
    t0 = time.perf_counter()
    tok = None
    for i, t in enumerate(prompt):
        tok, _ = m.decode_step(int(t), i, kc, vc, CACHE)
    t_prompt = time.perf_counter() - t0
    pos = PROMPT_LEN
    for _ in range(warmup):
        tok, _ = m.decode_step(tok, pos, kc, vc, CACHE)
        pos += 1
    n, t_dec = 0, 0.0
    steps = min(steps, GEN_PER_SEQ - warmup)
    while n < steps and pos < CACHE - 1:
        t1 = time.perf_counter()
        tok, _ = m.decode_step(tok, pos, kc, vc, CACHE)
        t_dec += time.perf_counter() - t1
        n += 1
        pos += 1
        if t_dec > budget_s:
            break
    # @run throughput of the configuration (32-token prompt + 256 generated),
    # from the measured prompt time and the sampled per-step time
    e2e = GEN_PER_SEQ / (t_prompt + GEN_PER_SEQ * t_dec / n)
    return {"tok_s": n / t_dec, "steps": n, "decode_s": t_dec, "prompt_s": t_prompt,
            "e2e_tok_s": e2e, "threads": O.num_threads(),
            "first_pos": PROMPT_LEN + warmup}


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def run_reference(args, d: Dist) -> None:
    """Reference arm: the reference's decode path on host cores.  IREE (the
    reference's runtime, needed for its llvm-cpu build) is not installed here,
    so this times the oracle port of that path, all host threads."""
    if d.rank != 0:
        return
    r = cpu_oracle_decode(args.steps, args.warmup, args.seed, budget_s=args.ref_budget)
    line = {
        "metric": METRIC, "impl": "reference", "value": r["tok_s"], "unit": UNIT,
        "n_gpus": args.gpus, "steps": r["steps"], "warmup": args.warmup,
        "ms_per_step": 1e3 / r["tok_s"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args),
        "cpu_baseline": {"value": r["tok_s"], "unit": UNIT, "cores": r["threads"], "kind": "port",
                         "sample": f"{r['steps']} decode steps from position {r['first_pos']} "
                                   f"after a {PROMPT_LEN}-token prompt, oracle/q3_oracle.c, "
                                   f"{r['threads']} threads on {cpu_model()}"},
        "e2e": {"value": r["e2e_tok_s"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit(line)


def config_dict(args) -> dict:
    return {"workload": "configs[2]: Qwen3-0.6B Q8_0 greedy decode, batch 1 per GPU, "
                        f"{PROMPT_LEN}-token prompt, {GEN_PER_SEQ} generated tokens per sequence, "
                        f"KV cache {CACHE}",
            "model": "Qwen3-0.6B (random init, Q8_0)", "global_batch": args.gpus,
            "seq_len": PROMPT_LEN + GEN_PER_SEQ, "parallelism": f"replicas x{args.gpus}",
            "l2": "inputs larger than L2: all 779 MB of weights are streamed every step"}


# ---------------------------------------------------------------- our path
# kernel kinds of the live trace (include/q3b200.h Q3_KIND_*)
TRACE_KINDS = {0: "qkv", 1: "attn", 2: "o", 3: "gate_up", 4: "down", 5: "vocab",
               7: "fused_attn", 8: "fused_ffn"}
KV_BYTES_W = 2 * KV_ROW  # K and V rows of one position, one layer


def kernel_alg_bytes(name: str, pos: float) -> float:
    """Algorithmic HBM bytes of one launch of a decode-step kernel at position
    pos: its weights (+ gammas) and the K/V rows it reads and writes."""
    gam = 2 * 1024 * 2
    kv = KV_BYTES_W * pos + KV_BYTES_W  # cached rows read, the new row written
    if name == "fused_attn":
        return Q8_BYTES["qkv"] + Q8_BYTES["o"] + gam / 2 + 2 * 128 * 2 + kv
    if name == "fused_ffn":
        return Q8_BYTES["gate_up"] + Q8_BYTES["down"] + gam / 2
    if name == "attn":
        return attn_bytes(int(pos))
    if name == "vocab":
        return VOCAB_BYTES
    return Q8_BYTES[name] + ACT_BYTES[name]


def live_kernels(dec, steps: int, pos: float) -> dict:
    """Per kernel kind of one decode step, from the live kernel trace (each
    kernel stamps the global timer; the step runs as in the timed loop):
    the time it adds to the step (its last CTA's end minus the previous
    kernel's), its share, and algorithmic bytes / that time."""
    t, kinds = dec.trace_kernels(steps)
    ends = t[:, 3].astype(np.float64)
    add = np.diff(np.concatenate([[0.0], ends]))
    step_ns = float(ends[-1])
    out = {}
    for k in sorted(set(kinds.tolist())):
        name = TRACE_KINDS.get(int(k), str(k))
        sel = add[kinds == k]
        b = kernel_alg_bytes(name, pos)
        avg_us = float(sel.mean()) / 1e3
        out[name] = {"launches_per_step": int(sel.size), "avg_us": avg_us,
                     "total_us_per_step": float(sel.sum()) / 1e3,
                     "share": float(sel.sum()) / step_ns, "alg_bytes_per_launch": b,
                     "achieved_gbs": b / (avg_us * 1e-6) / 1e9}
    return out


def step_roofline(bytes_per_step: float, ms_per_step: float, kern: dict, peak: float,
                  peak_src: str, engine: str, launches: int, traffic: dict) -> dict:
    """The headline roofline object: the whole decode step against the HBM
    roofline (the north star's per-token fraction), with the dominant kernel
    kind's own figures; traffic = ncu DRAM bytes per step from one-launch
    captures of each kernel kind (profiles/), or null."""
    ach = bytes_per_step / (ms_per_step * 1e-3) / 1e9
    dom = max(kern, key=lambda k: kern[k]["total_us_per_step"])
    tr = None
    if kern and all(k in traffic for k in kern):
        tr = sum(traffic[k] * kern[k]["launches_per_step"] for k in kern)
    d = dict(kern[dom])
    d["name"] = dom
    d["frac"] = d["achieved_gbs"] / peak
    d["traffic"] = traffic.get(dom)
    return {"bound": "hbm", "kernel": f"decode step ({engine} engine, {launches} launches)",
            "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
            "traffic": tr, "alg_bytes": bytes_per_step, "per": "step",
            "frac_of_8tbs": ach / NOMINAL_HBM_GBS, "peak_source": peak_src,
            "dominant_kernel": d,
            "timing": "achieved = algorithmic bytes of a step / measured step time (CUDA "
                      "events over the timed steps); kernel figures from the live trace"}


def run_ours(args, d: Dist) -> None:
    import q3b200
    from q3b200.weights import synthetic_weights

    q3b200.set_device(d.local)
    host = synthetic_weights(seed=args.seed)
    dw = q3b200.DeviceWeights(host)
    del host
    prompt = np.random.default_rng(args.seed).integers(0, 151936, PROMPT_LEN, dtype=np.int64)
    dec = q3b200.Qwen3Decoder(dw, max_seq_len=CACHE, engine=args.engine)
    ev = q3b200.Events()

    # warm-up: one short sequence
    dec.generate_begin(prompt, args.warmup, -1)
    dec.generate_steps(args.warmup)
    _, n = dec.generate_end(args.warmup)
    assert n == args.warmup

    chunks = [min(GEN_PER_SEQ, args.steps - i) for i in range(0, args.steps, GEN_PER_SEQ)]
    clocks = ClockSampler(d.local)
    d.barrier()
    dec.synchronize()
    clocks.start()
    launches0 = dec.kernel_launches()
    total_ms, done, bytes_total = 0.0, 0, 0
    for c in chunks:
        dec.generate_begin(prompt, c, -1)           # prompt ingestion: untimed
        ev.record_start(dec.stream)
        dec.generate_steps(c)
        ev.record_end(dec.stream)
        total_ms += ev.elapsed_ms()
        _, n = dec.generate_end(c)
        assert n == c, (n, c)
        done += c
        bytes_total += sum(step_bytes(PROMPT_LEN + i) for i in range(c))
    dec.synchronize()
    launches = dec.kernel_launches() - launches0
    clk = clocks.stop()
    d.barrier()
    t_max = d.max(total_ms)
    value = d.sum(done) / (t_max / 1e3)
    ms = t_max / (done if done else 1)

    # per-kernel figures from the live trace, at the middle of the timed positions
    tr_steps = 8
    mid = GEN_PER_SEQ // 2
    dec.generate_begin(prompt, mid + tr_steps + 1, -1)
    dec.generate_steps(mid)
    kern = live_kernels(dec, tr_steps, PROMPT_LEN + mid + tr_steps / 2)
    dec.generate_end(mid + tr_steps + 1)
    peak, peak_kind = load_peaks()
    peak_src = (f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                else "fallback 6.65 TB/s")
    roof = step_roofline(bytes_total / done, ms, kern, peak, peak_src, dec.engine,
                         dec.launches_per_step(), load_traffic())

    from q3b200.benchmark import gemv_pool, layer_bench

    configs0 = gemv_pool(seed=args.seed)
    for k in ("q3_gemv_q8_overlapped", "q3_gemv_q8"):
        configs0[k]["frac_of_measured"] = configs0[k]["gbs"] / peak
        configs0[k]["frac_of_8tbs"] = configs0[k]["gbs"] / NOMINAL_HBM_GBS
    configs1 = layer_bench(dw, seed=args.seed)
    configs1["frac_of_measured"] = configs1["gbs"] / peak
    # the same layer inside the decode step: the engine's kernels of one layer
    # at position 511 (512 keys attended), from the live trace
    pos1 = 511
    dec.generate_begin(prompt, pos1 - PROMPT_LEN + 8, -1)
    dec.generate_steps(pos1 - PROMPT_LEN - 2)
    k1 = live_kernels(dec, 4, pos1)
    dec.generate_end(pos1 - PROMPT_LEN + 8)
    per_layer = sum(v["total_us_per_step"] for k, v in k1.items() if k != "vocab") / 28
    b1 = 18825728
    configs1["in_engine"] = {"us_per_layer": per_layer, "gbs": b1 / (per_layer * 1e-6) / 1e9,
                             "frac_of_measured": b1 / (per_layer * 1e-6) / 1e9 / peak,
                             "how": "live trace of the decode step at position 511: the time the "
                                    "layer's kernels add to the step, averaged over the 28 layers"}
    # streaming GEMV bandwidth: 28 layers of one projection in one launch
    gemv_stream = measure_gemv_stream(q3b200, dw, peak) if not args.quick else {}
    batched = {} if args.no_batched else {
        k: measure_batched(q3b200, dw, d, k, args.seed, peak, args.warmup) for k in BATCHED}

    # end to end through the public call (host prompt in, host tokens out)
    e2e_vals = []
    for _ in range(3):
        dec.synchronize()
        d.barrier()
        t0 = time.perf_counter()
        out, n = dec.run(prompt, GEN_PER_SEQ, EOS)
        dt = time.perf_counter() - t0
        e2e_vals.append(n / dt)
    e2e_local = statistics.median(e2e_vals)
    e2e = d.sum(e2e_local) if d.world > 1 else e2e_local
    # the same call with the prompt ingested by the batched prefill (tensor-core
    # passes instead of one decode step per prompt token; tolerance-level cache)
    dec.set_prefill("batched")
    pf_vals = []
    for _ in range(3):
        dec.synchronize()
        d.barrier()
        t0 = time.perf_counter()
        out_pf, n_pf = dec.run(prompt, GEN_PER_SEQ, EOS)
        dt = time.perf_counter() - t0
        pf_vals.append(n_pf / dt)
    dec.set_prefill("steps")
    e2e_pf = d.sum(statistics.median(pf_vals)) if d.world > 1 else statistics.median(pf_vals)
    h2d = PROMPT_LEN * 8 + 48
    d2h = GEN_PER_SEQ * 8 + 48 + 4
    err = dec.device_error()

    cpu = None
    if d.world == 1 and not args.no_cpu_baseline:
        r = cpu_oracle_decode(args.steps, 0, args.seed, budget_s=args.cpu_budget)
        cpu = {"value": r["tok_s"], "unit": UNIT, "cores": r["threads"], "kind": "port",
               "sample": f"{r['steps']} decode steps from position {r['first_pos']} after a "
                         f"{PROMPT_LEN}-token prompt, oracle/q3_oracle.c, {r['threads']} threads "
                         f"on {cpu_model()}"}

    if d.rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": d.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": config_dict(args),
            "roofline": roof,
            "cpu_baseline": cpu,
            "clocks": clk,
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": h2d / GEN_PER_SEQ,
                    "d2h_bytes_per_step": d2h / GEN_PER_SEQ,
                    "call": f"q3_run: {PROMPT_LEN}-token host prompt in, {GEN_PER_SEQ} host "
                            "tokens out per call, wall clock incl. prompt ingestion"},
            "e2e_prefill_batched": {
                "value": e2e_pf, "unit": UNIT,
                "call": "q3_run with q3_model_set_prefill(Q3_PREFILL_BATCHED): the prompt's "
                        "first 31 positions in one tensor-core pass, then the same decode",
                "tokens_equal_to_steps_prefill": int(np.array_equal(out_pf[:n_pf], out[:n]))},
            "gpu_launches": launches,
            "engine": dec.engine,
            "kernels": kern,
            "configs0": configs0,
            "configs1": configs1,
            "gemv_stream": gemv_stream,
            "batched": batched,
            "device_error": err,
        }
        emit(line)
    dec.close()


BATCHED = {"b32": (32, 128, 2048, "configs[3]"), "b64": (64, 512, 4096, "configs[4]")}
BATCH_STEPS = 128
BATCH_KINDS = {0: "qkv", 1: "attn", 2: "o", 3: "gate_up", 4: "down", 5: "vocab", 6: "norm"}
# activation f16 elements (in, out) per sequence of the batched projections
BATCH_ACT = {"qkv": (1024, 4096), "o": (2048 + 1024, 1024), "gate_up": (1024, 3072),
             "down": (3072 + 1024, 1024)}


def batch_kernel_bytes(name: str, B: int, pos) -> float:
    """Algorithmic HBM bytes of one launch of a batched-step kernel; pos are
    the sequences' positions (each attends pos+1 keys)."""
    if name in Q8_BYTES:
        i, o = BATCH_ACT[name]
        return Q8_BYTES[name] + 2 * B * (i + o)
    if name == "attn":
        return float(sum(2 * KV_ROW * (int(p) + 1) + 2 * KV_ROW + 8192 + 4096 for p in pos))
    if name == "vocab":
        return 151936 * 1024 * 2 + B * 2048 + B * 16
    return B * (2048 + 2048) + 2048  # norm: x in, xn out, gamma


def measure_batched(q3b200, dw, d: Dist, key: str, seed: int, peak: float, warmup: int) -> dict:
    """B sequences whose cached contexts are
    U[lo, hi] positions of seeded pseudo-random K/V, 128 decode steps of all of
    them (tcgen05 projections, split-KV attention per sequence).  Device time
    of the 128 steps (CUDA events on the decoder's stream), max over ranks;
    tokens summed over ranks (replicas)."""
    B, lo, hi, cfg = BATCHED[key]
    rng = np.random.default_rng(seed + B)
    ctx = rng.integers(lo, hi + 1, size=B)
    tok = rng.integers(0, 151936, size=B)
    S = hi + BATCH_STEPS + warmup + 2
    bd = q3b200.BatchDecoder(dw, max_batch=B, max_seq_len=S)
    bd.begin_random(ctx, tok, seed=seed)
    bd.steps(warmup)
    bd.synchronize()
    ev = q3b200.Events()
    l0 = bd.kernel_launches()
    d.barrier()
    ev.record_start(bd.stream)
    bd.steps(BATCH_STEPS)
    ev.record_end(bd.stream)
    ms = ev.elapsed_ms()
    launches = bd.kernel_launches() - l0
    toks, pos = bd.read()
    assert (pos == ctx + warmup + BATCH_STEPS).all(), "batched positions did not advance"
    # per-kernel device times (serialised by events) over a few more steps
    prof_steps = 4
    times_us, kinds = bd.profile_steps(prof_steps)
    bd.close()
    ppos = ctx + warmup + BATCH_STEPS + prof_steps // 2
    kern = {}
    for kind, name in BATCH_KINDS.items():
        sel = times_us[kinds == kind]
        if sel.size == 0:
            continue
        b = batch_kernel_bytes(name, B, ppos)
        avg = float(sel.mean())
        kern[name] = {"launches_per_step": int(sel.size), "avg_us": avg,
                      "total_us_per_step": float(sel.sum()), "alg_bytes_per_launch": b,
                      "achieved_gbs": b / (avg * 1e-6) / 1e9}
    tot = float(times_us.sum())
    for k in kern.values():
        k["share"] = k["total_us_per_step"] / tot
    dom = max(kern, key=lambda k: kern[k]["total_us_per_step"])
    t_max = d.max(ms)
    w = sum(Q8_BYTES.values()) * 28 + VOCAB_BYTES + NORM_BYTES
    kv = sum(28 * (2 * KV_ROW * (int(c) + i + 1) + 2 * KV_ROW)
             for i in range(warmup, warmup + BATCH_STEPS) for c in ctx)
    step_b = (w * BATCH_STEPS + kv) / BATCH_STEPS
    gbs = step_b / (ms / BATCH_STEPS * 1e-3) / 1e9
    return {"workload": f"{cfg}: B={B} sequences, context U[{lo},{hi}], {BATCH_STEPS} decode steps",
            "tok_s": d.sum(B * BATCH_STEPS) / (t_max / 1e3), "ms_per_step": t_max / BATCH_STEPS,
            "alg_bytes_per_step": step_b, "achieved_gbs": gbs, "frac_of_measured": gbs / peak,
            "frac_of_8tbs": gbs / NOMINAL_HBM_GBS, "launches_per_step": launches / BATCH_STEPS,
            "gpu_launches": launches,
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": kern[dom]["achieved_gbs"],
                         "peak": peak, "unit": "GB/s",
                         "frac": kern[dom]["achieved_gbs"] / peak,
                         "traffic": batched_traffic(kern, dom),
                         "traffic_source": "one-launch ncu captures on a context-256 small "
                                           "case (profiles/k_bgemm_q8_b32.md, k_battn_b32.md); "
                                           "attention's DRAM/algorithmic ratio there times "
                                           "this launch's algorithmic bytes (its traffic grows "
                                           "with the context it streams)"},
            "kernels": kern,
            "l2": "inputs larger than L2 (779 MB of weights + the KV caches every step)"}


def batched_traffic(kern: dict, dom: str):
    """DRAM bytes per launch of the dominant batched kernel: the ratio of ncu
    DRAM bytes to algorithmic bytes in the one-launch small-case capture, times
    this launch's algorithmic bytes (attention's traffic scales with context)."""
    t = load_traffic()
    ratio = {"attn": t.get("b32_attn_c256", 0) / B32_ATTN_C256_ALG if "b32_attn_c256" in t else None}
    for k in ("qkv", "o", "gate_up", "down"):
        if f"b32_{k}_c256" in t:
            ratio[k] = t[f"b32_{k}_c256"] / B32_PROJ_ALG[k]
    r = ratio.get(dom)
    return None if r is None else r * kern[dom]["alg_bytes_per_launch"]


# algorithmic bytes of the captured small-case launches (B=32, context 256 + 3 warm-up + 1
# timed step of the benchmark twin at layer 4): K/V rows of every position, and the
# projections' weights + activations
B32_ATTN_C256_ALG = 32 * 8 * 2 * 256 * (256 + 4)  # (b, h) x K+V rows of 256 B x positions 0..259
B32_PROJ_ALG = {"qkv": 4456448 + 32 * 1024 * 2, "o": 2228224 + 32 * 2048 * 2 + 32 * 1024 * 2,
                "gate_up": 6684672 + 32 * 1024 * 2, "down": 3342336 + 32 * 3072 * 2 + 32 * 1024 * 2}


def measure_gemv_stream(q3b200, dw, peak: float) -> dict:
    """Each projection over all 28 layers in ONE launch, L2 flushed before
    every timed launch (q3b200.benchmark.gemv_stream)."""
    from q3b200.benchmark import GEMV_STREAM_SHAPES, gemv_stream

    out = {}
    for name in GEMV_STREAM_SHAPES:
        r = gemv_stream(dw, name)
        r["frac_of_measured"] = r["gbs"] / peak
        out[name] = r
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU decode time")
    ap.add_argument("--ref-budget", type=float, default=60.0, help="seconds, reference arm")
    ap.add_argument("--quick", action="store_true", help="skip the GEMV streaming sweep")
    ap.add_argument("--engine", default=None, choices=["fused", "graph", "persistent"],
                    help="decode engine (default: the library's, fused where available)")
    ap.add_argument("--no-batched", action="store_true", help="skip the B=32 / B=64 legs")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    route_stdout_to_stderr()
    d = Dist() if args.impl == "ours" else None
    if args.impl == "reference":
        class _D:
            rank = int(os.environ.get("RANK", "0"))
        run_reference(args, _D())
        return
    try:
        run_ours(args, d)
    finally:
        d.close()


if __name__ == "__main__":
    main()
