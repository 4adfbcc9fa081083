"""Host mirror of the reference module's public functions, over libq3b200.so.

The reference drives model/qwen3_full.mlir through iree.runtime:
``ctx.invoke(run, [tokens, n_tokens, max_tokens, eos])`` returns
``(tokens_out, n)`` (scripts/benchmark.py:52-81, scripts/chat.py:112-126).
``Qwen3Decoder`` offers the same calls -- run, decode, prefill_all,
init_chat, chat_turn -- backed by the sm_100a kernels and CUDA graphs of the
library, with numpy arrays in and out and no PyTorch.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import Weights, call, lib
from .device import DeviceArray
from .weights import VOCAB

WEIGHT_FIELDS = [
    ("token_embd", "token_embd.weight"), ("output_norm", "output_norm.weight"),
    ("output_T", "output_T.weight"), ("attn_norm", "stacked.attn_norm.weight"),
    ("ffn_norm", "stacked.ffn_norm.weight"), ("attn_q_norm", "stacked.attn_q_norm.weight"),
    ("attn_k_norm", "stacked.attn_k_norm.weight"), ("q8_attn_q", "stacked.q8.attn_q.weight"),
    ("q8_attn_k", "stacked.q8.attn_k.weight"), ("q8_attn_v", "stacked.q8.attn_v.weight"),
    ("q8_attn_output", "stacked.q8.attn_output.weight"),
    ("q8_ffn_gate_up", "stacked.q8.ffn_gate_up.weight"),
    ("q8_ffn_down", "stacked.q8.ffn_down.weight"),
]


class DeviceWeights:
    """Uploads a parameter dict once (tied tensors share one buffer)."""

    def __init__(self, host: dict[str, np.ndarray]):
        self.buffers: dict[str, DeviceArray] = {}
        by_id: dict[int, DeviceArray] = {}
        for _, name in WEIGHT_FIELDS:
            a = host[name]
            if id(a) not in by_id:
                by_id[id(a)] = DeviceArray.from_host(a)
            self.buffers[name] = by_id[id(a)]
        self.nbytes = sum(d.nbytes for d in by_id.values())
        self.struct = Weights(**{f: self.buffers[n].ptr for f, n in WEIGHT_FIELDS})


class Qwen3Decoder:
    """One decoder (KV cache, activations, graphs) on the current device."""

    def __init__(self, weights: DeviceWeights | dict, max_seq_len: int = 1024, stream=None,
                 engine: str | None = None, prefill: str | None = None):
        self.weights = weights if isinstance(weights, DeviceWeights) else DeviceWeights(weights)
        self.max_seq_len = int(max_seq_len)
        h = ctypes.c_void_p()
        call("q3_model_create", ctypes.byref(self.weights.struct), self.max_seq_len, stream,
             ctypes.byref(h))
        self.handle = h.value
        self.stream = lib().q3_model_stream(self.handle)
        if engine is not None:
            self.set_engine(engine)
        if prefill is not None:
            self.set_prefill(prefill)

    # -- @run (model/qwen3_full.mlir:2113-2167)
    def run(self, tokens, max_tokens: int, eos: int) -> tuple[np.ndarray, int]:
        t = np.ascontiguousarray(tokens, dtype=np.int64)
        out = np.zeros(max(int(max_tokens), 1), dtype=np.int64)
        n = ctypes.c_int64(0)
        call("q3_run", self.handle, t.ctypes.data, t.size, int(max_tokens), int(eos),
             out.ctypes.data, ctypes.byref(n))
        return out[:max(int(max_tokens), 0)], n.value

    # -- @decode (model/qwen3_full.mlir:1340-1394)
    def decode(self, token: int, pos: int, want_logits: bool = True):
        nxt = ctypes.c_int64(-1)
        logits = DeviceArray((VOCAB,), np.float16) if want_logits else None
        call("q3_decode", self.handle, int(token), int(pos), logits.ptr if logits else None,
             ctypes.byref(nxt))
        return (logits.download() if logits else None), nxt.value

    # -- @prefill_all (model/qwen3_full.mlir:1541-1570): token by token through @decode
    def prefill_all(self, tokens) -> np.ndarray:
        logits = None
        for i, t in enumerate(np.asarray(tokens, dtype=np.int64)):
            logits, _ = self.decode(int(t), i, want_logits=(i == len(tokens) - 1))
        return logits

    # -- @init_chat / @chat_turn (model/qwen3_full.mlir:2172-2222)
    def init_chat(self, max_ctx: int) -> None:
        call("q3_init_chat", self.handle, int(max_ctx))

    def chat_turn(self, tokens, max_gen: int, eos: int) -> tuple[np.ndarray, int]:
        t = np.ascontiguousarray(tokens, dtype=np.int64)
        out = np.zeros(max(int(max_gen), 1), dtype=np.int64)
        n = ctypes.c_int64(0)
        call("q3_chat_turn", self.handle, t.ctypes.data, t.size, int(max_gen), int(eos),
             out.ctypes.data, ctypes.byref(n))
        return out[:max(int(max_gen), 0)], n.value

    # -- step-level access for harnesses
    def generate_begin(self, tokens, max_gen: int, eos: int) -> None:
        t = np.ascontiguousarray(tokens, dtype=np.int64)
        call("q3_generate_begin", self.handle, t.ctypes.data, t.size, int(max_gen), int(eos))

    def generate_steps(self, steps: int) -> None:
        call("q3_generate_steps", self.handle, int(steps))

    def generate_end(self, max_gen: int) -> tuple[np.ndarray, int]:
        out = np.zeros(max(int(max_gen), 1), dtype=np.int64)
        n = ctypes.c_int64(0)
        call("q3_generate_end", self.handle, out.ctypes.data, ctypes.byref(n))
        return out[:n.value], n.value

    def profile_steps(self, steps: int) -> tuple[np.ndarray, np.ndarray]:
        """(per-kernel average microseconds, kinds) over `steps` generation steps."""
        cap = 512
        t = np.zeros(cap, np.float32)
        k = np.zeros(cap, np.int32)
        call("q3_model_profile_steps", self.handle, int(steps), t.ctypes.data, k.ctypes.data, cap)
        n = self.launches_per_step()
        return t[:n].copy(), k[:n].copy()

    ENGINES = {"graph": 0, "persistent": 1, "fused": 2}

    def set_engine(self, name: str) -> None:
        call("q3_model_set_engine", self.handle, self.ENGINES[name])

    PREFILL = {"steps": 0, "batched": 1}

    def set_prefill(self, name: str) -> None:
        """How prompts are ingested: "steps" (one decode step per token, the
        reference's @prefill_all route) or "batched" (tensor-core passes of up
        to 64 positions)."""
        call("q3_model_set_prefill", self.handle, self.PREFILL[name])

    @property
    def prefill_mode(self) -> str:
        e = ctypes.c_int(-1)
        call("q3_model_prefill_mode", self.handle, ctypes.byref(e))
        return {v: k for k, v in self.PREFILL.items()}[e.value]

    def prefill(self, tokens, pos0: int = 0) -> None:
        """Batched prefill: K/V rows of positions pos0 .. pos0+len(tokens)-1."""
        t = np.ascontiguousarray(tokens, dtype=np.int64)
        call("q3_model_prefill", self.handle, t.ctypes.data, int(pos0), t.size)

    @property
    def engine(self) -> str:
        e = ctypes.c_int(-1)
        call("q3_model_engine", self.handle, ctypes.byref(e))
        return {v: k for k, v in self.ENGINES.items()}[e.value]

    def trace_steps(self, steps: int, trace_step: int) -> np.ndarray:
        """Persistent engine: [ctas, phases, 4] SM-clock stamps of one step."""
        cap = 1024 * 160 * 4
        out = np.zeros(cap, np.int64)
        c, p = ctypes.c_int(), ctypes.c_int()
        call("q3_model_trace_steps", self.handle, int(steps), int(trace_step), out.ctypes.data,
             cap, ctypes.byref(c), ctypes.byref(p))
        return out[:c.value * p.value * 4].reshape(c.value, p.value, 4)

    def trace_phases(self, steps: int = 4) -> np.ndarray:
        """Fused engine: [56 launches, 128 CTAs, phases] global-timer stamps (ns)
        of the last of `steps` steps."""
        cap = 56 * 128 * 16
        out = np.zeros(cap, np.int64)
        nl, c, p = ctypes.c_int64(), ctypes.c_int(), ctypes.c_int()
        call("q3_model_trace_phases", self.handle, int(steps), out.ctypes.data, cap,
             ctypes.byref(nl), ctypes.byref(c), ctypes.byref(p))
        return out[:nl.value * c.value * p.value].reshape(nl.value, c.value, p.value)

    def kernel_launches(self) -> int:
        n = ctypes.c_int64(0)
        call("q3_model_kernel_launches", self.handle, ctypes.byref(n))
        return n.value

    def trace_kernels(self, steps: int = 4):
        """(times [n, 6] ns, kinds [n]): per kernel of a graph-engine step, its
        first CTA start, first and last release from the wait on the previous
        kernel, last CTA end, last CTA start and first CTA end, from the
        step's first kernel start."""
        cap = 512
        out = np.zeros((cap, 6), np.int64)
        kinds = np.zeros(cap, np.int32)
        n = ctypes.c_int64(0)
        call("q3_model_trace_kernels", self.handle, int(steps), out.ctypes.data, kinds.ctypes.data,
             cap, ctypes.byref(n))
        return out[:n.value].copy(), kinds[:n.value].copy()

    def launches_per_step(self) -> int:
        n = ctypes.c_int64(0)
        call("q3_model_launches_per_step", self.handle, ctypes.byref(n))
        return n.value

    def device_error(self) -> int:
        c = ctypes.c_int(0)
        call("q3_model_device_error", self.handle, ctypes.byref(c))
        return c.value

    def synchronize(self) -> None:
        call("q3_stream_synchronize", self.stream)

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib().q3_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class BatchDecoder:
    """B independent sequences decoded together (B <= 64): tcgen05 tensor-core
    projections and vocab head; attention per sequence over its own cache."""

    def __init__(self, weights: DeviceWeights | dict, max_batch: int, max_seq_len: int,
                 stream=None):
        self.weights = weights if isinstance(weights, DeviceWeights) else DeviceWeights(weights)
        self.max_batch, self.max_seq_len = int(max_batch), int(max_seq_len)
        h = ctypes.c_void_p()
        call("q3_batch_create", ctypes.byref(self.weights.struct), self.max_batch,
             self.max_seq_len, stream, ctypes.byref(h))
        self.handle = h.value
        self.stream = lib().q3_batch_stream(self.handle)
        self.B = 0

    def begin(self, prompts: list) -> None:
        """Sequence b starts at position 0 with prompt tokens prompts[b]."""
        B = len(prompts)
        width = max(len(p) for p in prompts)
        tab = np.zeros((B, width), np.int64)
        lens = np.array([len(p) for p in prompts], np.int64)
        for b, p in enumerate(prompts):
            tab[b, :len(p)] = p
        call("q3_batch_begin", self.handle, B, tab.ctypes.data, width, lens.ctypes.data)
        self.B = B

    def begin_random(self, ctx_lens, tokens, seed: int = 0) -> None:
        """Sequence b has a context of ctx_lens[b] pseudo-random cached positions."""
        c = np.ascontiguousarray(ctx_lens, np.int64)
        t = np.ascontiguousarray(tokens, np.int64)
        call("q3_batch_begin_random", self.handle, c.size, c.ctypes.data, t.ctypes.data, seed)
        self.B = c.size

    def steps(self, n: int) -> None:
        call("q3_batch_steps", self.handle, int(n))

    def read(self):
        """(tokens [B, S+1], positions [B]); raises on a device error word."""
        toks = np.zeros((self.B, self.max_seq_len + 1), np.int64)
        pos = np.zeros(self.B, np.int64)
        err = ctypes.c_int(0)
        call("q3_batch_read", self.handle, toks.ctypes.data, pos.ctypes.data, ctypes.byref(err))
        if err.value:
            raise RuntimeError(f"device error word {err.value}")
        return toks, pos

    def profile_steps(self, steps: int):
        """(times_us, kinds) per kernel of one step, averaged over `steps`
        decode steps (which advance the sequences)."""
        cap = 512
        t = np.zeros(cap, np.float32)
        k = np.zeros(cap, np.int32)
        n = ctypes.c_int64(0)
        call("q3_batch_profile_steps", self.handle, int(steps), t.ctypes.data, k.ctypes.data, cap,
             ctypes.byref(n))
        return t[:n.value].copy(), k[:n.value].copy()

    def trace_kernels(self, steps: int = 4):
        """(times [n, 6] ns, kinds [n]) per kernel of a batched step, as
        Qwen3Decoder.trace_kernels."""
        cap = 512
        out = np.zeros((cap, 6), np.int64)
        kinds = np.zeros(cap, np.int32)
        n = ctypes.c_int64(0)
        call("q3_batch_trace_kernels", self.handle, int(steps), out.ctypes.data, kinds.ctypes.data,
             cap, ctypes.byref(n))
        return out[:n.value].copy(), kinds[:n.value].copy()

    def read_argmax(self) -> np.ndarray:
        """[B, S+1]: entry p+1 is the greedy token after feeding position p."""
        out = np.zeros((self.B, self.max_seq_len + 1), np.int64)
        call("q3_batch_read_argmax", self.handle, out.ctypes.data)
        return out

    def trace_phases(self, steps: int = 4):
        """(stamps [launches, 512 CTAs, 8] global-timer ns, kinds [launches]) of
        the batched projections and attention in the last of `steps` steps."""
        nmax = 5 * 28
        out = np.zeros(nmax * 512 * 8, np.int64)
        kinds = np.zeros(nmax, np.int32)
        n = ctypes.c_int64(0)
        call("q3_batch_trace_phases", self.handle, int(steps), out.ctypes.data, kinds.ctypes.data,
             out.size, ctypes.byref(n))
        return out[:n.value * 512 * 8].reshape(n.value, 512, 8), kinds[:n.value].copy()

    def kernel_launches(self) -> int:
        n = ctypes.c_int64(0)
        call("q3_batch_kernel_launches", self.handle, ctypes.byref(n))
        return n.value

    def synchronize(self) -> None:
        call("q3_stream_synchronize", self.stream)

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib().q3_batch_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
