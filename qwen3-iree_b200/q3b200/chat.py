"""ctypes twin of the reference's scripts/chat.py.

The reference reads a line, wraps it in the chat template, calls `@run`
(prompt ids, length, max tokens, end-of-text id), cuts the output at the
first end-of-text token, prints it and "[n tok, t s, r tok/s]"
(scripts/chat.py:103-138); "quit", "exit" or "q" ends the loop.  This twin
does the same through libq3b200.so (q3_run).

With --tokenizer PATH (a tokenizer.json; the `tokenizers` package) lines are
text; without one (none ships here) a line is a list of token ids and the
reply is printed as ids.  Weights: the reference's .irpa archives with --irpa,
a Q8_0 GGUF checkpoint with --gguf, else
the seeded random-init model.

  python -m q3b200.chat [--max-tokens 256] [--tokenizer tokenizer.json]
"""
from __future__ import annotations

import argparse
import sys
import time

import numpy as np

from .benchmark import CHAT_TEMPLATE, EOS_TOKEN, load_tokenizer, load_weights, trim_eos

QUIT_WORDS = ("quit", "exit", "q")


def parse_ids(text: str) -> list[int]:
    """Token ids from a line: whitespace- or comma-separated integers."""
    return [int(t) for t in text.replace(",", " ").split()]


def encode_line(text: str, tokenizer) -> list[int]:
    if tokenizer is not None:
        return tokenizer.encode(CHAT_TEMPLATE.format(text)).ids
    return parse_ids(text)


def reply(dec, tokens: list[int], max_tokens: int, eos: int = EOS_TOKEN):
    """One @run call: (kept output tokens, seconds)."""
    t0 = time.perf_counter()
    out, n = dec.run(np.asarray(tokens, np.int64), max_tokens, eos)
    dt = time.perf_counter() - t0
    return trim_eos(out[:n], eos), dt


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Chat with Qwen3-0.6B Q8_0 via libq3b200.so")
    ap.add_argument("--tokenizer", default=None, help="tokenizer.json path")
    ap.add_argument("--max-tokens", type=int, default=256, help="max tokens to generate")
    ap.add_argument("--max-seq-len", type=int, default=1024)
    ap.add_argument("--seed", type=int, default=0, help="random-init weights")
    ap.add_argument("--gguf", default=None, help="Qwen3-0.6B Q8_0 GGUF checkpoint (else random init)")
    ap.add_argument("--irpa", nargs="+", default=None,
                    help="the reference's .irpa archive(s) (tools/create_q8_irpa.py output)")
    ap.add_argument("--device", type=int, default=0)
    args = ap.parse_args(argv)

    from . import DeviceWeights, Qwen3Decoder, set_device

    tokenizer = load_tokenizer(args.tokenizer)
    set_device(args.device)
    dec = Qwen3Decoder(DeviceWeights(load_weights(args)),
                       max_seq_len=args.max_seq_len)
    mode = "text" if tokenizer is not None else "token ids"
    print(f"Qwen3-0.6B Q8_0 on libq3b200.so ({mode}; type 'quit' to exit)\n", flush=True)
    while True:
        try:
            text = input("> ")
        except (EOFError, KeyboardInterrupt):
            break
        if text.strip().lower() in QUIT_WORDS:
            break
        if not text.strip():
            continue
        try:
            tokens = encode_line(text, tokenizer)
        except ValueError:
            print("expected token ids (integers), or pass --tokenizer", flush=True)
            continue
        if not tokens or len(tokens) + args.max_tokens > args.max_seq_len:
            print(f"prompt of {len(tokens)} ids does not fit a {args.max_seq_len}-position cache",
                  flush=True)
            continue
        out, dt = reply(dec, tokens, args.max_tokens)
        print(tokenizer.decode(out) if tokenizer is not None else " ".join(map(str, out)))
        print(f"[{len(out)} tok, {dt:.1f}s, {len(out) / dt:.1f} tok/s]\n", flush=True)
    dec.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
