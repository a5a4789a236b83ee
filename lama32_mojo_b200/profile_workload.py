"""Profiling workload: a random-init model of a preset's shapes (optionally
fewer layers / a smaller vocabulary so that ncu captures stay small), one
prefill of `--ctx` tokens per sequence (`--batch` sequences), then `--steps`
greedy decode steps launched one by one (no CUDA graph, so every kernel shows
up in a launch list).

    python -m lama32_mojo_b200.profile_workload --model llama-3.1-8b --layers 2 --vocab 16384 --ctx 2100
    ncu --set full --clock-control none -k regex:k_gemv_d -s 1 -c 4 -o out \\
        python -m lama32_mojo_b200.profile_workload --model llama-3.1-8b --layers 2 --vocab 16384 --ctx 2100
"""
from __future__ import annotations

import argparse
import dataclasses
import sys


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--model", default="llama-3.1-8b")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (0: the preset's)")
    ap.add_argument("--vocab", type=int, default=0, help="override the vocabulary size (0: the preset's)")
    ap.add_argument("--ctx", type=int, default=2100, help="prompt length (prefill tokens + 8)")
    ap.add_argument("--steps", type=int, default=2, help="greedy decode steps after the prefill")
    ap.add_argument("--max-tokens", type=int, default=2048, help="prefill chunk size")
    ap.add_argument("--batch", type=int, default=1, help="sequences decoded together")
    a = ap.parse_args(argv)

    import numpy as np

    from .config import PRESETS
    from .model import load_synthetic

    cfg = PRESETS[a.model]
    if a.layers:
        cfg = dataclasses.replace(cfg, layers=a.layers)
    if a.vocab:
        cfg = dataclasses.replace(cfg, vocab=a.vocab)
    B = max(1, a.batch)
    m = load_synthetic(cfg, device=0, seed=0, maxlen=a.ctx + a.steps + 16, max_seqs=B, max_tokens=a.max_tokens)
    rng = np.random.default_rng(1)
    first = []
    for s in range(B):
        lg = m.forward(rng.integers(0, cfg.vocab, size=max(1, a.ctx - 8)).tolist(), seq=s)
        if not np.isfinite(lg).all():
            print("non-finite logits", file=sys.stderr)
            return 1
        first.append(int(np.argmax(lg)))
    if B == 1:
        t = first[0]
        for _ in range(a.steps):
            t = m.forward_argmax([t])
        print("ok", t)
    else:
        cur = first
        for _ in range(a.steps):
            cur = m.decode(cur, list(range(B))).tolist()
        print("ok", cur)
    m.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
