"""Q8 GEMV/GEMM kernel sweep (benchmark config[1]).

    python -m lama32_mojo_b200.sweep [--shapes 1b,3b] [--m 1,8,64,512,4096] [--one K,N,M] [--iters 20]
    python -m lama32_mojo_b200.sweep --sample [--rows 1,8,64] [--iters 20]

Every projection shape of Llama-3.2-1B / 3B (K x N), int8 weights from N(0, 0.02)
with group-64 f16 scales packed by the GPU packer, bf16 activations N(0, 1),
M tokens.  Each case times ``q8op_gemm`` with CUDA events on the current stream
after warm-up (the timed launches captured in one CUDA graph), rotating over
enough weight copies that every launch reads weights from HBM (> 126 MB L2
per rotation), and prints one JSON line with the
achieved HBM GB/s (algorithmic bytes: codes + scales + activations + output)
and TFLOP/s (2*M*N*K).  ``--one`` runs a single case (the small command used
for ncu captures).

``--sample`` times ``q8op_sample`` (temperature 1, top-p 0.9) on rows of the
Llama-3 vocabulary (128256 logits): "peaked" rows (N(0, 2) plus 300 logits
raised by 25, a few hundred candidates within 16 of the maximum) and "flat"
rows (N(0, 0.5): every logit is a candidate, the sequential sums run over the
whole row).  Bytes are the logits read once.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

SHAPES = {
    "1b": [(2048, 3072), (2048, 2048), (2048, 512), (2048, 16384), (2048, 8192), (8192, 2048)],
    "3b": [(3072, 5120), (3072, 3072), (3072, 1024), (3072, 16384), (3072, 8192), (8192, 3072)],
}


def peaks():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def run_case(K, N, M, iters=20, warmup=5):
    import torch
    from . import ops
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(K * 7 + N)
    wbytes = N * (K + K // 32)
    copies = max(1, -(-300 * 2 ** 20 // wbytes))  # > 2x L2 per rotation
    copies = min(copies, 64)
    ws = [ops.pack_q8((torch.randn((N, K), generator=g, device=dev) * 0.02).to(torch.bfloat16))
          for _ in range(copies)]
    x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
    y = torch.empty((M, N), device=dev)
    for i in range(warmup):
        ops.mm_q8(x, ws[i % copies], K, out=y)
    torch.cuda.synchronize()
    # the timed launches replay a CUDA graph, so that the host's launch rate
    # (a ctypes call per GEMM) does not leave the GPU idle between kernels
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(iters):
            ops.mm_q8(x, ws[i % copies], K, out=y)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    bytes_ = wbytes + M * K * 2 + M * N * 4
    return {"K": K, "N": N, "M": M, "us": round(ms * 1e3, 2), "GB_s": round(bytes_ / (ms / 1e3) / 1e9, 1),
            "TFLOP_s": round(2.0 * M * N * K / (ms / 1e3) / 1e12, 2)}


def run_sample(kind: str, rows: int, iters: int = 20, warmup: int = 3):
    import ctypes as C

    import torch

    from . import _lib
    dev = torch.device("cuda", 0)
    V = 128256
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn((rows, V), generator=g, device=dev)
    if kind == "peaked":
        x *= 2.0
        hot = torch.randperm(V, generator=g, device=dev)[:300]
        x[:, hot] += 25.0
    else:
        x *= 0.5
    u = torch.rand(rows, generator=g, device=dev)
    out = torch.empty(rows, dtype=torch.int32, device=dev)
    L = _lib.lib()

    def call():
        st = torch.cuda.current_stream().cuda_stream
        _lib.check(L.q8op_sample(C.c_void_p(x.data_ptr()), rows, V, V, 1.0, 0.9, C.c_void_p(u.data_ptr()),
                                 C.c_void_p(out.data_ptr()), C.c_void_p(st)))

    for _ in range(warmup):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        call()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    cand = int((x >= x.max(dim=1, keepdim=True).values - 16.0).sum(dim=1).max().item())
    return {"op": "sample", "kind": kind, "rows": rows, "vocab": V, "max_candidates": cand,
            "us": round(ms * 1e3, 1), "GB_s": round(rows * V * 4 / (ms / 1e3) / 1e9, 1)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="1b,3b")
    ap.add_argument("--m", default="1,8,64,512,4096")
    ap.add_argument("--one", default=None, help="K,N,M")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--sample", action="store_true")
    ap.add_argument("--rows", default="1,8,64")
    a = ap.parse_args()
    if a.sample:
        for kind in ("peaked", "flat"):
            for rows in (int(v) for v in a.rows.split(",")):
                print(json.dumps(run_sample(kind, rows, iters=a.iters)), flush=True)
        return 0
    hbm, tc, kind = peaks()
    if a.one:
        K, N, M = (int(v) for v in a.one.split(","))
        cases = [(K, N, M)]
    else:
        cases = [(K, N, M) for s in a.shapes.split(",") for (K, N) in SHAPES[s]
                 for M in (int(v) for v in a.m.split(","))]
    for K, N, M in cases:
        r = run_case(K, N, M, iters=a.iters)
        bound = "hbm" if 2 * M < 140 else "tensor"
        r["bound"] = bound
        r["frac"] = round(r["GB_s"] / hbm, 4) if bound == "hbm" else round(r["TFLOP_s"] / tc, 4)
        r["peak_source"] = kind
        print(json.dumps(r), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
