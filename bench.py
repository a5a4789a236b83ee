#!/usr/bin/env python3
"""Decode throughput of the B200 Q8 path (BASELINE metric: decode tok/s,
Llama-3.1-8B Q8, 1/2/4/8 B200; Q8 GEMV HBM GB/s vs peak).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--ctx C] [--impl ours|reference]

Workload (config[3]): Llama-3.1-8B architecture, random-init N(0, 0.02) weights
quantized by the GPU packer (Q8 group 64, f16 scales), KV cache capacity 4096
per sequence (f32, as the reference), a random prompt prefilled to
``ctx - warmup - steps`` tokens, then greedy decode of batch B.  A step = one
decode token for each of the B sequences.  Tensor parallel over N GPUs (one
process per GPU, NCCL), so per-GPU weight bytes shrink with N ("strong").

* value     : tokens/s with the loop resident on the device (q8_generate: the
              argmax of each step feeds the next on the GPU), CUDA events on the
              model stream, barrier + sync on both sides, max over ranks.
* e2e       : tokens/s through the public per-step API (q8_decode with host
              ids in pinned staging and the argmax read back every step).
* roofline  : the Q8 GEMV kernels (dominant): algorithmic bytes (codes + f16
              scales + activations + outputs) / their CUDA-event durations,
              from per-launch events of profiled steps after the timed region.
* cpu_baseline : the CPU port of the reference path (oracle/q8_ref.c, pthreads,
              all host threads) timed on a bounded sample of the same decode
              step (a few full-width layers + the lm_head), scaled by layers.
* --impl reference : that CPU port alone as the reference arm.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=4096, help="KV capacity per sequence")
    ap.add_argument("--model", default="llama-3.1-8b")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-layers", type=int, default=0, help="layers in the CPU baseline (0: all)")
    ap.add_argument("--batches", default="8,64",
                    help="extra decode batch sizes reported beside the headline batch ('' for none)")
    ap.add_argument("--extra-steps", type=int, default=32, help="timed steps of each extra batch")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=32)
    return ap.parse_args()


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                if out:
                    self.samples.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 5 + i and s[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ----------------------------------------------------------------------------- CPU arm
def cpu_baseline(cfg, batch: int, ctx: int, layers: int, steps: int = 2):
    """The CPU port (oracle/q8_ref.c) on a bounded sample of one decode step."""
    from oracle import q8_ref
    r = q8_ref.time_decode_sample(cfg, batch=batch, ctx=ctx, sample_layers=layers, steps=steps)
    return r


PROFILED_STEPS = 4  # decode steps run with per-launch profiling after the timed region


def workload(a, world: int):
    """The decode workload both arms report: prompt length, the context at the
    middle of the timed steps, and the config object of the JSON line."""
    prompt = a.ctx - a.warmup - a.steps - a.e2e_steps - 8
    ctx_mid = prompt + a.warmup + a.steps // 2
    config = {"workload": f"{a.model} Q8 greedy decode, batch {a.batch}, KV capacity {a.ctx}, "
                          f"context {prompt}..{prompt + a.warmup + a.steps + a.e2e_steps + PROFILED_STEPS}",
              "model": a.model, "global_batch": a.batch, "seq_len": a.ctx, "prompt": prompt,
              "parallelism": f"tp{world}", "kv_dtype": "f32",
              "l2": "weights+KV per step > 126 MB L2 (no flush needed)"}
    return prompt, ctx_mid, config


def run_reference_arm(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from lama32_mojo_b200.config import PRESETS
    cfg = PRESETS[a.model]
    # the same workload as the GPU arm, sampled at the middle of its timed steps
    _, ctx, config = workload(a, a.gpus)
    r = cpu_baseline(cfg, a.batch, ctx, a.cpu_layers, steps=max(1, min(a.steps, 3)))
    line = {
        "impl": "reference", "metric": "decode tok/s", "value": r["tok_s"], "unit": "tok/s",
        "n_gpus": a.gpus, "steps": r["steps"], "warmup": 1, "ms_per_step": r["ms_per_step"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": config,
        "cpu_baseline": {"value": r["tok_s"], "unit": "tok/s", "cores": r["threads"], "kind": "port",
                         "sample": r["sample"]},
        "e2e": {"value": r["tok_s"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- GPU arm
def tp_parity(world, rank, local, dist):
    """Tensor-parallel parity before the timed region: a small model whose
    heads and vocabulary split over 8 ranks ("tiny-tp8": 8 kv heads, untied
    vocabulary-parallel head) runs at TP = world (NCCL prefill, the P2P decode
    exchange) and, on rank 0's GPU, at TP = 1 with the same GPU-made weights.
    The single-GPU path is the one the parity tests pin to the oracle.
    Returns (rank 0) the relative L2 of the layer-1 residual and the last
    prefill logits, and whether 8 greedy tokens agree."""
    import numpy as np

    from lama32_mojo_b200.config import PRESETS
    from lama32_mojo_b200.model import load_synthetic, nccl_unique_id

    tcfg = PRESETS["tiny-tp8"]
    uid = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    ids = np.random.default_rng(7).integers(0, tcfg.vocab, size=12).tolist()

    def run(mod):
        h1 = mod.forward_hidden(ids, 1)
        lg = mod.forward(ids)
        toks = [int(np.argmax(lg))]
        for _ in range(7):
            toks.append(int(mod.decode([toks[-1]], [0])[0]))
        mod.close()
        return h1, lg, toks

    got = run(load_synthetic(tcfg, device=local, seed=5, maxlen=64, max_seqs=1, tp_rank=rank, tp_size=world,
                             nccl_id=uid[0]))
    out = None
    if rank == 0:
        ref = run(load_synthetic(tcfg, device=local, seed=5, maxlen=64, max_seqs=1))
        rl2 = lambda x, y: float(np.linalg.norm(np.asarray(x, np.float64) - y) / max(np.linalg.norm(y), 1e-30))
        out = {"config": "tiny-tp8 (hidden 512, 2 layers, 8/8 heads, vocab 2048 untied)", "tp": world,
               "reference": "TP=1 on rank 0 (the oracle-pinned single-GPU path), same weights",
               "rel_l2_hidden_layer1": rl2(got[0], ref[0]), "rel_l2_logits": rl2(got[1], ref[1]),
               "tokens_equal": got[2] == ref[2], "tokens": got[2]}
        out["pass"] = bool(out["rel_l2_hidden_layer1"] <= 1e-5 and out["rel_l2_logits"] <= 1e-5
                           and out["tokens_equal"])
    dist.barrier()
    return out


def main():
    a = parse()
    if a.impl == "reference":
        return run_reference_arm(a)

    import numpy as np
    import torch
    import torch.distributed as dist
    from lama32_mojo_b200.config import PRESETS
    from lama32_mojo_b200.model import Q8Model, load_synthetic, nccl_unique_id

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=300))
        uid = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        nid = uid[0]
    else:
        nid = None

    cfg = PRESETS[a.model]
    B = a.batch
    batches = [int(v) for v in a.batches.split(",") if v.strip()] if a.batches else []
    prompt, ctx_mid, config = workload(a, world)
    assert prompt > 0, "ctx too small for warmup+steps"
    tpp = tp_parity(world, rank, local, dist) if world > 1 else None
    m = load_synthetic(cfg, device=local, seed=0, maxlen=a.ctx, max_seqs=max([B] + batches), max_tokens=2048,
                       tp_rank=rank, tp_size=world, nccl_id=nid)
    rng = np.random.default_rng(1)
    first = []
    ext = torch.cuda.ExternalStream(m.stream, device=dev)
    # prompt prefill (tensor-core GEMMs for chunks of >= 128 tokens): timed with
    # CUDA events, the last sequence's kernels profiled for the GEMM share
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    m.set_profiling(True)
    p0.record(ext)
    for b in range(B):
        ids = rng.integers(0, cfg.vocab, size=prompt).tolist()
        lg = m.forward(ids, seq=b)
        if not np.isfinite(lg).all():
            raise SystemExit("prefill produced non-finite logits: the workload is invalid")
        first.append(int(np.argmax(lg)))
    p1.record(ext)
    torch.cuda.synchronize()
    m.set_profiling(False)
    prefill_ms = p0.elapsed_time(p1)
    pprof = m.profile()
    seqs = list(range(B))

    def barrier():
        if world > 1:
            dist.barrier()

    # warmup (graph capture + clocks)
    toks = m.generate(first, seqs, a.warmup)
    cur = toks[-1].tolist()

    # ---- timed region: value (device-resident greedy loop)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.nvtx.range_push("decode_timed")
        e0.record(ext)
        toks = m.generate(cur, seqs, a.steps)
        e1.record(ext)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    if toks.min() < 0 or toks.max() >= cfg.vocab:
        raise SystemExit("decode produced out-of-range tokens: the workload is invalid")
    cur = toks[-1].tolist()
    ms_per_step = ms / a.steps
    value = B * a.steps / (ms / 1e3)

    # ---- e2e: per-step public API, host ids in, host argmax out
    barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(ext)
    for _ in range(a.e2e_steps):
        cur = m.decode(cur, seqs).tolist()
    f1.record(ext)
    torch.cuda.synchronize()
    barrier()
    ems = f0.elapsed_time(f1)
    if world > 1:
        t = torch.tensor([ems], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t.item())
    e2e = B * a.e2e_steps / (ems / 1e3)

    # ---- roofline of the dominant kernel (Q8 GEMV), per-launch CUDA events
    m.set_profiling(True)
    agg = {}
    nprof = PROFILED_STEPS
    for _ in range(nprof):
        cur = m.decode(cur, seqs).tolist()
        for k, (kms, kb, kl) in m.profile().items():
            s = agg.setdefault(k, [0.0, 0.0, 0])
            s[0] += kms
            s[1] += kb
            s[2] += kl
    m.set_profiling(False)
    # dominant kernel: the one-launch weight-ring decode step when it runs
    # (every GEMV, attention and norm of a step), else the Q8 GEMV launches
    dom = ["decode_step"] if "decode_step" in agg else [k for k in agg if k.startswith("gemv_")]
    dom_name = ("k_decode_ring (one-launch decode step: weights + KV of the whole step)"
                if dom == ["decode_step"] else "k_gemv_d (all Q8 GEMV launches of a decode step)")
    g_ms = sum(agg[k][0] for k in dom)
    g_b = sum(agg[k][1] for k in dom)
    g_l = sum(agg[k][2] for k in dom)
    peak, peak_kind = load_peaks()
    achieved = g_b / (g_ms / 1e3) / 1e9 if g_ms > 0 else 0.0
    # "phase:*" entries split the ring step's time (no launches of their own)
    step_ms_prof = sum(v[0] for k, v in agg.items() if not k.startswith("phase:")) / nprof
    breakdown = {k: {"ms_per_step": round(v[0] / nprof, 4), "launches_per_step": v[2] // nprof,
                     "GB_s": round(v[1] / (v[0] / 1e3) / 1e9, 1) if v[0] > 0 else None} for k, v in agg.items()}
    # DRAM traffic per launch of the dominant kernel: the ncu capture's
    # traffic / algorithmic ratio (profiles/decode_traffic.json) times this
    # launch's algorithmic bytes; null where no capture covers the kernel
    traffic = None
    tp = os.path.join(REPO, "profiles", "decode_traffic.json")
    if dom == ["decode_step"] and g_l > 0 and os.path.exists(tp):
        ratio = json.load(open(tp)).get("k_decode_ring")
        if ratio:
            traffic = round(ratio * g_b / g_l)

    # launches per step: our kernels inside the generate graph = the profiled
    # decode launches + the on-device step epilogue (k_step_end), which the
    # one-launch ring step does itself
    launches_per_step = sum(v[2] for v in agg.values()) // nprof + (0 if "decode_step" in agg else 1)
    gpu_launches = launches_per_step * a.steps

    # prefill summary: algorithmic GEMM flops (2*M*N*K; the split-operand mode
    # issues three tensor-core MMAs per product) over the profiled GEMM time
    H, F, L = cfg.hidden, cfg.inter // world, cfg.layers
    qd, kvd = cfg.n_heads * cfg.head_dim // world, cfg.n_kv * cfg.head_dim // world
    kn = {"gemm_qkv": H * (qd + 2 * kvd), "gemm_o": qd * H, "gemm_gateup": H * 2 * F, "gemm_down": F * H}
    g_ms = sum(pprof[k][0] for k in kn if k in pprof)
    g_fl = sum(2.0 * prompt * kn[k] * L for k in kn if k in pprof)
    tot_ms = sum(v[0] for v in pprof.values())
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    tc_peak = float(peaks.get("bf16_tflops", 1590.0))
    prefill = {"tokens": prompt * B, "ms": round(prefill_ms, 2), "tok_s": round(prompt * B / (prefill_ms / 1e3), 1),
               "chunk_tokens": 2048,
               "gemm_tflops": round(g_fl / (g_ms / 1e3) / 1e12, 1) if g_ms > 0 else None,
               "gemm_peak_tflops": tc_peak, "gemm_frac": round(g_fl / (g_ms / 1e3) / 1e12 / tc_peak, 4) if g_ms > 0 else None,
               "gemm_mode": "split operands (hi*hi + hi*lo + lo*hi tcgen05 MMAs, f32-accurate)",
               "share": {k: round(v[0] / tot_ms, 3) for k, v in pprof.items()} if tot_ms > 0 else None}

    step_bytes = cfg.decode_bytes(B, ctx_mid, tp=world)
    peak_bw = load_peaks()[0]

    # ---- the other config[3] batch sizes: fresh prompts, device-resident loop
    extra = {}
    for Bx in batches:
        xs = list(range(Bx))
        xprompt = a.ctx - a.warmup - a.extra_steps - 8
        firsts = []
        for s in xs:
            m.reset(s)
            lg = m.forward(rng.integers(0, cfg.vocab, size=xprompt).tolist(), seq=s)
            firsts.append(int(np.argmax(lg)))
        cur_x = m.generate(firsts, xs, a.warmup)[-1].tolist()
        barrier()
        torch.cuda.synchronize()
        x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        x0.record(ext)
        tx = m.generate(cur_x, xs, a.extra_steps)
        x1.record(ext)
        torch.cuda.synchronize()
        barrier()
        xms = x0.elapsed_time(x1)
        if world > 1:
            t = torch.tensor([xms], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            xms = float(t.item())
        if tx.min() < 0 or tx.max() >= cfg.vocab:
            raise SystemExit("decode produced out-of-range tokens: the workload is invalid")
        xmid = xprompt + a.warmup + a.extra_steps // 2
        xb = cfg.decode_bytes(Bx, xmid, tp=world)
        xstep = xms / a.extra_steps
        extra[str(Bx)] = {"value": round(Bx * a.extra_steps / (xms / 1e3), 2), "unit": "tok/s",
                          "ms_per_step": round(xstep, 4), "steps": a.extra_steps,
                          "context": f"{xprompt}..{xprompt + a.warmup + a.extra_steps}",
                          "step_roofline": {"bytes_per_step": xb,
                                            "achieved_GB_s": round(xb / (xstep / 1e3) / 1e9, 1),
                                            "frac": round(xb / (xstep / 1e3) / 1e9 / peak_bw, 4)}}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu:
        try:
            r = cpu_baseline(cfg, B, ctx_mid, a.cpu_layers)
            cpu = {"value": r["tok_s"], "unit": "tok/s", "cores": r["threads"], "kind": "port",
                   "sample": r["sample"]}
        except Exception as ex:  # the GPU number stands without it
            cpu = {"value": None, "unit": "tok/s", "cores": None, "kind": "port", "sample": f"failed: {ex}"}

    if rank == 0:
        line = {
            "metric": "decode tok/s", "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8xf32",
            "data": "synthetic (random-init N(0,0.02) weights, random prompt ids)",
            "config": config,
            "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 12 * B,
                    "d2h_bytes_per_step": 4 * B},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": dom_name,
                         "peak_source": f"{peak_kind} hbm_gbs", "launches_per_step": g_l // nprof},
            "step_roofline": {"bytes_per_step": step_bytes, "achieved_GB_s": round(step_bytes / (ms_per_step / 1e3) / 1e9, 1),
                              "frac": round(step_bytes / (ms_per_step / 1e3) / 1e9 / peak, 4)},
            "kernels": breakdown, "profiled_step_ms": round(step_ms_prof, 4),
            "gpu_launches": gpu_launches, "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "prefill": prefill,
            "batches": extra,
        }
        if tpp is not None:
            line["tp_parity"] = tpp
        print(json.dumps(line), flush=True)
    m.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
