"""Tensor-parallel partitioning on CPU ranks (gloo, world_size 2 and 4).

Each rank takes its shard of every weight exactly as the library's loader
does (``q8_shard_plan``: column-parallel q/k/v/gate/up rows, row-parallel
o/down K slices of whole 64-groups, vocab-parallel untied lm_head), runs the
layer math on its heads / FFN slice in numpy, sums the row-parallel partials
with an all-reduce and gathers the vocab shards.  The result must equal the
unsharded oracle: the sharding plan partitions the computation exactly.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lama32_mojo_b200 import PRESETS
from lama32_mojo_b200.model import shard_plan
from oracle import q8_oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _slice(cfg, name, full, r, t):
    p = shard_plan(cfg, r, t, name)
    if full.ndim == 1:
        return full
    return full[p["row0"]:p["row0"] + p["nrows"], p["k0"]:p["k0"] + p["kl"]]


def _allreduce(a):
    t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
    dist.all_reduce(t)
    return t.numpy()


def _rank_main(rank, world, port, cfgname, ids, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = PRESETS[cfgname]
        ocfg = O.PRESETS[cfgname]
        ck = O.make_q8_checkpoint(ocfg)
        full = O.OracleModel(ocfg, ck)
        W = lambda n: _slice(cfg, n, full.W(n), rank, world)  # noqa: E731
        nh, nkv, hd = cfg.n_heads // world, cfg.n_kv // world, cfg.head_dim
        inv = O.inv_freq(ocfg)
        x = O.embed_q8(ck["model.embed_tokens.weight"], cfg.hidden, ids)  # replicated embedding
        s = len(ids)
        for L in range(cfg.layers):
            p = f"model.layers.{L}."
            xn = O.rmsnorm(x, W(p + "input_layernorm.weight"), cfg.eps)
            q = (xn @ W(p + "self_attn.q_proj.weight").T).reshape(s, nh, hd)
            k = (xn @ W(p + "self_attn.k_proj.weight").T).reshape(s, nkv, hd)
            v = (xn @ W(p + "self_attn.v_proj.weight").T).reshape(s, nkv, hd)
            if cfg.qk_norm:
                q = O.rmsnorm(q, W(p + "self_attn.q_norm.weight"), cfg.eps)
                k = O.rmsnorm(k, W(p + "self_attn.k_norm.weight"), cfg.eps)
            q, k = O.rope(q, 0, inv), O.rope(k, 0, inv)
            ao = O.attention(q, k, v, nh // nkv).reshape(s, nh * hd)
            x = x + _allreduce(ao @ W(p + "self_attn.o_proj.weight").T)
            xn = O.rmsnorm(x, W(p + "post_attention_layernorm.weight"), cfg.eps)
            g = xn @ W(p + "mlp.gate_proj.weight").T
            u = xn @ W(p + "mlp.up_proj.weight").T
            x = x + _allreduce(O.silu_mul(g, u) @ W(p + "mlp.down_proj.weight").T)
        h = O.rmsnorm(x[-1:], W("model.norm.weight"), cfg.eps)
        head = "model.embed_tokens.weight" if cfg.tied else "lm_head.weight"
        if cfg.tied:  # the tied head reads the replicated embedding's vocab shard
            vl = cfg.vocab // world
            local = (h @ full.W(head)[rank * vl:(rank + 1) * vl].T)[0]
        else:
            local = (h @ W(head).T)[0]
        parts = [torch.zeros(len(local)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(local.astype(np.float32)))
        if rank == 0:
            out_q.put(torch.cat(parts).numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cfgname,world", [("tiny-llama-untied", 2), ("tiny-qwen3", 2), ("tiny-llama", 2)])
def test_tp_sharded_forward_equals_oracle(cfgname, world):
    ocfg = O.PRESETS[cfgname]
    ids = O.random_ids(ocfg, 5, seed=21)
    ref = O.OracleModel(ocfg, O.make_q8_checkpoint(ocfg)).forward(ids)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, cfgname, ids, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert O.rel_l2(got, ref) < 1e-5


def test_tp_partial_sums_are_exact_partition():
    """Row-parallel K slices of the packed rows reassemble the full product (tp 4)."""
    cfg = PRESETS["tiny-llama-untied"]
    ocfg = O.PRESETS["tiny-llama-untied"]
    ck = O.make_q8_checkpoint(ocfg)
    name = "model.layers.0.mlp.down_proj.weight"
    full = O.dequant_q8(ck[name], cfg.inter)
    x = np.random.default_rng(0).standard_normal((3, cfg.inter)).astype(np.float32)
    acc = np.zeros((3, cfg.hidden), np.float32)
    for r in range(4):
        p = shard_plan(cfg, r, 4, name)
        acc += x[:, p["k0"]:p["k0"] + p["kl"]] @ full[:, p["k0"]:p["k0"] + p["kl"]].T
    assert O.rel_l2(acc, x @ full.T) < 1e-6
