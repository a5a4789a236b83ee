"""Generate the committed golden fixtures by running the REFERENCE's own Python.

Run in a container where the reference checkout is available (it is never
read at test time):

    python tests/golden/make_golden.py --ref <path to lama32_mojo checkout> [--big]

What runs, all from the reference tree, unmodified:

* ``qwen3_mojo/scripts/quantize.py:pack_q8``  -> bit-exact packed Q8 golden
  vectors (random, zero, underflowing, overflowing, tie-at-.5 groups) and
  the sha256 of every packed tensor of the seeded synthetic checkpoints.
* ``scripts/gen_oracle.py:layer`` (Llama-3.2 tied), ``llama31_mojo/scripts/
  gen_oracle.py:layer`` (Llama-3.1 untied) and ``qwen3_mojo/scripts/
  gen_oracle.py:layer`` (Qwen3 QK-norm) -> after_layer0/1 and last logits of a
  prefill at position 0, with ``W()`` returning the Q8-dequantized weights
  (the reference f32 path on Q8 weights).
* ``qwen3_mojo/scripts/bench_python.py:forward`` (torch CPU, KV cache) ->
  logits of a prefill followed by cached greedy decode steps.

The reference scripts compute ``ROOT`` from ``__file__`` and open a model
file at import; they are executed with ``__file__`` pointing into a scratch
directory holding a one-tensor dummy safetensors file, then their module
constants (dims, eps, theta, inverse frequencies) are set for the synthetic
config and ``W`` / ``load_w`` are replaced by the synthetic weights.

``--big`` adds config[0] (Llama-3.2-1B dims, seed 0, 16-token prompt from
seed 1): reference prefill outputs plus 32 greedy decode steps of the oracle.

bf16 weights (the reference's non-Q8 path): the same two reference scripts
with ``W`` / ``load_w`` returning the bf16 checkpoint widened to f32 — which
is what they compute on a real bf16 checkpoint — over seeded checkpoints
whose norm weights are 1 + N(0, 0.1):
``scripts/gen_oracle.py:layer`` on tiny-llama -> tiny_llama_bf16_prefill.npz,
``qwen3_mojo/scripts/bench_python.py:forward`` on tiny-qwen3 ->
tiny_qwen3_bf16_decode.npz.  ``--bf16-only`` writes just these two.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import q8_oracle as O  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# --------------------------------------------------------------------------- reference loading

def load_pack_q8(ref: str):
    path = os.path.join(ref, "qwen3_mojo", "scripts", "quantize.py")
    spec = importlib.util.spec_from_file_location("ref_quantize", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.pack_q8


def ref_pack(pack_q8, w_bf16_u16: np.ndarray) -> np.ndarray:
    import torch
    t = torch.from_numpy(w_bf16_u16.astype(np.int16)).view(torch.bfloat16)
    out = pack_q8(t)
    return out.view(torch.int16).numpy().view(np.uint16).copy()


def exec_ref_script(ref: str, rel: str, scratch: str) -> dict:
    """Execute a reference script with ROOT redirected to ``scratch``."""
    import torch
    from safetensors.torch import save_file
    mdir = os.path.join(scratch, "assets", "model")
    os.makedirs(mdir, exist_ok=True)
    os.makedirs(os.path.join(scratch, "scripts"), exist_ok=True)
    dummy = os.path.join(mdir, "model.safetensors")
    if not os.path.exists(dummy):
        save_file({"dummy": torch.zeros(2, dtype=torch.bfloat16)}, dummy)
    src_path = os.path.join(ref, rel)
    src = open(src_path).read()
    ns = {"__file__": os.path.join(scratch, "scripts", os.path.basename(rel)),
          "__name__": "ref_" + os.path.basename(rel).replace(".py", "")}
    exec(compile(src, src_path, "exec"), ns)
    return ns


def set_llama_consts(ns: dict, cfg: O.Config):
    ns.update(H=cfg.hidden, LAYERS=cfg.layers, NH=cfg.n_heads, NKV=cfg.n_kv, HD=cfg.head_dim,
              INTER=cfg.inter, VOCAB=cfg.vocab, EPS=cfg.eps, THETA=cfg.theta,
              FACTOR=cfg.rope_factor, LOW_FF=cfg.low_ff, HIGH_FF=cfg.high_ff,
              ORIG_CTX=int(cfg.orig_ctx))
    ns["INV_FREQ"] = ns["llama3_inv_freq"]()


def set_qwen_consts(ns: dict, cfg: O.Config):
    ns.update(H=cfg.hidden, LAYERS=cfg.layers, NH=cfg.n_heads, NKV=cfg.n_kv, HD=cfg.head_dim,
              INTER=cfg.inter, VOCAB=cfg.vocab, EPS=cfg.eps, THETA=cfg.theta,
              QD=cfg.q_dim, KVD=cfg.kv_dim)
    ns["INV_FREQ"] = ns["inv_freq"]()


def checkpoint_via_reference(pack_q8, cfg: O.Config, seed: int = 0):
    """The seeded synthetic bf16 checkpoint, 2-D tensors packed by the reference."""
    ck, shas = {}, {}
    for name, w in O.make_bf16_weights(cfg, seed):
        ck[name] = ref_pack(pack_q8, w) if w.ndim == 2 else w
        shas[name] = sha(ck[name])
    return ck, shas


def make_W(cfg: O.Config, ck: dict):
    cache = {}

    def W(name):
        if name not in cache:
            shp = O.tensor_shape(cfg, name)
            a = ck[name]
            if len(shp) == 1 or cfg.weights == "bf16":
                cache[name] = O.bf16_to_f32(a).reshape(shp)
            else:
                cache[name] = O.dequant_q8(a, shp[1])
        return cache[name].copy()
    return W


def ref_prefill(ns: dict, cfg: O.Config, ck: dict, ids, head: str):
    """gen_oracle main() body (scripts/gen_oracle.py:111-127) without tokenizer/dumps."""
    W = make_W(cfg, ck)
    ns["W"] = W
    x = W("model.embed_tokens.weight")[ids].astype(np.float32)
    out = {"ids": np.asarray(ids, np.int32)}
    for L in range(cfg.layers):
        x = ns["layer"](x, L)
        if L in (0, 1):
            out[f"after_layer{L}"] = x.astype(np.float32)
    h = ns["rmsnorm"](x, W("model.norm.weight"))
    out["last_logits"] = (h[-1] @ W(head).T).astype(np.float32)
    return out


def ref_cached_decode_qwen(ns: dict, cfg: O.Config, ck: dict, ids, steps: int):
    """bench_python main() decode loop (qwen3_mojo/scripts/bench_python.py:173-195)."""
    import torch
    W = make_W(cfg, ck)
    ns["load_w"] = lambda name: torch.from_numpy(W(name))
    ns["_WEIGHTS"].clear()
    # module-level INV_FREQ of bench_python.py:31-35 for this config
    ns["INV_FREQ"] = torch.tensor(
        1.0 / (cfg.theta ** (np.arange(0, cfg.head_dim, 2, dtype=np.float64) / cfg.head_dim)),
        dtype=torch.float32)
    ns.update(H=cfg.hidden, LAYERS=cfg.layers, NH=cfg.n_heads, NKV=cfg.n_kv, HD=cfg.head_dim,
              VOCAB=cfg.vocab, EPS=cfg.eps, THETA=cfg.theta, QD=cfg.q_dim)
    cache = ns["KVCache"]()
    logits = ns["forward"](cache, list(ids))
    all_logits = [logits.numpy().astype(np.float32)]
    toks = []
    tok = int(torch.argmax(logits).item())
    for _ in range(steps):
        toks.append(tok)
        logits = ns["forward"](cache, [tok])
        all_logits.append(logits.numpy().astype(np.float32))
        tok = int(torch.argmax(logits).item())
    toks.append(tok)
    return {"ids": np.asarray(ids, np.int32), "tokens": np.asarray(toks, np.int32),
            "logits": np.stack(all_logits)}


# --------------------------------------------------------------------------- pack cases

def pack_cases(pack_q8) -> dict:
    rng = np.random.default_rng(123)
    cases = {}

    def add(name, w32):
        wb = O.bf16_round(np.asarray(w32, np.float32))
        cases[name + "_in"] = wb
        cases[name + "_out"] = ref_pack(pack_q8, wb)

    add("rand_64x128", rng.standard_normal((64, 128), dtype=np.float32) * 0.02)
    add("rand_33x2048", rng.standard_normal((33, 2048), dtype=np.float32))
    add("rand_7x4096_wide", rng.standard_normal((7, 4096), dtype=np.float32) * 30.0)
    add("rand_5x1792", rng.standard_normal((5, 1792), dtype=np.float32) * 0.5)
    # special groups: zero, scale underflowing f16 (-> x/0), subnormal scale,
    # overflowing scale (f16 inf), exact .5 ties, signed zeros, saturation.
    sp = np.zeros((8, 128), np.float32)
    sp[1, :64] = 0.0
    sp[1, 64:] = -0.0
    sp[2, :5] = [1e-7, -2e-6, 0.0, 3e-7, -0.0]          # scale -> 0 in f16
    sp[2, 64:70] = [1e-3, -5e-4, 2e-4, 0, 7e-4, -1e-3]   # subnormal f16 scale
    sp[3, :4] = [1e7, -3e6, 2.0, -1e5]                   # scale overflows to inf
    sp[3, 64:] = np.linspace(-1, 1, 64)
    sp[4, :64] = np.arange(64) - 31.5                    # many .5 ties after scaling
    sp[4, 64:] = 127.0 * (np.arange(64) % 3 - 1) + 0.5
    sp[5, :] = rng.standard_normal(128).astype(np.float32) * 1e-4
    sp[6, :] = 2.0 ** np.arange(-60, 68, dtype=np.float32) * np.where(np.arange(128) % 2, 1, -1)
    sp[7, :] = 65504.0 * 127.0
    add("special_8x128", sp)
    return cases


# --------------------------------------------------------------------------- bf16 path

def bf16_fixtures(ref: str, scratch: str):
    """Reference outputs on bf16 weights (the checkpoint as stored, no packing)."""
    cfg = O.PRESETS["tiny-llama"].replace(weights="bf16")
    ck = O.make_bf16_checkpoint(cfg, seed=5, norm_std=0.1)
    ns = exec_ref_script(ref, "scripts/gen_oracle.py", os.path.join(scratch, "llama32bf"))
    set_llama_consts(ns, cfg)
    np.savez_compressed(os.path.join(HERE, "tiny_llama_bf16_prefill.npz"),
                        **ref_prefill(ns, cfg, ck, O.random_ids(cfg, 11), "model.embed_tokens.weight"))
    cfg = O.PRESETS["tiny-qwen3"].replace(weights="bf16")
    ck = O.make_bf16_checkpoint(cfg, seed=6, norm_std=0.1)
    nsb = exec_ref_script(ref, "qwen3_mojo/scripts/bench_python.py", os.path.join(scratch, "qwen3bf"))
    np.savez_compressed(os.path.join(HERE, "tiny_qwen3_bf16_decode.npz"),
                        **ref_cached_decode_qwen(nsb, cfg, ck, O.random_ids(cfg, 7), 6))


# --------------------------------------------------------------------------- main

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True)
    ap.add_argument("--big", action="store_true")
    ap.add_argument("--bf16-only", action="store_true")
    a = ap.parse_args()
    ref = a.ref
    pack_q8 = load_pack_q8(ref)
    scratch = tempfile.mkdtemp(prefix="q8golden_")
    if a.bf16_only:
        bf16_fixtures(ref, scratch)
        print("wrote bf16 fixtures to", HERE)
        return

    np.savez_compressed(os.path.join(HERE, "pack_cases.npz"), **pack_cases(pack_q8))

    manifest = {"generator": "tests/golden/make_golden.py", "checkpoints": {}}

    # --- tiny Llama-3.2 shape, tied head: scripts/gen_oracle.py
    cfg = O.PRESETS["tiny-llama"]
    ck, shas = checkpoint_via_reference(pack_q8, cfg)
    manifest["checkpoints"][cfg.name] = shas
    ns = exec_ref_script(ref, "scripts/gen_oracle.py", os.path.join(scratch, "llama32"))
    set_llama_consts(ns, cfg)
    np.savez_compressed(os.path.join(HERE, "tiny_llama_prefill.npz"),
                        **ref_prefill(ns, cfg, ck, O.random_ids(cfg, 11), "model.embed_tokens.weight"))

    # --- tiny Llama-3.1 shape, untied head: llama31_mojo/scripts/gen_oracle.py
    cfg = O.PRESETS["tiny-llama-untied"]
    ck, shas = checkpoint_via_reference(pack_q8, cfg)
    manifest["checkpoints"][cfg.name] = shas
    ns = exec_ref_script(ref, "llama31_mojo/scripts/gen_oracle.py", os.path.join(scratch, "llama31"))
    set_llama_consts(ns, cfg)
    np.savez_compressed(os.path.join(HERE, "tiny_llama_untied_prefill.npz"),
                        **ref_prefill(ns, cfg, ck, O.random_ids(cfg, 9), "lm_head.weight"))

    # --- tiny Qwen3 shape: qwen3_mojo/scripts/gen_oracle.py and bench_python.py
    cfg = O.PRESETS["tiny-qwen3"]
    ck, shas = checkpoint_via_reference(pack_q8, cfg)
    manifest["checkpoints"][cfg.name] = shas
    ns = exec_ref_script(ref, "qwen3_mojo/scripts/gen_oracle.py", os.path.join(scratch, "qwen3"))
    set_qwen_consts(ns, cfg)
    np.savez_compressed(os.path.join(HERE, "tiny_qwen3_prefill.npz"),
                        **ref_prefill(ns, cfg, ck, O.random_ids(cfg, 13), "model.embed_tokens.weight"))
    nsb = exec_ref_script(ref, "qwen3_mojo/scripts/bench_python.py", os.path.join(scratch, "qwen3b"))
    np.savez_compressed(os.path.join(HERE, "tiny_qwen3_decode.npz"),
                        **ref_cached_decode_qwen(nsb, cfg, ck, O.random_ids(cfg, 7), 6))

    bf16_fixtures(ref, scratch)

    if a.big:
        # --- config[0]: Llama-3.2-1B dims, 16-token prompt, 32 greedy steps
        cfg = O.PRESETS["llama-3.2-1b"]
        ck, shas = checkpoint_via_reference(pack_q8, cfg)
        manifest["checkpoints"][cfg.name] = shas
        ids = O.random_ids(cfg, 16)
        ns = exec_ref_script(ref, "scripts/gen_oracle.py", os.path.join(scratch, "llama32big"))
        set_llama_consts(ns, cfg)
        pre = ref_prefill(ns, cfg, ck, ids, "model.embed_tokens.weight")
        ns = None
        m = O.OracleModel(cfg, ck)
        toks, margins, logits = O.greedy_generate(m, ids, 32)
        top = np.stack([np.argsort(-lg)[:8] for lg in logits]).astype(np.int32)
        topv = np.stack([lg[np.argsort(-lg)[:8]] for lg in logits]).astype(np.float32)
        np.savez_compressed(os.path.join(HERE, "config0_llama1b.npz"), **pre,
                            oracle_prefill_logits=logits[0].astype(np.float32),
                            tokens=np.asarray(toks, np.int32),
                            margins=np.asarray(margins, np.float32),
                            top_ids=top, top_vals=topv)
    else:
        old = os.path.join(HERE, "manifest.json")
        if os.path.exists(old):
            prev = json.load(open(old)).get("checkpoints", {})
            for k, v in prev.items():
                manifest["checkpoints"].setdefault(k, v)

    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
