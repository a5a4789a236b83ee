"""CPU oracle for the Q8 (W8A32, group-64) decode/prefill path — TEST INFRASTRUCTURE.

This module is a checker, never a product path: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import it.  The CUDA library (``libq8cuda.so``) never calls into it.

It restates, in numpy, the reference algorithm of plutonium-guy/lama32_mojo:

* quantizer ``pack_q8``            qwen3_mojo/scripts/quantize.py:31-43
* packed row layout               src/llama_q8.mojo:26-42
* Q8 matmul ``k_mm_q8``            src/llama_q8.mojo:54-93
* Q8 embedding gather             src/llama_q8.mojo:96-109
* RMSNorm                          scripts/gen_oracle.py:37-39 (k_rmsnorm_w src/llama_common.mojo:197-225)
* llama3 / plain RoPE frequencies  scripts/gen_oracle.py:42-55, qwen3_mojo/scripts/bench_python.py:31-35
* rotate-half RoPE                 scripts/gen_oracle.py:61-69
* Qwen3 per-head QK RMSNorm        qwen3_mojo/scripts/gen_oracle.py:69-70
* GQA causal attention             scripts/gen_oracle.py:79-89, cached form qwen3_mojo/scripts/bench_python.py:77-93
* SwiGLU + residual                scripts/gen_oracle.py:90-95
* layer / cached decode loop       qwen3_mojo/scripts/bench_python.py:96-130
* final norm + (un)tied lm_head    scripts/gen_oracle.py:126-127, llama31_mojo/scripts/gen_oracle.py:133
* temperature + nucleus sampling   src/sample.mojo:15-59 (``sample_literal``; no golden
                                   vectors exist for it: parity unpinned, cross-checked
                                   against the C restatement ``oracle/q8_ref.c``)

Parity is pinned by ``tests/golden/make_golden.py``, which runs the
reference's own Python (``pack_q8``, ``gen_oracle.layer``,
``bench_python.forward``) on seeded inputs and commits the outputs.
"""
from __future__ import annotations

import dataclasses
import math
from typing import Dict, List, Optional

import numpy as np

QG = 64  # quantization group along K (src/llama_q8.mojo:23, quantize.py:28)


# --------------------------------------------------------------------------- bf16 / f16 helpers

def bf16_round(x: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bits (uint16), round-to-nearest-even (torch's .to(bfloat16))."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u.astype(np.uint64) + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r


def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    """bf16 bits -> f32 (exact), as gen_oracle.W does (scripts/gen_oracle.py:32-33)."""
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# --------------------------------------------------------------------------- quantizer

def q8_rowstride(m: int) -> int:
    """Packed row length in u16 elements (src/llama_q8.mojo:26-28)."""
    return m // QG + m // 2


def pack_q8(w_bf16: np.ndarray) -> np.ndarray:
    """Restates quantize.pack_q8 (qwen3_mojo/scripts/quantize.py:31-43).

    ``w_bf16``: uint16 bf16 bits, shape [n, m].  Returns uint16 [n, m/64 + m/2]:
    per row the m/64 f16 group scales, then the m int8 codes (two per u16).

      scale_g = f16(max(f32(absmax_g) / 127, 1e-8))        (:36-37)
      q       = clip(rint(x / f32(scale_g)), -127, 127)     (:38-39)

    Edge case kept bit-exact: a scale that rounds to 0 in f16 gives x/0, i.e.
    +-inf -> +-127 and NaN (x == 0) -> 0 on x86 numpy.
    """
    n, m = w_bf16.shape
    assert m % QG == 0 and m % 2 == 0, (n, m)
    x = bf16_to_f32(w_bf16).reshape(n, m // QG, QG)
    scale = np.abs(x).max(axis=2) / np.float32(127.0)
    scale = np.maximum(scale, np.float32(1e-8)).astype(np.float16)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.rint(x / scale[:, :, None].astype(np.float32))
    q = np.where(np.isnan(q), 0.0, q)
    q = np.clip(q, -127, 127).astype(np.int8).reshape(n, m)
    return np.concatenate([scale.view(np.uint16), q.view(np.uint16)], axis=1)


def unpack_q8(packed: np.ndarray, m: int):
    """Split packed rows into (f16 scales [n, m/64], int8 codes [n, m])."""
    packed = np.ascontiguousarray(packed, dtype=np.uint16)
    n = packed.shape[0]
    assert packed.shape[1] == q8_rowstride(m), (packed.shape, m)
    scales = packed[:, : m // QG].copy().view(np.float16)
    codes = packed[:, m // QG:].copy().view(np.int8).reshape(n, m)
    return scales, codes


def dequant_q8(packed: np.ndarray, m: int) -> np.ndarray:
    """w = f32(int8) * f32(f16 scale) — the dequant of src/llama_q8.mojo:9."""
    scales, codes = unpack_q8(packed, m)
    n = codes.shape[0]
    s = scales.astype(np.float32)
    return (codes.reshape(n, m // QG, QG).astype(np.float32) * s[:, :, None]).reshape(n, m)


def mm_q8(x: np.ndarray, packed: np.ndarray, m: int) -> np.ndarray:
    """y[s, n] = sum_g f16(s[n,g]) * sum_{k in g} x[s,k] * q[n,k]  (k_mm_q8, src/llama_q8.mojo:54-93).

    Group-major like the reference: the unscaled int8 dot of each 64-wide group
    is accumulated in f32, then multiplied by that group's scale.
    """
    scales, codes = unpack_q8(packed, m)
    n = codes.shape[0]
    x = np.ascontiguousarray(x, dtype=np.float32)
    s = x.shape[0]
    g = m // QG
    out = np.zeros((s, n), dtype=np.float32)
    step = max(1, (1 << 26) // max(1, m))  # bound the temporary
    for j0 in range(0, n, step):
        c = codes[j0:j0 + step].reshape(-1, g, QG).astype(np.float32)
        part = np.einsum("sgk,ngk->sng", x.reshape(s, g, QG), c, optimize=True)
        out[:, j0:j0 + step] = (part * scales[j0:j0 + step].astype(np.float32)[None]).sum(-1)
    return out


def embed_q8(packed_emb: np.ndarray, d: int, ids) -> np.ndarray:
    """k_embed_gather_q8 (src/llama_q8.mojo:96-109): f32(int8) * f16 scale."""
    rows = np.asarray(packed_emb)[np.asarray(ids, dtype=np.int64)]
    return dequant_q8(rows, d)


# --------------------------------------------------------------------------- model config

@dataclasses.dataclass(frozen=True)
class Config:
    """Mirror of ``Config`` (src/llama_common.mojo:26-52) plus the family flags."""
    name: str
    hidden: int
    layers: int
    n_heads: int
    n_kv: int
    head_dim: int
    inter: int
    vocab: int
    eps: float
    theta: float
    rope_type: str = "llama3"      # "llama3" (llama_common.mojo:618) or "default" (:609)
    rope_factor: float = 1.0
    low_ff: float = 1.0
    high_ff: float = 4.0
    orig_ctx: float = 8192.0
    qk_norm: bool = False          # Qwen3 per-head RMSNorm (llama_q8.mojo:171)
    tied: bool = True              # lm_head = embed_tokens (qwen_q8.mojo:143-145)
    weights: str = "q8"            # "q8": packed Q8 matrices; "bf16": the non-Q8 path
                                   # (run_layer / mm_op, src/llama_common.mojo:636-780)

    @property
    def q_dim(self):
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self):
        return self.n_kv * self.head_dim

    @property
    def group(self):
        return self.n_heads // self.n_kv

    def replace(self, **kw) -> "Config":
        return dataclasses.replace(self, **kw)


PRESETS: Dict[str, Config] = {
    # config[0] / the llama32 shell (src/llama_gpu.mojo:29-31, assets/model/config.json)
    "llama-3.2-1b": Config("llama-3.2-1b", 2048, 16, 32, 8, 64, 8192, 128256, 1e-5, 500000.0,
                           "llama3", 32.0, 1.0, 4.0, 8192.0, False, True),
    # config[2]
    "llama-3.2-3b": Config("llama-3.2-3b", 3072, 28, 24, 8, 128, 8192, 128256, 1e-5, 500000.0,
                           "llama3", 32.0, 1.0, 4.0, 8192.0, False, True),
    # config[3] (llama31_mojo/src/llama_gpu.mojo:46-48, untied head)
    "llama-3.1-8b": Config("llama-3.1-8b", 4096, 32, 32, 8, 128, 14336, 128256, 1e-5, 500000.0,
                           "llama3", 8.0, 1.0, 4.0, 8192.0, False, False),
    # config[4] (Qwen3 family: QK-norm, plain RoPE theta 1e6, qwen_q8.mojo:30-32)
    "qwen3-8b": Config("qwen3-8b", 4096, 36, 32, 8, 128, 12288, 151936, 1e-6, 1000000.0,
                       "default", 1.0, 1.0, 4.0, 8192.0, True, False),
    # Qwen3-0.6B: the model the reference's own Q8 shell runs (qwen_q8.mojo:30-32)
    "qwen3-0.6b": Config("qwen3-0.6b", 1024, 28, 16, 8, 128, 3072, 151936, 1e-6, 1000000.0,
                         "default", 1.0, 1.0, 4.0, 8192.0, True, True),
    # small shapes of the same families, for fast exhaustive tests
    "tiny-llama": Config("tiny-llama", 512, 2, 8, 2, 64, 1024, 1000, 1e-5, 500000.0,
                         "llama3", 32.0, 1.0, 4.0, 8192.0, False, True),
    "tiny-llama-untied": Config("tiny-llama-untied", 512, 3, 4, 2, 128, 1536, 2048, 1e-5, 500000.0,
                                "llama3", 8.0, 1.0, 4.0, 8192.0, False, False),
    "tiny-qwen3": Config("tiny-qwen3", 256, 2, 4, 2, 128, 768, 1200, 1e-6, 1000000.0,
                         "default", 1.0, 1.0, 4.0, 8192.0, True, True),
    # small shapes the one-launch decode step takes (widths multiples of 512)
    "small-llama": Config("small-llama", 1024, 3, 16, 4, 64, 2048, 2048, 1e-5, 500000.0,
                          "llama3", 32.0, 1.0, 4.0, 8192.0, False, True),
    "small-qwen3": Config("small-qwen3", 1024, 2, 8, 2, 128, 1536, 3072, 1e-6, 1000000.0,
                          "default", 1.0, 1.0, 4.0, 8192.0, True, False),
    # q width (384) and FFN width (768) that the ring layout pads to 512 / 1024
    "small-pad": Config("small-pad", 512, 2, 6, 2, 64, 768, 1024, 1e-5, 500000.0,
                        "llama3", 32.0, 1.0, 4.0, 8192.0, False, True),
    # heads, FFN rows and vocabulary that split over 8 tensor-parallel ranks
    "tiny-tp8": Config("tiny-tp8", 512, 2, 8, 8, 64, 1024, 2048, 1e-5, 500000.0,
                       "llama3", 32.0, 1.0, 4.0, 8192.0, False, False),
}


def weight_names(cfg: Config) -> List[str]:
    """Tensor order of ``weight_names()`` (src/llama_gpu.mojo:34-49, qwen_q8.mojo:35-52);
    an untied model appends ``lm_head.weight`` (llama31_mojo/src/llama_gpu.mojo:150)."""
    names = ["model.embed_tokens.weight", "model.norm.weight"]
    for L in range(cfg.layers):
        p = f"model.layers.{L}."
        names += [p + "input_layernorm.weight", p + "post_attention_layernorm.weight"]
        if cfg.qk_norm:
            names += [p + "self_attn.q_norm.weight", p + "self_attn.k_norm.weight"]
        names += [p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight",
                  p + "self_attn.v_proj.weight", p + "self_attn.o_proj.weight",
                  p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight",
                  p + "mlp.down_proj.weight"]
    if not cfg.tied:
        names.append("lm_head.weight")
    return names


def tensor_shape(cfg: Config, name: str):
    H, QD, KVD, F = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.inter
    if name in ("model.embed_tokens.weight", "lm_head.weight"):
        return (cfg.vocab, H)
    if name == "model.norm.weight" or name.endswith("layernorm.weight"):
        return (H,)
    if name.endswith("q_norm.weight") or name.endswith("k_norm.weight"):
        return (cfg.head_dim,)
    tail = name.split(".")[-2]
    return {"q_proj": (QD, H), "k_proj": (KVD, H), "v_proj": (KVD, H), "o_proj": (H, QD),
            "gate_proj": (F, H), "up_proj": (F, H), "down_proj": (H, F)}[tail]


def make_bf16_weights(cfg: Config, seed: int = 0, std: float = 0.02, norm_std: float = 0.0):
    """Seeded synthetic checkpoint: every 2-D tensor is N(0, std) f32 from
    ``default_rng(seed)`` drawn in ``weight_names`` order, rounded to bf16 (RNE);
    norm weights are 1.0 (HF init), or 1 + N(0, norm_std) drawn in the same
    stream when ``norm_std`` > 0.  Yields (name, bf16 uint16 array)."""
    rng = np.random.default_rng(seed)
    for name in weight_names(cfg):
        shp = tensor_shape(cfg, name)
        if len(shp) == 1:
            v = np.ones(shp, np.float32)
            if norm_std > 0:
                v = v + rng.standard_normal(shp, dtype=np.float32) * np.float32(norm_std)
            yield name, bf16_round(v)
        else:
            w = rng.standard_normal(shp, dtype=np.float32) * np.float32(std)
            yield name, bf16_round(w)


def make_bf16_checkpoint(cfg: Config, seed: int = 0, std: float = 0.02,
                         norm_std: float = 0.0) -> Dict[str, np.ndarray]:
    """The synthetic checkpoint as stored for the bf16 path: every tensor bf16 bits."""
    return dict(make_bf16_weights(cfg, seed, std, norm_std))


def make_q8_checkpoint(cfg: Config, seed: int = 0, std: float = 0.02) -> Dict[str, np.ndarray]:
    """quantize.py main (qwen3_mojo/scripts/quantize.py:46-64) over the synthetic
    checkpoint: 2-D -> packed Q8 (uint16 bits of the F16-typed tensor), 1-D -> bf16 bits."""
    out = {}
    for name, w in make_bf16_weights(cfg, seed, std):
        out[name] = pack_q8(w) if w.ndim == 2 else w
    return out


def random_ids(cfg: Config, n: int, seed: int = 1) -> List[int]:
    return [int(t) for t in np.random.default_rng(seed).integers(0, cfg.vocab, size=n)]


# --------------------------------------------------------------------------- layer math

def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """scripts/gen_oracle.py:37-39."""
    v = x.astype(np.float32)
    return w * (v / np.sqrt((v * v).mean(-1, keepdims=True) + np.float32(eps)))


def inv_freq(cfg: Config) -> np.ndarray:
    """RoPE inverse frequencies, f64 math -> f32.

    default: 1/theta^(2d/hd) (src/llama_common.mojo:609-615, bench_python.py:31-35)
    llama3 : wavelength-scaled (scripts/gen_oracle.py:42-55, llama_common.mojo:618-633)
    """
    hd = cfg.head_dim
    inv = 1.0 / (cfg.theta ** (np.arange(0, hd, 2, dtype=np.float64) / hd))
    if cfg.rope_type == "default":
        return inv.astype(np.float32)
    wavelen = 2 * np.pi / inv
    smooth = (cfg.orig_ctx / wavelen - cfg.low_ff) / (cfg.high_ff - cfg.low_ff)
    scaled = np.where(wavelen < cfg.orig_ctx / cfg.high_ff, inv,
                      np.where(wavelen > cfg.orig_ctx / cfg.low_ff, inv / cfg.rope_factor,
                               (1 - smooth) * inv / cfg.rope_factor + smooth * inv))
    return scaled.astype(np.float32)


def rope(x: np.ndarray, pos0: int, inv: np.ndarray) -> np.ndarray:
    """HF rotate-half RoPE on x (s, nh, hd) at positions pos0.. (scripts/gen_oracle.py:61-69)."""
    s, hd = x.shape[0], x.shape[-1]
    t = np.arange(pos0, pos0 + s, dtype=np.float32)[:, None]
    freqs = t * inv[None, :]
    cos = np.cos(freqs)[:, None, :]
    sin = np.sin(freqs)[:, None, :]
    x0, x1 = x[..., : hd // 2], x[..., hd // 2:]
    return np.concatenate([x0 * cos - x1 * sin, x1 * cos + x0 * sin], -1)


def attention(q: np.ndarray, k_all: np.ndarray, v_all: np.ndarray, group: int) -> np.ndarray:
    """Causal GQA over the cache: q (s, nh, hd), k/v (t, nkv, hd), query i sits at
    position t - s + i (bench_python.py:77-93; max-subtracted softmax as gen_oracle.py:85-89)."""
    s, nh, hd = q.shape
    t = k_all.shape[0]
    out = np.empty((s, nh, hd), dtype=np.float32)
    mask = np.triu(np.full((s, t), -np.inf, dtype=np.float32), t - s + 1)
    for h in range(nh):
        kv = h // group
        # np.sqrt(int) is a float64 scalar: under NumPy 2 promotion the scores and
        # softmax run in f64, exactly as in the reference oracle expression.
        sc = q[:, h] @ k_all[:, kv].T / np.sqrt(hd) + mask
        sc = sc - sc.max(-1, keepdims=True)
        p = np.exp(sc)
        p /= p.sum(-1, keepdims=True)
        out[:, h] = p @ v_all[:, kv]
    return out


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """k_swiglu_mul (src/llama_common.mojo:476-481) / gen_oracle.py:94."""
    return g / (np.float32(1) + np.exp(-g)) * u


# --------------------------------------------------------------------------- model

class OracleModel:
    """f32 forward over dequantized Q8 weights with a KV cache (one sequence).

    Mirrors the reference model shell API: ``forward(ids) -> logits``,
    ``forward_argmax(ids) -> int``, ``n_cached`` (qwen3_mojo/src/qwen_q8.mojo:126-162).
    Weights are dequantized once (``q * f32(scale)``) so the matmuls are the
    reference f32 path on Q8 weights.  With ``cfg.weights == "bf16"`` every
    tensor is bf16 bits widened to f32 (the reference's bf16 shells,
    src/llama_gpu.mojo:103-155 over run_layer, src/llama_common.mojo:697-780).
    """

    def __init__(self, cfg: Config, ckpt: Dict[str, np.ndarray], maxlen: int = 1 << 30):
        self.cfg = cfg
        self.maxlen = maxlen
        self._ck = ckpt
        self._w: Dict[str, np.ndarray] = {}
        self.inv = inv_freq(cfg)
        self.k_cache: List[Optional[np.ndarray]] = [None] * cfg.layers
        self.v_cache: List[Optional[np.ndarray]] = [None] * cfg.layers
        self.n_cached = 0
        self.trace: Dict[str, np.ndarray] = {}

    def W(self, name: str) -> np.ndarray:
        if name not in self._w:
            a = self._ck[name]
            shp = tensor_shape(self.cfg, name)
            if len(shp) == 1 or self.cfg.weights == "bf16":
                self._w[name] = bf16_to_f32(a).reshape(shp)
            else:
                self._w[name] = dequant_q8(a, shp[1])
        return self._w[name]

    def reset(self):
        self.k_cache = [None] * self.cfg.layers
        self.v_cache = [None] * self.cfg.layers
        self.n_cached = 0

    def layer(self, x: np.ndarray, L: int, pos: int) -> np.ndarray:
        """One pre-norm GQA block (bench_python.py:96-119, gen_oracle.py:72-95)."""
        c = self.cfg
        p = f"model.layers.{L}."
        s = x.shape[0]
        xn = rmsnorm(x, self.W(p + "input_layernorm.weight"), c.eps)
        q = (xn @ self.W(p + "self_attn.q_proj.weight").T).reshape(s, c.n_heads, c.head_dim)
        k = (xn @ self.W(p + "self_attn.k_proj.weight").T).reshape(s, c.n_kv, c.head_dim)
        v = (xn @ self.W(p + "self_attn.v_proj.weight").T).reshape(s, c.n_kv, c.head_dim)
        if c.qk_norm:
            q = rmsnorm(q, self.W(p + "self_attn.q_norm.weight"), c.eps)
            k = rmsnorm(k, self.W(p + "self_attn.k_norm.weight"), c.eps)
        q, k = rope(q, pos, self.inv), rope(k, pos, self.inv)
        if self.k_cache[L] is None:
            self.k_cache[L], self.v_cache[L] = k, v
        else:
            self.k_cache[L] = np.concatenate([self.k_cache[L], k], 0)
            self.v_cache[L] = np.concatenate([self.v_cache[L], v], 0)
        out = attention(q, self.k_cache[L], self.v_cache[L], c.group)
        x = x + out.reshape(s, c.q_dim) @ self.W(p + "self_attn.o_proj.weight").T
        xn = rmsnorm(x, self.W(p + "post_attention_layernorm.weight"), c.eps)
        g = xn @ self.W(p + "mlp.gate_proj.weight").T
        u = xn @ self.W(p + "mlp.up_proj.weight").T
        return x + silu_mul(g, u) @ self.W(p + "mlp.down_proj.weight").T

    def forward_hidden(self, ids) -> np.ndarray:
        c = self.cfg
        s = len(ids)
        if self.n_cached + s > self.maxlen:
            raise RuntimeError("KV cache full")  # qwen_q8.mojo:128-129
        if c.weights == "bf16":  # k_embed_gather (src/llama_common.mojo:183-194)
            x = bf16_to_f32(np.asarray(self._ck["model.embed_tokens.weight"])[np.asarray(ids, np.int64)])
        else:
            x = embed_q8(self._ck["model.embed_tokens.weight"], c.hidden, ids)
        pos = self.n_cached
        for L in range(c.layers):
            x = self.layer(x, L, pos)
            self.trace[f"after_layer{L}"] = x
        self.n_cached += s
        return x

    def forward(self, ids) -> np.ndarray:
        """Logits of the last token (qwen_q8.mojo:126-156)."""
        x = self.forward_hidden(ids)
        h = rmsnorm(x[-1:], self.W("model.norm.weight"), self.cfg.eps)
        head = "model.embed_tokens.weight" if self.cfg.tied else "lm_head.weight"
        return (h @ self.W(head).T)[0]

    def forward_argmax(self, ids) -> int:
        return int(np.argmax(self.forward(ids)))


def greedy_generate(model: OracleModel, prompt, steps: int):
    """Prefill + ``steps`` greedy decode steps; returns (tokens, top2 margins, logits list)."""
    logits = model.forward(prompt)
    toks, margins, all_logits = [], [], [logits]
    for i in range(steps + 1):
        top2 = np.partition(logits, -2)[-2:]
        margins.append(float(top2[1] - top2[0]))
        t = int(np.argmax(logits))
        toks.append(t)
        if i == steps:
            break
        logits = model.forward([t])
        all_logits.append(logits)
    return toks, margins, all_logits


def sample_literal(logits, temp: float, top_p: float, u: float) -> int:
    """sample() of src/sample.mojo:15-59 in float32 scalar steps, loop for loop
    (pure Python: small rows only); u is the uniform draw the reference takes
    from random_float64() (:55)."""
    x = [np.float32(v) for v in np.asarray(logits, np.float32).ravel()]

    def argmax(v):  # :7-12, first maximum
        best = 0
        for i in range(1, len(v)):
            if v[i] > v[best]:
                best = i
        return best

    if temp <= 0:
        return argmax(x)
    t = np.float32(temp)
    mx = x[argmax(x)]
    cutoff = np.float32(mx - np.float32(16.0))
    cand_idx, cand_p = [], []
    total = np.float32(0.0)
    for i, v in enumerate(x):
        if v < cutoff:
            continue
        p = np.float32(np.exp(np.float32(np.float32(v - mx) / t)))
        cand_idx.append(i)
        cand_p.append(p)
        total = np.float32(total + p)
    if not cand_idx:
        return argmax(x)
    target = np.float32(total * np.float32(top_p))
    nuc_idx, nuc_p = [], []
    cum = np.float32(0.0)
    while cum < target and cand_idx:
        b = 0
        for i in range(1, len(cand_p)):
            if cand_p[i] > cand_p[b]:
                b = i
        cum = np.float32(cum + cand_p[b])
        nuc_idx.append(cand_idx[b])
        nuc_p.append(cand_p[b])
        cand_idx[b] = cand_idx[-1]
        cand_p[b] = cand_p[-1]
        cand_idx.pop()
        cand_p.pop()
    r = np.float32(np.float32(u) * cum)
    acc = np.float32(0.0)
    for i in range(len(nuc_idx)):
        acc = np.float32(acc + nuc_p[i])
        if r <= acc:
            return nuc_idx[i]
    return nuc_idx[-1]


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def decode_step_bytes(cfg: Config, batch: int, ctx: int, kv_bytes: int = 4, tp: int = 1) -> int:
    """Algorithmic HBM bytes of one decode step per GPU: every Q8 weight byte once
    (codes + f16 scales) plus the KV cache read for ``ctx`` positions per sequence."""
    H, QD, KVD, F = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.inter
    per_layer = (QD + 2 * KVD) * H + H * QD + 2 * F * H + H * F
    head = cfg.vocab * H
    w = (per_layer * cfg.layers + head) * (1 + 2 / QG) / tp
    kv = batch * ctx * cfg.layers * 2 * (KVD // tp) * kv_bytes
    return int(w + kv)


def q8_param_count(cfg: Config) -> int:
    H, QD, KVD, F = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.inter
    per_layer = (QD + 2 * KVD) * H + H * QD + 2 * F * H + H * F
    return per_layer * cfg.layers + cfg.vocab * H


def _selftest():  # pragma: no cover - manual sanity
    cfg = PRESETS["tiny-llama"]
    ck = make_q8_checkpoint(cfg)
    m = OracleModel(cfg, ck)
    toks, margins, _ = greedy_generate(m, random_ids(cfg, 8), 4)
    print(toks, [round(x, 4) for x in margins], math.isfinite(sum(margins)))


if __name__ == "__main__":
    _selftest()
