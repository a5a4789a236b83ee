"""Model configurations of the Q8 path.

``Config`` mirrors the reference's ``Config`` struct (src/llama_common.mojo:26-52)
and the family switches its shells hard-code: Qwen3 per-head QK-norm
(``LayerOffs.q_norm >= 0``, src/llama_q8.mojo:171) and tied vs untied lm_head
(qwen3_mojo/src/qwen_q8.mojo:143-145, llama31_mojo/src/llama_gpu.mojo:150).
Presets carry the dimensions of the models in the benchmark configurations.
"""
from __future__ import annotations

import dataclasses
import json
import os
from typing import Dict, List

from . import _lib


@dataclasses.dataclass(frozen=True)
class Config:
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
    rope_type: str = "llama3"
    rope_factor: float = 1.0
    low_ff: float = 1.0
    high_ff: float = 4.0
    orig_ctx: float = 8192.0
    qk_norm: bool = False
    tied: bool = True
    # "q8": packed Q8 matrices (the default); "bf16": the reference's non-Q8
    # path (run_layer / mm_op, src/llama_common.mojo:636-780), weights kept bf16
    weights: str = "q8"

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv * self.head_dim

    def replace(self, **kw) -> "Config":
        return dataclasses.replace(self, **kw)

    def to_c(self) -> _lib.q8_config:
        return _lib.q8_config(
            self.hidden, self.layers, self.n_heads, self.n_kv, self.head_dim, self.inter, self.vocab,
            self.eps, self.theta, self.rope_factor, self.low_ff, self.high_ff, self.orig_ctx,
            _lib.Q8_ROPE_LLAMA3 if self.rope_type == "llama3" else _lib.Q8_ROPE_DEFAULT,
            int(self.qk_norm), int(self.tied),
            _lib.Q8_BF16 if self.weights == "bf16" else _lib.Q8_PACKED)

    def weight_names(self) -> List[str]:
        """Tensor names the model loads (src/llama_gpu.mojo:34-49, qwen_q8.mojo:35-52)."""
        names = ["model.embed_tokens.weight", "model.norm.weight"]
        for L in range(self.layers):
            p = f"model.layers.{L}."
            names += [p + "input_layernorm.weight", p + "post_attention_layernorm.weight"]
            if self.qk_norm:
                names += [p + "self_attn.q_norm.weight", p + "self_attn.k_norm.weight"]
            names += [p + s for s in ("self_attn.q_proj.weight", "self_attn.k_proj.weight",
                                      "self_attn.v_proj.weight", "self_attn.o_proj.weight",
                                      "mlp.gate_proj.weight", "mlp.up_proj.weight",
                                      "mlp.down_proj.weight")]
        if not self.tied:
            names.append("lm_head.weight")
        return names

    def tensor_shape(self, name: str):
        H, QD, KVD, F = self.hidden, self.q_dim, self.kv_dim, self.inter
        if name in ("model.embed_tokens.weight", "lm_head.weight"):
            return (self.vocab, H)
        if name == "model.norm.weight" or name.endswith("layernorm.weight"):
            return (H,)
        if name.endswith("q_norm.weight") or name.endswith("k_norm.weight"):
            return (self.head_dim,)
        tail = name.split(".")[-2]
        return {"q_proj": (QD, H), "k_proj": (KVD, H), "v_proj": (KVD, H), "o_proj": (H, QD),
                "gate_proj": (F, H), "up_proj": (F, H), "down_proj": (H, F)}[tail]

    def q8_params(self) -> int:
        """Weights streamed per decode step: all linear layers + the lm_head
        (the embedding gather touches only the looked-up rows)."""
        H, QD, KVD, F = self.hidden, self.q_dim, self.kv_dim, self.inter
        per_layer = (QD + 2 * KVD) * H + H * QD + 2 * F * H + H * F
        return per_layer * self.layers + self.vocab * H

    def decode_bytes(self, batch: int, ctx: int, tp: int = 1, kv_bytes: int = 4) -> float:
        """Algorithmic HBM bytes of one decode step per GPU: every weight byte
        once (Q8: int8 codes + f16 group scales; bf16: 2 bytes) plus the KV read
        of ``ctx`` positions."""
        H, QD, KVD, F = self.hidden, self.q_dim, self.kv_dim, self.inter
        per_layer = (QD + 2 * KVD) * H + H * QD + 2 * F * H + H * F
        wb = 2.0 if self.weights == "bf16" else 1 + 2 / 64
        w = (per_layer * self.layers + self.vocab * H) * wb / tp
        kv = batch * ctx * self.layers * 2 * (KVD / tp) * kv_bytes
        return w + kv


PRESETS: Dict[str, Config] = {
    "llama-3.2-1b": Config("llama-3.2-1b", 2048, 16, 32, 8, 64, 8192, 128256, 1e-5, 500000.0,
                           "llama3", 32.0, 1.0, 4.0, 8192.0, False, True),
    "llama-3.2-3b": Config("llama-3.2-3b", 3072, 28, 24, 8, 128, 8192, 128256, 1e-5, 500000.0,
                           "llama3", 32.0, 1.0, 4.0, 8192.0, False, True),
    "llama-3.1-8b": Config("llama-3.1-8b", 4096, 32, 32, 8, 128, 14336, 128256, 1e-5, 500000.0,
                           "llama3", 8.0, 1.0, 4.0, 8192.0, False, False),
    "qwen3-8b": Config("qwen3-8b", 4096, 36, 32, 8, 128, 12288, 151936, 1e-6, 1000000.0,
                       "default", 1.0, 1.0, 4.0, 8192.0, True, False),
    "qwen3-0.6b": Config("qwen3-0.6b", 1024, 28, 16, 8, 128, 3072, 151936, 1e-6, 1000000.0,
                         "default", 1.0, 1.0, 4.0, 8192.0, True, True),
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


def from_hf_config(path: str, name: str = "hf") -> Config:
    """Config from a HuggingFace config.json (Llama / Qwen3 families)."""
    with open(path) as f:
        j = json.load(f)
    rs = j.get("rope_scaling") or {}
    llama3 = rs.get("rope_type", rs.get("type")) == "llama3"
    hd = j.get("head_dim") or j["hidden_size"] // j["num_attention_heads"]
    return Config(name, j["hidden_size"], j["num_hidden_layers"], j["num_attention_heads"],
                  j.get("num_key_value_heads", j["num_attention_heads"]), hd, j["intermediate_size"],
                  j["vocab_size"], float(j["rms_norm_eps"]), float(j.get("rope_theta", 10000.0)),
                  "llama3" if llama3 else "default", float(rs.get("factor", 1.0)),
                  float(rs.get("low_freq_factor", 1.0)), float(rs.get("high_freq_factor", 4.0)),
                  float(rs.get("original_max_position_embeddings", 8192)),
                  j.get("model_type") == "qwen3", bool(j.get("tie_word_embeddings", False)))


def from_model_dir(model_dir: str) -> Config:
    return from_hf_config(os.path.join(model_dir, "config.json"), os.path.basename(model_dir.rstrip("/")))
