"""ctypes wrapper of the C restatement (oracle/q8_ref.c) — TEST INFRASTRUCTURE.

Used as a second checker (the reference's exact k_mm_q8 accumulation order)
and as the timed CPU baseline / reference arm of bench.py.  Built by
``make -C oracle`` into ``oracle/_build/libq8ref.so``.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SO = os.path.join(HERE, "_build", "libq8ref.so")
_lib = None


class LayerW(C.Structure):
    _fields_ = [("qkv", C.c_void_p), ("o", C.c_void_p), ("gu", C.c_void_p), ("down", C.c_void_p),
                ("in_norm", C.c_void_p), ("post_norm", C.c_void_p), ("q_norm", C.c_void_p),
                ("k_norm", C.c_void_p)]


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True, capture_output=True)
    return SO


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(SO) or os.path.getmtime(SO) < os.path.getmtime(os.path.join(HERE, "q8_ref.c")):
            build()
        L = C.CDLL(SO)
        P, I, F = C.c_void_p, C.c_int, C.c_float
        L.q8r_threads.restype = I
        L.q8r_set_threads.argtypes = [I]
        L.q8r_gemv.argtypes = [P, I, I, P, I, P]
        L.q8r_embed.argtypes = [P, I, P, I, P]
        L.q8r_rmsnorm.argtypes = [P, P, I, I, F, P]
        L.q8r_attend.argtypes = [P, P, P, I, I, I, I, P]
        L.q8r_swiglu.argtypes = [P, P, I]
        L.q8r_argmax.argtypes = [P, I]
        L.q8r_argmax.restype = I
        L.q8r_sample.argtypes = [P, I, F, F, F, C.POINTER(C.c_double)]
        L.q8r_sample.restype = I
        L.q8r_layer.argtypes = [C.POINTER(LayerW), P, I, I, I, I, I, F, I, P, P, P, P]
        _lib = L
    return _lib


def _p(a):
    return C.c_void_p(a.ctypes.data) if a is not None else None


def gemv(x: np.ndarray, packed: np.ndarray, m: int) -> np.ndarray:
    """y = x . W^T in the reference k_mm_q8 accumulation order."""
    x = np.ascontiguousarray(x, np.float32)
    packed = np.ascontiguousarray(packed)
    n = packed.shape[0]
    y = np.empty((x.shape[0], n), np.float32)
    lib().q8r_gemv(_p(x), x.shape[0], m, _p(packed), n, _p(y))
    return y


def sample(logits: np.ndarray, temp: float, top_p: float, u: float):
    """Token of sample() (src/sample.mojo:15-59) for one logits row and the
    uniform draw u, with the decision margin (see q8r_sample)."""
    x = np.ascontiguousarray(logits, np.float32).ravel()
    mg = C.c_double()
    tok = lib().q8r_sample(_p(x), x.size, float(temp), float(top_p), float(np.float32(u)), C.byref(mg))
    return int(tok), float(mg.value)


def _rand_packed(rng, n, m):
    """Random packed rows: f16 scales ~ 0.02*2.5/127 and uniform int8 codes in
    [-127, 127] (random bytes, -128 moved to -127 as the quantizer never
    writes it)."""
    sc = (np.full((n, m // 64), 0.02 * 2.5 / 127, np.float32)).astype(np.float16).view(np.uint16)
    out = np.empty((n, m // 32 + m), np.uint8)
    out[:, : m // 32] = sc.view(np.uint8).reshape(n, m // 32)
    q = np.frombuffer(rng.bytes(n * m), np.int8).reshape(n, m)
    out[:, m // 32:] = np.maximum(q, np.int8(-127)).view(np.uint8)
    return out


def time_decode_sample(cfg, batch: int, ctx: int, sample_layers: int = 0, steps: int = 2, seed: int = 0):
    """Time the CPU port of decode steps: ``sample_layers`` full-width layers
    (0: every layer of the model; the reference's run_layer_q8 for one token)
    plus the final norm + lm_head GEMV + argmax, with a ``ctx``-long f32 KV
    cache.  With fewer layers than the model the step time is layers_time *
    (cfg.layers / sample_layers) + head_time; batch B is B single-sequence
    decodes (the reference decodes one sequence).  Returns tok/s and the
    sample description."""
    L = lib()
    rng = np.random.default_rng(seed)
    H, QD, KVD, F, hd = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.inter, cfg.head_dim
    ls = cfg.layers if sample_layers <= 0 else max(1, min(sample_layers, cfg.layers))
    ones = np.full(H, 0x3F80, np.uint16)
    hones = np.full(hd, 0x3F80, np.uint16)
    keep = []
    layers = []
    for _ in range(ls):
        w = dict(qkv=_rand_packed(rng, QD + 2 * KVD, H), o=_rand_packed(rng, H, QD),
                 gu=_rand_packed(rng, 2 * F, H), down=_rand_packed(rng, H, F))
        keep.append(w)
        layers.append(LayerW(w["qkv"].ctypes.data, w["o"].ctypes.data, w["gu"].ctypes.data,
                             w["down"].ctypes.data, ones.ctypes.data, ones.ctypes.data,
                             hones.ctypes.data if cfg.qk_norm else None,
                             hones.ctypes.data if cfg.qk_norm else None))
    head = _rand_packed(rng, cfg.vocab, H)
    kc = [rng.standard_normal((ctx + steps + 1, KVD)).astype(np.float32) for _ in range(ls)]
    vc = [rng.standard_normal((ctx + steps + 1, KVD)).astype(np.float32) for _ in range(ls)]
    inv = (1.0 / (cfg.theta ** (np.arange(0, hd, 2) / hd))).astype(np.float32)
    scratch = np.zeros(2 * H + 2 * QD + 2 * KVD + 2 * F + 64, np.float32)
    logits = np.zeros(cfg.vocab, np.float32)
    xn = np.zeros(H, np.float32)
    t_layers = t_head = 0.0
    nrun = 0
    for s in range(steps + 1):  # first step is warm-up
        for b in range(batch):
            h = rng.standard_normal(H).astype(np.float32)
            t0 = time.perf_counter()
            for li in range(ls):
                L.q8r_layer(C.byref(layers[li]), _p(h), H, cfg.n_heads, cfg.n_kv, hd, F, cfg.eps, ctx + s,
                            _p(inv), _p(kc[li]), _p(vc[li]), _p(scratch))
            t1 = time.perf_counter()
            L.q8r_rmsnorm(_p(h), _p(ones), 1, H, cfg.eps, _p(xn))
            L.q8r_gemv(_p(xn), 1, H, _p(head), cfg.vocab, _p(logits))
            L.q8r_argmax(_p(logits), cfg.vocab)
            t2 = time.perf_counter()
            if s > 0:
                t_layers += t1 - t0
                t_head += t2 - t1
                nrun += 1
    per_tok = (t_layers / nrun) * (cfg.layers / ls) + t_head / nrun
    return {"tok_s": 1.0 / per_tok, "ms_per_step": per_tok * batch * 1e3, "threads": L.q8r_threads(),
            "steps": steps,
            "sample": (f"full {cfg.layers}-layer decode step + lm_head per token at ctx {ctx}, "
                       f"{steps} timed steps x batch {batch} (random packed weights, one warm-up step)"
                       if ls == cfg.layers else
                       f"{ls} of {cfg.layers} full-width layers + lm_head per token at ctx {ctx}, "
                       f"{steps} timed steps x batch {batch}; layer time scaled by {cfg.layers}/{ls}")}


class RefModel:
    """Whole-model forward on the C restatement (q8r_embed, q8r_layer,
    q8r_rmsnorm, q8r_gemv): the reference model shell's loop
    (qwen3_mojo/src/qwen_q8.mojo:126-162) one token at a time, each token
    through run_layer_q8 at s == 1 (src/llama_q8.mojo:144-230) with an f32 KV
    cache per layer, then the final norm and the Q8 lm_head
    (qwen_q8.mojo:141-156).  The checker of the full-size parity tests: all
    host threads, int8 codes read directly, no dequantized copy of the
    weights.  ``tensors`` maps checkpoint names to packed rows (uint8 or the
    uint16 bits of quantize.py's F16 tensor) for 2-D weights and bf16 bits for
    norm vectors; ``inv`` is the RoPE inverse-frequency table."""

    def __init__(self, cfg, tensors, inv, maxlen: int):
        self.cfg = cfg
        L = lib()
        self._L = L
        H, QD, KVD, F = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.inter
        u8 = lambda a: np.ascontiguousarray(a).view(np.uint8)
        u16 = lambda a: np.ascontiguousarray(a).view(np.uint16)
        self._keep = []
        self.layers = []
        for i in range(cfg.layers):
            p = f"model.layers.{i}."
            qkv = np.concatenate([u8(tensors[p + f"self_attn.{n}_proj.weight"]) for n in "qkv"], 0)
            gu = np.concatenate([u8(tensors[p + f"mlp.{n}_proj.weight"]) for n in ("gate", "up")], 0)
            o, down = u8(tensors[p + "self_attn.o_proj.weight"]), u8(tensors[p + "mlp.down_proj.weight"])
            inn, post = u16(tensors[p + "input_layernorm.weight"]), u16(tensors[p + "post_attention_layernorm.weight"])
            qn = u16(tensors[p + "self_attn.q_norm.weight"]) if cfg.qk_norm else None
            kn = u16(tensors[p + "self_attn.k_norm.weight"]) if cfg.qk_norm else None
            self._keep += [qkv, gu, o, down, inn, post, qn, kn]
            self.layers.append(LayerW(qkv.ctypes.data, o.ctypes.data, gu.ctypes.data, down.ctypes.data,
                                      inn.ctypes.data, post.ctypes.data,
                                      qn.ctypes.data if qn is not None else None,
                                      kn.ctypes.data if kn is not None else None))
        self.embed = u8(tensors["model.embed_tokens.weight"])
        self.head = self.embed if cfg.tied else u8(tensors["lm_head.weight"])
        self.fnorm = u16(tensors["model.norm.weight"])
        self.inv = np.ascontiguousarray(inv, np.float32)
        self.maxlen = maxlen
        self.kc = [np.zeros((maxlen, KVD), np.float32) for _ in range(cfg.layers)]
        self.vc = [np.zeros((maxlen, KVD), np.float32) for _ in range(cfg.layers)]
        self.scratch = np.zeros(2 * H + 2 * QD + 2 * KVD + 2 * F + 64, np.float32)
        self.n_cached = 0

    def token(self, tok: int, keep=(), logits: bool = True):
        """Logits after one token at position n_cached (None when ``logits``
        is False); ``keep`` lists layers whose output residual is returned too
        ({layer: h})."""
        c, L = self.cfg, self._L
        if self.n_cached >= self.maxlen:
            raise RuntimeError("KV cache full")
        h = np.zeros(c.hidden, np.float32)
        ids = np.array([tok], np.int32)
        L.q8r_embed(_p(self.embed), c.hidden, _p(ids), 1, _p(h))
        kept = {}
        for i in range(c.layers):
            L.q8r_layer(C.byref(self.layers[i]), _p(h), c.hidden, c.n_heads, c.n_kv, c.head_dim, c.inter, c.eps,
                        self.n_cached, _p(self.inv), _p(self.kc[i]), _p(self.vc[i]), _p(self.scratch))
            if i in keep:
                kept[i] = h.copy()
        self.n_cached += 1
        if not logits:
            return (None, kept) if keep else None
        xn = np.zeros(c.hidden, np.float32)
        L.q8r_rmsnorm(_p(h), _p(self.fnorm), 1, c.hidden, c.eps, _p(xn))
        logits = np.zeros(self.head.shape[0], np.float32)
        L.q8r_gemv(_p(xn), 1, c.hidden, _p(self.head), self.head.shape[0], _p(logits))
        return (logits, kept) if keep else logits

    def prefill(self, ids, keep=()):
        """Logits of the last token and {layer: [len(ids), H]} residuals."""
        rows = {i: [] for i in keep}
        lg = None
        for n, t in enumerate(ids):
            lg, kept = self.token(int(t), keep=tuple(keep) or (-1,), logits=n == len(ids) - 1)
            for i in keep:
                rows[i].append(kept[i])
        return lg, {i: np.stack(v) for i, v in rows.items()}
