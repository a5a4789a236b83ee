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
    """Random packed rows: f16 scales ~ 0.02*2.5/127 and uniform int8 codes."""
    sc = (np.full((n, m // 64), 0.02 * 2.5 / 127, np.float32)).astype(np.float16).view(np.uint16)
    q = rng.integers(-127, 128, size=(n, m), dtype=np.int8).view(np.uint8)
    out = np.empty((n, m // 32 + m), np.uint8)
    out[:, : m // 32] = sc.view(np.uint8).reshape(n, m // 32)
    out[:, m // 32:] = q
    return out


def time_decode_sample(cfg, batch: int, ctx: int, sample_layers: int = 2, steps: int = 2, seed: int = 0):
    """Time the CPU port of one decode step on a bounded sample: ``sample_layers``
    full-width layers (the reference's run_layer_q8 for one token) plus the
    final norm + lm_head GEMV + argmax, with a ``ctx``-long f32 KV cache.  The
    full-model step time is layers_time * (cfg.layers / sample_layers) +
    head_time; batch B is B single-sequence decodes (the reference decodes one
    sequence).  Returns tok/s and the sample description."""
    L = lib()
    rng = np.random.default_rng(seed)
    H, QD, KVD, F, hd = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.inter, cfg.head_dim
    ls = max(1, min(sample_layers, cfg.layers))
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
            "sample": f"{ls} of {cfg.layers} full-width layers + lm_head per token at ctx {ctx}, "
                      f"{steps} timed steps x batch {batch}; layer time scaled by {cfg.layers}/{ls}"}
