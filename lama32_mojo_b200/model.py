"""Model-level host API — the B200 counterpart of the reference Q8 model shells.

``Q8Model`` keeps the reference's API (qwen3_mojo/src/qwen_q8.mojo:55-177,
src/llama_gpu.mojo:52-170): ``forward(ids) -> logits`` of the last token,
``forward_argmax(ids) -> int``, and the read/write ``n_cached`` counter; loading
is ``load_q8(model_dir, maxlen)`` (``load_qwen_q8`` / ``load_llama``).  It adds
multi-sequence decode (``decode``), on-device generation (``generate``), device
sampling (``set_sampling``, the chat REPLs' ``sample``) and tensor parallelism
(``tp_rank``/``tp_size``).  All compute
runs in libq8cuda.so; errors raise ``Q8Error`` (``KVCacheFull`` for the
reference's "KV cache full").
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import numpy as np

from . import _lib
from ._lib import check, lib
from .config import Config, from_model_dir


_M64 = (1 << 64) - 1


def sample_draw(seed: int, seq: int, pos: int) -> np.float32:
    """The uniform draw the library uses when sampling the row of sequence
    ``seq`` whose fed token sits at position ``pos`` (q8_set_sampling)."""
    key = ((seq & 0xFFFFFFFF) << 32) | (pos & 0xFFFFFFFF)
    z = (seed + (key + 1) * 0x9E3779B97F4A7C15) & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    z ^= z >> 31
    return np.float32((z >> 40) / 16777216.0)


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


class Q8Model:
    def __init__(self, cfg: Config, device: int = 0, maxlen: int = 2048, max_seqs: int = 1,
                 max_tokens: int = 2048, tp_rank: int = 0, tp_size: int = 1, nccl_id: Optional[bytes] = None):
        self.cfg = cfg
        self.device = device
        self.maxlen = maxlen
        self.max_seqs = max_seqs
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self._c = cfg.to_c()
        ctx = C.c_void_p()
        idbuf = C.create_string_buffer(bytes(nccl_id), 128) if nccl_id is not None else None
        check(lib().q8_create(C.byref(self._c), device, max_seqs, maxlen, max_tokens, tp_rank, tp_size,
                              C.cast(idbuf, C.c_void_p) if idbuf is not None else None, C.byref(ctx)))
        self._ctx = ctx

    # ------------------------------------------------------------------ lifetime
    def close(self):
        if getattr(self, "_ctx", None):
            lib().q8_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def _check(self, s):
        check(s, self._ctx)

    # ------------------------------------------------------------------ weights
    def load_tensor(self, name: str, data, packed: bool, on_device: bool = False, shape=None):
        """Upload one tensor.  ``data``: numpy array or torch tensor; ``packed``:
        True for Q8-packed rows (uint16/int16/f16 [n, m/64+m/2]), False for bf16."""
        if shape is None:
            shape = self.cfg.tensor_shape(name)
        rows = shape[0]
        cols = shape[1] if len(shape) > 1 else 1
        if hasattr(data, "data_ptr"):
            ptr = data.data_ptr()
            on_device = data.is_cuda
            keep = data
        else:
            keep = np.ascontiguousarray(data)
            ptr = keep.ctypes.data
        dtype = _lib.Q8_PACKED if packed else _lib.Q8_BF16
        self._check(lib().q8_load_tensor(self._ctx, name.encode(), dtype, rows, cols, C.c_void_p(ptr),
                                         int(on_device)))
        del keep

    def load_safetensors(self, model_dir: str):
        """SafeTensors + Weights.upload_all (src/safetensors.mojo:40-96, src/resident.mojo:30-60)."""
        self._check(lib().q8_load_safetensors(self._ctx, model_dir.encode()))

    # ------------------------------------------------------------------ reference API
    def forward(self, ids: Sequence[int], seq: int = 0) -> np.ndarray:
        """Logits of the last token (QwenQ8.forward, qwen_q8.mojo:154-156)."""
        ids = _i32(ids)
        out = np.empty(self.cfg.vocab, np.float32)
        self._check(lib().q8_forward(self._ctx, ids.ctypes.data, len(ids), seq, out.ctypes.data, None))
        return out

    def forward_argmax(self, ids: Sequence[int], seq: int = 0) -> int:
        """Greedy next token (QwenQ8.forward_argmax, qwen_q8.mojo:158-162)."""
        ids = _i32(ids)
        am = np.zeros(1, np.int32)
        self._check(lib().q8_forward(self._ctx, ids.ctypes.data, len(ids), seq, None, am.ctypes.data))
        return int(am[0])

    def forward_hidden(self, ids: Sequence[int], layer: int, seq: int = 0) -> np.ndarray:
        """Residual stream after ``layer`` for a prefill of ``ids`` at the current
        position (the oracle's after_layer{L}); does not advance n_cached."""
        ids = _i32(ids)
        out = np.empty((len(ids), self.cfg.hidden), np.float32)
        self._check(lib().q8_forward_hidden(self._ctx, ids.ctypes.data, len(ids), seq, layer, out.ctypes.data))
        return out

    def get_n_cached(self, seq: int = 0) -> int:
        v = C.c_int()
        self._check(lib().q8_n_cached(self._ctx, seq, C.byref(v)))
        return v.value

    def set_n_cached(self, n: int, seq: int = 0):
        if n == 0:
            self._check(lib().q8_reset(self._ctx, seq))
        else:
            self._check(lib().q8_set_n_cached(self._ctx, seq, n))

    n_cached = property(lambda self: self.get_n_cached(0), lambda self, n: self.set_n_cached(n, 0))

    def reset(self, seq: int = 0):
        self._check(lib().q8_reset(self._ctx, seq))

    def set_sampling(self, temp: float, top_p: float = 1.0, seed: int = 0):
        """Sample every picked token (temperature + nucleus, src/sample.mojo:15-59)
        on the device; temp <= 0 restores greedy argmax.  Draws: sample_draw()."""
        self._check(lib().q8_set_sampling(self._ctx, float(temp), float(top_p), int(seed) & (2**64 - 1)))

    # ------------------------------------------------------------------ batched / on-device
    def decode(self, ids: Sequence[int], seqs: Sequence[int], logits: bool = False):
        """One token for each of B sequences.  Returns argmax [B] (and logits [B, V])."""
        ids, seqs = _i32(ids), _i32(seqs)
        B = len(ids)
        am = np.zeros(B, np.int32)
        lg = np.empty((B, self.cfg.vocab), np.float32) if logits else None
        self._check(lib().q8_decode(self._ctx, ids.ctypes.data, seqs.ctypes.data, B,
                                    lg.ctypes.data if logits else None, am.ctypes.data))
        return (am, lg) if logits else am

    def generate(self, first_ids: Sequence[int], seqs: Sequence[int], steps: int) -> np.ndarray:
        """``steps`` greedy decode steps on the device; returns tokens [steps, B]."""
        first, seqs = _i32(first_ids), _i32(seqs)
        B = len(first)
        out = np.zeros((steps, B), np.int32)
        self._check(lib().q8_generate(self._ctx, first.ctypes.data, seqs.ctypes.data, B, steps, out.ctypes.data))
        return out

    def chat_generate(self, ids: Sequence[int], temp: float = 0.0, top_p: float = 1.0, eos: int = -1,
                      seed: int = 0, max_new: Optional[int] = None, seq: int = 0) -> list:
        """One assistant turn of the chat REPLs' generate() (qwen3_mojo/src/chat_q8.mojo:53-97,
        src/chat.mojo): prefill ``ids`` after the cached context, then one token per
        forward until ``eos`` or a full context (n_cached == maxlen), each token
        picked on the device (greedy for temp <= 0, else sample() with ``top_p``
        and draws from ``seed``).  Returns the tokens produced; ``eos`` is not
        included.  ``max_new`` optionally caps the count."""
        self.set_sampling(temp, top_p, seed)
        out = []
        nxt = self.forward_argmax(ids, seq)
        while self.get_n_cached(seq) < self.maxlen:
            if nxt == eos or (max_new is not None and len(out) >= max_new):
                break
            out.append(nxt)
            nxt = self.forward_argmax([nxt], seq)
        return out

    @property
    def stream(self) -> int:
        p = C.c_void_p()
        self._check(lib().q8_stream(self._ctx, C.byref(p)))
        return p.value or 0

    def set_profiling(self, on: bool):
        self._check(lib().q8_set_profiling(self._ctx, int(on)))

    def profile(self):
        """Per kernel class of the last step run with profiling on:
        {name: (ms, algorithmic bytes, launches)}."""
        cap = 64
        names = (C.c_char_p * cap)()
        ms = (C.c_double * cap)()
        by = (C.c_double * cap)()
        ln = (C.c_int * cap)()
        n = C.c_int()
        self._check(lib().q8_profile(self._ctx, cap, names, ms, by, ln, C.byref(n)))
        return {names[i].decode(): (ms[i], by[i], ln[i]) for i in range(n.value)}


def shard_plan(cfg: Config, tp_rank: int, tp_size: int, name: str) -> dict:
    """Tensor-parallel placement the loader applies to ``name`` (host-only)."""
    v = [C.c_int64() for _ in range(7)]
    slot = C.create_string_buffer(32)
    c = cfg.to_c()
    check(lib().q8_shard_plan(C.byref(c), tp_rank, tp_size, name.encode(), *[C.byref(x) for x in v], slot, 32))
    keys = ["n", "m", "row0", "nrows", "k0", "kl", "dst_row"]
    d = {k: x.value for k, x in zip(keys, v)}
    d["slot"] = slot.value.decode()
    return d


def inspect_checkpoint(model_dir: str) -> list:
    """Host-only safetensors scan: [(name, dtype, shape, begin, end)]."""
    cap = 1 << 22
    buf = C.create_string_buffer(cap)
    n = C.c_int()
    check(lib().q8_inspect_checkpoint(model_dir.encode(), buf, cap, C.byref(n)))
    out = []
    for line in buf.value.decode().splitlines():
        name, dt, shp, b, e = line.split(" ")
        out.append((name, dt, tuple(int(x) for x in shp.split(",")) if shp else (), int(b), int(e)))
    return out


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    check(lib().q8_nccl_unique_id(C.cast(buf, C.c_void_p)))
    return buf.raw


def load_q8(model_dir: str, maxlen: int, device: int = 0, cfg: Optional[Config] = None, **kw) -> Q8Model:
    """load_qwen_q8 / load_llama (qwen3_mojo/src/qwen_q8.mojo:165-177, src/llama_gpu.mojo:158-170):
    config.json + (packed Q8 or bf16) safetensors -> resident model."""
    cfg = cfg or from_model_dir(model_dir)
    m = Q8Model(cfg, device=device, maxlen=maxlen, **kw)
    m.load_safetensors(model_dir)
    return m


def load_synthetic(cfg: Config, device: int = 0, seed: int = 0, std: float = 0.02, **kw) -> Q8Model:
    """Random-init model: every 2-D tensor N(0, std) generated in bf16 on the GPU
    (torch RNG) and quantized on load by the GPU packer; norm weights 1.0."""
    import torch
    m = Q8Model(cfg, device=device, **kw)
    g = torch.Generator(device=f"cuda:{device}")
    g.manual_seed(seed)
    for name in cfg.weight_names():
        shp = cfg.tensor_shape(name)
        if len(shp) == 1:
            t = torch.ones(shp, dtype=torch.bfloat16, device=f"cuda:{device}")
        else:
            t = (torch.randn(shp, generator=g, dtype=torch.float32, device=f"cuda:{device}") * std).to(
                torch.bfloat16)
        m.load_tensor(name, t, packed=False)
        del t
    torch.cuda.synchronize(device)
    return m
