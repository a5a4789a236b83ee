"""Op-level entry points on CUDA tensors (thin wrappers over the C ABI).

Names follow the reference kernels they replace: ``pack_q8`` (quantize.py:31),
``mm_q8`` (k_mm_q8 / mm_q8_op, src/llama_q8.mojo:54-141), ``embed_q8``
(k_embed_gather_q8, :96), ``rmsnorm`` (k_rmsnorm_w, src/llama_common.mojo:197),
``rmsnorm_heads`` (k_rmsnorm2_w, :228), ``rope_kv_append`` (k_rope_qk_copy2,
:299), ``attention`` (k_scores/k_softmax_rows/k_att_out, :402-473),
``argmax`` (k_argmax, :493).  Tensors are torch CUDA tensors (torch provides
device memory and the stream); every kernel is in libq8cuda.so.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import check, lib

QG = 64


def _stream(t: torch.Tensor):
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _p(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("libq8cuda ops take CUDA tensors")


def row_u16(m: int) -> int:
    return m // QG + m // 2


def pack_q8(w_bf16: torch.Tensor) -> torch.Tensor:
    """bf16 [n, m] -> packed int16 [n, m/64 + m/2] (bit pattern of the reference's F16 tensor)."""
    _need_cuda(w_bf16)
    assert w_bf16.dtype == torch.bfloat16 and w_bf16.dim() == 2
    w = w_bf16.contiguous()
    n, m = w.shape
    out = torch.empty((n, row_u16(m)), dtype=torch.int16, device=w.device)
    check(lib().q8op_pack(_p(w), n, m, _p(out), _stream(w)))
    return out


def dequant_q8(packed: torch.Tensor, m: int) -> torch.Tensor:
    _need_cuda(packed)
    n = packed.shape[0]
    out = torch.empty((n, m), dtype=torch.float32, device=packed.device)
    check(lib().q8op_dequant(_p(packed), n, m, _p(out), _stream(packed)))
    return out


_DT = {torch.float32: _lib.Q8_F32, torch.bfloat16: _lib.Q8_BF16, torch.float16: _lib.Q8_F16}


def mm_q8(x: torch.Tensor, packed: torch.Tensor, m: int, out: torch.Tensor = None) -> torch.Tensor:
    """y[s, n] = x[s, m] . W[n, m]^T with W packed Q8."""
    _need_cuda(x, packed)
    assert x.dim() == 2 and x.shape[1] == m and x.stride(1) == 1
    n = packed.shape[0]
    s = x.shape[0]
    y = out if out is not None else torch.empty((s, n), dtype=torch.float32, device=x.device)
    check(lib().q8op_gemm(_p(x), _DT[x.dtype], x.stride(0), s, m, _p(packed), n, _p(y), y.stride(0), _stream(x)))
    return y


def mm_bf16(x: torch.Tensor, w_bf16: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
    """y[s, n] = x[s, m] . W[n, m]^T with f32 x and plain bf16 W (mm_op,
    src/llama_common.mojo:636-684)."""
    _need_cuda(x, w_bf16)
    assert x.dtype == torch.float32 and w_bf16.dtype == torch.bfloat16 and x.stride(1) == 1
    assert w_bf16.is_contiguous() and x.shape[1] == w_bf16.shape[1]
    s, m = x.shape
    n = w_bf16.shape[0]
    y = out if out is not None else torch.empty((s, n), dtype=torch.float32, device=x.device)
    check(lib().q8op_gemm_bf16(_p(x), x.stride(0), s, m, _p(w_bf16), n, _p(y), y.stride(0), _stream(x)))
    return y


def mm_q8_swiglu(x: torch.Tensor, packed_gu: torch.Tensor, m: int) -> torch.Tensor:
    """silu(x.Wg^T) * (x.Wu^T) with the F gate rows then F up rows in ``packed_gu``."""
    _need_cuda(x, packed_gu)
    F = packed_gu.shape[0] // 2
    s = x.shape[0]
    y = torch.empty((s, F), dtype=torch.float32, device=x.device)
    check(lib().q8op_gemm_swiglu(_p(x), _DT[x.dtype], x.stride(0), s, m, _p(packed_gu), F, _p(y), F,
                                 _stream(x)))
    return y


def embed_q8(packed_emb: torch.Tensor, d: int, ids: torch.Tensor) -> torch.Tensor:
    _need_cuda(packed_emb, ids)
    ids = ids.to(torch.int32).contiguous()
    y = torch.empty((ids.numel(), d), dtype=torch.float32, device=ids.device)
    check(lib().q8op_embed(_p(packed_emb), packed_emb.shape[0], d, _p(ids), ids.numel(), _p(y), _stream(ids)))
    return y


def rmsnorm(x: torch.Tensor, w_bf16: torch.Tensor, eps: float, resid: torch.Tensor = None) -> torch.Tensor:
    """y = w * x / sqrt(mean(x^2) + eps); with ``resid`` x is first updated in place to x + resid."""
    _need_cuda(x, w_bf16, resid)
    assert x.is_contiguous()
    y = torch.empty_like(x)
    rows, d = x.shape
    check(lib().q8op_rmsnorm(_p(x), _p(resid), _p(w_bf16), rows, d, eps, _p(y), _stream(x)))
    return y


def rmsnorm_heads(x: torch.Tensor, w_bf16: torch.Tensor, eps: float) -> torch.Tensor:
    _need_cuda(x, w_bf16)
    hd = x.shape[-1]
    y = torch.empty_like(x)
    check(lib().q8op_rmsnorm_heads(_p(x), _p(w_bf16), x.numel() // hd, hd, eps, _p(y), _stream(x)))
    return y


def rope_inv_freq(cfg) -> torch.Tensor:
    import numpy as np
    out = np.zeros(cfg.head_dim // 2, np.float32)
    c = cfg.to_c()
    check(lib().q8_rope_inv_freq(C.byref(c), out.ctypes.data_as(C.c_void_p)))
    return torch.from_numpy(out)


def rope_kv_append(qkv, pos, seq, n_heads, n_kv, hd, inv_freq, q_norm, k_norm, eps, k_pages, v_pages, page,
                   block_table):
    _need_cuda(qkv, pos, seq, inv_freq, k_pages, v_pages, block_table)
    T = qkv.shape[0]
    check(lib().q8op_rope_kv_append(_p(qkv), qkv.stride(0), T, _p(pos), _p(seq), n_heads, n_kv, hd, _p(inv_freq),
                                    _p(q_norm), _p(k_norm), eps, _p(k_pages), _p(v_pages), page, _p(block_table),
                                    block_table.shape[1], _stream(qkv)))


def attention(q, pos, seq, n_heads, n_kv, hd, k_pages, v_pages, page, block_table) -> torch.Tensor:
    _need_cuda(q, pos, seq, k_pages, v_pages, block_table)
    T = q.shape[0]
    out = torch.empty((T, n_heads * hd), dtype=torch.float32, device=q.device)
    check(lib().q8op_attention(_p(q), q.stride(0), T, _p(pos), _p(seq), n_heads, n_kv, hd, _p(k_pages),
                               _p(v_pages), page, _p(block_table), block_table.shape[1], _p(out), out.stride(0),
                               _stream(q)))
    return out


def argmax(logits: torch.Tensor) -> torch.Tensor:
    _need_cuda(logits)
    if logits.dim() == 1:
        logits = logits[None]
    out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    check(lib().q8op_argmax(_p(logits), logits.shape[0], logits.shape[1], logits.stride(0), _p(out),
                            _stream(logits)))
    return out


def device_status() -> None:
    """Synchronize the current device and raise if a tensor-core GEMM's bounded
    pipeline wait timed out since the last poll (q8_device_status)."""
    check(lib().q8_device_status())
