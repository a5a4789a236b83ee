"""The allocation-free GEMM entry point, called through the C ABI.

Callers that cannot allocate device memory (a host with its own fixed device
memory pool, or code that must not trigger cudaMalloc's implicit
synchronization) use q8op_gemm_noalloc, which stages activations in a static
device array instead of a cudaMalloc'd buffer.  Its output must match
q8op_gemm on two calls in a row (the second call reuses the static array the
first one left behind).  This file is collected last on purpose.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from lama32_mojo_b200 import _lib, ops
from oracle import q8_oracle as O

pytestmark = pytest.mark.gpu

MAX_ELEMS = 2 * 1024 * 1024  # Q8_NOALLOC_MAX_ELEMS in include/q8cuda.h


def _call(fn, x, packed, K, y):
    s = torch.cuda.current_stream().cuda_stream
    dt = _lib.Q8_BF16 if x.dtype == torch.bfloat16 else _lib.Q8_F32
    return fn(C.c_void_p(x.data_ptr()), dt, x.stride(0), x.shape[0], K, C.c_void_p(packed.data_ptr()),
              packed.shape[0], C.c_void_p(y.data_ptr()), y.stride(0), C.c_void_p(s))


# decode shapes of Llama-3.1-8B, a bf16 input, and M*K at the static capacity
# (512 x 4096 == Q8_NOALLOC_MAX_ELEMS: 64 eight-row blocks of the GEMV)
CASES = [(1, 4096, 6144, torch.float32), (8, 14336, 4096, torch.float32), (3, 2048, 2048, torch.bfloat16),
         (512, 4096, 256, torch.float32)]


@pytest.mark.parametrize("M,K,N,dt", CASES)
def test_noalloc_gemm_matches_gemm_and_oracle_twice(cuda, M, K, N, dt):
    assert M * K <= MAX_ELEMS
    L = _lib.lib()
    g = torch.Generator(device=cuda).manual_seed(123 + M)
    w = (torch.randn((N, K), generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    p = ops.pack_q8(w)
    x = torch.randn((M, K), generator=g, device=cuda).to(dt)
    y_ref = torch.empty((M, N), device=cuda)
    _lib.check(_call(L.q8op_gemm, x, p, K, y_ref))
    torch.cuda.synchronize()
    b = y_ref.cpu().numpy()
    want = O.mm_q8(x.float().cpu().numpy(), p.cpu().numpy().view(np.uint16), K)
    for _ in range(2):  # the second call reuses the static array the first one left behind
        y_new = torch.full((M, N), float("nan"), device=cuda)
        _lib.check(_call(L.q8op_gemm_noalloc, x, p, K, y_new))
        torch.cuda.synchronize()
        a = y_new.cpu().numpy()
        assert np.isfinite(a).all()
        # q8op_gemm takes the tensor-core GEMM from M = 128 (a different
        # accumulation order): the kernel tests' GEMM tolerance
        assert O.rel_l2(a, b) <= 1e-4 and np.abs(a - b).max() <= 1e-3, (M, K, N)
        assert O.rel_l2(a, want) <= 1e-4 and np.abs(a - want).max() <= 1e-3, (M, K, N)


def test_noalloc_gemm_rejects_oversize(cuda):
    L = _lib.lib()
    K = 4096
    M = MAX_ELEMS // K + 1
    x = torch.zeros((M, K), device=cuda)
    p = torch.zeros((16, K // 64 + K // 2), dtype=torch.int16, device=cuda)
    y = torch.zeros((M, 16), device=cuda)
    st = _call(L.q8op_gemm_noalloc, x, p, K, y)
    assert st == _lib.Q8_ERR_ARG
    assert "static staging capacity" in _lib.last_error()
