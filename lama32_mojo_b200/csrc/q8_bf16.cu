// bf16-weight matrix products: the reference's non-Q8 path.
//
// Replaces k_mm_w / k_mm_tile and their dispatch mm_op
// (src/llama_common.mojo:89-162, :636-684): y[m, n] = sum_k x[m, k] * w[n, k]
// with f32 activations, bf16 weights (exactly f32 after widening) and f32
// accumulation, plus the epilogues run_layer applies behind them (store,
// residual add k_res_add / k_add, SwiGLU k_swiglu_mul; :354-358, :396-399,
// :476-481).
//
// Work split.  A CTA of 8 warps covers 16 output rows (2 per warp) for up to
// 8 tokens (grid.y walks token blocks); lane l reads 16-byte chunks l, l + 32,
// .. of each row (8 weights) and the matching 8 activations of every token
// (L1-resident: every warp of the CTA reads the same x rows), keeping 2 x 8
// partial sums; a butterfly reduction finishes each sum (lane order, fixed:
// results do not depend on timing).  At decode (one token) the kernel streams
// the weights once with 4 chunks in flight per row; prefill-sized batches
// re-read the weights once per 8 tokens.
#include "q8_kernels.h"

namespace q8 {

constexpr int BF_WARPS = 8;
constexpr int BF_R = 2;   // rows per warp
constexpr int BF_MT = 8;  // tokens per CTA

__device__ __forceinline__ void bf_widen(uint4 q, float (&w)[8]) {
  const uint32_t v[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    w[2 * i] = __uint_as_float(v[i] << 16);
    w[2 * i + 1] = __uint_as_float(v[i] & 0xFFFF0000u);
  }
}

// rows of the CTA: STORE/ADD rows n, SwiGLU pairs (gate n, up F2 + n)
template <int EPI>
__global__ void __launch_bounds__(BF_WARPS * 32) k_gemm_bf16(const uint16_t* __restrict__ W, int K, int N, int F2,
                                                             const float* __restrict__ x, int64_t ldx, int M,
                                                             float* __restrict__ y, int64_t ldy) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = (blockIdx.x * BF_WARPS + warp) * (EPI == EPI_SWIGLU ? 1 : BF_R);
  const int m0 = blockIdx.y * BF_MT;
  const int mt = min(BF_MT, M - m0);
  int rows[BF_R];
  bool live[BF_R];
#pragma unroll
  for (int r = 0; r < BF_R; ++r) {
    if constexpr (EPI == EPI_SWIGLU) {
      rows[r] = r == 0 ? n0 : F2 + n0;
      live[r] = n0 < N;
    } else {
      rows[r] = n0 + r;
      live[r] = n0 + r < N;
    }
    if (!live[r]) rows[r] = 0;
  }
  float acc[BF_R][BF_MT];
#pragma unroll
  for (int r = 0; r < BF_R; ++r)
#pragma unroll
    for (int t = 0; t < BF_MT; ++t) acc[r][t] = 0.f;
  const int nch = K / 8;  // 16-byte chunks per row
#pragma unroll 2
  for (int ch = lane; ch < nch; ch += 32) {
    uint4 q[BF_R];
#pragma unroll
    for (int r = 0; r < BF_R; ++r)
      q[r] = __ldg(reinterpret_cast<const uint4*>(W + (int64_t)rows[r] * K) + ch);
#pragma unroll
    for (int t = 0; t < BF_MT; ++t) {
      if (t < mt) {
        const float4* xp = reinterpret_cast<const float4*>(x + (int64_t)(m0 + t) * ldx + ch * 8);
        const float4 a = __ldg(xp), b = __ldg(xp + 1);
        const float xv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int r = 0; r < BF_R; ++r) {
          float w[8];
          bf_widen(q[r], w);
          float s = acc[r][t];
#pragma unroll
          for (int i = 0; i < 8; ++i) s = fmaf(xv[i], w[i], s);
          acc[r][t] = s;
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < BF_R; ++r)
#pragma unroll
    for (int t = 0; t < BF_MT; ++t) acc[r][t] = warp_sum(acc[r][t]);
  if (lane != 0) return;
#pragma unroll
  for (int t = 0; t < BF_MT; ++t) {
    if (t >= mt) break;
    float* yr = y + (int64_t)(m0 + t) * ldy;
    if constexpr (EPI == EPI_SWIGLU) {
      if (live[0]) yr[n0] = silu_mul(acc[0][t], acc[1][t]);
    } else {
#pragma unroll
      for (int r = 0; r < BF_R; ++r) {
        if (!live[r]) continue;
        if constexpr (EPI == EPI_ADD) yr[n0 + r] += acc[r][t];
        else yr[n0 + r] = acc[r][t];
      }
    }
  }
}

// y = x . W^T (+ y for ADD; SwiGLU: W holds 2N rows, gate then up).  x f32
// rows [M][ldx]; K a multiple of 8 and 16-byte aligned rows.
int gemm_bf16_launch(int epi, const float* x, int64_t ldx, int M, int K, const uint16_t* W, int N, float* y,
                     int64_t ldy, cudaStream_t st) {
  if (M <= 0 || N <= 0) return Q8_OK;
  Q8_CHECK_ARG(K % 8 == 0 && ((uintptr_t)W & 15) == 0 && ((uintptr_t)x & 15) == 0 && ldx % 4 == 0,
               "gemm_bf16: K must be a multiple of 8 and x / W 16-byte aligned");
  const int rows_per_cta = BF_WARPS * (epi == EPI_SWIGLU ? 1 : BF_R);
  const dim3 grid(ceil_div(N, rows_per_cta), ceil_div(M, BF_MT));
  if (epi == EPI_SWIGLU) k_gemm_bf16<EPI_SWIGLU><<<grid, BF_WARPS * 32, 0, st>>>(W, K, N, N, x, ldx, M, y, ldy);
  else if (epi == EPI_ADD) k_gemm_bf16<EPI_ADD><<<grid, BF_WARPS * 32, 0, st>>>(W, K, N, 0, x, ldx, M, y, ldy);
  else k_gemm_bf16<EPI_STORE><<<grid, BF_WARPS * 32, 0, st>>>(W, K, N, 0, x, ldx, M, y, ldy);
  return launch_check("k_gemm_bf16");
}

// Embedding gather of bf16 rows into f32 (the reference's bf16 embed).
__global__ void k_embed_bf16(const uint16_t* __restrict__ E, int64_t d, const int32_t* __restrict__ ids,
                             float* __restrict__ y) {
  const int64_t row = ids[blockIdx.x];
  for (int64_t i = threadIdx.x; i < d; i += blockDim.x)
    y[(int64_t)blockIdx.x * d + i] = bf16_bits_to_f32(E[row * d + i]);
}

int embed_bf16_launch(const uint16_t* E, int64_t d, const int32_t* ids, int64_t s, float* y, cudaStream_t st) {
  if (s <= 0) return Q8_OK;
  k_embed_bf16<<<(unsigned)s, 256, 0, st>>>(E, d, ids, y);
  return launch_check("k_embed_bf16");
}

}  // namespace q8

using namespace q8;

extern "C" int q8op_gemm_bf16(const float* x, int64_t ldx, int64_t M, int64_t K, const void* w_bf16, int64_t N,
                              float* y, int64_t ldy, void* stream) {
  Q8_CHECK_ARG(x && w_bf16 && y && M > 0 && K > 0 && N > 0 && ldx >= K && ldy >= N, "q8op_gemm_bf16: bad argument");
  Q8_CHECK_ARG(M < (1 << 30) && K < (1 << 30) && N < (1 << 30), "q8op_gemm_bf16: dims too large");
  return gemm_bf16_launch(EPI_STORE, x, ldx, (int)M, (int)K, (const uint16_t*)w_bf16, (int)N, y, ldy,
                          (cudaStream_t)stream);
}
