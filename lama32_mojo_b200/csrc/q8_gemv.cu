// Decode Q8 GEMV/GEMM for small token counts (M <= 16 per CTA row of tiles).
//
// Replaces k_mm_q8 / mm_q8_op (src/llama_q8.mojo:54-93, :124-141):
//   y[m, n] = sum_g f16(s[n,g]) * sum_{k in g} x[m,k] * q[n,k]
//
// B200 design (HBM-bound: every weight byte is read exactly once):
//  * Each warp owns a 16-row x (K/KS) slab.  Per 64-wide group a lane loads 16
//    contiguous int8 codes of two rows (g and g+8) with one 128-bit load each,
//    converts them to f16 in registers (byte-permute into a 1024+b f16 bit
//    pattern, one f16x2 subtract: exact for |b| <= 127) and feeds four
//    m16n8k16 tensor-core MMAs.  The order of k inside a 64-group is free for
//    a dot product, so lane (g,t) uses the 16 physical k's [16t, 16t+16) of a
//    group; the activation fragment is built with the same permutation.
//  * Activations arrive in the split-f16 "XS" layout (hi = f16(x), lo =
//    f16(x - hi)); hi and lo run as two MMAs into the same f32 accumulator, so
//    the dot product carries the f32 activations of the reference (W8A32).
//  * The unscaled group partial of each row is multiplied by its f16 group
//    scale in f32 (same association as the reference: scale * group dot).
//  * The KS warps of a row tile reduce through shared memory; epilogues:
//    plain store (q|k|v, lm_head), residual add (o_proj, down: h += y) and
//    SwiGLU over (gate row p, up row F+p) pairs held by the same lane
//    (k_swiglu_mul, src/llama_common.mojo:476-481), written as XS for down.
#include "q8_kernels.h"
#include <algorithm>
#include <mutex>

namespace q8 {

struct GemvParams {
  const __half* xs;  // XS activations, token stride 2K halves
  int M, K;
  const uint8_t* W;  // packed rows
  int64_t rb;        // row bytes = K*33/32
  int N;             // output rows (SWIGLU: pairs F)
  float* y;          // f32 output (nullable for SWIGLU)
  int64_t ldy;
  __half* ys;        // XS output (SWIGLU only, K' = N)
  int ks, rt;        // k-split warps per row tile, row tiles per CTA (ks*rt == 8)
  int tiles;         // number of 16-row (8-pair for SWIGLU) tiles
};

__device__ __forceinline__ uint32_t cvt_s8x2_to_f16x2(uint32_t w_biased, uint32_t sel) {
  // w_biased = 4 int8 codes XOR 0x80 (offset binary).  Place two of them in
  // the low mantissa byte of f16 1024.0 (0x6400) -> 1024 + b + 128, then
  // subtract 1152: exact integer b in f16.
  uint32_t r = __byte_perm(w_biased, 0x64646464u, sel);
  __half2 h = *reinterpret_cast<__half2*>(&r);
  const uint32_t k1152 = 0x64806480u;
  h = __hsub2(h, *reinterpret_cast<const __half2*>(&k1152));
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void mma16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int VEC>
__device__ __forceinline__ void load_codes16(const uint8_t* p, uint32_t c[4]) {
  if constexpr (VEC == 16) {
    uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    c[0] = v.x; c[1] = v.y; c[2] = v.z; c[3] = v.w;
  } else if constexpr (VEC == 8) {
    uint2 v0 = __ldg(reinterpret_cast<const uint2*>(p));
    uint2 v1 = __ldg(reinterpret_cast<const uint2*>(p + 8));
    c[0] = v0.x; c[1] = v0.y; c[2] = v1.x; c[3] = v1.y;
  } else if constexpr (VEC == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) c[i] = __ldg(reinterpret_cast<const uint32_t*>(p + 4 * i));
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t lo = __ldg(reinterpret_cast<const uint16_t*>(p + 4 * i));
      uint32_t hi = __ldg(reinterpret_cast<const uint16_t*>(p + 4 * i + 2));
      c[i] = lo | (hi << 16);
    }
  }
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

template <int EPI, int VEC>
__global__ void __launch_bounds__(256) k_gemv_q8(GemvParams p) {
  __shared__ float red[8][32][4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rtw = warp / p.ks, ksw = warp % p.ks;
  const int tile = blockIdx.x * p.rt + rtw;
  const int m0 = blockIdx.y * 8;  // first token of this CTA's n8 tile
  const bool tile_ok = tile < p.tiles;

  int rowA, rowB;
  if constexpr (EPI == EPI_SWIGLU) {
    const int pr = min(tile * 8 + g, p.N - 1);
    rowA = pr;
    rowB = p.N + pr;
  } else {
    rowA = min(tile * 16 + g, p.N - 1);
    rowB = min(tile * 16 + g + 8, p.N - 1);
  }
  if (!tile_ok) rowA = rowB = 0;
  const uint8_t* baseA = p.W + (int64_t)rowA * p.rb;
  const uint8_t* baseB = p.W + (int64_t)rowB * p.rb;
  const __half* sclA = reinterpret_cast<const __half*>(baseA);
  const __half* sclB = reinterpret_cast<const __half*>(baseB);
  const uint8_t* codA = baseA + p.K / 32 + 16 * t;
  const uint8_t* codB = baseB + p.K / 32 + 16 * t;

  const int ngroups = p.K / Q8_QG;
  const int gbeg = (int)((int64_t)ksw * ngroups / p.ks);
  const int gend = (int)((int64_t)(ksw + 1) * ngroups / p.ks);
  const int m = m0 + g;
  const bool has_x = (m < p.M) && tile_ok;
  const uint4* xrow = reinterpret_cast<const uint4*>(p.xs + (int64_t)(has_x ? m : 0) * 2 * p.K);

  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
  for (int gi = gbeg; gi < gend; ++gi) {
    uint32_t ca[4], cb[4];
    load_codes16<VEC>(codA + gi * Q8_QG, ca);
    load_codes16<VEC>(codB + gi * Q8_QG, cb);
    const float sa = __half2float(sclA[gi]);
    const float sb = __half2float(sclB[gi]);
    uint4 h0 = make_uint4(0, 0, 0, 0), h1 = h0, l0 = h0, l1 = h0;
    if (has_x) {
      const uint4* xp = xrow + (int64_t)(4 * gi + t) * 4;  // 64 B = hi[16] | lo[16]
      h0 = __ldg(xp + 0); h1 = __ldg(xp + 1); l0 = __ldg(xp + 2); l1 = __ldg(xp + 3);
    }
    const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
    float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const uint32_t wa = ca[s] ^ 0x80808080u, wb = cb[s] ^ 0x80808080u;
      uint32_t a[4];
      a[0] = cvt_s8x2_to_f16x2(wa, 0x5140);  // row g,   phys k 4s+0, 4s+1
      a[1] = cvt_s8x2_to_f16x2(wb, 0x5140);  // row g+8
      a[2] = cvt_s8x2_to_f16x2(wa, 0x5342);  // row g,   phys k 4s+2, 4s+3
      a[3] = cvt_s8x2_to_f16x2(wb, 0x5342);  // row g+8
      mma16816(d, a, hw[2 * s], hw[2 * s + 1]);
      mma16816(d, a, lw[2 * s], lw[2 * s + 1]);
    }
    acc[0] = fmaf(sa, d[0], acc[0]);
    acc[1] = fmaf(sa, d[1], acc[1]);
    acc[2] = fmaf(sb, d[2], acc[2]);
    acc[3] = fmaf(sb, d[3], acc[3]);
  }

  if (p.ks > 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) red[warp][lane][i] = acc[i];
    __syncthreads();
    if (ksw != 0) return;
    for (int j = 1; j < p.ks; ++j) {
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] += red[warp + j][lane][i];
    }
  }
  if (!tile_ok) return;

  const int tok0 = m0 + 2 * t;
  if constexpr (EPI == EPI_SWIGLU) {
    const int pr = tile * 8 + g;
    if (pr >= p.N) return;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int mm = tok0 + j;
      if (mm >= p.M) continue;
      const float v = silu_mul(acc[j], acc[2 + j]);
      if (p.y) p.y[(int64_t)mm * p.ldy + pr] = v;
      if (p.ys) {
        __half hi, lo;
        split_f16(v, hi, lo);
        p.ys[xs_index(mm, pr, p.N, 0)] = hi;
        p.ys[xs_index(mm, pr, p.N, 1)] = lo;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int mm = tok0 + (i & 1);
      const int row = tile * 16 + g + 8 * (i >> 1);
      if (mm >= p.M || row >= p.N) continue;
      float* dst = p.y + (int64_t)mm * p.ldy + row;
      if constexpr (EPI == EPI_ADD) *dst += acc[i];
      else *dst = acc[i];
    }
  }
}

// ---------------------------------------------------------------- activation -> XS
__global__ void k_to_xs(const void* __restrict__ x, int dtype, int64_t ldx, int M, int K,
                        __half* __restrict__ xs) {
  const int64_t total = (int64_t)M * K;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / K, k = i % K;
    float v;
    if (dtype == Q8_F32) v = reinterpret_cast<const float*>(x)[m * ldx + k];
    else if (dtype == Q8_BF16) v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[m * ldx + k]);
    else v = __half2float(reinterpret_cast<const __half*>(x)[m * ldx + k]);
    __half hi, lo;
    split_f16(v, hi, lo);
    xs[xs_index(m, k, K, 0)] = hi;
    xs[xs_index(m, k, K, 1)] = lo;
  }
}

int to_xs_launch(const void* x, int dtype, int64_t ldx, int M, int K, __half* xs, cudaStream_t st) {
  const int64_t total = (int64_t)M * K;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 16);
  k_to_xs<<<blocks, 256, 0, st>>>(x, dtype, ldx, M, K, xs);
  return launch_check("k_to_xs");
}

static int pick_vec(const void* W, int64_t K) {
  const uint64_t a = (uint64_t)(uintptr_t)W | (uint64_t)q8_row_bytes(K) | (uint64_t)(K / 32);
  if ((a & 15) == 0) return 16;
  if ((a & 7) == 0) return 8;
  if ((a & 3) == 0) return 4;
  return 2;
}

template <int EPI>
static void launch_vec(int vec, dim3 grid, cudaStream_t st, const GemvParams& p) {
  switch (vec) {
    case 16: k_gemv_q8<EPI, 16><<<grid, 256, 0, st>>>(p); break;
    case 8: k_gemv_q8<EPI, 8><<<grid, 256, 0, st>>>(p); break;
    case 4: k_gemv_q8<EPI, 4><<<grid, 256, 0, st>>>(p); break;
    default: k_gemv_q8<EPI, 2><<<grid, 256, 0, st>>>(p); break;
  }
}

// Generic launcher: epi in {EPI_STORE, EPI_ADD, EPI_SWIGLU}.  xs holds M tokens
// of K in XS layout.  N = output rows (pairs for SWIGLU).
int gemv_launch(int epi, const __half* xs, int M, int K, const void* W, int N, float* y,
                int64_t ldy, __half* ys, cudaStream_t st) {
  Q8_CHECK_ARG(K % Q8_QG == 0 && K > 0 && N > 0 && M > 0, "gemv: bad shape M=%d K=%d N=%d", M, K, N);
  Q8_CHECK_ARG(((uintptr_t)W & 1) == 0, "gemv: packed weights must be 2-byte aligned");
  GemvParams p;
  p.xs = xs; p.M = M; p.K = K; p.W = (const uint8_t*)W; p.rb = q8_row_bytes(K);
  p.N = N; p.y = y; p.ldy = ldy; p.ys = ys;
  const int ngroups = K / Q8_QG;
  int ks = 8;
  while (ks > 1 && ngroups / ks < 4) ks >>= 1;
  p.ks = ks; p.rt = 8 / ks;
  p.tiles = (epi == EPI_SWIGLU) ? ceil_div(N, 8) : ceil_div(N, 16);
  dim3 grid(ceil_div(p.tiles, p.rt), ceil_div(M, 8));
  const int vec = pick_vec(W, K);
  if (epi == EPI_STORE) launch_vec<EPI_STORE>(vec, grid, st, p);
  else if (epi == EPI_ADD) launch_vec<EPI_ADD>(vec, grid, st, p);
  else launch_vec<EPI_SWIGLU>(vec, grid, st, p);
  return launch_check("k_gemv_q8");
}

// Small-M tensor-core GEMV for every M until the tcgen05 tile GEMM takes the
// large-M (prefill / wide batch) shapes.
int gemm_dispatch(int epi, const __half* xs, int M, int K, const void* W, int N, float* y,
                  int64_t ldy, __half* ys, cudaStream_t st) {
  return gemv_launch(epi, xs, M, K, W, N, y, ldy, ys, st);
}

// Per-device scratch for the op-level entry points (XS copy of x).
struct OpScratch {
  void* ptr = nullptr;
  size_t bytes = 0;
};
static OpScratch g_op_scratch[64];

int op_scratch(size_t bytes, void** out) {
  int dev = 0;
  Q8_CUDA(cudaGetDevice(&dev));
  OpScratch& s = g_op_scratch[dev & 63];
  if (s.bytes < bytes) {
    if (s.ptr) Q8_CUDA(cudaFree(s.ptr));
    s.ptr = nullptr;
    s.bytes = 0;
    if (cudaMalloc(&s.ptr, bytes) != cudaSuccess) {
      cudaGetLastError();
      set_error("op scratch: cudaMalloc(%zu) failed", bytes);
      return Q8_ERR_OOM;
    }
    s.bytes = bytes;
  }
  *out = s.ptr;
  return Q8_OK;
}

}  // namespace q8

using namespace q8;

static int op_gemm_common(int epi, const void* x, int x_dtype, int64_t ldx, int64_t M, int64_t K,
                          const void* w, int64_t N, float* y, int64_t ldy, void* stream) {
  Q8_CHECK_ARG(x && w && y, "q8op_gemm: null pointer");
  Q8_CHECK_ARG(x_dtype == Q8_F32 || x_dtype == Q8_BF16 || x_dtype == Q8_F16, "q8op_gemm: bad x_dtype");
  Q8_CHECK_ARG(M > 0 && K > 0 && N > 0 && K % Q8_QG == 0 && ldx >= K && ldy >= (epi == EPI_SWIGLU ? N : N),
               "q8op_gemm: bad shape");
  Q8_CHECK_ARG(M < (1 << 30) && K < (1 << 30) && N < (1 << 30), "q8op_gemm: dims too large");
  cudaStream_t st = (cudaStream_t)stream;
  void* xs = nullptr;
  Q8_TRY(op_scratch((size_t)M * K * 4, &xs));
  Q8_TRY(to_xs_launch(x, x_dtype, ldx, (int)M, (int)K, (__half*)xs, st));
  return gemm_dispatch(epi, (const __half*)xs, (int)M, (int)K, w, (int)N, y, ldy, nullptr, st);
}

extern "C" int q8op_gemm(const void* x, int x_dtype, int64_t ldx, int64_t M, int64_t K,
                         const void* packed_w, int64_t N, float* y, int64_t ldy, void* stream) {
  return op_gemm_common(EPI_STORE, x, x_dtype, ldx, M, K, packed_w, N, y, ldy, stream);
}

extern "C" int q8op_gemm_swiglu(const void* x, int x_dtype, int64_t ldx, int64_t M, int64_t K,
                                const void* packed_gu, int64_t F, float* act, int64_t ld_act,
                                void* stream) {
  return op_gemm_common(EPI_SWIGLU, x, x_dtype, ldx, M, K, packed_gu, F, act, ld_act, stream);
}

// ---------------------------------------------------------------- allocation-free entry
// Staging for q8op_gemm_noalloc: x converted to split-f16 (2 halves per
// element).  A file-scope device array, so the entry point never allocates.
static __device__ __align__(256) __half g_noalloc_xs[2 * Q8_NOALLOC_MAX_ELEMS];

namespace q8 {
// Device address of g_noalloc_xs per device.  In host code the symbol is only
// a host-side shadow; the device address comes from cudaGetSymbolAddress,
// resolved once per device with that device current.
static __half* g_noalloc_dev[64];
static std::mutex g_noalloc_mu;

static int noalloc_staging(__half** out) {
  int dev = 0;
  Q8_CUDA(cudaGetDevice(&dev));
  Q8_CHECK_ARG(dev >= 0 && dev < 64, "q8op_gemm_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_dev[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_xs);
    if (e != cudaSuccess || !p) {
      set_error("q8op_gemm_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return Q8_ERR_CUDA;
    }
    g_noalloc_dev[dev] = (__half*)p;
  }
  *out = g_noalloc_dev[dev];
  return Q8_OK;
}
}  // namespace q8

extern "C" int q8op_gemm_noalloc(const void* x, int x_dtype, int64_t ldx, int64_t M, int64_t K,
                                 const void* packed_w, int64_t N, float* y, int64_t ldy, void* stream) {
  Q8_CHECK_ARG(x && packed_w && y, "q8op_gemm_noalloc: null pointer");
  Q8_CHECK_ARG(x_dtype == Q8_F32 || x_dtype == Q8_BF16 || x_dtype == Q8_F16, "q8op_gemm_noalloc: bad x_dtype");
  Q8_CHECK_ARG(M > 0 && K > 0 && N > 0 && K % Q8_QG == 0 && ldx >= K && ldy >= N, "q8op_gemm_noalloc: bad shape");
  Q8_CHECK_ARG(N < (1 << 30), "q8op_gemm_noalloc: N too large");
  Q8_CHECK_ARG(M * K <= (int64_t)Q8_NOALLOC_MAX_ELEMS,
               "q8op_gemm_noalloc: M*K = %lld exceeds the static staging capacity of %d elements",
               (long long)(M * K), (int)Q8_NOALLOC_MAX_ELEMS);
  cudaStream_t st = (cudaStream_t)stream;
  __half* xs = nullptr;
  Q8_TRY(noalloc_staging(&xs));
  // every staged element is written before it is read: nothing to clear
  Q8_TRY(to_xs_launch(x, x_dtype, ldx, (int)M, (int)K, xs, st));
  return gemm_dispatch(EPI_STORE, xs, (int)M, (int)K, packed_w, (int)N, y, ldy, nullptr, st);
}
