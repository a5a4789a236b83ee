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
#include "q8_gemv_core.cuh"
#include "q8_kernels.h"
#include <algorithm>
#include <mutex>

namespace q8 {

struct GemvParams {
  const float* x32;  // f32 activations [M, ldx32] (int8-digit kernel, XSRC_GLOBAL)
  int64_t ldx32;
  const __half* xs;  // XS activations, token stride 2K halves (split-f16 kernel, XSRC_GLOBAL)
  int M, K;
  const uint8_t* W;  // packed rows
  int64_t rb;        // row bytes = K*33/32
  int N;             // output rows (SWIGLU: pairs F)
  float* y;          // f32 output (nullable for SWIGLU)
  int64_t ldy;
  __half* ys;        // XS output (SWIGLU only, K' = N)
  int ks, rt;        // k-split warps per row tile, row tiles per CTA tile (ks*rt == 8)
  int tiles;         // 16-row (8-pair for SWIGLU) row tiles
  int ctiles;        // CTA tiles = ceil(tiles / rt); CTAs loop over them
  int stage_x;       // 1: this CTA's token rows of x are staged in shared memory
  // fused RMSNorm prologue (XSRC_RMS): x = w * h / sqrt(mean(h^2) + eps), h f32 [M, K]
  const float* h;
  int64_t ldh;
  const uint16_t* nw;
  float eps;
};

enum { XSRC_GLOBAL = 0, XSRC_RMS = 1 };
constexpr int GEMV_P = 8;  // 64-wide groups whose codes a lane loads before computing

template <int EPI>
__device__ __forceinline__ void tile_rows(const GemvParams& p, int tile, int g, int t, const uint8_t*& codA,
                                          const uint8_t*& codB, const __half*& sclA, const __half*& sclB) {
  int rowA, rowB;
  if constexpr (EPI == EPI_SWIGLU) {
    const int pr = min(tile * 8 + g, p.N - 1);
    rowA = pr;
    rowB = p.N + pr;
  } else {
    rowA = min(tile * 16 + g, p.N - 1);
    rowB = min(tile * 16 + g + 8, p.N - 1);
  }
  if (tile >= p.tiles) rowA = rowB = 0;
  const uint8_t* baseA = p.W + (int64_t)rowA * p.rb;
  const uint8_t* baseB = p.W + (int64_t)rowB * p.rb;
  sclA = reinterpret_cast<const __half*>(baseA);
  sclB = reinterpret_cast<const __half*>(baseB);
  codA = baseA + p.K / 32 + 16 * t;
  codB = baseB + p.K / 32 + 16 * t;
}

template <int VEC, int NP>
__device__ __forceinline__ void load_batch_n(const uint8_t* codA, const uint8_t* codB, const __half* sclA,
                                             const __half* sclB, int g0, int gend, uint32_t (&ca)[NP][4],
                                             uint32_t (&cb)[NP][4], __half2 (&sab)[NP]) {
#pragma unroll
  for (int q = 0; q < NP; ++q) {
    const int gi = min(g0 + q, gend - 1);
    load_codes16<VEC>(codA + gi * Q8_QG, ca[q]);
    load_codes16<VEC>(codB + gi * Q8_QG, cb[q]);
    sab[q] = __halves2half2(__ldg(sclA + gi), __ldg(sclB + gi));
  }
}

template <int VEC>
__device__ __forceinline__ void load_batch(const uint8_t* codA, const uint8_t* codB, const __half* sclA,
                                           const __half* sclB, int g0, int gend, uint32_t (&ca)[GEMV_P][4],
                                           uint32_t (&cb)[GEMV_P][4], __half2 (&sab)[GEMV_P]) {
#pragma unroll
  for (int q = 0; q < GEMV_P; ++q) {
    const int gi = min(g0 + q, gend - 1);
    load_codes16<VEC>(codA + gi * Q8_QG, ca[q]);
    load_codes16<VEC>(codB + gi * Q8_QG, cb[q]);
    sab[q] = __halves2half2(__ldg(sclA + gi), __ldg(sclB + gi));  // (row g, row g+8) scales
  }
}

// Persistent small-M GEMV.  CTA = 8 warps = rt row tiles x ks K-slices; each
// CTA loops over CTA tiles.  Per CTA, once: the weight batch of its first
// tile is issued (weights do not depend on the previous kernel, so this runs
// before griddepcontrol.wait), then the CTA's token rows of x are staged in
// shared memory (a copy of the XS rows, or RMSNorm of the f32 residual rows
// for XSRC_RMS).  Per tile, each warp computes its K-slice from registers and
// issues the next batch (or the next tile's first batch) before the
// cross-warp reduction and epilogue, so memory stays busy during them.
template <int EPI, int VEC, int XSRC>
__global__ void __launch_bounds__(256, 2) k_gemv_q8(GemvParams p) {
  __shared__ float red[8][32][4];
  __shared__ float inv_s[8];
  extern __shared__ __align__(16) uint8_t xs_smem[];
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rtw = warp / p.ks, ksw = warp % p.ks;
  const int m0 = blockIdx.y * 8;
  const int ngroups = p.K / Q8_QG;
  const int gbeg = (int)((int64_t)ksw * ngroups / p.ks);
  const int gend = (int)((int64_t)(ksw + 1) * ngroups / p.ks);
  const int nb = (gend - gbeg + GEMV_P - 1) / GEMV_P;
  int ct = blockIdx.x;

  uint32_t ca[GEMV_P][4], cb[GEMV_P][4];
  __half2 sab[GEMV_P];
  const uint8_t *codA, *codB;
  const __half *sclA, *sclB;
  tile_rows<EPI>(p, ct * p.rt + rtw, g, t, codA, codB, sclA, sclB);
  if (nb > 0) load_batch<VEC>(codA, codB, sclA, sclB, gbeg, gend, ca, cb, sab);

  pdl_wait();  // activations below are written by the previous kernel

  const int mcount = min(8, p.M - m0);
  const int m = m0 + g;
  const bool has_x = m < p.M;
  const uint4* xrow;
  if constexpr (XSRC == XSRC_RMS) {
    // k_rmsnorm_w (src/llama_common.mojo:197-225) fused in front of the
    // matmul: warp w reduces sum(h^2) of token m0+w, then the CTA writes the
    // normalized rows as split-f16 chunks into shared memory.
    if (warp < mcount) {
      const float* hr = p.h + (int64_t)(m0 + warp) * p.ldh;
      float ss = 0.f;
      for (int k = lane * 4; k < p.K; k += 128) {
        const float4 v = *reinterpret_cast<const float4*>(hr + k);
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
      }
      ss = warp_sum(ss);
      if (lane == 0) inv_s[warp] = 1.0f / sqrtf(ss / (float)p.K + p.eps);
    }
    __syncthreads();
    __half* xsm = reinterpret_cast<__half*>(xs_smem);
    const int k4n = p.K / 4;
    for (int i = threadIdx.x; i < mcount * k4n; i += blockDim.x) {
      const int mm = i / k4n, k = (i % k4n) * 4;
      const float4 v = *reinterpret_cast<const float4*>(p.h + (int64_t)(m0 + mm) * p.ldh + k);
      const uint2 wb = *reinterpret_cast<const uint2*>(p.nw + k);
      const float inv = inv_s[mm];
      const float yv[4] = {__uint_as_float(wb.x << 16) * v.x * inv, __uint_as_float(wb.x & 0xffff0000u) * v.y * inv,
                           __uint_as_float(wb.y << 16) * v.z * inv, __uint_as_float(wb.y & 0xffff0000u) * v.w * inv};
      __half hi[4], lo[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) split_f16(yv[e], hi[e], lo[e]);
      // 4 consecutive k stay inside one 16-chunk: 8-byte stores of hi and lo
      *reinterpret_cast<uint2*>(xsm + xs_index(mm, k, p.K, 0)) = *reinterpret_cast<uint2*>(hi);
      *reinterpret_cast<uint2*>(xsm + xs_index(mm, k, p.K, 1)) = *reinterpret_cast<uint2*>(lo);
    }
    __syncthreads();
    xrow = reinterpret_cast<const uint4*>(xsm + (int64_t)(has_x ? g : 0) * 2 * p.K);
  } else {
    if (p.stage_x) {
      uint4* dst = reinterpret_cast<uint4*>(xs_smem);
      const uint4* src = reinterpret_cast<const uint4*>(p.xs + (int64_t)m0 * 2 * p.K);
      const int n16 = mcount * p.K / 4;  // 2K halves per token = K/4 uint4
      for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = __ldg(src + i);
      __syncthreads();
      xrow = reinterpret_cast<const uint4*>(xs_smem) + (int64_t)(has_x ? g : 0) * (p.K / 4);
    } else {
      xrow = reinterpret_cast<const uint4*>(p.xs + (int64_t)(has_x ? m : 0) * 2 * p.K);
    }
  }
  const bool x_in_smem = (XSRC == XSRC_RMS) || p.stage_x;

  for (; ct < p.ctiles; ct += gridDim.x) {
    const int tile = ct * p.rt + rtw;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int b = 0; b < nb; ++b) {
      const int g0 = gbeg + b * GEMV_P;
#pragma unroll
      for (int q = 0; q < GEMV_P; ++q) {
        // groups past gend were loaded clamped; their scale is zeroed below
        const int gi = min(g0 + q, gend - 1);
        const bool valid = g0 + q < gend;
        uint4 h0 = make_uint4(0, 0, 0, 0), h1 = h0, l0 = h0, l1 = h0;
        if (has_x) {
          const uint4* xp = xrow + (int64_t)(4 * gi + t) * 4;  // 64 B = hi[16] | lo[16]
          if (x_in_smem) {
            h0 = xp[0]; h1 = xp[1]; l0 = xp[2]; l1 = xp[3];
          } else {
            h0 = __ldg(xp + 0); h1 = __ldg(xp + 1); l0 = __ldg(xp + 2); l1 = __ldg(xp + 3);
          }
        }
        const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
        // hi and lo products accumulate in separate registers: two short
        // dependent MMA chains per group, independent across groups
        float dh[4] = {0.f, 0.f, 0.f, 0.f}, dl[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const uint32_t wa = ca[q][s] ^ 0x80808080u, wb = cb[q][s] ^ 0x80808080u;
          uint32_t a[4];
          a[0] = cvt_s8x2_to_f16x2(wa, 0x5140);  // row g,   phys k 4s+0, 4s+1
          a[1] = cvt_s8x2_to_f16x2(wb, 0x5140);  // row g+8
          a[2] = cvt_s8x2_to_f16x2(wa, 0x5342);  // row g,   phys k 4s+2, 4s+3
          a[3] = cvt_s8x2_to_f16x2(wb, 0x5342);  // row g+8
          mma16816(dh, a, hw[2 * s], hw[2 * s + 1]);
          mma16816(dl, a, lw[2 * s], lw[2 * s + 1]);
        }
        float2 sc = __half22float2(sab[q]);
        if (!valid) sc = make_float2(0.f, 0.f);
        acc[0] = fmaf(sc.x, dh[0] + dl[0], acc[0]);
        acc[1] = fmaf(sc.x, dh[1] + dl[1], acc[1]);
        acc[2] = fmaf(sc.y, dh[2] + dl[2], acc[2]);
        acc[3] = fmaf(sc.y, dh[3] + dl[3], acc[3]);
      }
      // keep the weight stream going: next batch of this tile, or the first
      // batch of this CTA's next tile, before the reduction / epilogue
      if (b + 1 < nb) {
        load_batch<VEC>(codA, codB, sclA, sclB, g0 + GEMV_P, gend, ca, cb, sab);
      } else if (ct + (int)gridDim.x < p.ctiles) {
        tile_rows<EPI>(p, (ct + gridDim.x) * p.rt + rtw, g, t, codA, codB, sclA, sclB);
        load_batch<VEC>(codA, codB, sclA, sclB, gbeg, gend, ca, cb, sab);
      }
    }

    bool owner = true;
    if (p.ks > 1) {
#pragma unroll
      for (int i = 0; i < 4; ++i) red[warp][lane][i] = acc[i];
      __syncthreads();
      owner = ksw == 0;
      if (owner) {
        for (int j = 1; j < p.ks; ++j) {
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[i] += red[warp + j][lane][i];
        }
      }
    }
    if (owner && tile < p.tiles) {
      const int tok0 = m0 + 2 * t;
      if constexpr (EPI == EPI_SWIGLU) {
        const int pr = tile * 8 + g;
        if (pr < p.N) {
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
    if (p.ks > 1) __syncthreads();  // red[] is reused by the next tile
  }
}

// ---------------------------------------------------------------- int8-digit GEMV
// Decode GEMV for M <= 8 tokens per CTA row of tiles.
//
// Arithmetic: the int8 weight codes go to the tensor core unchanged
// (mma.m16n8k32 s8 x s8 -> s32).  Each activation group of 64 values is
// written as three int8 digits with one f32 scale e:
//     x ~= e * (a0 + a1/254 + a2/254^2),   e = max|x| / 127,
// a0 = rint(x/e), a1 = rint(254 (x/e - a0)), a2 = rint(254 (254 (x/e - a0) - a1)).
// The representation error is <= 0.5/254^2 of e (~2^-24 of the group
// maximum) and the integer dot products are exact, so the result carries the
// f32 activations of the reference (W8A32) to ~1e-7.  The three digits of a
// token are three MMA columns (the n=8 columns are otherwise idle at decode
// batch sizes); per group and column the s32 partial is scaled in f32 by
// (f16 weight scale) x (e / 254^digit) — the reference's association,
// scale x group dot (src/llama_q8.mojo:76-83).  No weight conversion is
// needed, which keeps the instruction count per weight byte low enough for
// the tensor-core path to keep up with HBM.
//
// Structure: persistent CTAs of 8 warps (rt row tiles x ks K-slices).  Per
// CTA, once: the first weight batch is issued into registers (before
// griddepcontrol.wait — weights do not depend on the previous kernel), then
// the CTA's token rows are turned into digits in shared memory (RMSNorm fused
// in for XSRC_RMS).  Per tile, each warp computes its K-slice and issues the
// next batch before the reduction / epilogue.
__device__ __forceinline__ void imma16832(int d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ int8_t digit8(float v) { return (int8_t)max(-127, min(127, __float2int_rn(v))); }

// shared-memory layout of the int8-digit kernel (byte offsets, 16-aligned)
struct R8Layout {
  int fcol, red, total;
};
__host__ __device__ inline R8Layout r8_layout(int mcount, int K, int nt) {
  R8Layout L;
  const int ngroups = K / Q8_QG;
  L.fcol = (mcount * K * 3 + 15) & ~15;      // after the digits [m][group][digit][64]
  L.red = L.fcol + ngroups * nt * 8 * 4;     // f32 [group][nt*8]
  L.total = L.red + 8 * 16 * nt * 8 * 4;     // f32 [warp][16 rows][nt*8]
  return L;
}

constexpr int R8_P = 4;  // groups per register batch (two batches in flight per warp)

// one register batch of R8_P groups against the staged digits
template <int NT>
__device__ __forceinline__ void r8_compute(const uint32_t (&ca)[R8_P][4], const uint32_t (&cb)[R8_P][4],
                                           const __half2 (&sab)[R8_P], int g0, int gend, int g, int t, int mcount,
                                           int ngroups, const int8_t* xq, const float* fcol, float (&acc)[NT][4]) {
#pragma unroll
  for (int q = 0; q < R8_P; ++q) {
    const int gi = min(g0 + q, gend - 1);  // groups past gend were loaded clamped: scale 0
    float2 sc = __half22float2(sab[q]);
    if (g0 + q >= gend) sc = make_float2(0.f, 0.f);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int col = nt * 8 + g;  // B column of this lane: token col/3, digit col%3
      uint4 bx = make_uint4(0, 0, 0, 0);
      if (col < 3 * mcount)
        bx = *reinterpret_cast<const uint4*>(xq + ((int64_t)((col / 3) * ngroups + gi) * 3 + col % 3) * Q8_QG +
                                             16 * t);
      int d[4] = {0, 0, 0, 0};
      imma16832(d, ca[q][0], cb[q][0], ca[q][1], cb[q][1], bx.x, bx.y);  // physical k 16t+0..7
      imma16832(d, ca[q][2], cb[q][2], ca[q][3], cb[q][3], bx.z, bx.w);  // physical k 16t+8..15
      const float2 f = *reinterpret_cast<const float2*>(fcol + gi * NT * 8 + nt * 8 + 2 * t);
      acc[nt][0] = fmaf(__int2float_rn(d[0]), sc.x * f.x, acc[nt][0]);
      acc[nt][1] = fmaf(__int2float_rn(d[1]), sc.x * f.y, acc[nt][1]);
      acc[nt][2] = fmaf(__int2float_rn(d[2]), sc.y * f.x, acc[nt][2]);
      acc[nt][3] = fmaf(__int2float_rn(d[3]), sc.y * f.y, acc[nt][3]);
    }
  }
}

template <int EPI, int VEC, int XSRC, int NT>
__global__ void __launch_bounds__(256, 2) k_gemv_q8_r8(GemvParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float inv_s[8];
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rtw = warp / p.ks, ksw = warp % p.ks;
  const int m0 = blockIdx.y * 8;
  const int mcount = min(8, p.M - m0);
  const int ngroups = p.K / Q8_QG;
  const int gbeg = (int)((int64_t)ksw * ngroups / p.ks);
  const int gend = (int)((int64_t)(ksw + 1) * ngroups / p.ks);
  const int nb = (gend - gbeg + R8_P - 1) / R8_P;  // batches per tile
  const int my_ctiles = (p.ctiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int n_items = my_ctiles * nb;               // (tile, batch) items of this warp, in order
  const R8Layout L = r8_layout(mcount, p.K, NT);
  int8_t* xq = reinterpret_cast<int8_t*>(smem);
  float* fcol = reinterpret_cast<float*>(smem + L.fcol);
  float* red = reinterpret_cast<float*>(smem + L.red);

  // item i -> (tile, first group); rows are re-derived when the tile changes
  auto item_tile = [&](int i) { return ((int)blockIdx.x + (i / nb) * (int)gridDim.x) * p.rt + rtw; };
  auto item_g0 = [&](int i) { return gbeg + (i % nb) * R8_P; };
  uint32_t ca0[R8_P][4], cb0[R8_P][4], ca1[R8_P][4], cb1[R8_P][4];
  __half2 s0[R8_P], s1[R8_P];
  const uint8_t *codA, *codB;
  const __half *sclA, *sclB;
  int rows_tile = -1;
  auto load = [&](int i, uint32_t (&ca)[R8_P][4], uint32_t (&cb)[R8_P][4], __half2 (&sab)[R8_P]) {
    const int tl = item_tile(i);
    if (tl != rows_tile) {
      tile_rows<EPI>(p, tl, g, t, codA, codB, sclA, sclB);
      rows_tile = tl;
    }
    load_batch_n<VEC, R8_P>(codA, codB, sclA, sclB, item_g0(i), gend, ca, cb, sab);
  };
  if (n_items > 0) load(0, ca0, cb0, s0);
  if (n_items > 1) load(1, ca1, cb1, s1);

  pdl_wait();  // activations below are written by the previous kernel

  if constexpr (XSRC == XSRC_RMS) {
    // k_rmsnorm_w (src/llama_common.mojo:197-225) fused in front of the matmul
    if (warp < mcount) {
      const float* hr = p.h + (int64_t)(m0 + warp) * p.ldh;
      float ss = 0.f;
      for (int k = lane * 4; k < p.K; k += 128) {
        const float4 v = *reinterpret_cast<const float4*>(hr + k);
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
      }
      ss = warp_sum(ss);
      if (lane == 0) inv_s[warp] = 1.0f / sqrtf(ss / (float)p.K + p.eps);
    }
    __syncthreads();
  }
  // activation digits: one warp per (token, group), two values per lane
  for (int it = warp; it < mcount * ngroups; it += 8) {
    const int mm = it / ngroups, gi = it % ngroups;
    const int k = gi * Q8_QG + 2 * lane;
    float v0, v1;
    if constexpr (XSRC == XSRC_RMS) {
      const float2 hv = *reinterpret_cast<const float2*>(p.h + (int64_t)(m0 + mm) * p.ldh + k);
      const uint32_t wb = *reinterpret_cast<const uint32_t*>(p.nw + k);
      v0 = __uint_as_float(wb << 16) * hv.x * inv_s[mm];
      v1 = __uint_as_float(wb & 0xffff0000u) * hv.y * inv_s[mm];
    } else {
      const float2 xv = *reinterpret_cast<const float2*>(p.x32 + (int64_t)(m0 + mm) * p.ldx32 + k);
      v0 = xv.x;
      v1 = xv.y;
    }
    const float amax = warp_max(fmaxf(fabsf(v0), fabsf(v1)));
    const float e = amax / 127.0f;
    const float ie = amax > 0.f ? 127.0f / amax : 0.f;
    float u0 = v0 * ie, u1 = v1 * ie;
    int8_t* dq = xq + ((int64_t)(mm * ngroups + gi) * 3) * Q8_QG + 2 * lane;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int8_t d0 = digit8(u0), d1 = digit8(u1);
      *reinterpret_cast<uint16_t*>(dq + j * Q8_QG) = (uint16_t)(uint8_t)d0 | ((uint16_t)(uint8_t)d1 << 8);
      u0 = (u0 - (float)d0) * 254.0f;
      u1 = (u1 - (float)d1) * 254.0f;
    }
    if (lane < 3) fcol[gi * NT * 8 + 3 * mm + lane] = lane == 0 ? e : (lane == 1 ? e / 254.0f : e / 64516.0f);
  }
  for (int i = threadIdx.x; i < ngroups * NT * 8; i += blockDim.x)  // unused columns contribute 0
    if (i % (NT * 8) >= 3 * mcount) fcol[i] = 0.f;
  __syncthreads();

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;

  // tile epilogue: park partials, reduce the K-slices and the three digit columns
  auto finish = [&](int i) {
    const int tile = item_tile(i);
    float* rw = red + warp * 16 * NT * 8;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      rw[g * NT * 8 + nt * 8 + 2 * t] = acc[nt][0];
      rw[g * NT * 8 + nt * 8 + 2 * t + 1] = acc[nt][1];
      rw[(g + 8) * NT * 8 + nt * 8 + 2 * t] = acc[nt][2];
      rw[(g + 8) * NT * 8 + nt * 8 + 2 * t + 1] = acc[nt][3];
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
    }
    if (p.ks > 1) __syncthreads();
    else __syncwarp();
    if (ksw == 0 && tile < p.tiles) {
      auto val = [&](int r, int mm) {
        float v = 0.f;
        for (int j = 0; j < p.ks; ++j) {
          const float* rj = red + (warp + j) * 16 * NT * 8 + r * NT * 8 + 3 * mm;
          v += rj[0] + rj[1] + rj[2];
        }
        return v;
      };
      if constexpr (EPI == EPI_SWIGLU) {
        for (int it = lane; it < 8 * mcount; it += 32) {
          const int r = it & 7, mm = it >> 3;
          const int pr = tile * 8 + r;
          if (pr >= p.N) continue;
          const float v = silu_mul(val(r, mm), val(r + 8, mm));
          const int tok = m0 + mm;
          if (p.y) p.y[(int64_t)tok * p.ldy + pr] = v;
          if (p.ys) {
            __half hi, lo;
            split_f16(v, hi, lo);
            p.ys[xs_index(tok, pr, p.N, 0)] = hi;
            p.ys[xs_index(tok, pr, p.N, 1)] = lo;
          }
        }
      } else {
        for (int it = lane; it < 16 * mcount; it += 32) {
          const int r = it & 15, mm = it >> 4;
          const int row = tile * 16 + r;
          if (row >= p.N) continue;
          float* dst = p.y + (int64_t)(m0 + mm) * p.ldy + row;
          if constexpr (EPI == EPI_ADD) *dst += val(r, mm);
          else *dst = val(r, mm);
        }
      }
    }
    if (p.ks > 1) __syncthreads();  // red[] is reused by the next tile
    else __syncwarp();
  };

  // two register batches in flight: the next batch is always requested
  // before the current one is computed
  for (int i = 0; i < n_items; i += 2) {
    r8_compute<NT>(ca0, cb0, s0, item_g0(i), gend, g, t, mcount, ngroups, xq, fcol, acc);
    if (i + 2 < n_items) load(i + 2, ca0, cb0, s0);
    if (i % nb == nb - 1) finish(i);
    if (i + 1 >= n_items) break;
    r8_compute<NT>(ca1, cb1, s1, item_g0(i + 1), gend, g, t, mcount, ngroups, xq, fcol, acc);
    if (i + 3 < n_items) load(i + 3, ca1, cb1, s1);
    if ((i + 1) % nb == nb - 1) finish(i + 1);
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

__global__ void k_to_f32(const void* __restrict__ x, int dtype, int64_t ldx, int M, int K, float* __restrict__ y) {
  const int64_t total = (int64_t)M * K;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / K, k = i % K;
    float v;
    if (dtype == Q8_F32) v = reinterpret_cast<const float*>(x)[m * ldx + k];
    else if (dtype == Q8_BF16) v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[m * ldx + k]);
    else v = __half2float(reinterpret_cast<const __half*>(x)[m * ldx + k]);
    y[i] = v;
  }
}

int to_f32_launch(const void* x, int dtype, int64_t ldx, int M, int K, float* y, cudaStream_t st) {
  const int64_t total = (int64_t)M * K;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 16);
  k_to_f32<<<blocks, 256, 0, st>>>(x, dtype, ldx, M, K, y);
  return launch_check("k_to_f32");
}

__global__ void k_to_f16(const void* __restrict__ x, int dtype, int64_t ldx, int M, int K, __half* __restrict__ y,
                         int64_t ylo) {
  const int64_t total = (int64_t)M * K;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / K, k = i % K;
    if (dtype == Q8_F16) {  // exact in f16: the remainder is zero
      y[i] = reinterpret_cast<const __half*>(x)[m * ldx + k];
      if (ylo) y[ylo + i] = __float2half_rn(0.f);
      continue;
    }
    const float v = dtype == Q8_F32 ? reinterpret_cast<const float*>(x)[m * ldx + k]
                                    : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[m * ldx + k]);
    const __half hv = __float2half_rn(v);
    y[i] = hv;
    if (ylo) y[ylo + i] = __float2half_rn(v - __half2float(hv));
  }
}

int to_f16_launch(const void* x, int dtype, int64_t ldx, int M, int K, __half* y, cudaStream_t st, int64_t ylo) {
  const int64_t total = (int64_t)M * K;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 16);
  k_to_f16<<<blocks, 256, 0, st>>>(x, dtype, ldx, M, K, y, ylo);
  return launch_check("k_to_f16");
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

// int8-digit GEMV: plans the launch, returns 1 if the shape does not qualify.
static constexpr size_t kR8SmemMax = 200 * 1024;
struct R8Plan {
  int nt, vec;
  size_t smem;
  dim3 grid;
};
static dim3 plan_gemv(GemvParams& p, int epi, int M, int K, int N, size_t smem);
static int pick_vec(const void* W, int64_t K);
static int r8_plan(GemvParams& p, int epi, int M, int K, int N, const void* W, R8Plan* out) {
  if (M > 8) return 1;
  const int nt = ceil_div(3 * M, 8);
  const size_t smem = (size_t)r8_layout(M, K, nt).total;
  if (smem > kR8SmemMax) return 1;
  const dim3 grid = plan_gemv(p, epi, M, K, N, smem);
  // building the digits costs O(K) per CTA: worth it only when every CTA
  // goes on to stream several row tiles (the vocabulary-sized head)
  if (p.ctiles < 3 * (int)grid.x) return 1;
  out->nt = nt;
  out->vec = pick_vec(W, K);
  out->smem = smem;
  out->grid = grid;
  return 0;
}

template <int EPI, int XSRC, int NT>
static int r8_attr() {
  Q8_CUDA(cudaFuncSetAttribute(k_gemv_q8_r8<EPI, 16, XSRC, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)kR8SmemMax));
  Q8_CUDA(cudaFuncSetAttribute(k_gemv_q8_r8<EPI, 8, XSRC, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)kR8SmemMax));
  Q8_CUDA(cudaFuncSetAttribute(k_gemv_q8_r8<EPI, 4, XSRC, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)kR8SmemMax));
  Q8_CUDA(cudaFuncSetAttribute(k_gemv_q8_r8<EPI, 2, XSRC, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)kR8SmemMax));
  return Q8_OK;
}

template <int EPI, int XSRC>
static int r8_attr_all() {
  Q8_TRY((r8_attr<EPI, XSRC, 1>()));
  Q8_TRY((r8_attr<EPI, XSRC, 2>()));
  Q8_TRY((r8_attr<EPI, XSRC, 3>()));
  return Q8_OK;
}

template <int EPI, int XSRC, int NT>
static int r8_launch_nt(const R8Plan& pl, cudaStream_t st, const GemvParams& p) {
  const dim3 blk(256);
  switch (pl.vec) {
    case 16: return launch_pdl("k_gemv_q8_r8", k_gemv_q8_r8<EPI, 16, XSRC, NT>, pl.grid, blk, pl.smem, st, p);
    case 8: return launch_pdl("k_gemv_q8_r8", k_gemv_q8_r8<EPI, 8, XSRC, NT>, pl.grid, blk, pl.smem, st, p);
    case 4: return launch_pdl("k_gemv_q8_r8", k_gemv_q8_r8<EPI, 4, XSRC, NT>, pl.grid, blk, pl.smem, st, p);
    default: return launch_pdl("k_gemv_q8_r8", k_gemv_q8_r8<EPI, 2, XSRC, NT>, pl.grid, blk, pl.smem, st, p);
  }
}

template <int EPI, int XSRC>
static int r8_launch(const R8Plan& pl, cudaStream_t st, const GemvParams& p) {
  if (pl.nt == 1) return r8_launch_nt<EPI, XSRC, 1>(pl, st, p);
  if (pl.nt == 2) return r8_launch_nt<EPI, XSRC, 2>(pl, st, p);
  return r8_launch_nt<EPI, XSRC, 3>(pl, st, p);
}

// Largest shared-memory staging of x per CTA (2 CTAs of 256 threads fit an SM
// with this much each; larger stagings fall back to reading x from L2).
static constexpr size_t kStageMax = 100 * 1024;
// Largest K the fused-RMSNorm GEMV accepts (8 tokens x K x 4 B staged).
static constexpr int kRmsMaxK = 6144;

template <int EPI, int VEC, int XSRC>
static int launch_one(dim3 grid, size_t smem, cudaStream_t st, const GemvParams& p) {
  return launch_pdl("k_gemv_q8", k_gemv_q8<EPI, VEC, XSRC>, grid, dim3(256), smem, st, p);
}

template <int EPI, int XSRC>
static int launch_vec(int vec, dim3 grid, size_t smem, cudaStream_t st, const GemvParams& p) {
  switch (vec) {
    case 16: return launch_one<EPI, 16, XSRC>(grid, smem, st, p);
    case 8: return launch_one<EPI, 8, XSRC>(grid, smem, st, p);
    case 4: return launch_one<EPI, 4, XSRC>(grid, smem, st, p);
    default: return launch_one<EPI, 2, XSRC>(grid, smem, st, p);
  }
}

template <int EPI, int VEC, int XSRC>
static int set_smem_attr(int bytes) {
  Q8_CUDA(cudaFuncSetAttribute(k_gemv_q8<EPI, VEC, XSRC>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  return Q8_OK;
}

template <int EPI, int XSRC>
static int set_smem_attr_all(int bytes) {
  Q8_TRY((set_smem_attr<EPI, 16, XSRC>(bytes)));
  Q8_TRY((set_smem_attr<EPI, 8, XSRC>(bytes)));
  Q8_TRY((set_smem_attr<EPI, 4, XSRC>(bytes)));
  Q8_TRY((set_smem_attr<EPI, 2, XSRC>(bytes)));
  return Q8_OK;
}

// Opt every GEMV variant into large dynamic shared memory on the current
// device (once, before any launch or capture).
int gemv_init() {
  static bool done[64] = {false};
  int dev = 0;
  Q8_CUDA(cudaGetDevice(&dev));
  if (done[dev & 63]) return Q8_OK;
  const int rms = 8 * kRmsMaxK * 4;
  Q8_TRY((set_smem_attr_all<EPI_STORE, XSRC_GLOBAL>((int)kStageMax)));
  Q8_TRY((set_smem_attr_all<EPI_ADD, XSRC_GLOBAL>((int)kStageMax)));
  Q8_TRY((set_smem_attr_all<EPI_SWIGLU, XSRC_GLOBAL>((int)kStageMax)));
  Q8_TRY((set_smem_attr_all<EPI_STORE, XSRC_RMS>(rms)));
  Q8_TRY((set_smem_attr_all<EPI_SWIGLU, XSRC_RMS>(rms)));
  Q8_TRY((r8_attr_all<EPI_STORE, XSRC_GLOBAL>()));
  Q8_TRY((r8_attr_all<EPI_ADD, XSRC_GLOBAL>()));
  Q8_TRY((r8_attr_all<EPI_SWIGLU, XSRC_GLOBAL>()));
  Q8_TRY((r8_attr_all<EPI_STORE, XSRC_RMS>()));
  Q8_TRY((r8_attr_all<EPI_SWIGLU, XSRC_RMS>()));
  done[dev & 63] = true;
  return Q8_OK;
}

static dim3 plan_gemv(GemvParams& p, int epi, int M, int K, int N, size_t smem) {
  const int ngroups = K / Q8_QG;
  const int tiles = (epi == EPI_SWIGLU) ? ceil_div(N, 8) : ceil_div(N, 16);
  // Split K across the warps of a CTA only when whole-row warps would leave
  // the GPU short of warps (each split costs a CTA barrier per tile).
  const int want_warps = 8 * num_sms();
  int ks = 1;
  while (ks < 8 && tiles * ks < want_warps && ngroups / (2 * ks) >= 4) ks <<= 1;
  p.ks = ks;
  p.rt = 8 / ks;
  p.tiles = (epi == EPI_SWIGLU) ? ceil_div(N, 8) : ceil_div(N, 16);
  p.ctiles = ceil_div(p.tiles, p.rt);
  const int per_sm = smem <= kStageMax ? 2 : 1;
  return dim3(std::min(p.ctiles, per_sm * num_sms()), ceil_div(M, 8));
}

// GEMV with the RMSNorm of f32 rows h[M, K] (weight nw) fused in its prologue.
int gemv_rms_launch(int epi, const float* h, int64_t ldh, const uint16_t* nw, float eps, int M, int K,
                    const void* W, int N, float* y, int64_t ldy, __half* ys, cudaStream_t st) {
  Q8_CHECK_ARG(K % Q8_QG == 0 && K > 0 && K <= kRmsMaxK && N > 0 && M > 0, "gemv_rms: bad shape M=%d K=%d", M, K);
  Q8_CHECK_ARG(epi != EPI_ADD, "gemv_rms: residual epilogue not supported");
  Q8_CHECK_ARG(((uintptr_t)h & 15) == 0 && (ldh % 4) == 0 && ((uintptr_t)nw & 7) == 0, "gemv_rms: alignment");
  if (gemv_d_enabled() && ((uintptr_t)nw & 15) == 0 && gemv_d_supported(M, K, N, true, W))
    return gemv_d_launch(epi, true, nullptr, 0, h, ldh, nw, eps, M, K, W, N, y, ldy, ys, st);
  Q8_TRY(gemv_init());
  GemvParams p{};
  p.M = M; p.K = K; p.W = (const uint8_t*)W; p.rb = q8_row_bytes(K);
  p.N = N; p.y = y; p.ldy = ldy; p.ys = ys; p.h = h; p.ldh = ldh; p.nw = nw; p.eps = eps;
  {
    R8Plan pl;
    if (r8_plan(p, epi, M, K, N, W, &pl) == 0) {
      if (epi == EPI_STORE) return r8_launch<EPI_STORE, XSRC_RMS>(pl, st, p);
      return r8_launch<EPI_SWIGLU, XSRC_RMS>(pl, st, p);
    }
  }
  const size_t smem = (size_t)std::min(8, M) * K * 4;
  const dim3 grid = plan_gemv(p, epi, M, K, N, smem);
  const int vec = pick_vec(W, K);
  if (epi == EPI_STORE) return launch_vec<EPI_STORE, XSRC_RMS>(vec, grid, smem, st, p);
  return launch_vec<EPI_SWIGLU, XSRC_RMS>(vec, grid, smem, st, p);
}

// Generic launcher: epi in {EPI_STORE, EPI_ADD, EPI_SWIGLU}.  xs holds M tokens
// of K in XS layout.  N = output rows (pairs for SWIGLU).
int gemv_launch(int epi, const float* x32, int64_t ldx32, const __half* xs, int M, int K, const void* W, int N,
                float* y, int64_t ldy, __half* ys, cudaStream_t st) {
  Q8_CHECK_ARG(K % Q8_QG == 0 && K > 0 && N > 0 && M > 0, "gemv: bad shape M=%d K=%d N=%d", M, K, N);
  Q8_CHECK_ARG(((uintptr_t)W & 1) == 0, "gemv: packed weights must be 2-byte aligned");
  Q8_CHECK_ARG(((uintptr_t)xs & 15) == 0 && ((uintptr_t)x32 & 7) == 0 && (ldx32 % 2) == 0,
               "gemv: activation alignment");
  if (gemv_d_enabled() && x32 && ((uintptr_t)x32 & 15) == 0 && (ldx32 % 4) == 0 &&
      gemv_d_supported(M, K, N, false, W))
    return gemv_d_launch(epi, false, x32, ldx32, nullptr, 0, nullptr, 0.f, M, K, W, N, y, ldy, ys, st);
  Q8_TRY(gemv_init());
  GemvParams p{};
  p.xs = xs; p.M = M; p.K = K; p.W = (const uint8_t*)W; p.rb = q8_row_bytes(K);
  p.N = N; p.y = y; p.ldy = ldy; p.ys = ys;
  if (x32) {
    p.x32 = x32;
    p.ldx32 = ldx32;
    R8Plan pl;
    if (r8_plan(p, epi, M, K, N, W, &pl) == 0) {
      if (epi == EPI_STORE) return r8_launch<EPI_STORE, XSRC_GLOBAL>(pl, st, p);
      if (epi == EPI_ADD) return r8_launch<EPI_ADD, XSRC_GLOBAL>(pl, st, p);
      return r8_launch<EPI_SWIGLU, XSRC_GLOBAL>(pl, st, p);
    }
  }
  Q8_CHECK_ARG(xs, "gemv: shape needs split-f16 activations (none given)");
  const size_t stage = (size_t)std::min(8, M) * K * 4;
  p.stage_x = stage <= kStageMax ? 1 : 0;
  const size_t smem = p.stage_x ? stage : 0;
  const dim3 grid = plan_gemv(p, epi, M, K, N, smem);
  const int vec = pick_vec(W, K);
  if (epi == EPI_STORE) return launch_vec<EPI_STORE, XSRC_GLOBAL>(vec, grid, smem, st, p);
  if (epi == EPI_ADD) return launch_vec<EPI_ADD, XSRC_GLOBAL>(vec, grid, smem, st, p);
  return launch_vec<EPI_SWIGLU, XSRC_GLOBAL>(vec, grid, smem, st, p);
}

// Small-M tensor-core GEMV for every M until the tcgen05 tile GEMM takes the
// large-M (prefill / wide batch) shapes.
int gemm_dispatch(int epi, const float* x32, int64_t ldx32, const __half* xs, int M, int K, const void* W, int N,
                  float* y, int64_t ldy, __half* ys, cudaStream_t st) {
  return gemv_launch(epi, x32, ldx32, xs, M, K, W, N, y, ldy, ys, st);
}

// Per-device scratch for the op-level entry points (XS copy of x).  Growing
// it retires the old buffer instead of freeing it, so a graph that captured
// an earlier op-level call keeps a valid pointer.
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
  if (M >= tc_min_tokens() && K % 512 == 0 && ((uintptr_t)w & 15) == 0) {
    // prefill-sized batch: f16 rows (split hi + lo unless fast mode) ->
    // tensor-core GEMM
    const int64_t lo = gemm_tc_exact() ? M * K : 0;
    Q8_TRY(op_scratch((size_t)M * K * 4, &xs));
    Q8_TRY(to_f16_launch(x, x_dtype, ldx, (int)M, (int)K, (__half*)xs, st, lo));
    return gemm_tc_launch(epi, (const __half*)xs, K, lo, (int)M, (int)K, w, (int)N, y, ldy, nullptr, 0, 0, st);
  }
  Q8_TRY(op_scratch((size_t)M * K * 8, &xs));
  Q8_TRY(to_xs_launch(x, x_dtype, ldx, (int)M, (int)K, (__half*)xs, st));
  // f32 rows for the int8-digit kernel: the caller's x when it is f32, else a
  // converted copy after the XS rows in the same scratch
  const float* x32 = (const float*)x;
  int64_t ld32 = ldx;
  if (!(x_dtype == Q8_F32 && ((uintptr_t)x & 7) == 0 && (ldx % 2) == 0)) {
    float* conv = (float*)((char*)xs + (size_t)M * K * 4);
    Q8_TRY(to_f32_launch(x, x_dtype, ldx, (int)M, (int)K, conv, st));
    x32 = conv;
    ld32 = K;
  }
  return gemm_dispatch(epi, x32, ld32, (const __half*)xs, (int)M, (int)K, w, (int)N, y, ldy, nullptr, st);
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
  return gemm_dispatch(EPI_STORE, nullptr, 0, xs, (int)M, (int)K, packed_w, (int)N, y, ldy, nullptr, st);
}
