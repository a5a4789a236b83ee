// Decode Q8 GEMV for 1-2 tokens on the int8 tensor cores ("digit" GEMV).
//
// Replaces k_mm_q8 / mm_q8_op at decode batch sizes (src/llama_q8.mojo:54-93,
// :124-141), with k_rmsnorm_w (src/llama_common.mojo:197-225) fused in front
// for the q|k|v and gate|up inputs and k_swiglu_mul (:476) / k_res_add
// (:354-358) fused behind:
//   y[m, n] (+)= sum_g f16(s[n,g]) * sum_{k in g} x[m,k] * q[n,k]
//
// Arithmetic.  The int8 weight codes go to the tensor core unchanged
// (mma.m16n8k32 s8 x s8 -> s32).  Each activation group of 64 values is
// written as three int8 digits with one f32 scale e = max|x|/127:
//     x ~= e (a0 + a1/254 + a2/254^2),
// a0 = rint(x/e), a1 = rint(254 (x/e - a0)), a2 = rint(254 (254 (x/e - a0) - a1)),
// a representation error of <= 0.5/254^2 of e (~2^-24 of the group maximum);
// the integer dot products are exact, so the result carries the f32
// activations of the reference.  The three digits of token m are MMA columns
// 3m..3m+2 (the n=8 columns are otherwise idle at decode), and per group and
// column the s32 partial is scaled in f32 by (f16 weight scale) x
// (e / 254^digit): the reference's association, scale x group dot.
//
// Work split.  Units are (16-row tile, 64-group); a matrix has U = tiles x
// groups.  CTA c owns the quad-aligned range [c U/G, (c+1) U/G) (4 units = 4
// consecutive groups of one tile, one register batch) and its 8 warps split it
// again, so every warp streams the same number of weight bytes whatever the
// shape.  Per warp two batches are in flight: 4 groups x 16 codes of rows g
// and g+8 per lane (two 16 B loads per group) plus their 4 + 4 group scales
// (two 8 B loads).  The first two batches are requested before
// griddepcontrol.wait: weights never depend on the previous kernel.
// Tiles a warp holds whole are finished in registers; tiles shared by warps
// are summed in shared memory in warp order; a tile shared by CTAs is parked
// as per-CTA partials and finished by the last CTA to arrive (ticket
// counter), which sums the partials in CTA order.  Every sum has a fixed
// order: results do not depend on timing.
#include "q8_gemv_core.cuh"
#include "q8_kernels.h"

#include <mutex>

namespace q8 {

constexpr int GD_THREADS = 256;
constexpr int GD_WARPS = GD_THREADS / 32;
constexpr int GD_UB = 4;           // groups per register batch (one quad)
constexpr int GD_MB = 2;           // tokens per launch
constexpr int GD_GPW = 8;          // digitization: groups per warp per iteration
constexpr int GD_GIT = GD_GPW * GD_WARPS;
constexpr int GD_SL = 4;           // partial slots per split tile

enum { GD_X_F32 = 0, GD_X_RMS = 1 };

struct GdParams {
  const uint8_t* W;   // packed rows
  int64_t rb;
  int K, N;           // N output rows (SwiGLU: pairs; W holds 2N rows)
  int T, ng, U;       // tiles, groups per row, units
  int M;              // tokens (1..GD_MB)
  const float* x;     // GD_X_F32: activations [M][ldx]
  int64_t ldx;
  const float* h;     // GD_X_RMS: residual rows [M][ldh], norm weight nw (bf16)
  int64_t ldh;
  const uint16_t* nw;
  float eps;
  float* y;           // output [M][ldy] (store / add / SwiGLU f32)
  int64_t ldy;
  __half* ys;         // optional split-f16 copy of the SwiGLU output (K' = N)
  float* part;        // split-tile partials [T][GD_SL][16][GD_MB]
  int* ticket;        // [T], zero at rest
  int aligned;        // CTA ranges of whole tiles (no tile is shared by CTAs)
};

// ------------------------------------------------------------------ unit ranges
// Tile-aligned ranges (CTA c owns tiles [c T/G, (c+1) T/G)) keep every tile
// inside one CTA; quad-balanced ranges split the units evenly and let tiles
// straddle CTAs.
__host__ __device__ inline int gd_cu0(int U, int c, int G) {
  return 4 * (int)(((unsigned)c * (unsigned)(U / 4)) / (unsigned)G);
}
__host__ __device__ inline int gd_cta_of(int U, int x, int G) {
  return (int)((((unsigned)(x / 4) + 1u) * (unsigned)G - 1u) / (unsigned)(U / 4));
}
__host__ __device__ inline int gd_range0(const GdParams& p, int c, int G) {
  return p.aligned ? p.ng * (int)(((unsigned)c * (unsigned)p.T) / (unsigned)G) : gd_cu0(p.U, c, G);
}
__device__ __forceinline__ int gd_wu0(int w, int cu0, int ncu) {
  return cu0 + 4 * (int)(((unsigned)(ncu / 4) * (unsigned)w) / (unsigned)GD_WARPS);
}
__device__ __forceinline__ int gd_warp_of(int x, int cu0, int ncu) {
  return (int)((((unsigned)((x - cu0) / 4) + 1u) * (unsigned)GD_WARPS - 1u) / (unsigned)(ncu / 4));
}

__device__ __forceinline__ void gd_imma(int d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ------------------------------------------------------------------ activation digits
// 4 lanes per (token, group), 16 values per lane: digits into xq
// [M][group][digit][64] and e/254^digit into fcol [group][8] (0 for unused
// columns).  Every lane takes part (the group maximum is a shuffle).
__device__ __forceinline__ void gd_digits16(const float (&v)[16], bool valid, int mm, int gi, int sq, int ng,
                                            int8_t* xq, float* fcol) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  if (!valid) return;
  const float e = amax / 127.0f;
  const float ie = amax > 0.f ? 127.0f / amax : 0.f;
  uint32_t w[3][4];
#pragma unroll
  for (int i4 = 0; i4 < 4; ++i4) {
    uint32_t p0 = 0, p1 = 0, p2 = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      float u = v[4 * i4 + b] * ie;
      const int d0 = max(-127, min(127, __float2int_rn(u)));
      u = (u - (float)d0) * 254.0f;
      const int d1 = max(-127, min(127, __float2int_rn(u)));
      u = (u - (float)d1) * 254.0f;
      const int d2 = max(-127, min(127, __float2int_rn(u)));
      p0 |= (uint32_t)(d0 & 0xFF) << (8 * b);
      p1 |= (uint32_t)(d1 & 0xFF) << (8 * b);
      p2 |= (uint32_t)(d2 & 0xFF) << (8 * b);
    }
    w[0][i4] = p0;
    w[1][i4] = p1;
    w[2][i4] = p2;
  }
  int8_t* dq = xq + ((int64_t)(mm * ng + gi) * 3) * 64 + 16 * sq;
#pragma unroll
  for (int j = 0; j < 3; ++j) *reinterpret_cast<uint4*>(dq + j * 64) = make_uint4(w[j][0], w[j][1], w[j][2], w[j][3]);
  if (sq < 3) fcol[gi * 8 + 3 * mm + sq] = sq == 0 ? e : (sq == 1 ? e / 254.0f : e / 64516.0f);
}

// x = w * h / sqrt(mean(h^2) + eps) (RMSNorm, values kept in registers
// between the two passes; M * K / 64 <= 2 * GD_GIT).
__device__ __forceinline__ void gd_stage_rms(const GdParams& p, int8_t* xq, float* fcol, float* scr) {
  constexpr int IT = 2;
  const int ng = p.K / 64, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sq = lane & 3;
  float v[IT][16];
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int item = it * GD_GIT + warp * GD_GPW + (lane >> 2);
    if (item < p.M * ng) {
      const int m = item / ng, k0 = (item % ng) * 64 + 16 * sq;
      const float4* hp = reinterpret_cast<const float4*>(p.h + (int64_t)m * p.ldh + k0);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 a = hp[i];
        v[it][4 * i] = a.x; v[it][4 * i + 1] = a.y; v[it][4 * i + 2] = a.z; v[it][4 * i + 3] = a.w;
      }
    }
  }
  const int nq = ng * 4;  // quarter-groups per token
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int item = it * GD_GIT + warp * GD_GPW + (lane >> 2);
    if (item < p.M * ng) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) ss = fmaf(v[it][i], v[it][i], ss);
      scr[(item / ng) * nq + (item % ng) * 4 + sq] = ss;
    }
  }
  for (int i = threadIdx.x; i < ng * 8; i += GD_THREADS)
    if (i % 8 >= 3 * p.M) fcol[i] = 0.f;
  __syncthreads();
  float* inv = scr + GD_MB * nq;
  if (warp < p.M) {  // per-token sum of squares in a fixed order
    float t = 0.f;
    for (int i = lane; i < nq; i += 32) t += scr[warp * nq + i];
    t = warp_sum(t);
    if (lane == 0) inv[warp] = 1.0f / sqrtf(t / (float)p.K + p.eps);
  }
  __syncthreads();
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int item = it * GD_GIT + warp * GD_GPW + (lane >> 2);
    const bool valid = item < p.M * ng;
    const int m = valid ? item / ng : 0, gi = valid ? item % ng : 0;
    if (valid) {
      const int k0 = gi * 64 + 16 * sq;
      const uint4 w0 = __ldg(reinterpret_cast<const uint4*>(p.nw + k0));
      const uint4 w1 = __ldg(reinterpret_cast<const uint4*>(p.nw + k0 + 8));
      const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      const float r = inv[m];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[it][2 * i] = __uint_as_float(ww[i] << 16) * v[it][2 * i] * r;
        v[it][2 * i + 1] = __uint_as_float(ww[i] & 0xFFFF0000u) * v[it][2 * i + 1] * r;
      }
    }
    gd_digits16(v[it], valid, m, gi, sq, ng, xq, fcol);
  }
  __syncthreads();
}

// f32 activations -> digits, in rounds of two iterations whose loads are all
// issued before any digit is made.
__device__ __forceinline__ void gd_stage_f32(const GdParams& p, int8_t* xq, float* fcol) {
  constexpr int IT = 2;
  const int ng = p.K / 64, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sq = lane & 3;
  for (int i = threadIdx.x; i < ng * 8; i += GD_THREADS)
    if (i % 8 >= 3 * p.M) fcol[i] = 0.f;
  for (int base = 0; base * GD_GIT < p.M * ng; base += IT) {
    float v[IT][16];
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int item = (base + it) * GD_GIT + warp * GD_GPW + (lane >> 2);
      if (item < p.M * ng) {
        const int m = item / ng, k0 = (item % ng) * 64 + 16 * sq;
        const float4* sp = reinterpret_cast<const float4*>(p.x + (int64_t)m * p.ldx + k0);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 a = sp[i];
          v[it][4 * i] = a.x; v[it][4 * i + 1] = a.y; v[it][4 * i + 2] = a.z; v[it][4 * i + 3] = a.w;
        }
      }
    }
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int item = (base + it) * GD_GIT + warp * GD_GPW + (lane >> 2);
      const bool valid = item < p.M * ng;
      gd_digits16(v[it], valid, valid ? item / ng : 0, valid ? item % ng : 0, sq, ng, xq, fcol);
    }
  }
  __syncthreads();
}

// ------------------------------------------------------------------ epilogues
// One finished output: row r of tile tl (SwiGLU: pair r with its up value vu).
template <int EPI>
__device__ __forceinline__ void gd_store(const GdParams& p, int tl, int r, int m, float v, float vu) {
  if (m >= p.M) return;
  if constexpr (EPI == EPI_SWIGLU) {
    const int pr = tl * 8 + r;
    if (pr >= p.N) return;
    const float a = silu_mul(v, vu);
    if (p.y) p.y[(int64_t)m * p.ldy + pr] = a;
    if (p.ys) {
      __half hi, lo;
      split_f16(a, hi, lo);
      p.ys[xs_index(m, pr, p.N, 0)] = hi;
      p.ys[xs_index(m, pr, p.N, 1)] = lo;
    }
  } else {
    const int row = tl * 16 + r;
    if (row >= p.N) return;
    float* dst = p.y + (int64_t)m * p.ldy + row;
    if constexpr (EPI == EPI_ADD) *dst += v;
    else *dst = v;
  }
}

template <int EPI>
__device__ __forceinline__ void gd_rows(const GdParams& p, int tl, int gq, int& ra, int& rbw) {
  if constexpr (EPI == EPI_SWIGLU) {
    const int pr = min(tl * 8 + gq, p.N - 1);
    ra = pr;
    rbw = p.N + pr;
  } else {
    ra = min(tl * 16 + gq, p.N - 1);
    rbw = min(tl * 16 + gq + 8, p.N - 1);
  }
}

__device__ __forceinline__ float gd_scale(uint2 s, int q) {
  const uint32_t v = q < 2 ? s.x : s.y;
  return __half2float(__ushort_as_half((unsigned short)((q & 1) ? (v >> 16) : (v & 0xFFFFu))));
}

struct GdWarp {
  int wu0, wu1, ng, first_tile, gq, t, warp, lu, cur, seg0;
  bool has_col;
};

template <int EPI, int VEC>
__device__ __forceinline__ void gd_load_quad(const GdParams& p, GdWarp& w, uint32_t (&ca)[GD_UB][4],
                                             uint32_t (&cb)[GD_UB][4], uint2& sa, uint2& sb) {
  const int u = min(w.lu, w.wu1 - GD_UB);  // past the range: reload the last quad (unused)
  const int tl = u / w.ng, g0 = u % w.ng;
  int ra, rbw;
  gd_rows<EPI>(p, tl, w.gq, ra, rbw);
  const uint8_t* rowa = p.W + (int64_t)ra * p.rb;
  const uint8_t* rowb = p.W + (int64_t)rbw * p.rb;
  const uint8_t* pa = rowa + p.K / 32 + g0 * 64 + 16 * w.t;
  const uint8_t* pb = rowb + p.K / 32 + g0 * 64 + 16 * w.t;
#pragma unroll
  for (int q = 0; q < GD_UB; ++q) {
    load_codes16<VEC>(pa + q * 64, ca[q]);
    load_codes16<VEC>(pb + q * 64, cb[q]);
  }
  if constexpr (VEC >= 8) {
    sa = __ldg(reinterpret_cast<const uint2*>(rowa) + g0 / 4);
    sb = __ldg(reinterpret_cast<const uint2*>(rowb) + g0 / 4);
  } else {
    const uint32_t* s32a = reinterpret_cast<const uint32_t*>(rowa) + g0 / 2;
    const uint32_t* s32b = reinterpret_cast<const uint32_t*>(rowb) + g0 / 2;
    sa = make_uint2(__ldg(s32a), __ldg(s32a + 1));
    sb = make_uint2(__ldg(s32b), __ldg(s32b + 1));
  }
  w.lu += GD_UB;
}

// Segment [s0, s1) of tile ftl done: each token's three digit columns (held by
// the four t-lanes of the row) summed in column order; lane t < M writes token t.
template <int EPI>
__device__ __forceinline__ void gd_flush(const GdParams& p, float* red, const GdWarp& w, int ftl, int s0, int s1,
                                         const float (&acc)[4]) {
  float c0[8], c1[8];
#pragma unroll
  for (int cc = 0; cc < 8; ++cc) {
    const int src = (w.gq << 2) | (cc >> 1);
    c0[cc] = __shfl_sync(0xffffffffu, acc[cc & 1], src);
    c1[cc] = __shfl_sync(0xffffffffu, acc[2 + (cc & 1)], src);
  }
  const float a = w.t == 0 ? c0[0] + c0[1] + c0[2] : c0[3] + c0[4] + c0[5];
  const float bv = w.t == 0 ? c1[0] + c1[1] + c1[2] : c1[3] + c1[4] + c1[5];
  if (w.t >= GD_MB) return;
  if (s0 == ftl * w.ng && s1 == (ftl + 1) * w.ng) {
    if constexpr (EPI == EPI_SWIGLU) {
      gd_store<EPI>(p, ftl, w.gq, w.t, a, bv);
    } else {
      gd_store<EPI>(p, ftl, w.gq, w.t, a, 0.f);
      gd_store<EPI>(p, ftl, w.gq + 8, w.t, bv, 0.f);
    }
  } else {  // shared tile: first segment -> slot 0, last -> slot 1
    float* rw = red + (w.warp * 2 + (ftl == w.first_tile ? 0 : 1)) * 16 * GD_MB;
    rw[w.gq * GD_MB + w.t] = a;
    rw[(w.gq + 8) * GD_MB + w.t] = bv;
  }
}

template <int EPI>
__device__ __forceinline__ void gd_compute_quad(const GdParams& p, const int8_t* xcol, const float* fcol,
                                                float* red, GdWarp& w, int u0, float (&acc)[4],
                                                const uint32_t (&ca)[GD_UB][4], const uint32_t (&cb)[GD_UB][4],
                                                uint2 sa, uint2 sb) {
  const int tl = u0 / w.ng, g0 = u0 % w.ng;
  if (tl != w.cur) {
    if (w.cur >= 0) gd_flush<EPI>(p, red, w, w.cur, w.seg0, u0, acc);
    w.cur = tl;
    w.seg0 = u0;
    acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
  }
#pragma unroll
  for (int q = 0; q < GD_UB; ++q) {
    uint4 bx = make_uint4(0, 0, 0, 0);
    if (w.has_col) bx = *reinterpret_cast<const uint4*>(xcol + (int64_t)(g0 + q) * 3 * 64);
    int d[4] = {0, 0, 0, 0};
    gd_imma(d, ca[q][0], cb[q][0], ca[q][1], cb[q][1], bx.x, bx.y);  // physical k 16t+0..7
    gd_imma(d, ca[q][2], cb[q][2], ca[q][3], cb[q][3], bx.z, bx.w);  // physical k 16t+8..15
    const float s0 = gd_scale(sa, q), s1 = gd_scale(sb, q);
    const float2 f = *reinterpret_cast<const float2*>(fcol + (g0 + q) * 8 + 2 * w.t);
    acc[0] = fmaf(__int2float_rn(d[0]), s0 * f.x, acc[0]);
    acc[1] = fmaf(__int2float_rn(d[1]), s0 * f.y, acc[1]);
    acc[2] = fmaf(__int2float_rn(d[2]), s1 * f.x, acc[2]);
    acc[3] = fmaf(__int2float_rn(d[3]), s1 * f.y, acc[3]);
  }
}

template <int EPI, int VEC, int XSRC>
__global__ void __launch_bounds__(GD_THREADS, 2) k_gemv_d(GdParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[GD_WARPS * 2 * 16 * GD_MB];
  __shared__ float scr[GD_MB * 4 * 64 + GD_MB];  // RMSNorm: quarter-group sums of squares (K <= 4096)
  __shared__ int s_last[2];
  pdl_trigger();
  const int G = gridDim.x, c = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ng = p.ng;
  const int cu0 = gd_range0(p, c, G), cu1 = gd_range0(p, c + 1, G), ncu = cu1 - cu0;
  int8_t* xq = reinterpret_cast<int8_t*>(smem);
  float* fcol = reinterpret_cast<float*>(smem + (((size_t)p.M * p.K * 3 + 15) & ~(size_t)15));

  GdWarp w;
  w.wu0 = gd_wu0(warp, cu0, ncu);
  w.wu1 = gd_wu0(warp + 1, cu0, ncu);
  w.ng = ng;
  w.first_tile = w.wu0 / ng;
  w.gq = lane >> 2;
  w.t = lane & 3;
  w.warp = warp;
  w.has_col = w.gq < 3 * p.M;
  w.lu = w.wu0;
  w.cur = -1;
  w.seg0 = 0;
  const int8_t* xcol = xq + ((int64_t)(w.gq / 3) * ng * 3 + w.gq % 3) * 64 + 16 * w.t;

  // weights do not depend on the previous kernel: request them first
  uint32_t ca0[GD_UB][4], cb0[GD_UB][4], ca1[GD_UB][4], cb1[GD_UB][4];
  uint2 sa0 = make_uint2(0, 0), sb0 = sa0, sa1 = sa0, sb1 = sa0;
  if (w.wu0 < w.wu1) {
    gd_load_quad<EPI, VEC>(p, w, ca0, cb0, sa0, sb0);
    gd_load_quad<EPI, VEC>(p, w, ca1, cb1, sa1, sb1);
  }
  pdl_wait();  // activations and tickets below are written by earlier kernels
  if (ncu == 0) return;  // uniform across the CTA
  if constexpr (XSRC == GD_X_RMS) gd_stage_rms(p, xq, fcol, scr);
  else gd_stage_f32(p, xq, fcol);

  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (w.wu0 < w.wu1) {
    for (int u0 = w.wu0; u0 < w.wu1; u0 += 2 * GD_UB) {
      gd_compute_quad<EPI>(p, xcol, fcol, red, w, u0, acc, ca0, cb0, sa0, sb0);
      if (u0 + 2 * GD_UB < w.wu1) gd_load_quad<EPI, VEC>(p, w, ca0, cb0, sa0, sb0);
      if (u0 + GD_UB >= w.wu1) break;
      gd_compute_quad<EPI>(p, xcol, fcol, red, w, u0 + GD_UB, acc, ca1, cb1, sa1, sb1);
      if (u0 + 3 * GD_UB < w.wu1) gd_load_quad<EPI, VEC>(p, w, ca1, cb1, sa1, sb1);
    }
  }
  if (w.cur >= 0) gd_flush<EPI>(p, red, w, w.cur, w.seg0, w.wu1, acc);  // whole warp: shuffles
  __syncthreads();

  // tiles shared by warps: sum the warp partials in warp order; tiles also
  // shared by other CTAs become this CTA's partial slot
  constexpr int RP = (EPI == EPI_SWIGLU) ? 8 : 16;
  const int t_lo = cu0 / ng, t_hi = (cu1 - 1) / ng;
  const int nitems = (t_hi - t_lo + 1) * RP * p.M;
  bool wrote_part = false;
  for (int idx = threadIdx.x; idx < nitems; idx += GD_THREADS) {
    const int m = idx % p.M, r = (idx / p.M) % RP, ctl = t_lo + idx / (p.M * RP);
    const int tu0 = max(cu0, ctl * ng), tu1 = min(cu1, (ctl + 1) * ng);
    const int wa = gd_warp_of(tu0, cu0, ncu), wb = gd_warp_of(tu1 - 1, cu0, ncu);
    const bool cta_whole = tu0 == ctl * ng && tu1 == (ctl + 1) * ng;
    if (wa == wb && cta_whole) continue;  // finished in registers
    float v = 0.f, vu = 0.f;
    for (int ww = wa; ww <= wb; ++ww) {
      const int w0 = gd_wu0(ww, cu0, ncu);
      if (w0 == gd_wu0(ww + 1, cu0, ncu)) continue;  // empty warp range
      const float* rw = red + (ww * 2 + (ctl == w0 / ng ? 0 : 1)) * 16 * GD_MB;
      v += rw[r * GD_MB + m];
      if constexpr (EPI == EPI_SWIGLU) vu += rw[(r + 8) * GD_MB + m];
    }
    if (cta_whole) {
      gd_store<EPI>(p, ctl, r, m, v, vu);
    } else {
      float* slot = p.part + ((int64_t)ctl * GD_SL + (c - gd_cta_of(p.U, ctl * ng, G))) * 16 * GD_MB;
      slot[r * GD_MB + m] = v;
      if constexpr (EPI == EPI_SWIGLU) slot[(r + 8) * GD_MB + m] = vu;
      wrote_part = true;
    }
  }
  // tiles shared by CTAs (at most the first and the last of this range):
  // the last CTA to arrive sums the slots in CTA order and finishes the tile
  const bool split_lo = cu0 % ng != 0 || (cu1 < (t_lo + 1) * ng);
  const bool split_hi = t_hi != t_lo && cu1 % ng != 0;
  (void)wrote_part;
  if (!split_lo && !split_hi) return;
  // the CTA's partial stores happen before the barrier; thread 0 then
  // publishes them with a gpu-scope fence ahead of the ticket increment, and
  // the last CTA's fence after the increment orders its reads of the others
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
#pragma unroll
    for (int side = 0; side < 2; ++side) {
      const int tl = side == 0 ? t_lo : t_hi;
      const bool mine = side == 0 ? split_lo : split_hi;
      s_last[side] = 0;
      if (mine) {
        const int cf = gd_cta_of(p.U, tl * ng, G), cl = gd_cta_of(p.U, (tl + 1) * ng - 1, G);
        s_last[side] = atomicAdd(p.ticket + tl, 1) == cl - cf;
      }
    }
    __threadfence();
  }
  __syncthreads();
#pragma unroll
  for (int side = 0; side < 2; ++side) {
    if (!s_last[side]) continue;
    const int tl = side == 0 ? t_lo : t_hi;
    const int cf = gd_cta_of(p.U, tl * ng, G), cl = gd_cta_of(p.U, (tl + 1) * ng - 1, G);
    const float* base = p.part + (int64_t)tl * GD_SL * 16 * GD_MB;
    for (int idx = threadIdx.x; idx < RP * p.M; idx += GD_THREADS) {
      const int m = idx % p.M, r = idx / p.M;
      float v = 0.f, vu = 0.f;
      for (int s = 0; s <= cl - cf; ++s) {
        if (gd_cu0(p.U, cf + s, G) == gd_cu0(p.U, cf + s + 1, G)) continue;  // empty CTA range: no slot
        v += __ldcg(base + (int64_t)s * 16 * GD_MB + r * GD_MB + m);
        if constexpr (EPI == EPI_SWIGLU) vu += __ldcg(base + (int64_t)s * 16 * GD_MB + (r + 8) * GD_MB + m);
      }
      gd_store<EPI>(p, tl, r, m, v, vu);
    }
    if (threadIdx.x == 0) p.ticket[tl] = 0;  // ready for the next launch
  }
}

// ------------------------------------------------------------------ host side
template <int EPI, int VEC, int XSRC>
static int gd_attr(int smem) {
  Q8_CUDA(cudaFuncSetAttribute(k_gemv_d<EPI, VEC, XSRC>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  return Q8_OK;
}

constexpr int GD_SMEM_MAX = 100 * 1024;  // two CTAs per SM

static int gd_init() {
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  Q8_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  if (done[dev & 63]) return Q8_OK;
  Q8_TRY((gd_attr<EPI_STORE, 16, GD_X_F32>(GD_SMEM_MAX)));
  Q8_TRY((gd_attr<EPI_ADD, 16, GD_X_F32>(GD_SMEM_MAX)));
  Q8_TRY((gd_attr<EPI_SWIGLU, 16, GD_X_F32>(GD_SMEM_MAX)));
  Q8_TRY((gd_attr<EPI_STORE, 16, GD_X_RMS>(GD_SMEM_MAX)));
  Q8_TRY((gd_attr<EPI_SWIGLU, 16, GD_X_RMS>(GD_SMEM_MAX)));
  Q8_TRY((gd_attr<EPI_STORE, 8, GD_X_F32>(GD_SMEM_MAX)));
  Q8_TRY((gd_attr<EPI_ADD, 8, GD_X_F32>(GD_SMEM_MAX)));
  Q8_TRY((gd_attr<EPI_SWIGLU, 8, GD_X_F32>(GD_SMEM_MAX)));
  Q8_TRY((gd_attr<EPI_STORE, 8, GD_X_RMS>(GD_SMEM_MAX)));
  Q8_TRY((gd_attr<EPI_SWIGLU, 8, GD_X_RMS>(GD_SMEM_MAX)));
  done[dev & 63] = true;
  return Q8_OK;
}

// Shape / alignment limits of the digit GEMV (else the caller uses the
// split-f16 kernels).
bool gemv_d_supported(int M, int K, int N, bool rms, const void* W) {
  if (M < 1 || M > GD_MB || K % 256 != 0 || N < 1) return false;
  if (((uintptr_t)W & 15) != 0) return false;
  if ((size_t)M * K * 3 + (size_t)(K / 64) * 32 + 16 > (size_t)GD_SMEM_MAX) return false;
  if (rms && (K > 4096 || M * (K / 64) > 2 * GD_GIT)) return false;
  return true;
}

// Scratch per device: split-tile partials and tickets (tickets zero at rest).
// Growing it never frees the previous buffers: CUDA graphs captured earlier
// (decode steps of any context on the device) keep their pointers, so the old
// buffers stay allocated until the process exits.  The scratch is shared by
// every context and op-level call on the device: launches that use it must
// not run concurrently (the library's model calls run on one stream per
// context; contexts on one device must not decode at the same time on
// different streams).
struct GdScratch {
  float* part = nullptr;
  int* ticket = nullptr;
  int tiles = 0;
};
static GdScratch g_gd[64];
static std::mutex g_gd_mu;

static int gd_scratch(int tiles, float** part, int** ticket) {
  int dev = 0;
  Q8_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_gd_mu);
  GdScratch& s = g_gd[dev & 63];
  if (s.tiles < tiles) {
    // grown only outside stream capture (the first calls of a shape run
    // eagerly); the old buffers are retired, not freed
    s.part = nullptr;
    s.ticket = nullptr;
    s.tiles = 0;
    const int nt = std::max(tiles, 16384);
    if (cudaMalloc(&s.part, (size_t)nt * GD_SL * 16 * GD_MB * 4) != cudaSuccess ||
        cudaMalloc(&s.ticket, (size_t)nt * 4) != cudaSuccess || cudaMemset(s.ticket, 0, (size_t)nt * 4) != cudaSuccess) {
      cudaGetLastError();
      set_error("gemv_d: scratch allocation failed");
      return Q8_ERR_OOM;
    }
    s.tiles = nt;
  }
  *part = s.part;
  *ticket = s.ticket;
  return Q8_OK;
}

// Q8_GD=0 keeps decode GEMVs on the split-f16 kernels (A/B comparisons).
bool gemv_d_enabled() {
  static const bool on = [] {
    const char* e = getenv("Q8_GD");
    return !(e && e[0] == '0');
  }();
  return on;
}

int gemv_d_prepare(int max_tiles) {
  Q8_TRY(gd_init());
  float* part;
  int* ticket;
  return gd_scratch(max_tiles, &part, &ticket);
}

template <int EPI, int XSRC>
static int gd_launch_vec(int vec, int grid, int smem, cudaStream_t st, const GdParams& p) {
  if (vec == 16) return launch_pdl("k_gemv_d", k_gemv_d<EPI, 16, XSRC>, dim3(grid), dim3(GD_THREADS), smem, st, p);
  return launch_pdl("k_gemv_d", k_gemv_d<EPI, 8, XSRC>, dim3(grid), dim3(GD_THREADS), smem, st, p);
}

// y = x . W^T (epi STORE / ADD / SWIGLU).  rms: x = RMSNorm(h) * nw, else x.
int gemv_d_launch(int epi, bool rms, const float* x, int64_t ldx, const float* h, int64_t ldh, const uint16_t* nw,
                  float eps, int M, int K, const void* W, int N, float* y, int64_t ldy, __half* ys, cudaStream_t st) {
  Q8_CHECK_ARG(gemv_d_supported(M, K, N, rms, W), "gemv_d: unsupported shape");
  Q8_TRY(gd_init());
  GdParams p{};
  p.W = (const uint8_t*)W;
  p.rb = q8_row_bytes(K);
  p.K = K;
  p.N = N;
  p.ng = K / 64;
  p.T = epi == EPI_SWIGLU ? ceil_div(N, 8) : ceil_div(N, 16);
  p.U = p.T * p.ng;
  p.M = M;
  p.x = x;
  p.ldx = ldx;
  p.h = h;
  p.ldh = ldh;
  p.nw = nw;
  p.eps = eps;
  p.y = y;
  p.ldy = ldy;
  p.ys = ys;
  Q8_TRY(gd_scratch(p.T, &p.part, &p.ticket));
  const int smem = (int)((((size_t)M * K * 3 + 15) & ~(size_t)15) + (size_t)(K / 64) * 32);
  static const int per_sm = [] {
    const char* e = getenv("Q8_GD_CTAS");  // CTAs per SM (1: the next kernel's CTAs can be co-resident)
    return e ? std::max(1, std::min(2, atoi(e))) : 2;
  }();
  // Q8_GD_BALANCED=1: quad-balanced ranges with tiles shared by CTAs
  static const bool balanced = getenv("Q8_GD_BALANCED") != nullptr;
  int G;
  if (!balanced) {
    // whole tiles per CTA, equal counts: G = ceil(T / ceil(T / Gmax))
    const int gmax = per_sm * num_sms();
    const int k = ceil_div(p.T, gmax);
    G = ceil_div(p.T, k);
    p.aligned = 1;
  } else {
    G = std::min(per_sm * num_sms(), p.U / 4);
    // a tile may be shared by at most GD_SL CTAs (its partial slots): with at
    // least qmin quads per CTA a tile of qt quads spans <= ceil((qt-1)/qmin)+1
    const int qt = p.ng / 4, need = ceil_div(qt - 1, GD_SL - 1);
    if (need > 0) G = std::max(1, std::min(G, (p.U / 4) / need));
  }
  const int vec = (q8_row_bytes(K) % 16 == 0 && (K / 32) % 16 == 0) ? 16 : 8;
  if (rms) {
    if (epi == EPI_SWIGLU) return gd_launch_vec<EPI_SWIGLU, GD_X_RMS>(vec, G, smem, st, p);
    return gd_launch_vec<EPI_STORE, GD_X_RMS>(vec, G, smem, st, p);
  }
  if (epi == EPI_SWIGLU) return gd_launch_vec<EPI_SWIGLU, GD_X_F32>(vec, G, smem, st, p);
  if (epi == EPI_ADD) return gd_launch_vec<EPI_ADD, GD_X_F32>(vec, G, smem, st, p);
  return gd_launch_vec<EPI_STORE, GD_X_F32>(vec, G, smem, st, p);
}

}  // namespace q8
