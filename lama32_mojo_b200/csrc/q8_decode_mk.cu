// Persistent decode step: one cooperative launch runs every layer of a
// decode step for B <= 8 tokens (one per sequence).
//
// Replaces, for small token batches, the per-op dispatch chain of
// run_layer_q8 (src/llama_q8.mojo:144-230) and the model shell's forward
// (qwen3_mojo/src/qwen_q8.mojo:126-162): embed -> L x [RMSNorm, q|k|v,
// QK-norm + RoPE + KV append, GQA attention, o_proj + residual, RMSNorm,
// gate|up + SwiGLU, down + residual] -> final RMSNorm -> lm_head -> argmax.
//
// Why one launch: at batch 1 every per-layer matrix is small (17-120 MB for
// Llama-3.1-8B, 3-18 us at HBM speed), so separate kernels pay their launch,
// their serialized activation staging and their ramp/tail on every op.  Here
// one CTA per SM loops over the phases of the step; phases are separated by
// a grid barrier, and before arriving at each barrier a CTA asks L2 to fetch
// the weight rows of its next GEMV (cp.async.bulk.prefetch.L2), so HBM keeps
// streaming while the grid synchronizes.
//
// GEMV phases split the (16-row tile x 64-group) units of a matrix evenly
// over all warps of the grid: CTA c owns units [c*U/G, (c+1)*U/G) and its 16
// warps split that range again.  A warp computes a run of units with the
// split-f16 m16n8k16 MMA of the standalone GEMV; tiles a warp covers whole are
// finished in registers, tiles shared by warps are summed in shared memory in
// warp order, and tiles shared by CTAs are written to per-CTA partial slots
// that the consuming phase sums in CTA order.  Every sum has a fixed order:
// results do not depend on timing.  Residual adds fold into the next phase's
// RMSNorm prologue (each CTA normalizes the whole row itself and writes back
// its slice of the updated residual, ping-ponging between two buffers).
//
// Every wait is bounded: a barrier that does not complete within ~1 s sets
// the device status word, after which all later waits return at once; the
// host reports Q8_ERR_TIMEOUT.  No load uses cluster multicast.
#include "q8_decode_mk.h"
#include "q8_gemv_core.cuh"
#include "q8_kernels.h"

#include <algorithm>
#include <mutex>

namespace q8 {

// ------------------------------------------------------------------ unit ranges
struct MkGemv {
  const uint8_t* W;
  int64_t rb;
  int K, N;     // N output rows (SwiGLU: gate/up pairs; W holds 2N rows)
  int T, ng;    // 16-row tiles (8-pair tiles for SwiGLU), 64-groups per row
  int U;        // T * ng units
  int aligned;  // CTA ranges on tile boundaries (epilogue needs whole tiles)
};

__host__ __device__ inline MkGemv mk_desc(const uint8_t* W, int K, int N, bool swiglu, bool aligned) {
  MkGemv g;
  g.W = W;
  g.rb = (int64_t)K / 32 + K;
  g.K = K;
  g.N = N;
  g.ng = K / 64;
  g.T = swiglu ? (N + 7) / 8 : (N + 15) / 16;
  g.U = g.T * g.ng;
  g.aligned = aligned ? 1 : 0;
  return g;
}

// First unit of CTA c's range.  Ranges are whole quads of 4 units (4
// consecutive groups of one tile: K % 256 == 0 makes ng a multiple of 4), so a
// 4-unit register batch never crosses a tile.  U * G < 2^31 is checked on the
// host, so the products stay in 32 bits.
__host__ __device__ inline int mk_cu0(const MkGemv& g, int c, int G) {
  if (g.aligned) return g.ng * (int)(((unsigned)c * (unsigned)g.T) / (unsigned)G);
  return 4 * (int)(((unsigned)c * (unsigned)(g.U / 4)) / (unsigned)G);
}

// Whether some CTA ranges are empty (fewer quads / tiles than CTAs).
__host__ __device__ inline bool mk_sparse(const MkGemv& g, int G) { return g.aligned ? g.T < G : g.U / 4 < G; }

// The CTA whose range holds unit x (largest c with mk_cu0(c) <= x).
__host__ __device__ inline int mk_cta_of(const MkGemv& g, int x, int G) {
  if (g.aligned) return (int)((((unsigned)(x / g.ng) + 1u) * (unsigned)G - 1u) / (unsigned)g.T);
  return (int)((((unsigned)(x / 4) + 1u) * (unsigned)G - 1u) / (unsigned)(g.U / 4));
}

// ------------------------------------------------------------------ small helpers
__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int ld_volatile_i32(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// Grid barrier over a monotonic arrival counter (zeroed before the launch).
// Bounded: gives up after ~2^31 cycles, or at once when the status word is
// already set, so a fault never turns into a hang.
__device__ __forceinline__ void mk_barrier(const MkParams& P, unsigned int& target) {
  target += gridDim.x;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(P.bar, 1u);
    if (ld_volatile_i32(P.status) == 0) {
      const long long t0 = clock64();
      while (ld_acquire_u32(P.bar) < target) {
        if (ld_volatile_i32(P.status) != 0) break;
        if (clock64() - t0 > (1ll << 31)) {
          atomicExch(P.status, Q8_ERR_TIMEOUT);
          break;
        }
      }
    }
    __threadfence();
    if (P.ts && blockIdx.x == 0) {  // phase trace: time at which this barrier completed
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      P.ts[target / gridDim.x] = t;
    }
  }
  __syncthreads();
}

// Sub-phase trace (CTA 0, thread 0): P.ts2[phase * 4 + j].
__device__ __forceinline__ void mk_mark(const MkParams& P, int phase, int j) {
  if (P.ts2 && blockIdx.x == 0 && threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    P.ts2[phase * 4 + j] = t;
  }
}

// Ask L2 to fetch this CTA's weight rows of the next GEMV (at most `budget`
// bytes): rows are contiguous, so a few bulk prefetches cover them.
__device__ __forceinline__ void mk_prefetch_rows(const uint8_t* base, int64_t row0, int64_t row1, int64_t rb,
                                                 int64_t budget) {
  if (row1 <= row0 || budget <= 0) return;
  uint64_t a0 = (uint64_t)(base + row0 * rb), a1 = (uint64_t)(base + row1 * rb);
  a0 = (a0 + 15) & ~15ull;  // inside the matrix: round the start up, the end down
  a1 &= ~15ull;
  if (a1 > a0 + (uint64_t)budget) a1 = (a0 + (uint64_t)budget) & ~15ull;
  constexpr uint64_t kChunk = 32768;
  const int lane = threadIdx.x & 31;
  for (uint64_t a = a0 + (uint64_t)lane * kChunk; a < a1; a += 32 * kChunk) {
    const uint32_t n = (uint32_t)((a1 - a) < kChunk ? (a1 - a) : kChunk);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(n) : "memory");
  }
}

__device__ __forceinline__ void mk_prefetch(const MkGemv& g, bool swiglu, int budget) {
  if (threadIdx.x >= 32 || budget <= 0) return;
  const int G = gridDim.x, c = blockIdx.x;
  const int cu0 = mk_cu0(g, c, G), cu1 = mk_cu0(g, c + 1, G);
  if (cu0 >= cu1) return;
  const int t0 = cu0 / g.ng, t1 = (cu1 - 1) / g.ng;
  if (swiglu) {
    const int64_t p0 = (int64_t)t0 * 8, p1 = min((int64_t)g.N, (int64_t)(t1 + 1) * 8);
    mk_prefetch_rows(g.W, p0, p1, g.rb, budget / 2);
    mk_prefetch_rows(g.W, g.N + p0, g.N + p1, g.rb, budget / 2);
  } else {
    mk_prefetch_rows(g.W, (int64_t)t0 * 16, min((int64_t)g.N, (int64_t)(t1 + 1) * 16), g.rb, budget);
  }
}

// Sum of the cross-CTA partial slots of output row n (token b) of a GEMV
// phase with unit-balanced ranges, in CTA order.
__device__ __forceinline__ float mk_psum(const MkGemv& g, const float* part, int b, int n, int G) {
  const int t = n / 16;
  const int cf = mk_cta_of(g, t * g.ng, G), cl = mk_cta_of(g, (t + 1) * g.ng - 1, G);
  float v = 0.f;
  if (!mk_sparse(g, G)) {  // every CTA range is non-empty
    for (int s = 0; s <= cl - cf; ++s) v += __ldcg(part + ((int64_t)s * MK_BMAX + b) * g.N + n);
  } else {         // fewer units than CTAs: CTAs with empty ranges wrote no slot
    for (int s = 0; s <= cl - cf; ++s)
      if (mk_cu0(g, cf + s, G) != mk_cu0(g, cf + s + 1, G))
        v += __ldcg(part + ((int64_t)s * MK_BMAX + b) * g.N + n);
  }
  return v;
}

// ------------------------------------------------------------------ staging prologues
// The GEMV input of a phase is staged per CTA in shared memory as int8
// digits (see mk_digits16): xq [B][group][digit][64] int8 and the column
// factors fcol [group][8] f32.  Prologues issue all their loads before
// computing, so each costs about one L2 round trip.
struct MkStage {
  int8_t* xq;
  float* fcol;
};

__device__ __forceinline__ MkStage mk_stage_layout(uint8_t* smem, int B, int K) {
  MkStage st;
  st.xq = reinterpret_cast<int8_t*>(smem);
  st.fcol = reinterpret_cast<float*>(smem + (((size_t)B * K * 3 + 15) & ~(size_t)15));
  return st;
}

// x = RMSNorm(src) * w (k_rmsnorm_w, src/llama_common.mojo:197-225): src is
// the Q8 embedding row of each token (first layer) or h_in + the partial
// slots of the producing GEMV (its 16-row tiles are 16-element chunks here);
// CTA c also writes its chunks of src to h_out (the updated residual).
struct MkSrc {
  const uint8_t* embed;  // non-null: dequantized embedding rows of P.ids
  const float* h_in;
  const MkGemv* pg;      // producer of `part` (null: no partials)
  const float* part;
};

__device__ __forceinline__ void mk_add4(float (&v)[16], int i, float4 a) {
  v[4 * i] += a.x;
  v[4 * i + 1] += a.y;
  v[4 * i + 2] += a.z;
  v[4 * i + 3] += a.w;
}

__device__ __forceinline__ void mk_src_chunk(const MkParams& P, const MkSrc& s, int b, int ch, int G,
                                             float (&v)[16]) {
  const int k0 = ch * 16;
  if (s.embed) {
    // k_embed_gather_q8 (src/llama_q8.mojo:96-109): f32(int8) * f32(f16 scale)
    const uint8_t* r = s.embed + (int64_t)__ldg(P.ids + b) * ((int64_t)P.H / 32 + P.H);
    const float sc = __half2float(__ldg(reinterpret_cast<const __half*>(r) + k0 / 64));
    const uint2 q0 = __ldg(reinterpret_cast<const uint2*>(r + P.H / 32 + k0));
    const uint2 q1 = __ldg(reinterpret_cast<const uint2*>(r + P.H / 32 + k0 + 8));
    const uint32_t w[4] = {q0.x, q0.y, q1.x, q1.y};
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = (float)(int8_t)((w[i / 4] >> (8 * (i % 4))) & 0xFF) * sc;
    return;
  }
  const float4* hp = reinterpret_cast<const float4*>(s.h_in + (int64_t)b * P.H + k0);
  float4 a[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) a[i] = __ldcg(hp + i);
  int ns = 0;
  const float* pp = nullptr;
  int64_t sstride = 0;
  bool sparse = false;
  if (s.part) {
    const MkGemv& g = *s.pg;
    const int cf = mk_cta_of(g, ch * g.ng, G), cl = mk_cta_of(g, (ch + 1) * g.ng - 1, G);
    ns = cl - cf + 1;
    pp = s.part + (int64_t)b * g.N + k0;
    sstride = (int64_t)MK_BMAX * g.N;
    sparse = mk_sparse(g, G);  // CTAs with empty ranges wrote no slot
    if (sparse) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[4 * i] = a[i].x; v[4 * i + 1] = a[i].y; v[4 * i + 2] = a[i].z; v[4 * i + 3] = a[i].w;
      }
      for (int sl = 0; sl < ns; ++sl) {
        if (mk_cu0(g, cf + sl, G) == mk_cu0(g, cf + sl + 1, G)) continue;
#pragma unroll
        for (int i = 0; i < 4; ++i) mk_add4(v, i, __ldcg(reinterpret_cast<const float4*>(pp + sl * sstride) + i));
      }
      return;
    }
  }
  // slots 0 and 1 issued together with h (the common case), further slots after
  float4 p0[4], p1[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    p0[i] = ns > 0 ? __ldcg(reinterpret_cast<const float4*>(pp) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    p1[i] = ns > 1 ? __ldcg(reinterpret_cast<const float4*>(pp + sstride) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[4 * i] = a[i].x; v[4 * i + 1] = a[i].y; v[4 * i + 2] = a[i].z; v[4 * i + 3] = a[i].w;
  }
  if (ns > 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) mk_add4(v, i, p0[i]);
  }
  if (ns > 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) mk_add4(v, i, p1[i]);
  }
  for (int sl = 2; sl < ns; ++sl) {
#pragma unroll
    for (int i = 0; i < 4; ++i) mk_add4(v, i, __ldcg(reinterpret_cast<const float4*>(pp + sl * sstride) + i));
  }
}

// Activation digits.  A group of 64 values is x ~= e (a0 + a1/254 + a2/254^2)
// with e = max|x|/127, a0 = rint(x/e), a1 = rint(254 (x/e - a0)),
// a2 = rint(254 (254 (x/e - a0) - a1)): int8 digits, representation error
// <= 0.5/254^2 of e (~2^-24 of the group maximum).  Digit j of token m is B
// column 3m + j; fcol holds e/254^j per column (0 for unused columns).
//
// Work split: 4 lanes per (token, group), 16 values per lane, so a warp
// digitizes 8 groups at once; an item is (iteration, warp, lane / 4).
constexpr int MK_GPW = 8;                   // groups per warp per iteration
constexpr int MK_GIT = MK_GPW * MK_WARPS;   // groups per CTA per iteration

__device__ __forceinline__ void mk_digits16(const float (&v)[16], bool valid, int mm, int gi, int sq, int ng,
                                            const MkStage& st) {
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
  int8_t* dq = st.xq + ((int64_t)(mm * ng + gi) * 3) * 64 + 16 * sq;
#pragma unroll
  for (int j = 0; j < 3; ++j) *reinterpret_cast<uint4*>(dq + j * 64) = make_uint4(w[j][0], w[j][1], w[j][2], w[j][3]);
  if (sq < 3) st.fcol[gi * 8 + 3 * mm + sq] = sq == 0 ? e : (sq == 1 ? e / 254.0f : e / 64516.0f);
}

__device__ __forceinline__ void mk_fcol_zero(const MkStage& st, int B, int ng) {
  for (int i = threadIdx.x; i < ng * 8; i += MK_THREADS)
    if (i % 8 >= 3 * B) st.fcol[i] = 0.f;
}

// RMSNorm prologue: values stay in registers between the sum-of-squares pass
// and the digits (B * H / 64 <= 2 * MK_GIT is checked on the host).
// scr: >= MK_BMAX * (H / 16) + MK_BMAX floats.
template <int IT>
__device__ __noinline__ void mk_stage_rms_it(const MkParams& P, const MkSrc& s, float* h_out, const uint16_t* w,
                                const MkStage& st, float* scr) {
  const int G = gridDim.x, c = blockIdx.x, H = P.H, nch = H / 16, ng = H / 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sq = lane & 3;
  const int c0 = (int)(((unsigned)c * (unsigned)nch) / (unsigned)G);
  const int c1 = (int)(((unsigned)(c + 1) * (unsigned)nch) / (unsigned)G);
  float* inv = scr + MK_BMAX * nch;
  float v[IT][16];
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int item = it * MK_GIT + warp * MK_GPW + (lane >> 2);
    if (item < P.B * ng) {
      const int b = item / ng, ch = (item % ng) * 4 + sq;
      mk_src_chunk(P, s, b, ch, G, v[it]);
    }
  }
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int item = it * MK_GIT + warp * MK_GPW + (lane >> 2);
    if (item < P.B * ng) {
      const int b = item / ng, ch = (item % ng) * 4 + sq;
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) ss = fmaf(v[it][i], v[it][i], ss);
      scr[b * nch + ch] = ss;
      if (h_out && ch >= c0 && ch < c1) {
        float4* ho = reinterpret_cast<float4*>(h_out + (int64_t)b * H + ch * 16);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          ho[i] = make_float4(v[it][4 * i], v[it][4 * i + 1], v[it][4 * i + 2], v[it][4 * i + 3]);
      }
    }
  }
  __syncthreads();
  if (warp < P.B) {  // per-token sum of squares in chunk order
    float t = 0.f;
    for (int ch = lane; ch < nch; ch += 32) t += scr[warp * nch + ch];
    t = warp_sum(t);
    if (lane == 0) inv[warp] = 1.0f / sqrtf(t / (float)H + P.eps);
  }
  mk_fcol_zero(st, P.B, ng);
  __syncthreads();
#pragma unroll
  for (int it = 0; it < IT; ++it) {
    const int item = it * MK_GIT + warp * MK_GPW + (lane >> 2);
    const bool valid = item < P.B * ng;
    const int b = valid ? item / ng : 0, gi = valid ? item % ng : 0;
    if (valid) {
      const int k0 = gi * 64 + 16 * sq;
      const uint4 w0 = __ldg(reinterpret_cast<const uint4*>(w + k0));
      const uint4 w1 = __ldg(reinterpret_cast<const uint4*>(w + k0 + 8));
      const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      const float r = inv[b];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[it][2 * i] = __uint_as_float(ww[i] << 16) * v[it][2 * i] * r;
        v[it][2 * i + 1] = __uint_as_float(ww[i] & 0xFFFF0000u) * v[it][2 * i + 1] * r;
      }
    }
    mk_digits16(v[it], valid, b, gi, sq, ng, st);  // all lanes: the max is a shuffle
  }
  __syncthreads();
}

__device__ __forceinline__ void mk_stage_rms(const MkParams& P, const MkSrc& s, float* h_out, const uint16_t* w,
                                             const MkStage& st, float* scr) {
  if (P.B * (P.H / 64) <= MK_GIT) mk_stage_rms_it<1>(P, s, h_out, w, st, scr);
  else mk_stage_rms_it<2>(P, s, h_out, w, st, scr);
}

// f32 rows [B][K] written earlier in the launch -> digits, in rounds of two
// iterations whose loads are all issued before any digit is made.
__device__ __noinline__ void mk_stage_f32(const float* src, int B, int K, const MkStage& st) {
  constexpr int IT = 2;
  const int ng = K / 64, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sq = lane & 3;
  mk_fcol_zero(st, B, ng);
  for (int base = 0; base * MK_GIT < B * ng; base += IT) {
    float v[IT][16];
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int item = (base + it) * MK_GIT + warp * MK_GPW + (lane >> 2);
      if (item < B * ng) {
        const float4* sp = reinterpret_cast<const float4*>(src + (int64_t)item * 64 + 16 * sq);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 a = __ldcg(sp + i);
          v[it][4 * i] = a.x; v[it][4 * i + 1] = a.y; v[it][4 * i + 2] = a.z; v[it][4 * i + 3] = a.w;
        }
      }
    }
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int item = (base + it) * MK_GIT + warp * MK_GPW + (lane >> 2);
      const bool valid = item < B * ng;
      mk_digits16(v[it], valid, valid ? item / ng : 0, valid ? item % ng : 0, sq, ng, st);
    }
  }
  __syncthreads();
}

// ------------------------------------------------------------------ GEMV phase
enum { MK_PART = 0, MK_SWIGLU = 1, MK_LOGITS = 2 };

struct MkOut {
  float* part;     // MK_PART: slots [SL][MK_BMAX][N]
  float* act;      // MK_SWIGLU: f32 [B][N]
  float* logits;   // MK_LOGITS: [B][N]
};

// One finished output: row r of tile tl (SwiGLU: pair r with its up value).
template <int EPI>
__device__ __forceinline__ void mk_store(const MkGemv& g, const MkOut& o, int B, int slot, int tl, int r, int b,
                                         float v, float vu) {
  if (b >= B) return;
  if constexpr (EPI == MK_PART) {
    const int row = tl * 16 + r;
    if (row < g.N) o.part[((int64_t)slot * MK_BMAX + b) * g.N + row] = v;
  } else if constexpr (EPI == MK_SWIGLU) {
    const int pr = tl * 8 + r;
    if (pr < g.N) o.act[(int64_t)b * g.N + pr] = silu_mul(v, vu);
  } else {
    const int row = tl * 16 + r;
    if (row < g.N) o.logits[(int64_t)b * g.N + row] = v;
  }
}

template <int EPI>
__device__ __forceinline__ void mk_rows(const MkGemv& g, int tl, int gq, int& ra, int& rbw) {
  if constexpr (EPI == MK_SWIGLU) {
    const int pr = min(tl * 8 + gq, g.N - 1);
    ra = pr;
    rbw = g.N + pr;
  } else {
    ra = min(tl * 16 + gq, g.N - 1);
    rbw = min(tl * 16 + gq + 8, g.N - 1);
  }
}

// Warp ranges (whole quads) inside a CTA range of ncu units.
__device__ __forceinline__ int mk_warp_of(int x, int cu0, int ncu) {
  return (int)((((unsigned)((x - cu0) / 4) + 1u) * (unsigned)MK_WARPS - 1u) / (unsigned)(ncu / 4));
}

__device__ __forceinline__ int mk_wu0(int w, int cu0, int ncu) {
  return cu0 + 4 * (int)(((unsigned)(ncu / 4) * (unsigned)w) / (unsigned)MK_WARPS);
}

__device__ __forceinline__ void mk_imma(int d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

constexpr int MK_UB = 4;  // units per register batch = one quad (two batches in flight per warp)

// Per-warp state of the unit stream of one GEMV phase.
struct MkWarp {
  int wu0, wu1, ng, first_tile;
  int gq, t, warp;
  bool has_col;
  const int8_t* xcol;      // this lane's B column of the staged digits
  int lu;                  // next unit to load (quad-aligned)
  int cur, seg0;           // tile being accumulated, its first unit
};

// One quad: codes of rows g and g+8 for 4 groups, and their 4 + 4 group scales
// as two 8-byte loads.
template <int EPI, int VEC>
__device__ __forceinline__ void mk_load_quad(const MkGemv& g, MkWarp& w, uint32_t (&ca)[MK_UB][4],
                                             uint32_t (&cb)[MK_UB][4], uint2& sa, uint2& sb) {
  const int u = min(w.lu, w.wu1 - MK_UB);  // past the range: reload the last quad (unused)
  const int tl = u / w.ng, g0 = u % w.ng;
  int ra, rbw;
  mk_rows<EPI>(g, tl, w.gq, ra, rbw);
  const uint8_t* rowa = g.W + (int64_t)ra * g.rb;
  const uint8_t* rowb = g.W + (int64_t)rbw * g.rb;
  const uint8_t* pa = rowa + g.K / 32 + g0 * 64 + 16 * w.t;
  const uint8_t* pb = rowb + g.K / 32 + g0 * 64 + 16 * w.t;
#pragma unroll
  for (int q = 0; q < MK_UB; ++q) {
    load_codes16<VEC>(pa + q * 64, ca[q]);
    load_codes16<VEC>(pb + q * 64, cb[q]);
  }
  sa = __ldg(reinterpret_cast<const uint2*>(rowa) + g0 / 4);
  sb = __ldg(reinterpret_cast<const uint2*>(rowb) + g0 / 4);
  w.lu += MK_UB;
}

// Finished segment [s0, s1) of tile ftl: sum each token's three digit columns
// (held by the four t-lanes of the row) in column order; whole tiles are
// stored, shared ones parked in red (first segment slot 0, last slot 1).
template <int EPI>
__device__ __forceinline__ void mk_flush(const MkParams& P, const MkGemv& g, const MkOut& o, float* red,
                                         const MkWarp& w, int ftl, int s0, int s1, const float (&acc)[4]) {
  float c0[8], c1[8];
#pragma unroll
  for (int cc = 0; cc < 8; ++cc) {
    const int src = (w.gq << 2) | (cc >> 1);
    c0[cc] = __shfl_sync(0xffffffffu, acc[cc & 1], src);
    c1[cc] = __shfl_sync(0xffffffffu, acc[2 + (cc & 1)], src);
  }
  // lane t writes token t (<= 2 tokens per step on this path)
  const float a = w.t == 0 ? c0[0] + c0[1] + c0[2] : c0[3] + c0[4] + c0[5];
  const float bv = w.t == 0 ? c1[0] + c1[1] + c1[2] : c1[3] + c1[4] + c1[5];
  if (w.t >= 2) return;
  if (s0 == ftl * w.ng && s1 == (ftl + 1) * w.ng) {
    if constexpr (EPI == MK_SWIGLU) {
      mk_store<EPI>(g, o, P.B, 0, ftl, w.gq, w.t, a, bv);
    } else {
      mk_store<EPI>(g, o, P.B, 0, ftl, w.gq, w.t, a, 0.f);
      mk_store<EPI>(g, o, P.B, 0, ftl, w.gq + 8, w.t, bv, 0.f);
    }
  } else {
    float* rw = red + (w.warp * 2 + (ftl == w.first_tile ? 0 : 1)) * 16 * MK_BMAX;
    rw[w.gq * MK_BMAX + w.t] = a;
    rw[(w.gq + 8) * MK_BMAX + w.t] = bv;
  }
}

__device__ __forceinline__ float mk_scale(uint2 s, int q) {
  const uint32_t v = q < 2 ? s.x : s.y;
  return __half2float(__ushort_as_half((unsigned short)((q & 1) ? (v >> 16) : (v & 0xFFFFu))));
}

template <int EPI>
__device__ __forceinline__ void mk_compute_quad(const MkParams& P, const MkGemv& g, const MkStage& st,
                                                const MkOut& o, float* red, MkWarp& w, int u0, float (&acc)[4],
                                                const uint32_t (&ca)[MK_UB][4], const uint32_t (&cb)[MK_UB][4],
                                                uint2 sa, uint2 sb) {
  const int tl = u0 / w.ng, g0 = u0 % w.ng;
  if (tl != w.cur) {
    if (w.cur >= 0) mk_flush<EPI>(P, g, o, red, w, w.cur, w.seg0, u0, acc);
    w.cur = tl;
    w.seg0 = u0;
    acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
  }
#pragma unroll
  for (int q = 0; q < MK_UB; ++q) {
    uint4 bx = make_uint4(0, 0, 0, 0);
    if (w.has_col) bx = *reinterpret_cast<const uint4*>(w.xcol + (int64_t)(g0 + q) * 3 * 64);
    int d[4] = {0, 0, 0, 0};
    mk_imma(d, ca[q][0], cb[q][0], ca[q][1], cb[q][1], bx.x, bx.y);  // physical k 16t+0..7
    mk_imma(d, ca[q][2], cb[q][2], ca[q][3], cb[q][3], bx.z, bx.w);  // physical k 16t+8..15
    const float s0 = mk_scale(sa, q), s1 = mk_scale(sb, q);
    const float2 f = *reinterpret_cast<const float2*>(st.fcol + (g0 + q) * 8 + 2 * w.t);
    acc[0] = fmaf(__int2float_rn(d[0]), s0 * f.x, acc[0]);
    acc[1] = fmaf(__int2float_rn(d[1]), s0 * f.y, acc[1]);
    acc[2] = fmaf(__int2float_rn(d[2]), s1 * f.x, acc[2]);
    acc[3] = fmaf(__int2float_rn(d[3]), s1 * f.y, acc[3]);
  }
}

// Int8-digit GEMV over this CTA's unit range.  Per unit and lane: the 16
// int8 codes of rows g and g+8 at bytes [16t, 16t+16) of the group go to the
// tensor core unchanged (two m16n8k32 s8 MMAs; the k order inside a group is
// free for a dot product, and the digits use the same order), and the s32
// column partials are scaled in f32 by (f16 weight scale) x (e / 254^digit),
// the reference's association scale x group dot (src/llama_q8.mojo:76-83).
template <int EPI, int VEC>
__device__ void mk_gemv(const MkParams& P, const MkGemv& g, const MkStage& st, const MkOut& o, float* red, int ph) {
  mk_mark(P, ph, 0);
  const int G = gridDim.x, c = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cu0 = mk_cu0(g, c, G), cu1 = mk_cu0(g, c + 1, G), ncu = cu1 - cu0;
  const int ng = g.ng;
  MkWarp w;
  w.wu0 = mk_wu0(warp, cu0, ncu);
  w.wu1 = mk_wu0(warp + 1, cu0, ncu);
  w.ng = ng;
  w.first_tile = w.wu0 / ng;
  w.gq = lane >> 2;
  w.t = lane & 3;
  w.warp = warp;
  // B column of this lane = gq: token gq / 3, digit gq % 3 (unused columns read 0)
  w.has_col = w.gq < 3 * P.B;
  w.xcol = st.xq + ((int64_t)(w.gq / 3) * ng * 3 + w.gq % 3) * 64 + 16 * w.t;
  w.lu = w.wu0;
  w.cur = -1;
  w.seg0 = 0;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  uint32_t ca0[MK_UB][4], cb0[MK_UB][4], ca1[MK_UB][4], cb1[MK_UB][4];
  uint2 sa0, sb0, sa1, sb1;
  if (w.wu0 < w.wu1) {
    mk_load_quad<EPI, VEC>(g, w, ca0, cb0, sa0, sb0);
    mk_load_quad<EPI, VEC>(g, w, ca1, cb1, sa1, sb1);
    for (int u0 = w.wu0; u0 < w.wu1; u0 += 2 * MK_UB) {
      mk_compute_quad<EPI>(P, g, st, o, red, w, u0, acc, ca0, cb0, sa0, sb0);
      if (u0 + 2 * MK_UB < w.wu1) mk_load_quad<EPI, VEC>(g, w, ca0, cb0, sa0, sb0);
      if (u0 + MK_UB >= w.wu1) break;
      mk_compute_quad<EPI>(P, g, st, o, red, w, u0 + MK_UB, acc, ca1, cb1, sa1, sb1);
      if (u0 + 3 * MK_UB < w.wu1) mk_load_quad<EPI, VEC>(g, w, ca1, cb1, sa1, sb1);
    }
  }
  // the flush shuffles need the whole warp: every lane takes this branch together
  if (w.cur >= 0) mk_flush<EPI>(P, g, o, red, w, w.cur, w.seg0, w.wu1, acc);
  __syncthreads();
  mk_mark(P, ph, 1);

  // tiles shared by warps (or by CTAs): sum the warp partials in warp order
  if (ncu > 0) {
    constexpr int RP = (EPI == MK_SWIGLU) ? 8 : 16;
    const int t_lo = cu0 / ng, t_hi = (cu1 - 1) / ng;
    const int nitems = (t_hi - t_lo + 1) * RP * P.B;
    for (int idx = threadIdx.x; idx < nitems; idx += MK_THREADS) {
      const int b = idx % P.B, r = (idx / P.B) % RP, ctl = t_lo + idx / (P.B * RP);
      const int tu0 = max(cu0, ctl * ng), tu1 = min(cu1, (ctl + 1) * ng);
      const int wa = mk_warp_of(tu0, cu0, ncu), wb = mk_warp_of(tu1 - 1, cu0, ncu);
      const bool cta_whole = tu0 == ctl * ng && tu1 == (ctl + 1) * ng;
      if (wa == wb && cta_whole) continue;  // finished in registers
      float v = 0.f, vu = 0.f;
      for (int w = wa; w <= wb; ++w) {
        const int w0 = mk_wu0(w, cu0, ncu);
        if (w0 == mk_wu0(w + 1, cu0, ncu)) continue;  // empty warp range
        const float* rw = red + (w * 2 + (ctl == w0 / ng ? 0 : 1)) * 16 * MK_BMAX;
        v += rw[r * MK_BMAX + b];
        if constexpr (EPI == MK_SWIGLU) vu += rw[(r + 8) * MK_BMAX + b];
      }
      // only unit-balanced (MK_PART) phases share a tile between CTAs
      const int slot = cta_whole ? 0 : c - mk_cta_of(g, ctl * ng, G);
      mk_store<EPI>(g, o, P.B, slot, ctl, r, b, v, vu);
    }
  }

  if constexpr (EPI == MK_LOGITS) {
    // argmax over this CTA's logits rows, lowest index on ties
    // (k_argmax, src/llama_common.mojo:493-519), merged grid-wide as a packed
    // (order-preserving value bits, ~index) 64-bit atomicMax
    __syncthreads();
    __shared__ float s_bv[MK_WARPS];
    __shared__ int s_bi[MK_WARPS];
    if (ncu > 0) {
      const int r_lo = (cu0 / ng) * 16, r_hi = min(g.N, ((cu1 - 1) / ng + 1) * 16);
      for (int b = 0; b < P.B; ++b) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int row = r_lo + threadIdx.x; row < r_hi; row += MK_THREADS) {
          const float v = __ldcg(o.logits + (int64_t)b * g.N + row);
          if (v > bv || (v == bv && row < bi)) {
            bv = v;
            bi = row;
          }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
          if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
          }
        }
        if (lane == 0) {
          s_bv[warp] = bv;
          s_bi[warp] = bi;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
          for (int w = 1; w < MK_WARPS; ++w)
            if (s_bv[w] > bv || (s_bv[w] == bv && s_bi[w] < bi)) {
              bv = s_bv[w];
              bi = s_bi[w];
            }
          if (bi != 0x7fffffff) {
            const uint32_t u = __float_as_uint(bv);
            const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
            atomicMax(P.amax_key + b, ((unsigned long long)ord << 32) | (0xFFFFFFFFu - (uint32_t)bi));
          }
        }
        __syncthreads();
      }
    }
  }
  __syncthreads();  // red and the staging buffer are reused by the next phase
  mk_mark(P, ph, 2);
}

// ------------------------------------------------------------------ attention phase
// GQA attention of each step token over its paged KV (k_scores /
// k_softmax_rows / k_att_out, src/llama_common.mojo:402-473), with the RoPE +
// KV append of k_rope_qk_copy2 (:299-342) and Qwen3's QK-norm (k_rmsnorm2_w,
// :228-270) done by the task that owns the token's position.  Task = (token,
// kv head, context split): the CTA's 16 warps split the keys, merge in shared
// memory, and the last split to finish merges all splits (ticket counter).
template <int HD>
__device__ void mk_attention(const MkParams& P, const MkLayer& ly, const MkGemv& gqkv, uint8_t* smem, int ph) {
  constexpr int E = HD / 32, J = HD / 32;
  const int G = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Gq = P.nh / P.nkv;
  const int ntask = P.B * P.nkv * P.nsplit;
  float* qs = reinterpret_cast<float*>(smem);                 // [MK_GMAX][HD]
  float* sm_m = qs + MK_GMAX * HD;                            // [MK_WARPS][MK_GMAX]
  float* sm_l = sm_m + MK_WARPS * MK_GMAX;
  float* sm_o = sm_l + MK_WARPS * MK_GMAX;                    // [MK_WARPS][MK_GMAX][HD]
  float* s_w = sm_o + MK_WARPS * MK_GMAX * HD;                // [MK_GMAX][MK_MAXSPLIT]
  float* s_l = s_w + MK_GMAX * MK_MAXSPLIT;
  float* s_L = s_l + MK_GMAX * MK_MAXSPLIT;                   // [MK_GMAX]
  int* s_last = reinterpret_cast<int*>(s_L + MK_GMAX);
  const float qscale = 1.4426950408889634f / sqrtf((float)HD);  // log2(e)/sqrt(hd): exp2 domain

  for (int tk = blockIdx.x; tk < ntask; tk += G) {
    const int item = tk / P.nsplit, sp = tk % P.nsplit;
    const int b = item / P.nkv, kvh = item % P.nkv;
    const int p = __ldg(P.pos + b);
    const int kv_end = p + 1;
    const int per = (kv_end + P.nsplit - 1) / P.nsplit;
    const int k_lo = min(kv_end, sp * per), k_hi = min(kv_end, k_lo + per);
    const int32_t* btr = P.bt + (int64_t)__ldg(P.seq + b) * P.max_pages;
    const float fp = (float)p;

    // ---- q heads of this kv head (warps 0..Gq-1), new k/v (last warp)
    const bool own_new = p >= k_lo && p < k_hi;
    if (warp < Gq || (warp == MK_WARPS - 1 && own_new)) {
      const bool is_q = warp < Gq;
      const int row0 = is_q ? (kvh * Gq + warp) * HD : P.qd + kvh * HD;
      float v[J];
#pragma unroll
      for (int j = 0; j < J; ++j) v[j] = mk_psum(gqkv, P.pqkv, b, row0 + lane + 32 * j, G);
      const uint16_t* nw = is_q ? ly.q_norm : ly.k_norm;
      if (nw) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < J; ++j) ss = fmaf(v[j], v[j], ss);
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)HD + P.eps);
#pragma unroll
        for (int j = 0; j < J; ++j) v[j] = bf16_bits_to_f32(__ldg(nw + lane + 32 * j)) * v[j] * inv;
      }
#pragma unroll
      for (int j = 0; j < J / 2; ++j) {
        const int d = lane + 32 * j;
        float sn, cs;
        sincosf(fp * __ldg(P.inv_freq + d), &sn, &cs);
        const float x0 = v[j], x1 = v[j + J / 2];
        v[j] = x0 * cs - x1 * sn;
        v[j + J / 2] = x1 * cs + x0 * sn;
      }
      if (is_q) {
#pragma unroll
        for (int j = 0; j < J; ++j) qs[warp * HD + lane + 32 * j] = v[j] * qscale;
      } else {
        const int pg = __ldg(btr + p / P.page);
        const int64_t off = (((int64_t)pg * P.nkv + kvh) * P.page + (p % P.page)) * HD;
        const int vrow = P.qd + P.nkv * HD + kvh * HD;
#pragma unroll
        for (int j = 0; j < J; ++j) {
          ly.kp[off + lane + 32 * j] = v[j];
          ly.vp[off + lane + 32 * j] = mk_psum(gqkv, P.pqkv, b, vrow + lane + 32 * j, G);
        }
      }
    }
    __threadfence_block();
    __syncthreads();
    if (tk == (int)blockIdx.x) mk_mark(P, ph, 0);

    // ---- keys [k_lo, k_hi) split over the warps; online softmax per head
    const int wper = (k_hi - k_lo + MK_WARPS - 1) / MK_WARPS;
    const int w_lo = min(k_hi, k_lo + warp * wper), w_hi = min(k_hi, w_lo + wper);
    float q[MK_GMAX][E], o[MK_GMAX][E], m[MK_GMAX], l[MK_GMAX];
#pragma unroll
    for (int g = 0; g < MK_GMAX; ++g) {
      m[g] = -INFINITY;
      l[g] = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        o[g][e] = 0.f;
        q[g][e] = g < Gq ? qs[g * HD + lane * E + e] : 0.f;
      }
    }
    // two chunks of 4 keys in flight per warp: load the next while computing
    auto load = [&](int j0, float (&kr)[4][E], float (&vr)[4][E]) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int jj = min(j0 + u, w_hi - 1);
        const int64_t off =
            (((int64_t)__ldg(btr + jj / P.page) * P.nkv + kvh) * P.page + (jj % P.page)) * HD + lane * E;
        if constexpr (E == 4) {
          const float4 k4 = __ldcg(reinterpret_cast<const float4*>(ly.kp + off));
          const float4 v4 = __ldcg(reinterpret_cast<const float4*>(ly.vp + off));
          kr[u][0] = k4.x; kr[u][1] = k4.y; kr[u][2] = k4.z; kr[u][3] = k4.w;
          vr[u][0] = v4.x; vr[u][1] = v4.y; vr[u][2] = v4.z; vr[u][3] = v4.w;
        } else {
          const float2 k2 = __ldcg(reinterpret_cast<const float2*>(ly.kp + off));
          const float2 v2 = __ldcg(reinterpret_cast<const float2*>(ly.vp + off));
          kr[u][0] = k2.x; kr[u][1] = k2.y;
          vr[u][0] = v2.x; vr[u][1] = v2.y;
        }
      }
    };
    // online-softmax update of the Gq heads with 4 keys (exp2 domain)
    auto chunk = [&](int j0, const float (&kr)[4][E], const float (&vr)[4][E]) {
#pragma unroll
      for (int g = 0; g < MK_GMAX; ++g) {
        if (g >= Gq) break;
        float sc[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float d = 0.f;
#pragma unroll
          for (int e = 0; e < E; ++e) d = fmaf(q[g][e], kr[u][e], d);
          sc[u] = d;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
          for (int u = 0; u < 4; ++u) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], off);
        }
        float mx = m[g];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (j0 + u >= w_hi) sc[u] = -INFINITY;
          mx = fmaxf(mx, sc[u]);
        }
        const float corr = (m[g] == -INFINITY) ? 0.f : exp2f(m[g] - mx);
        float psum = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) o[g][e] *= corr;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float pz = (sc[u] == -INFINITY) ? 0.f : exp2f(sc[u] - mx);
          psum += pz;
#pragma unroll
          for (int e = 0; e < E; ++e) o[g][e] = fmaf(pz, vr[u][e], o[g][e]);
        }
        l[g] = l[g] * corr + psum;
        m[g] = mx;
      }
    };
    if (w_lo < w_hi) {
      float ka[4][E], va[4][E], kb[4][E], vb[4][E];
      load(w_lo, ka, va);
      for (int j0 = w_lo; j0 < w_hi; j0 += 8) {
        const int j1 = j0 + 4;
        if (j1 < w_hi) load(j1, kb, vb);
        chunk(j0, ka, va);
        if (j1 < w_hi) {
          if (j1 + 4 < w_hi) load(j1 + 4, ka, va);
          chunk(j1, kb, vb);
        }
      }
    }

    // ---- merge the warps
    if (tk == (int)blockIdx.x) mk_mark(P, ph, 1);
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g < MK_GMAX; ++g) {
        sm_m[warp * MK_GMAX + g] = m[g];
        sm_l[warp * MK_GMAX + g] = l[g];
      }
    }
#pragma unroll
    for (int g = 0; g < MK_GMAX; ++g) {
      if (g >= Gq) break;
#pragma unroll
      for (int e = 0; e < E; ++e) sm_o[(warp * MK_GMAX + g) * HD + lane * E + e] = o[g][e];
    }
    __syncthreads();
    const int W = Gq * HD + 2 * Gq;
    float* mypart = P.apart + ((int64_t)item * P.nsplit + sp) * W;
    for (int i = threadIdx.x; i < Gq * HD; i += MK_THREADS) {
      const int g = i / HD, d = i % HD;
      float M = -INFINITY;
      for (int w = 0; w < MK_WARPS; ++w) M = fmaxf(M, sm_m[w * MK_GMAX + g]);
      float L = 0.f, O = 0.f;
      if (M != -INFINITY) {
        for (int w = 0; w < MK_WARPS; ++w) {
          const float mw = sm_m[w * MK_GMAX + g];
          if (mw == -INFINITY) continue;
          const float f = exp2f(mw - M);
          L = fmaf(sm_l[w * MK_GMAX + g], f, L);
          O = fmaf(sm_o[(w * MK_GMAX + g) * HD + d], f, O);
        }
      }
      if (P.nsplit == 1) {
        P.ao[(int64_t)b * P.qd + (kvh * Gq + g) * HD + d] = L > 0.f ? O / L : 0.f;
      } else {
        mypart[i] = O;
        if (d == 0) {
          mypart[Gq * HD + g] = M;
          mypart[Gq * HD + Gq + g] = L;
        }
      }
    }
    if (P.nsplit > 1) {
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) *s_last = (atomicAdd(P.ticket + item, 1) == P.nsplit - 1);
      __syncthreads();
      if (*s_last) {
        __threadfence();
        const float* base = P.apart + (int64_t)item * P.nsplit * W;
        for (int idx = threadIdx.x; idx < Gq * P.nsplit; idx += MK_THREADS) {
          const int g = idx / P.nsplit, s2 = idx % P.nsplit;
          s_w[g * MK_MAXSPLIT + s2] = __ldcg(base + (int64_t)s2 * W + Gq * HD + g);
          s_l[g * MK_MAXSPLIT + s2] = __ldcg(base + (int64_t)s2 * W + Gq * HD + Gq + g);
        }
        __syncthreads();
        if (threadIdx.x < Gq) {
          const int g = threadIdx.x;
          float M = -INFINITY;
          for (int s2 = 0; s2 < P.nsplit; ++s2) M = fmaxf(M, s_w[g * MK_MAXSPLIT + s2]);
          float L = 0.f;
          for (int s2 = 0; s2 < P.nsplit; ++s2) {
            const float ms = s_w[g * MK_MAXSPLIT + s2];
            const float f = (M == -INFINITY || ms == -INFINITY) ? 0.f : exp2f(ms - M);
            s_w[g * MK_MAXSPLIT + s2] = f;
            L = fmaf(s_l[g * MK_MAXSPLIT + s2], f, L);
          }
          s_L[g] = L;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < Gq * HD; i += MK_THREADS) {
          const int g = i / HD;
          float O = 0.f;
          for (int s0 = 0; s0 < P.nsplit; s0 += 16) {  // 16 independent loads per round
            float pv[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) pv[u] = s0 + u < P.nsplit ? __ldcg(base + (int64_t)(s0 + u) * W + i) : 0.f;
#pragma unroll
            for (int u = 0; u < 16; ++u)
              if (s0 + u < P.nsplit) O = fmaf(pv[u], s_w[g * MK_MAXSPLIT + s0 + u], O);
          }
          const float L = s_L[g];
          P.ao[(int64_t)b * P.qd + kvh * Gq * HD + i] = L > 0.f ? O / L : 0.f;
        }
        if (threadIdx.x == 0) P.ticket[item] = 0;  // ready for the next launch
      }
    }
    __syncthreads();  // shared memory is reused by the next task
    if (tk == (int)blockIdx.x) mk_mark(P, ph, 2);
  }
}

// ------------------------------------------------------------------ the step kernel
template <int HD, int VEC>
__global__ void __launch_bounds__(MK_THREADS, 1) k_decode_step(MkParams P) {
  extern __shared__ __align__(16) uint8_t smem[];
  float* red = reinterpret_cast<float*>(smem + MK_XS_BYTES);
  float* scr = red;  // staging scratch: per-chunk sums of squares (red is idle then)
  unsigned int target = 0;
  if (blockIdx.x == 0 && threadIdx.x < MK_BMAX) P.amax_key[threadIdx.x] = 0ull;
  if (P.ts && blockIdx.x == 0 && threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    P.ts[0] = t;
  }
  const MkStage stH = mk_stage_layout(smem, P.B, P.H);
  const MkStage stQ = mk_stage_layout(smem, P.B, P.qd);
  const MkStage stF = mk_stage_layout(smem, P.B, P.F);

  MkGemv g_dn = mk_desc(nullptr, P.F, P.H, false, false);
  mk_prefetch(mk_desc(P.layers[0].qkv, P.H, P.nqkv, false, false), false, P.pf_bytes);
  const MkOut o_qkv{P.pqkv, nullptr, nullptr};
  const MkOut o_res{P.pres, nullptr, nullptr};
  const MkOut o_act{nullptr, P.act, nullptr};
  const MkOut o_lg{nullptr, nullptr, P.logits};

  for (int L = 0; L < P.L; ++L) {
    const MkLayer ly = P.layers[L];
    const MkGemv g_qkv = mk_desc(ly.qkv, P.H, P.nqkv, false, false);
    const MkGemv g_o = mk_desc(ly.o, P.qd, P.H, false, false);
    const MkGemv g_gu = mk_desc(ly.gu, P.H, P.F, true, true);
    // residual (+ previous down_proj partials) -> hB; x = RMSNorm -> q|k|v
    const MkSrc sA{L == 0 ? P.embed : nullptr, P.hA, L == 0 ? nullptr : &g_dn, L == 0 ? nullptr : P.pres};
    mk_stage_rms(P, sA, P.hB, ly.in_norm, stH, scr);
    mk_gemv<MK_PART, VEC>(P, g_qkv, stH, o_qkv, red, 5 * L);
    mk_prefetch(g_o, false, P.pf_bytes);
    mk_barrier(P, target);
    mk_attention<HD>(P, ly, g_qkv, smem, 5 * L + 1);
    mk_prefetch(g_gu, true, P.pf_bytes);
    mk_barrier(P, target);
    mk_stage_f32(P.ao, P.B, P.qd, stQ);
    mk_gemv<MK_PART, VEC>(P, g_o, stQ, o_res, red, 5 * L + 2);
    mk_barrier(P, target);
    // hB + o_proj partials -> hA; x = RMSNorm -> gate|up + SwiGLU
    const MkSrc sC{nullptr, P.hB, &g_o, P.pres};
    mk_stage_rms(P, sC, P.hA, ly.post_norm, stH, scr);
    mk_gemv<MK_SWIGLU, VEC>(P, g_gu, stH, o_act, red, 5 * L + 3);
    g_dn = mk_desc(ly.down, P.F, P.H, false, false);
    mk_prefetch(g_dn, false, P.pf_bytes);
    mk_barrier(P, target);
    mk_stage_f32(P.act, P.B, P.F, stF);
    mk_gemv<MK_PART, VEC>(P, g_dn, stF, o_res, red, 5 * L + 4);
    if (L + 1 < P.L) mk_prefetch(mk_desc(P.layers[L + 1].qkv, P.H, P.nqkv, false, false), false, P.pf_bytes);
    else mk_prefetch(mk_desc(P.lm_head, P.H, P.V, false, true), false, P.pf_bytes);
    mk_barrier(P, target);
  }
  // final RMSNorm of hA + last down_proj partials -> lm_head -> argmax
  const MkSrc sE{nullptr, P.hA, &g_dn, P.pres};
  mk_stage_rms(P, sE, nullptr, P.final_norm, stH, scr);
  mk_gemv<MK_LOGITS, VEC>(P, mk_desc(P.lm_head, P.H, P.V, false, true), stH, o_lg, red, 5 * P.L);
  mk_barrier(P, target);
  if (blockIdx.x == 0 && threadIdx.x < P.B)
    P.argmax[threadIdx.x] = (int32_t)(0xFFFFFFFFu - (uint32_t)(__ldcg(P.amax_key + threadIdx.x) & 0xFFFFFFFFull));
}

// ------------------------------------------------------------------ host side
int mk_slots(int K, int N, bool swiglu, bool aligned, int G) {
  const MkGemv g = mk_desc(nullptr, K, N, swiglu, aligned);
  if (aligned) return 1;
  int mx = 1;
  for (int t = 0; t < g.T; ++t)
    mx = std::max(mx, mk_cta_of(g, (t + 1) * g.ng - 1, G) - mk_cta_of(g, t * g.ng, G) + 1);
  return mx;
}

size_t mk_attn_part_floats(int nkv, int nsplit, int hd) {
  return (size_t)MK_BMAX * nkv * nsplit * (size_t)(MK_GMAX * hd + 2 * MK_GMAX);
}

int mk_smem_bytes() { return MK_SMEM; }

// Largest step batch (<= 2: the GEMV flush writes two tokens per quad) whose
// staged digits fit for every K and whose prologues fit their register
// iterations (RMSNorm: 2 x MK_GIT groups).
int mk_max_batch(int H, int qd, int F) {
  auto need = [](int B, int K) { return (((size_t)B * K * 3 + 15) & ~(size_t)15) + (size_t)(K / 64) * 32; };
  int b = 0;
  while (b < 2 && need(b + 1, H) <= MK_XS_BYTES && need(b + 1, qd) <= MK_XS_BYTES &&
         need(b + 1, F) <= MK_XS_BYTES && (b + 1) * (H / 64) <= 2 * MK_GIT)
    ++b;
  return b;
}

template <int HD, int VEC>
static int mk_attr() {
  Q8_CUDA(cudaFuncSetAttribute(k_decode_step<HD, VEC>, cudaFuncAttributeMaxDynamicSharedMemorySize, MK_SMEM));
  return Q8_OK;
}

static int mk_init() {
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  Q8_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  if (done[dev & 63]) return Q8_OK;
  Q8_TRY((mk_attr<64, 16>()));
  Q8_TRY((mk_attr<64, 8>()));
  Q8_TRY((mk_attr<128, 16>()));
  Q8_TRY((mk_attr<128, 8>()));
  done[dev & 63] = true;
  return Q8_OK;
}

template <int HD, int VEC>
static const void* mk_kernel() {
  return reinterpret_cast<const void*>(k_decode_step<HD, VEC>);
}

static const void* mk_pick(int hd, int vec) {
  if (hd == 64) return vec == 16 ? mk_kernel<64, 16>() : mk_kernel<64, 8>();
  return vec == 16 ? mk_kernel<128, 16>() : mk_kernel<128, 8>();
}

int mk_check_residency(int hd, int vec, int G, bool* ok) {
  *ok = false;
  if ((hd != 64 && hd != 128) || (vec != 16 && vec != 8)) return Q8_OK;
  Q8_TRY(mk_init());
  int dev = 0, coop = 0, per_sm = 0;
  Q8_CUDA(cudaGetDevice(&dev));
  Q8_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
  Q8_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mk_pick(hd, vec), MK_THREADS, MK_SMEM));
  *ok = coop != 0 && per_sm >= 1 && G <= per_sm * num_sms();
  return Q8_OK;
}

int mk_launch(const MkParams& p, int vec, int G, cudaStream_t st) {
  Q8_TRY(mk_init());
  Q8_CUDA(cudaMemsetAsync(p.bar, 0, sizeof(unsigned int), st));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(MK_THREADS);
  cfg.dynamicSmemBytes = MK_SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (p.hd == 64) {
    e = vec == 16 ? cudaLaunchKernelEx(&cfg, k_decode_step<64, 16>, p) : cudaLaunchKernelEx(&cfg, k_decode_step<64, 8>, p);
  } else {
    e = vec == 16 ? cudaLaunchKernelEx(&cfg, k_decode_step<128, 16>, p)
                  : cudaLaunchKernelEx(&cfg, k_decode_step<128, 8>, p);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("launch k_decode_step: %s", cudaGetErrorString(e));
    return Q8_ERR_CUDA;
  }
  return Q8_OK;
}

}  // namespace q8
