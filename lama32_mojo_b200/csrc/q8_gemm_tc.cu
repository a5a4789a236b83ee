// Prefill Q8 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Replaces k_mm_q8 / mm_q8_op for large token counts (src/llama_q8.mojo:54-141)
// and, with the SwiGLU epilogue, the gate/up GEMM + k_swiglu_mul pair
// (src/llama_common.mojo:476):
//   y[m, n] (+)= sum_k x16[m, k] * f16(q[n, k] * s[n, k/64])
//
// Tile: 128 weight rows (MMA M) x BN tokens (MMA N: 64, 128 or 256), K in steps
// of 64 (one quantization group).  Warp roles (320 threads):
//   warp 0     TMA producer: two int8 code boxes [64 rows x 64 B] (no swizzle)
//              and the f16 activation box [BN tokens x 128 B] (128 B swizzle)
//              into a 4-stage ring; completion counted in bytes on full[s].
//   warps 2-9  two groups of 4 converter warps, alternating k-tiles: dequantize
//              codes x f16 group scale -> f16 (one rounding of the exact
//              product) into the K-major 128 B-swizzled layout the tensor core
//              reads; fence to the async proxy; arrive conv[s].  Group scales
//              are fetched 8 k-tiles (one uint4 per row) ahead.
//   warp 1     allocates BN TMEM columns; one lane issues 4 x
//              tcgen05.mma.kind::f16 (K = 16 each, f32 accumulate in TMEM) per
//              stage and commits the stage back to empty[s].
// Epilogue (warps 2-9; each owns the 32 TMEM lanes = weight rows of its
// quadrant, the two groups split the token columns): tcgen05.ld.32x32b, then
// store / accumulate y[token][row] (consecutive lanes -> consecutive rows:
// coalesced).  SwiGLU tiles hold 64
// gate rows in lanes 0-63 and the matching up rows in lanes 64-127; the up
// quadrants hand their values to the gate quadrants through shared memory.
//
// Every barrier wait is bounded (mbar_wait): a lost completion records
// Q8_ERR_TIMEOUT in the device error word instead of hanging, and the CTA
// still releases its TMEM.  No load uses cluster multicast.
#include "q8_kernels.h"

#include <cuda.h>

#include <mutex>

namespace q8 {

constexpr int TC_BM = 128, TC_BK = 64;
constexpr int TC_CODES = TC_BM * TC_BK;  // 8 KB int8
constexpr int TC_A = TC_BM * TC_BK * 2;  // 16 KB f16, SW128

struct TcParams {
  const uint8_t* W;  // packed rows (group scales read from here)
  int64_t rb;        // packed row bytes
  int K, N, M;       // N: output rows (SwiGLU: pairs F; W holds 2F rows)
  float* y;          // f32 output [M][ldy] (nullable for SwiGLU)
  int64_t ldy;
  __half* y16;       // SwiGLU only: f16 copy of the output [M][ld16]
  int64_t ld16;
  int64_t y16lo;     // > 0: also the f16 remainder a - f16(a), at y16 + y16lo
  int ksplit;        // K split across gridDim.z CTAs (1: none)
  float* ws;         // split partials [tile][ksplit][TC_BM][BN]
  int* tickets;      // [tile], zero at rest
};

// split-K semaphore: release this CTA's partial stores (made visible to the
// calling thread by a barrier), acquire the other CTAs'
__device__ __forceinline__ int tc_ticket_add(int* t) {
  int old;
  asm volatile("fence.acq_rel.gpu;\n\tatom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(t) : "memory");
  return old;
}

// barrier 3 over the 8 converter / epilogue warps
__device__ __forceinline__ void epi_bar_all() { asm volatile("bar.sync 3, 256;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Shared-memory matrix descriptor, K-major with 128 B swizzle: start >> 4,
// LBO 16 B (ignored for swizzled K-major), SBO 1024 B (8 rows x 128 B),
// descriptor version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(const void* smem_ptr) {
  const uint64_t addr = smem_u32(smem_ptr);
  return ((addr >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void tc_mma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Named barrier of one 4-warp epilogue group (ids 1 and 2).
__device__ __forceinline__ void epi_bar(int grp) { asm volatile("bar.sync %0, 128;" ::"r"(grp + 1) : "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 int8 codes (one uint4) times the f16 group scale -> 16 f16 values.
// Bytes are biased to u8, placed as the low mantissa byte of 1024.0h and the
// 1152.0h bias removed: exact integers q, then one rounding of q * s.  With
// LO the rounding remainder q*s - f16(q*s) is produced too (one fused
// multiply-add: exact whenever it is an f16 normal, i.e. hi + lo = q*s to
// ~2^-22 relative for the scales of quantized weights).
template <bool LO>
__device__ __forceinline__ void dequant16x(uint4 c, __half2 s2, uint32_t (&h)[8], uint32_t (&l)[8]) {
  const uint32_t w[4] = {c.x ^ 0x80808080u, c.y ^ 0x80808080u, c.z ^ 0x80808080u, c.w ^ 0x80808080u};
  const uint32_t k1152 = 0x64806480u;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t lo = __byte_perm(w[j], 0x64646464u, 0x5140), hi = __byte_perm(w[j], 0x64646464u, 0x5342);
    const __half2 qa = __hsub2(*reinterpret_cast<__half2*>(&lo), *reinterpret_cast<const __half2*>(&k1152));
    const __half2 qb = __hsub2(*reinterpret_cast<__half2*>(&hi), *reinterpret_cast<const __half2*>(&k1152));
    const __half2 a = __hmul2(qa, s2);
    const __half2 b = __hmul2(qb, s2);
    h[2 * j] = *reinterpret_cast<const uint32_t*>(&a);
    h[2 * j + 1] = *reinterpret_cast<const uint32_t*>(&b);
    if constexpr (LO) {
      const __half2 ra = __hfma2(qa, s2, __hneg2(a));
      const __half2 rb = __hfma2(qb, s2, __hneg2(b));
      l[2 * j] = *reinterpret_cast<const uint32_t*>(&ra);
      l[2 * j + 1] = *reinterpret_cast<const uint32_t*>(&rb);
    }
  }
}

__device__ __forceinline__ void dequant16(uint4 c, __half2 s2, uint32_t (&h)[8]) {
  const uint32_t w[4] = {c.x ^ 0x80808080u, c.y ^ 0x80808080u, c.z ^ 0x80808080u, c.w ^ 0x80808080u};
  const uint32_t k1152 = 0x64806480u;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t lo = __byte_perm(w[j], 0x64646464u, 0x5140), hi = __byte_perm(w[j], 0x64646464u, 0x5342);
    __half2 a = __hsub2(*reinterpret_cast<__half2*>(&lo), *reinterpret_cast<const __half2*>(&k1152));
    __half2 b = __hsub2(*reinterpret_cast<__half2*>(&hi), *reinterpret_cast<const __half2*>(&k1152));
    a = __hmul2(a, s2);
    b = __hmul2(b, s2);
    h[2 * j] = *reinterpret_cast<uint32_t*>(&a);
    h[2 * j + 1] = *reinterpret_cast<uint32_t*>(&b);
  }
}

// Shared-memory bytes of one pipeline stage and of the whole ring for a
// token tile of BN.
// X (split operands): A and B each hold a hi and a lo tile.
template <int BN, bool X>
struct TcCfg {
  static constexpr int A = TC_A * (X ? 2 : 1);       // f16 weight tiles, SW128
  static constexpr int B1 = BN * TC_BK * 2;          // one f16 activation box, SW128
  static constexpr int B = B1 * (X ? 2 : 1);
  static constexpr int STAGE = A + B + TC_CODES;     // A | B | codes
  // An even stage count: converter group g owns the stages of k-tiles kt = g
  // (mod 2), so no group ever waits on a stage's mbarrier more than one phase
  // ahead (a parity wait cannot tell phase r from phase r + 2).
  static constexpr int S = X ? 2 : 4;
  static constexpr int SMEM = S * STAGE + 1024;      // + alignment slack
  static_assert(S % 2 == 0, "converter groups alternate k-tiles: the ring needs an even stage count");
  static_assert(STAGE % 1024 == 0, "stage must keep 1024 B alignment for SW128");
  static_assert(SMEM <= 227 * 1024, "ring exceeds shared memory");
};

// 8 group scales (one uint4 of a packed row's scale block) -> scale of k-tile
// 2*jj + grp.  jj comes from an unrolled loop (resolved at compile time); grp
// (0/1) picks the f16 in the word.
__device__ __forceinline__ __half pick_scale(uint4 b, int jj, int grp) {
  const uint32_t w = jj == 0 ? b.x : jj == 1 ? b.y : jj == 2 ? b.z : b.w;
  return __ushort_as_half((unsigned short)(grp ? (w >> 16) : (w & 0xFFFFu)));
}

template <int EPI, int BN, bool X>
__global__ void __launch_bounds__(320, 1) k_gemm_q8_tc(const __grid_constant__ CUtensorMap tm_codes,
                                                       const __grid_constant__ CUtensorMap tm_x,
                                                       const __grid_constant__ CUtensorMap tm_xlo, TcParams p) {
  using Cfg = TcCfg<BN, X>;
  constexpr int S = Cfg::S;
  extern __shared__ uint8_t smem_raw[];
  // 1024 B alignment of the shared-window address (the swizzle atom)
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ __align__(8) uint64_t full[S], conv[S], empty[S], accf;
  __shared__ uint32_t tmem_base;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // token tiles vary fastest: CTAs resident together share one weight tile
  const int m0 = blockIdx.x * BN;
  const int r0 = blockIdx.y * (EPI == EPI_SWIGLU ? TC_BM / 2 : TC_BM);  // first output row (pair)
  // weight rows of the two 64-row code boxes
  const int rowA = r0, rowB = (EPI == EPI_SWIGLU) ? p.N + r0 : r0 + 64;
  // K range of this CTA: whole blocks of 8 k-tiles (one uint4 of group scales)
  const int nkb = p.K / (8 * TC_BK);
  const int kb0 = (int)(((int64_t)blockIdx.z * nkb) / gridDim.z), kb1 = (int)(((int64_t)(blockIdx.z + 1) * nkb) / gridDim.z);
  const int kt0 = 8 * kb0, nk = 8 * (kb1 - kb0);  // k-tiles [kt0, kt0 + nk)
  __shared__ int s_last;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);  // the 4 warps of the converter group that owns stage s
      mbar_init(&empty[s], 1);
    }
    mbar_init(&accf, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      for (int lk = 0; lk < nk; ++lk) {
        const int kt = kt0 + lk, s = lk % S;
        const uint32_t ph = (lk / S) & 1;
        mbar_wait(&empty[s], ph ^ 1);
        uint8_t* st = smem + s * Cfg::STAGE;
        mbar_arrive_expect_tx(&full[s], TC_CODES + Cfg::B);
        tma_load_2d(st + Cfg::A + Cfg::B, &tm_codes, kt * TC_BK, rowA, &full[s]);
        tma_load_2d(st + Cfg::A + Cfg::B + TC_CODES / 2, &tm_codes, kt * TC_BK, rowB, &full[s]);
        tma_load_2d(st + Cfg::A, &tm_x, kt * TC_BK, m0, &full[s]);
        if constexpr (X) tma_load_2d(st + Cfg::A + Cfg::B1, &tm_xlo, kt * TC_BK, m0, &full[s]);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    // instruction descriptor: f32 accumulate, A = B = f16, both K-major,
    // N = BN (bits 17-22: N >> 3), M = 128 (bits 24-28: M >> 4)
    const uint32_t idesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
    if (lane == 0) {
      for (int lk = 0; lk < nk; ++lk) {
        const int s = lk % S;
        const uint32_t ph = (lk / S) & 1;
        mbar_wait(&full[s], ph);
        mbar_wait(&conv[s], ph);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        uint8_t* st = smem + s * Cfg::STAGE;
        const uint64_t da = sw128_desc(st), db = sw128_desc(st + Cfg::A);
#pragma unroll
        for (int k = 0; k < TC_BK / 16; ++k) {  // K = 16 -> 32 B further inside the swizzle atom
          tc_mma_f16(tmem, da + 2 * k, db + 2 * k, idesc, (lk | k) != 0);
          if constexpr (X) {
            // hi x lo and lo x hi; lo x lo is below the f32 accumulation error
            const uint64_t dal = sw128_desc(st + TC_A), dbl = sw128_desc(st + Cfg::A + Cfg::B1);
            tc_mma_f16(tmem, da + 2 * k, dbl + 2 * k, idesc, 1u);
            tc_mma_f16(tmem, dal + 2 * k, db + 2 * k, idesc, 1u);
          }
        }
        tc_commit(&empty[s]);
      }
      tc_commit(&accf);
    }
  } else {
    // ---------------- converters: two groups of 4 warps; group g converts the
    // k-tiles kt = g (mod 2), so each group has two MMA periods per tile
    const int grp = (warp - 2) >> 2;
    const int ct = threadIdx.x - 64 - 128 * grp;  // 0..127 within the group
    // item it of thread ct: A row (it*128 + ct) >> 2, 16-code chunk (it*128 + ct) & 3
    const uint4* srow[4];
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int row = (it * 128 + ct) >> 2;
      int n;
      bool ok;
      if constexpr (EPI == EPI_SWIGLU) {
        ok = r0 + (row & 63) < p.N;
        n = (row < 64 ? rowA : rowB) + (row & 63);
      } else {
        n = r0 + row;
        ok = n < p.N;
      }
      srow[it] = ok ? reinterpret_cast<const uint4*>(p.W + (int64_t)n * p.rb) : nullptr;
    }
    const uint4 zero4 = make_uint4(0, 0, 0, 0);
    uint4 snext[4];
#pragma unroll
    for (int it = 0; it < 4; ++it) snext[it] = srow[it] ? __ldg(srow[it] + kb0) : zero4;
    for (int kb = kb0; kb < kb1; ++kb) {
      // scales of k-tiles 8kb..8kb+7 (one uint4 per row); fetch the next block
      uint4 sblk[4];
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        sblk[it] = snext[it];
        snext[it] = (srow[it] && kb + 1 < kb1) ? __ldg(srow[it] + kb + 1) : zero4;
      }
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int lk = 8 * (kb - kb0) + 2 * jj + grp;
        const int s = lk % S;
        const uint32_t ph = (lk / S) & 1;
        __half sc[4];
#pragma unroll
        for (int it = 0; it < 4; ++it) sc[it] = pick_scale(sblk[it], jj, grp);
        mbar_wait(&full[s], ph);
        uint8_t* st = smem + s * Cfg::STAGE;
        const uint8_t* codes = st + Cfg::A + Cfg::B;
        uint4 c[4];
#pragma unroll
        for (int it = 0; it < 4; ++it) {
          const int idx = it * 128 + ct;
          c[it] = *reinterpret_cast<const uint4*>(codes + (idx >> 2) * TC_BK + (idx & 3) * 16);
        }
#pragma unroll
        for (int it = 0; it < 4; ++it) {
          const int idx = it * 128 + ct;
          const int row = idx >> 2, chunk = idx & 3;
          uint32_t h[8], l[8];
          dequant16x<X>(c[it], __halves2half2(sc[it], sc[it]), h, l);
          // 16 f16 = logical 16-byte chunks 2*chunk and 2*chunk+1 of the 128 B row
          uint8_t* arow = st + row * 128;
          const int o0 = ((2 * chunk) ^ (row & 7)) << 4, o1 = ((2 * chunk + 1) ^ (row & 7)) << 4;
          *reinterpret_cast<uint4*>(arow + o0) = make_uint4(h[0], h[1], h[2], h[3]);
          *reinterpret_cast<uint4*>(arow + o1) = make_uint4(h[4], h[5], h[6], h[7]);
          if constexpr (X) {
            *reinterpret_cast<uint4*>(arow + TC_A + o0) = make_uint4(l[0], l[1], l[2], l[3]);
            *reinterpret_cast<uint4*>(arow + TC_A + o1) = make_uint4(l[4], l[5], l[6], l[7]);
          }
        }
        fence_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
      }
    }
    // ---------------- epilogue: this warp's TMEM lanes are A rows 32q..32q+31;
    // group g stores token columns [g*BN/2, (g+1)*BN/2)
    mbar_wait(&accf, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int q = warp & 3;
    const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
    const int cbeg = grp * (BN / 2), cend = cbeg + BN / 2;
    // split K: every CTA parks its f32 tile; the last CTA of the tile (ticket)
    // sums the parked tiles in split order and runs the epilogue below
    const int tile = blockIdx.x + gridDim.x * blockIdx.y;
    const int arow = 32 * q + lane;  // accumulator row = TMEM lane
    float* wst = p.ksplit > 1 ? p.ws + (int64_t)tile * p.ksplit * TC_BM * BN : nullptr;
    bool run_epi = true;
    if (p.ksplit > 1) {
#pragma unroll 1
      for (int c0 = cbeg; c0 < cend; c0 += 32) {
        float v[32];
        tmem_ld32(tq + (uint32_t)c0, v);
        float4* dst = reinterpret_cast<float4*>(wst + ((int64_t)blockIdx.z * TC_BM + arow) * BN + c0);
#pragma unroll
        for (int j = 0; j < 8; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      }
      epi_bar_all();
      if (threadIdx.x == 64) s_last = tc_ticket_add(&p.tickets[tile]) == p.ksplit - 1;
      epi_bar_all();
      run_epi = s_last != 0;
      if (run_epi && threadIdx.x == 64) p.tickets[tile] = 0;  // ready for the next launch
    }
    // accumulator columns c0..c0+31 of this thread's row: TMEM, or the sum of
    // the parked split tiles in split order
    auto fetch = [&](int c0, float (&v)[32]) {
      if (p.ksplit <= 1) {
        tmem_ld32(tq + (uint32_t)c0, v);
        return;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = 0.f;
      for (int z = 0; z < p.ksplit; ++z) {
        const float4* src = reinterpret_cast<const float4*>(wst + ((int64_t)z * TC_BM + arow) * BN + c0);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 t = __ldcg(src + j);
          v[4 * j] += t.x;
          v[4 * j + 1] += t.y;
          v[4 * j + 2] += t.z;
          v[4 * j + 3] += t.w;
        }
      }
    };
    if (run_epi) {
    if constexpr (EPI == EPI_SWIGLU) {
      // every MMA has completed: stage memory is free for the hand-off
      float* xch = reinterpret_cast<float*>(smem) + grp * (64 * 33);  // [64 rows][33] per group
      const int pr = r0 + 32 * (q & 1) + lane;
#pragma unroll 1
      for (int c0 = cbeg; c0 < cend; c0 += 32) {
        float v[32];
        fetch(c0, v);
        if (q >= 2) {
#pragma unroll
          for (int j = 0; j < 32; ++j) xch[(32 * (q - 2) + lane) * 33 + j] = v[j];
        }
        epi_bar(grp);
        if (q < 2 && pr < p.N) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = m0 + c0 + j;
            if (m < p.M) {
              const float a = silu_mul(v[j], xch[(32 * q + lane) * 33 + j]);
              if (p.y) p.y[(int64_t)m * p.ldy + pr] = a;
              if (p.y16) {
                const __half hi = __float2half_rn(a);
                p.y16[(int64_t)m * p.ld16 + pr] = hi;
                if (p.y16lo) p.y16[p.y16lo + (int64_t)m * p.ld16 + pr] = __float2half_rn(a - __half2float(hi));
              }
            }
          }
        }
        epi_bar(grp);
      }
    } else {
      const int n = r0 + 32 * q + lane;
#pragma unroll 1
      for (int c0 = cbeg; c0 < cend; c0 += 32) {
        float v[32];
        fetch(c0, v);
        if (n < p.N) {
          float* col = p.y + (int64_t)(m0 + c0) * p.ldy + n;
          const int mcnt = min(32, p.M - (m0 + c0));
          if constexpr (EPI == EPI_ADD) {
            // all 32 residual reads in flight before the first store (the
            // stores may alias them, so the compiler would serialize them)
            float old[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) old[j] = j < mcnt ? col[(int64_t)j * p.ldy] : 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < mcnt) col[(int64_t)j * p.ldy] = old[j] + v[j];
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < mcnt) col[(int64_t)j * p.ldy] = v[j];
          }
        }
      }
    }
    }  // run_epi
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN) : "memory");
  }
}

// ---------------------------------------------------------------- host side
typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled_t encode_fn() {
  static PFN_encodeTiled_t fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_encodeTiled_t)f;
    else
      cudaGetLastError();
  });
  return fn;
}

// 2-D tensor map over `rows` rows of `inner` elements (dtype 0: u8, 1: u16,
// 2: f32), `row_bytes` apart; box box_inner x box_rows, optionally with the
// 128 B swizzle.
int tensor_map_2d(CUtensorMap* m, int dtype, const void* base, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                  uint32_t box_inner, uint32_t box_rows, bool swizzle128) {
  PFN_encodeTiled_t enc = encode_fn();
  if (!enc) {
    set_error("tensor map: cuTensorMapEncodeTiled unavailable");
    return Q8_ERR_CUDA;
  }
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t es[2] = {1, 1};
  const CUtensorMapDataType dt = dtype == 0 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT16
                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUresult r = enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("tensor map: encode failed (%d)", (int)r);
    return Q8_ERR_CUDA;
  }
  return Q8_OK;
}

// 2-D tensor map over `rows` rows of `inner` f32 elements, `row_bytes` apart
// (the decode attention's K pool); box box_inner x box_rows, 128 B swizzle.
int tensor_map_f32_rows(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                        uint32_t box_inner, uint32_t box_rows) {
  PFN_encodeTiled_t enc = encode_fn();
  if (!enc) {
    set_error("tensor map: cuTensorMapEncodeTiled unavailable");
    return Q8_ERR_CUDA;
  }
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("tensor map: encode failed (%d)", (int)r);
    return Q8_ERR_CUDA;
  }
  return Q8_OK;
}

template <int EPI, int BN, bool X>
static int tc_attr() {
  Q8_CUDA(cudaFuncSetAttribute(k_gemm_q8_tc<EPI, BN, X>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               TcCfg<BN, X>::SMEM));
  return Q8_OK;
}

template <bool X>
static int tc_attr_all() {
  Q8_TRY((tc_attr<EPI_STORE, 64, X>()));
  Q8_TRY((tc_attr<EPI_ADD, 64, X>()));
  Q8_TRY((tc_attr<EPI_SWIGLU, 64, X>()));
  Q8_TRY((tc_attr<EPI_STORE, 128, X>()));
  Q8_TRY((tc_attr<EPI_ADD, 128, X>()));
  Q8_TRY((tc_attr<EPI_SWIGLU, 128, X>()));
  Q8_TRY((tc_attr<EPI_STORE, 256, X>()));
  Q8_TRY((tc_attr<EPI_ADD, 256, X>()));
  Q8_TRY((tc_attr<EPI_SWIGLU, 256, X>()));
  return Q8_OK;
}

// split-K workspace per device: up to TC_WS_TILES parked 128 x 128 f32 tiles
constexpr int TC_WS_TILES = 320;
static float* g_tc_ws[64];
static int* g_tc_tickets[64];

static int tc_init() {
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  Q8_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  if (done[dev & 63]) return Q8_OK;
  Q8_TRY(tc_attr_all<false>());
  Q8_TRY(tc_attr_all<true>());
  cudaError_t e = cudaMalloc(&g_tc_ws[dev & 63], (size_t)TC_WS_TILES * TC_BM * 128 * 4);
  if (e == cudaSuccess) e = cudaMalloc(&g_tc_tickets[dev & 63], (size_t)TC_WS_TILES * 4);
  if (e == cudaSuccess) e = cudaMemset(g_tc_tickets[dev & 63], 0, (size_t)TC_WS_TILES * 4);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("gemm_tc: split-K workspace allocation failed: %s", cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? Q8_ERR_OOM : Q8_ERR_CUDA;
  }
  done[dev & 63] = true;
  return Q8_OK;
}

int gemm_tc_prepare() { return tc_init(); }

template <int BN, bool X>
static void tc_launch(int epi, dim3 grid, const CUtensorMap& tmc, const CUtensorMap& tmx, const CUtensorMap& tmxl,
                      const TcParams& p, cudaStream_t st) {
  constexpr int sm = TcCfg<BN, X>::SMEM;
  if (epi == EPI_STORE) k_gemm_q8_tc<EPI_STORE, BN, X><<<grid, 320, sm, st>>>(tmc, tmx, tmxl, p);
  else if (epi == EPI_ADD) k_gemm_q8_tc<EPI_ADD, BN, X><<<grid, 320, sm, st>>>(tmc, tmx, tmxl, p);
  else k_gemm_q8_tc<EPI_SWIGLU, BN, X><<<grid, 320, sm, st>>>(tmc, tmx, tmxl, p);
}

bool gemm_tc_supported(int K, const void* W, const __half* x16, int64_t ld16) {
  return K > 0 && K % 512 == 0 && ((uintptr_t)W & 15) == 0 && x16 && ((uintptr_t)x16 & 15) == 0 && ld16 >= K &&
         (ld16 * 2) % 16 == 0 && encode_fn() != nullptr;
}

// Split operands (activation hi/lo planes, weight hi/lo tiles, three MMAs)
// unless Q8_TC_FAST=1: single f16 operands, about 2^-12 relative per product.
bool gemm_tc_exact() {
  static const bool exact = [] {
    const char* e = getenv("Q8_TC_FAST");
    return !(e && e[0] == '1');
  }();
  return exact;
}

static int tc_x_map(PFN_encodeTiled_t enc, CUtensorMap* m, const __half* x16, int64_t ld16, int M, int K, int bn) {
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)(ld16 * 2)};
  cuuint32_t box[2] = {TC_BK, (cuuint32_t)bn};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void*)x16, dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("gemm_tc: activation tensor map encode failed (%d)", (int)r);
    return Q8_ERR_CUDA;
  }
  return Q8_OK;
}

int gemm_tc_launch(int epi, const __half* x16, int64_t ld16, int64_t x16lo, int M, int K, const void* W, int N,
                   float* y, int64_t ldy, __half* y16, int64_t ldy16, int64_t y16lo, cudaStream_t st) {
  if (M <= 0 || N <= 0) return Q8_OK;
  Q8_CHECK_ARG(gemm_tc_supported(K, W, x16, ld16),
               "gemm_tc: unsupported operands (K=%d must be a multiple of 512; 16-byte aligned W and x)", K);
  Q8_CHECK_ARG(epi == EPI_SWIGLU ? (y || y16) : y != nullptr, "gemm_tc: no output");
  Q8_CHECK_ARG(epi != EPI_SWIGLU || !y16 || (((uintptr_t)y16 & 1) == 0 && ldy16 >= N), "gemm_tc: bad y16");
  Q8_CHECK_ARG(x16lo >= 0 && (x16lo * 2) % 16 == 0, "gemm_tc: lo plane must be 16-byte aligned");
  Q8_TRY(tc_init());
  PFN_encodeTiled_t enc = encode_fn();
  const int64_t rb = q8_row_bytes(K);
  const int wrows = epi == EPI_SWIGLU ? 2 * N : N;
  const bool X = x16lo > 0;
  // 256-token tiles halve the dequantization work per MMA; decode batches of
  // <= 64 tokens take 64-token tiles (half the MMA work of a mostly empty 128)
  const int bn = M >= 256 ? 256 : (M <= 64 ? 64 : 128);
  CUtensorMap tmc, tmx, tmxl;
  {
    // codes of every row: K bytes after the K/32 bytes of f16 group scales
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)wrows};
    cuuint64_t strides[1] = {(cuuint64_t)rb};
    cuuint32_t box[2] = {TC_BK, TC_BM / 2};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(&tmc, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)((const uint8_t*)W + K / 32), dims, strides, box,
                     es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("gemm_tc: code tensor map encode failed (%d)", (int)r);
      return Q8_ERR_CUDA;
    }
  }
  Q8_TRY(tc_x_map(enc, &tmx, x16, ld16, M, K, bn));
  Q8_TRY(tc_x_map(enc, &tmxl, X ? x16 + x16lo : x16, ld16, M, K, bn));
  TcParams p{(const uint8_t*)W, rb, K, N, M, y, ldy, y16, ldy16, y16lo, 1, nullptr, nullptr};
  dim3 grid(ceil_div(M, bn), epi == EPI_SWIGLU ? ceil_div(N, TC_BM / 2) : ceil_div(N, TC_BM));
  // small batches leave SMs idle: split K (whole 8-tile scale blocks) until
  // the tiles cover the SMs; the last CTA of a tile sums the parts in order
  {
    const int ntile = (int)(grid.x * grid.y), nkb = K / (8 * TC_BK);
    int ks = 1;
    if (bn <= 128 && ntile < num_sms()) ks = std::min(nkb, std::max(1, num_sms() / ntile));
    while (ks > 1 && ntile * ks > TC_WS_TILES) --ks;
    if (ks > 1) {
      int dev = 0;
      Q8_CUDA(cudaGetDevice(&dev));
      p.ksplit = ks;
      p.ws = g_tc_ws[dev & 63];
      p.tickets = g_tc_tickets[dev & 63];
      grid.z = ks;
    }
  }
  if (X && bn == 256) tc_launch<256, true>(epi, grid, tmc, tmx, tmxl, p, st);
  else if (X && bn == 64) tc_launch<64, true>(epi, grid, tmc, tmx, tmxl, p, st);
  else if (X) tc_launch<128, true>(epi, grid, tmc, tmx, tmxl, p, st);
  else if (bn == 256) tc_launch<256, false>(epi, grid, tmc, tmx, tmxl, p, st);
  else if (bn == 64) tc_launch<64, false>(epi, grid, tmc, tmx, tmxl, p, st);
  else tc_launch<128, false>(epi, grid, tmc, tmx, tmxl, p, st);
  return launch_check("k_gemm_q8_tc");
}

int tc_min_tokens() {
  static const int v = [] {
    const char* e = getenv("Q8_TC_MIN");
    // the tensor-core GEMM (64-token tiles, split K) beats the split-f16
    // GEMV from 16 tokens, as in the model's decode batches
    return e ? std::max(1, atoi(e)) : kTcDecodeMinTokens;
  }();
  return v;
}

int gemm_tc_error_word(int** out) {
  Q8_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(out), g_q8_device_error));
  return Q8_OK;
}

int gemm_tc_poll_error() {
  int v = 0;
  Q8_CUDA(cudaMemcpyFromSymbol(&v, g_q8_device_error, sizeof(int)));
  if (v == 0) return Q8_OK;
  const int z = 0;
  Q8_CUDA(cudaMemcpyToSymbol(g_q8_device_error, &z, sizeof(int)));
  set_error("k_gemm_q8_tc: a pipeline barrier wait timed out (device status %d)", v);
  return v;
}

}  // namespace q8

extern "C" int q8_device_status(void) {
  Q8_CUDA(cudaDeviceSynchronize());
  const int a = q8::gemm_tc_poll_error();
  const int b = q8::attn_dec_poll_error();
  return a != 0 ? a : b;
}
