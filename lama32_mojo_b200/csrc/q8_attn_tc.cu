// Prefill attention on the tensor cores (mma.sync m16n8k16, f16 split operands).
//
// Replaces, for prompt chunks, k_scores + k_softmax_rows + k_att_out
// (src/llama_common.mojo:402-473): S = q.k / sqrt(hd) with the causal mask,
// row softmax, O = P.V, without a materialized score matrix.
//
// CTA = (query block, kv head, context split), 4 warps; the 64 rows of a CTA
// are (token, head) pairs of a query block and the G query heads that share
// the kv head (row r = token r / G, head r % G); warp w owns rows 16w..16w+15.
// Keys stream in tiles of 64: K and V rows (f32 in the paged cache) become
// f16 hi / lo planes (hi = f16(x), lo = f16(x - hi)) in shared memory, 16-byte
// chunks XOR-swizzled by row so that ldmatrix reads are conflict-free.
//   S  = Qh.Kh + Qh.Kl + Ql.Kh   (three MMAs per fragment; q is pre-scaled by
//                                 log2(e)/sqrt(hd): exp2-domain online softmax)
//   O += Ph.Vh + Ph.Vl + Pl.Vh   (P reused from the S accumulators as the A
//                                 operand, split the same way)
// Dropping only the lo.lo products leaves about 2^-22 relative error per
// product, i.e. f32-level results.  Row maxima are quad shuffles; row sums stay
// per thread until the end.  Splits write (o, m, l) partials in the layout of
// k_attn_combine (m in the natural-log domain).  Query blocks run longest
// first (they are issued in reverse) to shorten the causal tail.
#include "q8_kernels.h"

namespace q8 {

constexpr int ATC_ROWS = 64;     // query rows per CTA
constexpr int ATC_TK = 64;       // keys per tile
constexpr int ATC_THREADS = 128; // 4 warps x 16 rows

template <int HD>
struct AtcSmem {
  __half kh[ATC_TK * HD], kl[ATC_TK * HD], vh[ATC_TK * HD], vl[ATC_TK * HD];
  int qpos[ATC_ROWS];
};

// element (row, dim) of a swizzled [ATC_TK][HD] f16 plane
template <int HD>
__device__ __forceinline__ int atc_swz(int row, int dim) {
  return row * HD + ((((dim >> 3) ^ (row & 7))) << 3) + (dim & 7);
}

__device__ __forceinline__ void atc_ldsm_x4(uint32_t (&r)[4], const __half* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void atc_ldsm_x4_t(uint32_t (&r)[4], const __half* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void atc_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// (x0, x1) -> packed f16x2 hi and lo (lo = f16 of the remainder)
__device__ __forceinline__ void atc_split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
  const __half l0 = __float2half_rn(x0 - __half2float(h0)), l1 = __float2half_rn(x1 - __half2float(h1));
  hi = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
  lo = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
}

__device__ __forceinline__ void atc_write_out(const AttnArgs& a, int tok, int col, float v) {
  if (a.out32) a.out32[(int64_t)tok * a.ldo + col] = v;
  if (a.outxs) {
    __half hi, lo;
    split_f16(v, hi, lo);
    const int K = a.nh * a.hd;
    a.outxs[xs_index(tok, col, K, 0)] = hi;
    a.outxs[xs_index(tok, col, K, 1)] = lo;
  }
  if (a.out16) {
    const int64_t i = (int64_t)tok * (a.nh * a.hd) + col;
    const __half hv = __float2half_rn(v);
    a.out16[i] = hv;
    if (a.out16lo) a.out16[a.out16lo + i] = __float2half_rn(v - __half2float(hv));
  }
}

template <int HD>
__global__ void __launch_bounds__(ATC_THREADS, 2) k_attn_tc(AttnArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AtcSmem<HD>& S = *reinterpret_cast<AtcSmem<HD>*>(smem_raw);
  constexpr int KS = HD / 16;       // k-steps of QK^T over head dims
  constexpr int NT = ATC_TK / 8;    // score n-tiles per key tile
  constexpr int ON = HD / 8;        // output n-tiles
  const int qb = a.nqb - 1 - (int)blockIdx.x;  // longest query blocks first
  const int kvh = blockIdx.y, sp = blockIdx.z;
  const int G = a.nh / a.nkv;
  const int tok0 = a.qb_tok0 ? a.qb_tok0[qb] : qb;
  const int qlen = a.qb_tok0 ? a.qb_len[qb] : 1;
  const int R = qlen * G;
  const int sq = a.seq[tok0];
  const int kv_end = a.pos[tok0 + qlen - 1] + 1;
  const int ntile = (kv_end + ATC_TK - 1) / ATC_TK;
  const int per = (ntile + a.nsplit - 1) / a.nsplit;
  const int k_lo = sp * per * ATC_TK;
  const int k_hi = min(kv_end, (sp + 1) * per * ATC_TK);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int r0 = 16 * warp + g, r1 = r0 + 8;

  for (int r = threadIdx.x; r < ATC_ROWS; r += ATC_THREADS) S.qpos[r] = r < R ? a.pos[tok0 + r / G] : -1;

  // Q fragments (rows r0, r1), scaled into the exp2 domain and split
  uint32_t qh[KS][4], ql[KS][4];
  {
    const float qs = 1.4426950408889634f / sqrtf((float)HD);
    const float* q0 = r0 < R ? a.q + (int64_t)(tok0 + r0 / G) * a.ldq + (int64_t)(kvh * G + r0 % G) * HD : nullptr;
    const float* q1 = r1 < R ? a.q + (int64_t)(tok0 + r1 / G) * a.ldq + (int64_t)(kvh * G + r1 % G) * HD : nullptr;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float* qr = (i & 1) ? q1 : q0;
        const int col = 16 * kk + 2 * t + ((i >> 1) << 3);
        float2 v = make_float2(0.f, 0.f);
        if (qr) v = *reinterpret_cast<const float2*>(qr + col);
        atc_split2(v.x * qs, v.y * qs, qh[kk][i], ql[kk][i]);
      }
    }
  }

  float o[ON][4];
#pragma unroll
  for (int n = 0; n < ON; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int32_t* btr = a.bt + (int64_t)sq * a.max_pages;
  const int mi = lane >> 3, rr = lane & 7;  // ldmatrix: matrix and row this lane addresses

  for (int j0 = k_lo; j0 < k_hi; j0 += ATC_TK) {
    __syncthreads();  // the previous tile is consumed (first pass: qpos is visible)
    // four rows' loads in flight per thread before any conversion
    for (int i0 = threadIdx.x; i0 < ATC_TK * HD / 4; i0 += 4 * ATC_THREADS) {
      float4 kv[4], vv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * ATC_THREADS;
        const int jj = i / (HD / 4), d = (i % (HD / 4)) * 4, j = j0 + jj;
        kv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        vv[u] = kv[u];
        if (j < k_hi) {
          const int pg = btr[j / a.page];
          const int64_t off = (((int64_t)pg * a.nkv + kvh) * a.page + (j % a.page)) * HD + d;
          kv[u] = *reinterpret_cast<const float4*>(a.kp + off);
          vv[u] = *reinterpret_cast<const float4*>(a.vp + off);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * ATC_THREADS;
        const int jj = i / (HD / 4), d = (i % (HD / 4)) * 4;
        uint32_t h0, l0_, h1, l1_;
        const int e = atc_swz<HD>(jj, d);
        atc_split2(kv[u].x, kv[u].y, h0, l0_);
        atc_split2(kv[u].z, kv[u].w, h1, l1_);
        *reinterpret_cast<uint2*>(S.kh + e) = make_uint2(h0, h1);
        *reinterpret_cast<uint2*>(S.kl + e) = make_uint2(l0_, l1_);
        atc_split2(vv[u].x, vv[u].y, h0, l0_);
        atc_split2(vv[u].z, vv[u].w, h1, l1_);
        *reinterpret_cast<uint2*>(S.vh + e) = make_uint2(h0, h1);
        *reinterpret_cast<uint2*>(S.vl + e) = make_uint2(l0_, l1_);
      }
    }
    __syncthreads();

    // S = Q K^T for keys j0 .. j0 + 63
    float s[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      uint32_t bh[NT / 2][4], bl[NT / 2][4];
#pragma unroll
      for (int np = 0; np < NT; np += 2) {
        // matrices: (keys 8np.., dims 16kk..), (8np.., 16kk+8..), (8np+8.., 16kk..), (8np+8.., 16kk+8..)
        const int key = 8 * np + ((mi >> 1) << 3) + rr, dim = 16 * kk + ((mi & 1) << 3);
        atc_ldsm_x4(bh[np / 2], S.kh + atc_swz<HD>(key, dim));
        atc_ldsm_x4(bl[np / 2], S.kl + atc_swz<HD>(key, dim));
      }
      // one split term across all n-tiles before the next: independent MMAs back to back
#pragma unroll
      for (int n = 0; n < NT; ++n) atc_mma(s[n], qh[kk], bh[n / 2][(n & 1) * 2], bh[n / 2][(n & 1) * 2 + 1]);
#pragma unroll
      for (int n = 0; n < NT; ++n) atc_mma(s[n], qh[kk], bl[n / 2][(n & 1) * 2], bl[n / 2][(n & 1) * 2 + 1]);
#pragma unroll
      for (int n = 0; n < NT; ++n) atc_mma(s[n], ql[kk], bh[n / 2][(n & 1) * 2], bh[n / 2][(n & 1) * 2 + 1]);
    }

    // causal mask, online softmax (rows r0: c0/c1, r1: c2/c3)
    const int qp0 = S.qpos[r0], qp1 = S.qpos[r1];
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = j0 + 8 * n + 2 * t + e;
        if (key >= k_hi || key > qp0) s[n][e] = -INFINITY;
        if (key >= k_hi || key > qp1) s[n][2 + e] = -INFINITY;
        mx0 = fmaxf(mx0, s[n][e]);
        mx1 = fmaxf(mx1, s[n][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float c0 = mn0 == -INFINITY ? 0.f : exp2f(m0 - mn0);
    const float c1 = mn1 == -INFINITY ? 0.f : exp2f(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        s[n][e] = s[n][e] == -INFINITY ? 0.f : exp2f(s[n][e] - mn0);
        s[n][2 + e] = s[n][2 + e] == -INFINITY ? 0.f : exp2f(s[n][2 + e] - mn1);
        ps0 += s[n][e];
        ps1 += s[n][2 + e];
      }
    }
    l0 = fmaf(l0, c0, ps0);
    l1 = fmaf(l1, c1, ps1);
#pragma unroll
    for (int n = 0; n < ON; ++n) {
      o[n][0] *= c0;
      o[n][1] *= c0;
      o[n][2] *= c1;
      o[n][3] *= c1;
    }

    // O += P V (P from the score accumulators: k-step kk = keys 16kk .. 16kk+15)
#pragma unroll
    for (int kk = 0; kk < ATC_TK / 16; ++kk) {
      uint32_t ph[4], pl[4];
      atc_split2(s[2 * kk][0], s[2 * kk][1], ph[0], pl[0]);
      atc_split2(s[2 * kk][2], s[2 * kk][3], ph[1], pl[1]);
      atc_split2(s[2 * kk + 1][0], s[2 * kk + 1][1], ph[2], pl[2]);
      atc_split2(s[2 * kk + 1][2], s[2 * kk + 1][3], ph[3], pl[3]);
#pragma unroll
      for (int np = 0; np < ON; np += 4) {
        // matrices (transposed): (keys 16kk.., dims 8np..), (16kk+8.., 8np..), (16kk.., 8np+8..), (16kk+8.., 8np+8..)
        uint32_t vh[2][4], vl[2][4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int key = 16 * kk + ((mi & 1) << 3) + rr, dim = 8 * (np + 2 * h) + ((mi >> 1) << 3);
          atc_ldsm_x4_t(vh[h], S.vh + atc_swz<HD>(key, dim));
          atc_ldsm_x4_t(vl[h], S.vl + atc_swz<HD>(key, dim));
        }
#pragma unroll
        for (int n = 0; n < 4; ++n) atc_mma(o[np + n], ph, vh[n / 2][(n & 1) * 2], vh[n / 2][(n & 1) * 2 + 1]);
#pragma unroll
        for (int n = 0; n < 4; ++n) atc_mma(o[np + n], ph, vl[n / 2][(n & 1) * 2], vl[n / 2][(n & 1) * 2 + 1]);
#pragma unroll
        for (int n = 0; n < 4; ++n) atc_mma(o[np + n], pl, vh[n / 2][(n & 1) * 2], vh[n / 2][(n & 1) * 2 + 1]);
      }
    }
  }

  // row sums over the quad
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  if (a.nsplit == 1) {
#pragma unroll
    for (int n = 0; n < ON; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int d = 8 * n + 2 * t + e;
        if (r0 < R)
          atc_write_out(a, tok0 + r0 / G, (kvh * G + r0 % G) * HD + d, l0 > 0.f ? o[n][e] / l0 : 0.f);
        if (r1 < R)
          atc_write_out(a, tok0 + r1 / G, (kvh * G + r1 % G) * HD + d, l1 > 0.f ? o[n][2 + e] / l1 : 0.f);
      }
    }
    return;
  }
  // partial layout of k_attn_combine: per item 64*HD o, 64 m (natural log), 64 l
  const int64_t item = ((int64_t)qb * a.nkv + kvh) * a.nsplit + sp;
  float* po = a.part + item * (int64_t)(ATC_ROWS * HD + 2 * ATC_ROWS);
  constexpr float LN2 = 0.6931471805599453f;
#pragma unroll
  for (int n = 0; n < ON; ++n) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int d = 8 * n + 2 * t + e;
      po[r0 * HD + d] = o[n][e];
      po[r1 * HD + d] = o[n][2 + e];
    }
  }
  if (t == 0) {
    po[ATC_ROWS * HD + r0] = m0 == -INFINITY ? -INFINITY : m0 * LN2;
    po[ATC_ROWS * HD + r1] = m1 == -INFINITY ? -INFINITY : m1 * LN2;
    po[ATC_ROWS * HD + ATC_ROWS + r0] = l0;
    po[ATC_ROWS * HD + ATC_ROWS + r1] = l1;
  }
}

template <int HD>
static int atc_run(const AttnArgs& a, cudaStream_t st) {
  constexpr size_t smem = sizeof(AtcSmem<HD>);
  static bool attr_done[64] = {false};
  int dev = 0;
  Q8_CUDA(cudaGetDevice(&dev));
  if (!attr_done[dev & 63]) {
    Q8_CUDA(cudaFuncSetAttribute(k_attn_tc<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_done[dev & 63] = true;
  }
  k_attn_tc<HD><<<dim3(a.nqb, a.nkv, a.nsplit), ATC_THREADS, smem, st>>>(a);
  return launch_check("k_attn_tc");
}

// Tensor-core path for query blocks of up to 64 (token, head) rows; false when
// the shape is not covered (the caller keeps the SIMT kernel).
bool attention_tc_supported(const AttnArgs& a) {
  static const bool on = [] {
    const char* e = getenv("Q8_ATTN_TC");
    return !(e && e[0] == '0');
  }();
  const int G = a.nkv > 0 ? a.nh / a.nkv : 0;
  return on && (a.hd == 64 || a.hd == 128) && G > 0 && a.qb_max * G <= ATC_ROWS && a.qb_max * G > 8;
}

int attention_tc_launch(const AttnArgs& a, cudaStream_t st) {
  if (a.hd == 128) return atc_run<128>(a, st);
  return atc_run<64>(a, st);
}

}  // namespace q8
