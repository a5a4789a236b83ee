// Decode attention over the paged f32 KV cache: one query token per sequence.
//
// Replaces, for the decode step, k_scores + k_softmax_rows + k_att_out
// (src/llama_common.mojo:402-473) and, fused in front, the QK-norm of
// k_rmsnorm2_w (:228-270) and k_rope_qk_copy2 (:299-342) for the new token:
//   out[h] = sum_j softmax_j(q_h . k_j / sqrt(hd)) v_j,  j = 0..pos.
//
// Work split.  CTA = (token, kv head, context split), about one CTA per SM in
// total; the split's positions are cut into blocks of 16.  The last warp is
// the producer: it streams the blocks' K and V rows with the TMA engine into
// AD_R shared-memory slots per consumer warp (full / empty mbarrier pair per
// slot, transaction bytes counted on full), so up to AD_C * AD_R blocks are
// in flight per SM whatever the consumers are doing.  Block i belongs to
// consumer warp i % AD_C and each slot serves one warp in order, so no wait
// ever targets a barrier phase more than one ahead.  With pages of a multiple
// of 16 slots a block is 16 consecutive rows of one page: K comes as HD/32
// tensor-map boxes of 16 rows x 128 B with the 128 B swizzle (16-byte chunk c
// of row j lands at chunk c ^ (j & 7)), V as one bulk copy.  Otherwise each lane copies one
// row (K rows padded by 16 B).  Consumer warps take blocks w, w + AD_C, ..:
//   scores:  lanes 2j, 2j+1 = position j, each taking half of the 16-byte
//            chunks of the row (chunks with bit 2 clear / set), so every
//            8-lane phase of a shared-memory read touches 8 different bank
//            groups and q reads are broadcasts; all G query heads of the kv
//            group at once, one shuffle joins the halves;
//   softmax: one warp max per head per block (online, exp2 domain: q is
//            pre-scaled by log2(e)/sqrt(hd));
//   PV:      lane l owns head dims [E l, E l + E), probabilities broadcast
//            from shared memory;
// then the slot goes back to the producer.  The new position's k and v
// (rotated in the prologue, appended to the cache) are patched into the
// staged block from shared memory, so no copy depends on this kernel's own
// global writes.
// Consumer warps merge through shared memory; splits write (o, m, l)
// partials and the last CTA of a (token, kv head) merges them in split order
// (atomic ticket, reset by that CTA).  Every sum has a fixed order: results
// do not depend on timing.  Every barrier wait is bounded.
#include "q8_kernels.h"

#include <cuda.h>
#include <math.h>
#include <string.h>
#include <mutex>

namespace q8 {

int tensor_map_f32_rows(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                        uint32_t box_inner, uint32_t box_rows);

constexpr int AD_C = 8;                   // consumer warps
constexpr int AD_R = 1;                   // slots per consumer warp
constexpr int AD_S = AD_C * AD_R;         // slots (blocks in flight per CTA)
constexpr int AD_THREADS = (AD_C + 1) * 32;
constexpr int AD_KB = 16;                 // positions per block (two lanes each)
constexpr int AD_MAXSPLIT = 128;          // context splits per (token, kv head)

struct AdArgs {
  const float* q; int64_t ldq;       // q|k|v rows [T][ldq] (un-rotated when inv_freq is set)
  const int32_t* pos; const int32_t* seq;
  int T, nh, nkv;
  const float* kp; const float* vp; int page;   // pools [pages][nkv][page][HD]
  const int32_t* bt; int max_pages;
  float* part;      // [T*nkv][nsplit][ad_stride]
  int* ticket;      // [T*nkv], zero at rest
  float* out32; int64_t ldo;
  __half* outxs;
  __half* out16;           // optional f16 rows [T][nh*hd] (tensor-core GEMM input)
  int64_t out16lo;         // > 0: f16 remainders at out16 + out16lo
  const float* inv_freq;   // RoPE + QK-norm + KV append fused when set
  const uint16_t* qn;
  const uint16_t* kn;
  float eps;
  float* kw;
  float* vw;
};

__host__ __device__ constexpr int ad_stride(int G, int HD) { return G * HD + ((2 * G + 3) & ~3); }

// one ring slot (floats): K (swizzled boxes, or padded rows) then V rows
template <int HD, bool TM>
__host__ __device__ constexpr int ad_kslot() { return TM ? AD_KB * HD : AD_KB * (HD + 4); }
template <int HD, bool TM>
__host__ __device__ constexpr int ad_slot() { return ad_kslot<HD, TM>() + AD_KB * HD; }

template <int HD, int GMAX, bool TM>
constexpr size_t ad_smem_bytes() {
  return 1024                                          // alignment slack (swizzled boxes need 1 KB)
         + (size_t)AD_S * ad_slot<HD, TM>() * 4        // ring
         + (size_t)AD_C * GMAX * AD_KB * 4             // probabilities
         + (size_t)GMAX * HD * 4                       // q (scaled)
         + (size_t)2 * HD * 4                          // the new position's k, v
         + (size_t)2 * AD_S * 8;                       // mbarriers
}

__device__ __forceinline__ float ad_warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ void ad_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ticket increment with gpu-scope release (this CTA's earlier stores, made
// visible to thread 0 by a CTA barrier, are published first) and acquire
// (later reads see the other CTAs' published stores)
__device__ __forceinline__ int ad_ticket_add(int* t) {
  int old;
  asm volatile("fence.acq_rel.gpu;\n\tatom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(t) : "memory");
  return old;
}

// barrier 1 over the consumer warps only (the producer never joins)
__device__ __forceinline__ void ad_sync_consumers() { asm volatile("bar.sync 1, %0;" ::"n"(AD_C * 32) : "memory"); }

__device__ __forceinline__ void ad_tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void ad_write_out(const AdArgs& a, int K, int tok, int col, float v) {
  if (a.out32) a.out32[(int64_t)tok * a.ldo + col] = v;
  if (a.outxs) {
    __half hi, lo;
    split_f16(v, hi, lo);
    a.outxs[xs_index(tok, col, K, 0)] = hi;
    a.outxs[xs_index(tok, col, K, 1)] = lo;
  }
  if (a.out16) {
    const int64_t i = (int64_t)tok * K + col;
    const __half hv = __float2half_rn(v);
    a.out16[i] = hv;
    if (a.out16lo) a.out16[a.out16lo + i] = __float2half_rn(v - __half2float(hv));
  }
}

// float offset of 16-byte chunk c of row j in a slot's K part
template <int HD, bool TM>
__device__ __forceinline__ int ad_kofs(int j, int c) {
  if constexpr (TM) return (c >> 3) * (AD_KB * 32) + j * 32 + (((c & 7) ^ (j & 7)) << 2);
  else return j * (HD + 4) + 4 * c;
}

template <int HD, int GMAX, bool TM>
__global__ void __launch_bounds__(AD_THREADS, 1) k_attn_dec(AdArgs a, const __grid_constant__ CUtensorMap tmK) {
  constexpr int E = HD / 32, CH = HD / 4, J = HD / 32;
  constexpr int KS = ad_kslot<HD, TM>(), SL = ad_slot<HD, TM>();
  constexpr int MAXT = (GMAX + 1 + AD_C - 1) / AD_C;  // prologue tasks per consumer warp
  extern __shared__ uint8_t smem_raw[];
  float* ring = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  float* sP = ring + AD_S * SL;
  float* sQ = sP + AD_C * GMAX * AD_KB;
  float* sKn = sQ + GMAX * HD;
  float* sVn = sKn + HD;
  uint64_t* full = reinterpret_cast<uint64_t*>(sVn + HD);
  uint64_t* empty = full + AD_S;
  __shared__ float sm_m[AD_C][GMAX], sm_l[AD_C][GMAX];
  __shared__ int s_last;

  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == AD_C * 32) {
    for (int s = 0; s < AD_S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  const int item = blockIdx.x, sp = blockIdx.y, ns = gridDim.y;
  const int b = item / a.nkv, kvh = item % a.nkv, G = a.nh / a.nkv;
  pdl_wait();  // q, pos and the cache rows are written by earlier kernels

  const int p = a.pos[b], kv_end = p + 1;
  const int nb = (kv_end + AD_KB - 1) / AD_KB;
  const int bl0 = (int)((int64_t)sp * nb / ns), bl1 = (int)((int64_t)(sp + 1) * nb / ns);
  const int nblk = bl1 - bl0;
  const int32_t* btr = a.bt + (int64_t)a.seq[b] * a.max_pages;
  const bool own_new = a.inv_freq && p >= bl0 * AD_KB && p < bl1 * AD_KB;

  if (warp == AD_C) {
    // ---------------------------------------------------------------- producer
    // page-table entries 32 at a time: lane l holds btr[pg0 + l]
    int pg0 = -1, pgv = 0;
    for (int i = 0; i < nblk; ++i) {
      const int k = i / AD_C, slot = (i % AD_C) * AD_R + k % AD_R, u = k / AD_R;
      if (u > 0) mbar_wait(&empty[slot], (uint32_t)((u - 1) & 1));  // the slot's previous block consumed
      const int key0 = (bl0 + i) * AD_KB;
      const int nv = min(AD_KB, kv_end - key0);
      float* dk = ring + slot * SL;
      float* dv = dk + KS;
      if constexpr (TM) {
        const int pi = key0 / a.page;
        if (pg0 < 0 || pi >= pg0 + 32) {
          pg0 = pi;
          pgv = (pg0 + lane < a.max_pages) ? btr[pg0 + lane] : 0;
        }
        const int pg = __shfl_sync(0xffffffffu, pgv, pi - pg0);
        if (lane == 0) {
          const int64_t row0 = ((int64_t)pg * a.nkv + kvh) * a.page + (key0 % a.page);
          mbar_arrive_expect_tx(&full[slot], (uint32_t)(2 * AD_KB * HD * 4));
#pragma unroll
          for (int cb = 0; cb < HD / 32; ++cb) ad_tma_2d(dk + cb * AD_KB * 32, &tmK, cb * 32, (int)row0, &full[slot]);
          bulk_g2s(dv, a.vp + row0 * HD, AD_KB * HD * 4, &full[slot]);
        }
      } else {
        if (lane == 0) mbar_arrive_expect_tx(&full[slot], (uint32_t)(2 * nv * HD * 4));
        __syncwarp();
        if (lane < nv) {
          const int j = key0 + lane;
          const int64_t row = ((int64_t)btr[j / a.page] * a.nkv + kvh) * a.page + (j % a.page);
          bulk_g2s(dk + lane * (HD + 4), a.kp + row * HD, HD * 4, &full[slot]);
          bulk_g2s(dv + lane * HD, a.vp + row * HD, HD * 4, &full[slot]);
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  // prologue: q heads of the group -> sQ (QK-norm + RoPE when fused, scaled);
  // the split holding position p also rotates the new k and appends k, v to
  // the cache (and keeps them in sKn / sVn for its own block)
  {
    const float qscale = 1.4426950408889634f / sqrtf((float)HD);
    const int ntask = G + (own_new ? 1 : 0);
    float v[MAXT][J], vv[J];
#pragma unroll
    for (int i = 0; i < MAXT; ++i) {
      const int t = warp + AD_C * i;
      if (t < ntask) {
        const float* src = a.q + (int64_t)b * a.ldq + (t < G ? (int64_t)(kvh * G + t) * HD : (int64_t)(a.nh + kvh) * HD);
#pragma unroll
        for (int j = 0; j < J; ++j) v[i][j] = src[lane + 32 * j];
        if (t == G) {
          const float* vsrc = a.q + (int64_t)b * a.ldq + (int64_t)(a.nh + a.nkv + kvh) * HD;
#pragma unroll
          for (int j = 0; j < J; ++j) vv[j] = vsrc[lane + 32 * j];
        }
      }
    }
    float cs[J / 2], sn[J / 2];
    if (a.inv_freq && warp < ntask) {
      const float fp = (float)p;
#pragma unroll
      for (int j = 0; j < J / 2; ++j) sincosf(fp * a.inv_freq[lane + 32 * j], &sn[j], &cs[j]);
    }
#pragma unroll
    for (int i = 0; i < MAXT; ++i) {
      const int t = warp + AD_C * i;
      if (t >= ntask) break;
      if (a.inv_freq) {
        const uint16_t* nw = t < G ? a.qn : a.kn;
        if (nw) {
          float ss = 0.f;
#pragma unroll
          for (int j = 0; j < J; ++j) ss = fmaf(v[i][j], v[i][j], ss);
          ss = warp_sum(ss);
          const float inv = 1.0f / sqrtf(ss / (float)HD + a.eps);
#pragma unroll
          for (int j = 0; j < J; ++j) v[i][j] = bf16_bits_to_f32(nw[lane + 32 * j]) * v[i][j] * inv;
        }
        // rotate-half pairs (d, d + hd/2) sit in one lane: dims lane + 32 j
#pragma unroll
        for (int j = 0; j < J / 2; ++j) {
          const float x0 = v[i][j], x1 = v[i][j + J / 2];
          v[i][j] = x0 * cs[j] - x1 * sn[j];
          v[i][j + J / 2] = x1 * cs[j] + x0 * sn[j];
        }
      }
      if (t < G) {
#pragma unroll
        for (int j = 0; j < J; ++j) sQ[t * HD + lane + 32 * j] = v[i][j] * qscale;
      } else {
        const int64_t off = (((int64_t)btr[p / a.page] * a.nkv + kvh) * a.page + (p % a.page)) * HD;
#pragma unroll
        for (int j = 0; j < J; ++j) {
          a.kw[off + lane + 32 * j] = v[i][j];
          a.vw[off + lane + 32 * j] = vv[j];
          sKn[lane + 32 * j] = v[i][j];
          sVn[lane + 32 * j] = vv[j];
        }
      }
    }
    ad_sync_consumers();
  }

  float m[GMAX], l[GMAX], o[GMAX][E];
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) o[g][e] = 0.f;
  }
  float* pw = sP + warp * GMAX * AD_KB;
  const int jr = lane >> 1, hh = 4 * (lane & 1);
  const bool lead = (lane & 1) == 0;
  for (int i = warp, k = 0; i < nblk; i += AD_C, ++k) {
    const int slot = warp * AD_R + k % AD_R;
    const int key0 = (bl0 + i) * AD_KB;
    const int nv = min(AD_KB, kv_end - key0);
    float* kb = ring + slot * SL;
    float* vb = kb + KS;
    mbar_wait(&full[slot], (uint32_t)((k / AD_R) & 1));
    if (own_new && p >= key0 && p < key0 + AD_KB) {  // the appended row, from the prologue
      for (int c = lane; c < CH; c += 32) {
        *reinterpret_cast<float4*>(kb + ad_kofs<HD, TM>(p - key0, c)) = *reinterpret_cast<const float4*>(sKn + 4 * c);
        *reinterpret_cast<float4*>(vb + (p - key0) * HD + 4 * c) = *reinterpret_cast<const float4*>(sVn + 4 * c);
      }
      // generic writes land before the bulk copies that later refill the slot
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
    }

    // scores of position key0 + jr for every head of the group
    float s[GMAX];
    {
      float s0[GMAX], s1[GMAX];
#pragma unroll
      for (int g = 0; g < GMAX; ++g) s0[g] = s1[g] = 0.f;
      const float4* q4 = reinterpret_cast<const float4*>(sQ);
#pragma unroll 2
      for (int c = 0; c < CH / 2; c += 2) {
        const int c0 = ((c >> 2) << 3) + hh + (c & 3), c1 = c0 + 1;  // this lane's half of the chunks
        const float4 k0 = *reinterpret_cast<const float4*>(kb + ad_kofs<HD, TM>(jr, c0));
        const float4 k1 = *reinterpret_cast<const float4*>(kb + ad_kofs<HD, TM>(jr, c1));
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
          if (g < G) {
            const float4 qa = q4[g * CH + c0], qb = q4[g * CH + c1];
            s0[g] = fmaf(qa.w, k0.w, fmaf(qa.z, k0.z, fmaf(qa.y, k0.y, fmaf(qa.x, k0.x, s0[g]))));
            s1[g] = fmaf(qb.w, k1.w, fmaf(qb.z, k1.z, fmaf(qb.y, k1.y, fmaf(qb.x, k1.x, s1[g]))));
          }
        }
      }
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
        const float part = s0[g] + s1[g];
        const float other = __shfl_xor_sync(0xffffffffu, part, 1);
        s[g] = (lane & 1) ? other + part : part + other;  // the even lane's half first on both lanes
      }
    }

    // online softmax per head (warp-uniform max), probabilities to shared memory
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      if (g >= G) break;
      const float sc = jr < nv ? s[g] : -INFINITY;
      const float mn = fmaxf(m[g], ad_warp_max(sc));
      const float corr = exp2f(m[g] - mn);  // 0 on the first block (m = -inf)
      const float pz = jr < nv ? exp2f(sc - mn) : 0.f;
      l[g] = fmaf(l[g], corr, lead ? pz : 0.f);
#pragma unroll
      for (int e = 0; e < E; ++e) o[g][e] *= corr;
      m[g] = mn;
      if (lead) pw[g * AD_KB + jr] = pz;
    }
    __syncwarp();

    // o += p V over the block's valid positions
    for (int j0 = 0; j0 < nv; j0 += 4) {
      float4 pp[GMAX];
#pragma unroll
      for (int g = 0; g < GMAX; ++g)
        if (g < G) pp[g] = *reinterpret_cast<const float4*>(pw + g * AD_KB + j0);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (j0 + u < nv) {
          float x[E];
          const float* vr = vb + (j0 + u) * HD + lane * E;
          if constexpr (E == 4) {
            const float4 t = *reinterpret_cast<const float4*>(vr);
            x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
          } else {
            const float2 t = *reinterpret_cast<const float2*>(vr);
            x[0] = t.x; x[1] = t.y;
          }
#pragma unroll
          for (int g = 0; g < GMAX; ++g) {
            if (g < G) {
              const float pg = u == 0 ? pp[g].x : (u == 1 ? pp[g].y : (u == 2 ? pp[g].z : pp[g].w));
#pragma unroll
              for (int e = 0; e < E; ++e) o[g][e] = fmaf(pg, x[e], o[g][e]);
            }
          }
        }
      }
    }
    __syncwarp();  // slot and probabilities consumed
    if (lane == 0) ad_arrive(&empty[slot]);
  }
#pragma unroll
  for (int g = 0; g < GMAX; ++g) l[g] = warp_sum(l[g]);

  // merge the consumer warps: (m, l, o) per head; o staged over the ring
  // (every issued block has been waited for, so no copy is in flight)
  ad_sync_consumers();
  float* sO = ring;  // [AD_C][GMAX][HD]
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      sm_m[warp][g] = m[g];
      sm_l[warp][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    if (g >= G) break;
#pragma unroll
    for (int e = 0; e < E; ++e) sO[(warp * GMAX + g) * HD + lane * E + e] = o[g][e];
  }
  ad_sync_consumers();
  const int WS = ad_stride(G, HD);
  const int nthr = AD_C * 32;
  float* mypart = a.part + ((int64_t)item * ns + sp) * WS;
  for (int i = threadIdx.x; i < G * HD; i += nthr) {
    const int g = i / HD, d = i % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < AD_C; ++w) M = fmaxf(M, sm_m[w][g]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < AD_C; ++w) {
        if (sm_m[w][g] == -INFINITY) continue;
        const float f = exp2f(sm_m[w][g] - M);
        L = fmaf(sm_l[w][g], f, L);
        O = fmaf(sO[(w * GMAX + g) * HD + d], f, O);
      }
    }
    if (ns == 1) {
      ad_write_out(a, a.nh * HD, b, (kvh * G + g) * HD + d, L > 0.f ? O / L : 0.f);
    } else {
      mypart[i] = O;
      if (d == 0) {
        mypart[G * HD + g] = M;
        mypart[G * HD + G + g] = L;
      }
    }
  }
  if (ns == 1) return;
  // split-K semaphore: the CTA's partial stores, then one gpu-scope
  // release/acquire ticket (cumulative over the CTA through the barrier)
  ad_sync_consumers();
  if (threadIdx.x == 0) s_last = (ad_ticket_add(&a.ticket[item]) == ns - 1);
  ad_sync_consumers();
  if (!s_last) return;

  // merge the splits: the consumer threads take (float4 chunk, run of
  // splits) pairs; a run is folded in split order with an online rescale, all
  // of a batch's loads ((m, l) of the chunk's head and the o chunk of every
  // split) in flight together; the runs are then folded in run order
  const float* base = a.part + (int64_t)item * ns * WS;
  const int nchunk = G * HD / 4;
  const int nrun = max(1, min(ns, nthr / nchunk));
  float4* sred = reinterpret_cast<float4*>(ring + AD_C * GMAX * HD);   // [nrun][nchunk] o, past sO
  float2* sml = reinterpret_cast<float2*>(sred + nrun * nchunk);       // [nrun][nchunk] (m, l)
  for (int t = threadIdx.x; t < nrun * nchunk; t += nthr) {
    const int i4 = t % nchunk, run = t / nchunk;
    const int g = (4 * i4) / HD;
    const int r0 = run * ns / nrun, r1 = (run + 1) * ns / nrun;
    float M = -INFINITY, L = 0.f;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = r0; s0 < r1; s0 += 16) {
      float4 v[16];
      float ms[16], ls[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const bool ok = s0 + u < r1;
        const float* ps = base + (int64_t)(s0 + u) * WS;
        v[u] = ok ? __ldcg(reinterpret_cast<const float4*>(ps) + i4) : make_float4(0.f, 0.f, 0.f, 0.f);
        ms[u] = ok ? __ldcg(ps + G * HD + g) : -INFINITY;
        ls[u] = ok ? __ldcg(ps + G * HD + G + g) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        if (ms[u] == -INFINITY) continue;  // empty split (or past the run)
        const float mn = fmaxf(M, ms[u]);
        const float c = exp2f(M - mn), f = exp2f(ms[u] - mn);
        O.x = fmaf(v[u].x, f, O.x * c);
        O.y = fmaf(v[u].y, f, O.y * c);
        O.z = fmaf(v[u].z, f, O.z * c);
        O.w = fmaf(v[u].w, f, O.w * c);
        L = fmaf(ls[u], f, L * c);
        M = mn;
      }
    }
    sred[run * nchunk + i4] = O;
    sml[run * nchunk + i4] = make_float2(M, L);
  }
  ad_sync_consumers();
  for (int i4 = threadIdx.x; i4 < nchunk; i4 += nthr) {
    float4 O = sred[i4];
    float M = sml[i4].x, L = sml[i4].y;
    for (int run = 1; run < nrun; ++run) {
      const float2 ml = sml[run * nchunk + i4];
      if (ml.x == -INFINITY) continue;
      const float4 x = sred[run * nchunk + i4];
      const float mn = fmaxf(M, ml.x);
      const float c = exp2f(M - mn), f = exp2f(ml.x - mn);
      O.x = fmaf(x.x, f, O.x * c);
      O.y = fmaf(x.y, f, O.y * c);
      O.z = fmaf(x.z, f, O.z * c);
      O.w = fmaf(x.w, f, O.w * c);
      L = fmaf(ml.y, f, L * c);
      M = mn;
    }
    const int col = (kvh * G) * HD + 4 * i4;
    ad_write_out(a, a.nh * HD, b, col + 0, L > 0.f ? O.x / L : 0.f);
    ad_write_out(a, a.nh * HD, b, col + 1, L > 0.f ? O.y / L : 0.f);
    ad_write_out(a, a.nh * HD, b, col + 2, L > 0.f ? O.z / L : 0.f);
    ad_write_out(a, a.nh * HD, b, col + 3, L > 0.f ? O.w / L : 0.f);
  }
  if (threadIdx.x == 0) a.ticket[item] = 0;  // ready for the next launch
}

template <int HD, int GMAX, bool TM>
static int ad_launch(const AdArgs& a, const CUtensorMap& tm, dim3 grid, cudaStream_t st) {
  constexpr size_t smem = ad_smem_bytes<HD, GMAX, TM>();
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(k_attn_dec<HD, GMAX, TM>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  });
  if (attr != cudaSuccess) {
    set_error("k_attn_dec: shared memory attribute: %s", cudaGetErrorString(attr));
    return Q8_ERR_CUDA;
  }
  return launch_pdl("k_attn_dec", k_attn_dec<HD, GMAX, TM>, grid, dim3(AD_THREADS), smem, st, a, tm);
}

template <bool TM>
static int ad_dispatch(const AdArgs& a, const CUtensorMap& tm, int hd, dim3 grid, cudaStream_t st) {
  const bool g4 = a.nh / a.nkv <= 4;
  if (hd == 128) return g4 ? ad_launch<128, 4, TM>(a, tm, grid, st) : ad_launch<128, 8, TM>(a, tm, grid, st);
  if (hd == 64) return g4 ? ad_launch<64, 4, TM>(a, tm, grid, st) : ad_launch<64, 8, TM>(a, tm, grid, st);
  set_error("attention decode: head_dim %d unsupported (64/128)", hd);
  return Q8_ERR_ARG;
}

// Context splits per (token, kv head): one CTA per SM at a time, so the
// launch takes ceil(items * ns / SMs) waves of CTAs that each stream maxlen /
// ns positions after a fixed cost (launch, prologue, split merge) worth about
// AD_FIXED_KEYS positions; ns minimises waves x (AD_FIXED_KEYS + maxlen / ns).
// Batch 1 of 8 kv heads gets 18 splits (one wave), batch 64 gets 2 (seven
// nearly full waves instead of 3.5).
constexpr int AD_FIXED_KEYS = 300;

int attention_decode_nsplit(int items, int maxlen) {
  items = std::max(1, items);
  const int sms = num_sms();
  const int nmax = std::max(1, std::min(AD_MAXSPLIT, (maxlen + AD_KB - 1) / AD_KB));
  int best = 1;
  double best_cost = 1e300;
  for (int ns = 1; ns <= nmax; ++ns) {
    const double waves = (double)ceil_div((int64_t)items * ns, sms);
    const double cost = waves * (AD_FIXED_KEYS + (double)maxlen / ns);
    if (cost < best_cost * (1.0 - 1e-9)) {
      best_cost = cost;
      best = ns;
    }
  }
  return best;
}

size_t attention_decode_part_floats(int T, int nkv, int nsplit, int group, int hd) {
  return (size_t)T * nkv * nsplit * (size_t)ad_stride(group, hd);
}

int attention_decode_launch(const float* q, int64_t ldq, int T, const int32_t* pos, const int32_t* seq, int nh,
                            int nkv, int hd, const float* kp, const float* vp, int page, const int32_t* bt,
                            int max_pages, int nsplit, float* part, int* ticket, float* out32, int64_t ldo,
                            __half* outxs, cudaStream_t st, const AttnRope* rope, int64_t pool_rows,
                            __half* out16, int64_t out16lo) {
  Q8_CHECK_ARG(nkv > 0 && nh % nkv == 0 && nh / nkv <= 8, "attention decode: GQA group must be <= 8");
  Q8_CHECK_ARG(nsplit >= 1 && nsplit <= AD_MAXSPLIT && (nsplit == 1 || (part && ticket)),
               "attention decode: bad split count %d", nsplit);
  Q8_CHECK_ARG(page >= 1, "attention decode: bad page size %d", page);
  Q8_CHECK_ARG(((uintptr_t)kp & 15) == 0 && ((uintptr_t)vp & 15) == 0, "attention decode: pools must be 16-byte aligned");
  if (T <= 0) return Q8_OK;
  AdArgs a{q, ldq, pos, seq, T, nh, nkv, kp, vp, page, bt, max_pages, part, ticket, out32, ldo, outxs,
           out16, out16lo, nullptr, nullptr, nullptr, 0.f, nullptr, nullptr};
  if (rope) {
    Q8_CHECK_ARG(rope->inv_freq && rope->kw == kp && rope->vw == vp, "attention decode: bad rope arguments");
    a.inv_freq = rope->inv_freq;
    a.qn = rope->qn;
    a.kn = rope->kn;
    a.eps = rope->eps;
    a.kw = rope->kw;
    a.vw = rope->vw;
  }
  const dim3 grid(T * nkv, nsplit);
  CUtensorMap tm;
  memset(&tm, 0, sizeof(tm));
  // whole 16-row blocks per page: tensor-map K boxes and one bulk V copy per block
  if (pool_rows > 0 && page % AD_KB == 0 && pool_rows < (int64_t)1 << 31) {
    Q8_TRY(tensor_map_f32_rows(&tm, kp, (uint64_t)hd, (uint64_t)pool_rows, (uint64_t)hd * 4, 32, AD_KB));
    return ad_dispatch<true>(a, tm, hd, grid, st);
  }
  return ad_dispatch<false>(a, tm, hd, grid, st);
}

// Device address of this file's error word (per device, current device).
int attn_dec_error_word(int** out) {
  Q8_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(out), g_q8_device_error));
  return Q8_OK;
}

int attn_dec_poll_error() {
  int v = 0;
  Q8_CUDA(cudaMemcpyFromSymbol(&v, g_q8_device_error, sizeof(int)));
  if (v == 0) return Q8_OK;
  const int z = 0;
  Q8_CUDA(cudaMemcpyToSymbol(g_q8_device_error, &z, sizeof(int)));
  set_error("k_attn_dec: a staging barrier wait timed out (device status %d)", v);
  return v;
}

}  // namespace q8
