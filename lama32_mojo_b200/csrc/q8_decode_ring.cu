// Weight-ring decode step: one cooperative launch runs a whole decode step
// of one sequence (embed -> L x [RMSNorm, q|k|v, QK-norm + RoPE + KV append,
// GQA attention, o_proj + residual, RMSNorm, gate|up + SwiGLU, down +
// residual] -> final RMSNorm -> lm_head -> greedy argmax).
//
// Replaces, for batch-1 decode, the per-op dispatch chain of run_layer_q8
// (src/llama_q8.mojo:144-230) and the model shell's forward_argmax
// (qwen3_mojo/src/qwen_q8.mojo:126-162, src/llama_gpu.mojo:119-155), with
// the arithmetic of k_mm_q8 (src/llama_q8.mojo:54-93), k_rmsnorm_w / k_res_add
// (src/llama_common.mojo:197-225, :354-358), k_rmsnorm2_w (:228-270),
// k_rope_qk_copy2 (:299-342), k_scores / k_softmax_rows / k_att_out
// (:402-473), k_swiglu_mul (:476-481) and k_argmax (:493-519).
//
// Why one launch with a ring.  At batch 1 a decode step is a chain of ~160
// dependent operations over 7.7 GB of weights (Llama-3.1-8B); with one kernel
// per operation every boundary drains the memory pipeline (launch, ramp,
// activation staging, tail: ~11 us each).  Weight bytes never depend on the
// activations, so here one CTA per SM splits into
//   * a producer warp that walks the CTA's share of every phase of the step
//     in order (its tiles of each matrix, its KV blocks of each layer's
//     attention) and streams them with bulk copies (TMA engine) into a ring
//     of shared-memory slots, waiting only for free slots, and
//   * 8 consumer warps that wait for the previous phase of the whole grid
//     (a monotonic arrival counter), stage the phase's activation vector once
//     per CTA, and drain the ring.
// The producer therefore runs up to a ring's worth of bytes (128 KB per SM)
// ahead across phase and layer boundaries, and HBM keeps streaming while the
// grid synchronizes.
//
// Ring.  Consumer warp w owns slots 2w and 2w+1 (full / empty mbarrier pair
// each) and takes its items in order, alternating slots; the producer fills
// them in the same order, so no wait ever targets a phase more than one
// ahead.  A GEMV stage is one bulk copy of one 8448-byte block of the ring
// layout: every matrix is copied once, at load, into blocks of 16 weight
// rows x 512 codes stored as four 16 x 128 B boxes (16-byte chunk c of row r
// at chunk c ^ (r & 7), so ldmatrix is conflict-free) followed by the rows'
// 16 x 8 f16 group scales.  An attention block is 16 consecutive K rows of one
// page in one slot and the matching 16 V rows in the other (one bulk copy
// each).  Few large copies matter: the TMA engine's per-copy cost capped 2 KB
// boxes near 3.4 TB/s where 8 KB copies stream above 6 TB/s.
//
// GEMV arithmetic (as the standalone digit GEMV): int8 codes straight to
// mma.m16n8k32.s8 against the activations written as three int8 digits per
// value with one f32 scale per 64-group, x ~ e (a0 + a1/254 + a2/254^2), so
// the exact integer dot products carry the f32 activations; per group and
// digit column the s32 sum is scaled by (f16 weight scale) x (e / 254^d).
//
// Work split.  A matrix of T 16-row tiles (SwiGLU: 8 gate + 8 up rows) and C
// = K/512 chunks has T*C stages.  q|k|v, o_proj, gate|up and lm_head give
// each CTA whole tiles (so their epilogues finish rows: store, residual add,
// SwiGLU, logits + argmax); down_proj, whose tiles are 14336 codes deep,
// gives each CTA an even share of stages and parks partial rows in per-CTA
// slots that the next phase's staging adds to the residual in slot order.
// A CTA's stages are cut into 8 contiguous runs, one per consumer warp; a
// warp's per-tile sums go to shared memory and are added in warp order.
// The residual alternates between two buffers by layer, so a staging that
// folds the down partials into the residual never races with another CTA
// reading the old value.  Attention: CTA (kv head, context split), 16-
// position blocks, online softmax; the last split CTA of a kv head (release /
// acquire ticket) merges the splits in order.  Every sum has a fixed order:
// results do not depend on timing.
//
// Tensor parallelism.  Each rank runs the step on its shards (column-parallel
// q|k|v and gate|up rows, its kv heads, row-parallel K slices of o_proj and
// down_proj, its vocabulary rows).  The row-parallel phases end in an
// exchange inside the launch instead of a grid barrier: every CTA stores its
// partial rows into every rank's inbox (plain stores into peer memory mapped
// with CUDA IPC: no remote loads, no bulk copies from peers) and, after a CTA
// barrier, counts itself on every rank's arrival counter with one
// system-scope release per rank (cumulative over the CTA's stores); the next
// phase's staging waits (acquire) for the CTAs of all ranks and adds the
// partials in rank order, so every rank computes the same residual.  The
// lm_head phase ends with the ranks' argmax keys maxed into every rank's slot.
// Counters only grow: a step's targets derive from the rank's completed-step
// count, so no rank ever resets memory another rank may be counting into.
//
// Every wait is bounded (seconds): a wait that gives up sets the device
// status word, after which every other wait returns at once and the host
// reports Q8_ERR_TIMEOUT (Q8_ERR_COMM for a tensor-parallel peer that never
// arrived).  No load uses cluster multicast.
#include "q8_decode_ring.h"
#include "q8_kernels.h"

#include <algorithm>
#include <mutex>

namespace q8 {

enum { DP_QKV = 0, DP_ATTN = 1, DP_O = 2, DP_GU = 3, DP_DOWN = 4, DP_LM = 5 };

constexpr int DR_RING = DR_SLOTS * DR_SLOT_BYTES;
constexpr int DR_FCOL_BYTES = 256 * 16;  // K <= 16384
constexpr int DR_ATT_BYTES = (DR_GMAX * 128 + DR_CW * DR_GMAX * 16 + 2 * 128) * 4;
constexpr int DR_SMEM = 1024 + DR_RING + DR_XQ_BYTES + DR_FCOL_BYTES + DR_ATT_BYTES + 2 * DR_SLOTS * 8;

// ------------------------------------------------------------------ small helpers
__device__ __forceinline__ unsigned int dr_ld_acquire(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int dr_ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// barrier 1 over the 8 consumer warps (the producer never joins)
__device__ __forceinline__ void dr_csync() { asm volatile("bar.sync 1, %0;" ::"n"(DR_CW * 32) : "memory"); }

__device__ __forceinline__ void dr_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded mbarrier wait: gives up after ~2^34 cycles (~9 s, setting the
// status word) or as soon as another wait has given up (checked every 2^10
// polls).  The local bounds exceed the cross-rank exchange's (~2^33), so a
// rank that never arrives is reported as such.
__device__ __forceinline__ bool dr_mwait(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (unsigned it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 0x3FFu) == 0) {
      if (dr_ld_volatile(status)) return false;
      if (clock64() - t0 > (1ll << 34)) {
        atomicExch(status, Q8_ERR_TIMEOUT);
        return false;
      }
    }
  }
}

// Grid phase barrier (consumer warps only): wait until every CTA has arrived
// `target` times in total, then release the CTA's consumers.
__device__ __forceinline__ void dr_grid_wait(const DrParams& P, unsigned int target) {
  if (threadIdx.x == 0 && dr_ld_volatile(P.status) == 0) {
    const long long t0 = clock64();
    for (unsigned it = 1; dr_ld_acquire(P.bar) < target; ++it) {
      if ((it & 63u) == 0) {
        if (dr_ld_volatile(P.status)) break;
        if (clock64() - t0 > (1ll << 34)) {
          atomicExch(P.status, Q8_ERR_TIMEOUT);
          break;
        }
      }
    }
  }
  dr_csync();
}

// Cross-rank exchange (tensor parallelism): wait until this rank's counter
// `ctr` holds `target` arrivals of all ranks' CTAs (system-scope acquire).  The
// bound is longer than the grid barrier's: the ranks' launches may be skewed
// by their hosts.
__device__ __forceinline__ unsigned long long dr_ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void dr_xwait1(const DrParams& P, const unsigned long long* ctr, unsigned long long target) {
  if (dr_ld_volatile(P.status)) return;
  const long long t0 = clock64();
  for (unsigned it = 1; dr_ld_acquire_sys(ctr) < target; ++it) {
    if ((it & 63u) == 0) {
      if (dr_ld_volatile(P.status)) return;
      if (clock64() - t0 > (1ll << 33)) {
        atomicExch(P.status, Q8_ERR_COMM);
        return;
      }
    }
  }
}
__device__ __forceinline__ void dr_xwait(const DrParams& P, const unsigned long long* ctr, unsigned long long target) {
  if (threadIdx.x == 0) dr_xwait1(P, ctr, target);
  dr_csync();
}
// This CTA's arrival on every rank's counter `k` after the consumer threads'
// stores into the ranks' inboxes: the CTA barrier orders every thread's
// stores before the arriving threads, whose system-scope release increments
// are cumulative over what they observed (one release per rank instead of a
// system fence in every thread).
__device__ __forceinline__ void dr_xarrive(const DrParams& P, int k) {
  dr_csync();
  if (threadIdx.x < DR_MAXTP) {
    unsigned long long* ctr = nullptr;
#pragma unroll
    for (int r = 0; r < DR_MAXTP; ++r)  // static indices into the parameter arrays
      if (threadIdx.x == r && r < P.tp) ctr = P.xcnt[r];
    if (ctr) asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(ctr + k) : "memory");
  }
}

// Every consumer thread's stores of the phase (ordered before thread 0 by the
// CTA barrier), then one gpu-scope release increment.
__device__ __forceinline__ void dr_grid_arrive(const DrParams& P) {
  dr_csync();
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(P.bar) : "memory");
}

__device__ __forceinline__ void dr_ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void dr_imma(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// CTA 0's phase timeline (profiling): globaltimer into trace[ph * 4 + j].
__device__ __forceinline__ void dr_mark(const DrParams& P, int ph, int j) {
  if (P.trace && blockIdx.x == 0 && threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    P.trace[ph * 4 + j] = t;
  }
}

// ------------------------------------------------------------------ phases
// Phase ph of the step: layer ph / 5, kind ph % 5; the last phase is lm_head.
__device__ __forceinline__ int dr_kind(const DrParams& P, int ph) { return ph == 5 * P.L ? DP_LM : ph % 5; }

// CTAs a split phase of S stages (C per tile) spreads over: at most G, and
// few enough that every range holds at least ceil(C / 2) stages, so that a
// tile meets at most 3 ranges.
__host__ __device__ __forceinline__ int dr_split_ctas(long long S, int C, int G) {
  const long long per = (C + 1) / 2;
  const long long g = S / per;
  return (int)(g < G ? (g < 1 ? 1 : g) : G);
}

// One GEMV phase as one CTA sees it.
struct DrG {
  const uint8_t* W;  // the matrix in ring layout (block st at W + st * DR_BLOCK)
  int K, C, T;   // inputs, 512-code chunks per row, 16-row tiles
  int F2;        // SwiGLU: rows of tile t are gate t*8.. and up F2 + t*8..; 0: rows t*16..
  int s0, s1;    // this CTA's stages [s0, s1) of T*C
  int split;     // tiles may be shared by CTAs (partial rows into slots)
};

__device__ __forceinline__ DrG dr_gemv_desc(const DrParams& P, int kind, int L) {
  DrG d;
  int N;
  const DrLayer* ly = P.layers + (kind == DP_LM ? 0 : L);
  d.F2 = 0;
  d.split = 0;
  switch (kind) {
    case DP_QKV: d.W = ly->qkv; d.K = P.H; N = P.nqkv; break;
    case DP_O: d.W = ly->o; d.K = P.qdp; N = P.H; break;
    case DP_GU: d.W = ly->gu; d.K = P.H; N = P.F; d.F2 = P.F; break;
    case DP_DOWN: d.W = ly->down; d.K = P.Fp; N = P.H; d.split = dr_down_split(P.Fp); break;
    default: d.W = P.lm_head; d.K = P.H; N = P.V; break;
  }
  d.T = d.F2 ? N / 8 : N / 16;
  d.C = d.K / DR_CK;
  const int G = gridDim.x, c = blockIdx.x;
  if (d.split) {  // over the first dr_split_ctas CTAs: each range holds >= C/2 stages
    const long long S = (long long)d.T * d.C;
    const int Gs = dr_split_ctas(S, d.C, G);
    d.s0 = c < Gs ? (int)(S * c / Gs) : (int)S;
    d.s1 = c < Gs ? (int)(S * (c + 1) / Gs) : (int)S;
  } else {
    d.s0 = (int)((long long)d.T * c / G) * d.C;
    d.s1 = (int)((long long)d.T * (c + 1) / G) * d.C;
  }
  return d;
}

// CTA whose split range holds stage x: the largest c with floor(c S / Gs) <= x.
__device__ __forceinline__ int dr_cta_of(long long x, long long S, int C) {
  const long long Gs = dr_split_ctas(S, C, gridDim.x);
  return (int)(((x + 1) * Gs - 1) / S);
}

// ------------------------------------------------------------------ producer
__device__ __forceinline__ void dr_issue_stage(const DrParams& P, const DrG& d, int st, uint8_t* ring,
                                               uint64_t* full, uint64_t* empty, int slot, int use, int lane) {
  if (use > 0) dr_mwait(&empty[slot], (uint32_t)((use - 1) & 1), P.status);
  if (lane == 0) {
    mbar_arrive_expect_tx(&full[slot], DR_BLOCK);
    bulk_g2s(ring + slot * DR_SLOT_BYTES, d.W + (int64_t)st * DR_BLOCK, DR_BLOCK, &full[slot]);
  }
}

template <int HD>
__device__ __forceinline__ void dr_produce_attn(const DrParams& P, int L, uint8_t* ring, uint64_t* full,
                                                uint64_t* empty, int (&u)[DR_CW], int lane) {
  const int c = blockIdx.x, ns = P.nsplit;
  if (c >= P.nkv * ns) return;
  const int kvh = c / ns, sp = c % ns;
  const int p = P.pos[0], kv_end = p + 1, nb = (kv_end + 15) / 16;
  const int bl0 = (int)((long long)sp * nb / ns), bl1 = (int)((long long)(sp + 1) * nb / ns);
  const int32_t* btr = P.bt + (int64_t)P.seq[0] * P.max_pages;
  const float* kp = P.layers[L].kp;
  const float* vp = P.layers[L].vp;
  const int nblk = bl1 - bl0;
  for (int r = 0; r * DR_CW < nblk; ++r) {
#pragma unroll
    for (int w = 0; w < DR_CW; ++w) {
      const int i = r * DR_CW + w;
      if (i < nblk) {
        const int sk = 2 * w + (u[w] & 1), uk = u[w] >> 1;
        const int sv = 2 * w + ((u[w] + 1) & 1), uv = (u[w] + 1) >> 1;
        if (uk > 0) dr_mwait(&empty[sk], (uint32_t)((uk - 1) & 1), P.status);
        if (uv > 0) dr_mwait(&empty[sv], (uint32_t)((uv - 1) & 1), P.status);
        const int key0 = (bl0 + i) * 16;
        const int64_t row0 = ((int64_t)btr[key0 / P.page] * P.nkv + kvh) * P.page + (key0 % P.page);
        // 16 consecutive rows of one page: one bulk copy each for K and V
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[sk], 16 * HD * 4);
          bulk_g2s(ring + sk * DR_SLOT_BYTES, kp + row0 * HD, 16 * HD * 4, &full[sk]);
          mbar_arrive_expect_tx(&full[sv], 16 * HD * 4);
          bulk_g2s(ring + sv * DR_SLOT_BYTES, vp + row0 * HD, 16 * HD * 4, &full[sv]);
        }
        u[w] += 2;
      }
    }
  }
}

template <int HD>
__device__ void dr_producer(const DrParams& P, uint8_t* ring, uint64_t* full, uint64_t* empty) {
  const int lane = threadIdx.x & 31;
  int u[DR_CW];
#pragma unroll
  for (int w = 0; w < DR_CW; ++w) u[w] = 0;
  const int nphase = 5 * P.L + 1;
  for (int ph = 0; ph < nphase; ++ph) {
    if (dr_ld_volatile(P.status)) break;
    const int kind = dr_kind(P, ph), L = ph / 5;
    if (kind == DP_ATTN) {
      dr_produce_attn<HD>(P, L, ring, full, empty, u, lane);
      continue;
    }
    const DrG d = dr_gemv_desc(P, kind, L);
    const int n = d.s1 - d.s0, runs = (n + DR_CW - 1) / DR_CW;
    for (int r = 0; r < runs; ++r) {
#pragma unroll
      for (int w = 0; w < DR_CW; ++w) {
        const int a = d.s0 + (int)((long long)n * w / DR_CW), b = d.s0 + (int)((long long)n * (w + 1) / DR_CW);
        if (a + r < b) {
          dr_issue_stage(P, d, a + r, ring, full, empty, 2 * w + (u[w] & 1), u[w] >> 1, lane);
          ++u[w];
        }
      }
    }
  }
  // no copy may still be landing in this CTA's shared memory when it exits
#pragma unroll
  for (int w = 0; w < DR_CW; ++w) {
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const int uses = (u[w] + 1 - b) >> 1;
      if (uses > 0) dr_mwait(&full[2 * w + b], (uint32_t)((uses - 1) & 1), P.status);
    }
  }
}

// ------------------------------------------------------------------ activation staging
// Digits of one 64-group into xq [group][digit][64] with the k order the
// B fragments read (byte t*16 + j*4 + b holds k = 16 j + 4 t + b, so lane t
// of a quad gets both k32 halves of the group with one 16-byte load), and
// (e, e/254, e/254^2, 0) into fcol [group].  Four lanes per group (sq = lane &
// 3 holds k = 16 sq .. 16 sq + 15); every lane of the warp takes part.
__device__ __forceinline__ void dr_digits16(const float (&v)[16], bool valid, int gi, int sq, uint8_t* xq,
                                            float4* fcol) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  if (!valid) return;
  const float e = amax / 127.0f;
  const float ie = amax > 0.f ? 127.0f / amax : 0.f;
  uint8_t* dq = xq + (int64_t)gi * 192 + sq * 4;
  // Round-to-nearest-even through the f32 adder: for |x| < 2^22, y = x +
  // 1.5 * 2^23 holds rint(x) exactly, y - 1.5 * 2^23 is that integer as a
  // float and the low byte of y's bits is it modulo 256 (the conversion
  // instructions run at a fraction of the adder's rate).  Every digit is
  // within [-127, 127]: |x| <= 127 for the first, |residual| <= 0.5 * 254 for
  // the others.
  constexpr float kM = 12582912.0f;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    uint32_t y0[4], y1[4], y2[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const float x = v[4 * t + b] * ie;
      const float r0 = __fadd_rn(x, kM);
      const float x1 = __fmul_rn(__fsub_rn(x, __fsub_rn(r0, kM)), 254.0f);
      const float r1 = __fadd_rn(x1, kM);
      const float x2 = __fmul_rn(__fsub_rn(x1, __fsub_rn(r1, kM)), 254.0f);
      const float r2 = __fadd_rn(x2, kM);
      y0[b] = __float_as_uint(r0);
      y1[b] = __float_as_uint(r1);
      y2[b] = __float_as_uint(r2);
    }
    // low bytes of the four values, in value order
    *reinterpret_cast<uint32_t*>(dq + t * 16) =
        __byte_perm(__byte_perm(y0[0], y0[1], 0x0040), __byte_perm(y0[2], y0[3], 0x0040), 0x5410);
    *reinterpret_cast<uint32_t*>(dq + 64 + t * 16) =
        __byte_perm(__byte_perm(y1[0], y1[1], 0x0040), __byte_perm(y1[2], y1[3], 0x0040), 0x5410);
    *reinterpret_cast<uint32_t*>(dq + 128 + t * 16) =
        __byte_perm(__byte_perm(y2[0], y2[1], 0x0040), __byte_perm(y2[2], y2[3], 0x0040), 0x5410);
  }
  if (sq == 0) fcol[gi] = make_float4(e, e / 254.0f, e / 64516.0f, 0.f);
}

// 16 values x[k0 .. k0+15] of the phase's input vector: the step's Q8
// embedding row (embed), or src + nslots partial slots (stride H); every load
// of the item is in flight before the first is used.
template <bool XP>
__device__ __forceinline__ void dr_load16(const DrParams& P, bool embed, const float* src, const float* slots,
                                          int nslots, int k0, float (&v)[16]) {
  if (embed) {
    const int64_t rb = (int64_t)P.H + P.H / 32;
    const uint8_t* row = P.embed + (int64_t)P.ids[0] * rb;
    const float s = __half2float(__ushort_as_half(reinterpret_cast<const unsigned short*>(row)[k0 / 64]));
    const uint4 q = *reinterpret_cast<const uint4*>(row + P.H / 32 + k0);
    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = (float)(int8_t)((qw[i >> 2] >> (8 * (i & 3))) & 0xFF) * s;
    return;
  }
  else {
  float4 a[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) a[i] = __ldcg(reinterpret_cast<const float4*>(src + k0) + i);
  if constexpr (!XP) {  // + this GPU's partial slots (<= DR_NS), in slot order
    float4 pp[DR_NS][4];
#pragma unroll
    for (int sl = 0; sl < DR_NS; ++sl)
#pragma unroll
      for (int i = 0; i < 4; ++i)
        pp[sl][i] = sl < nslots ? __ldcg(reinterpret_cast<const float4*>(slots + (int64_t)sl * P.H + k0) + i)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int sl = 0; sl < DR_NS; ++sl) {
      if (sl < nslots) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          a[i].x += pp[sl][i].x; a[i].y += pp[sl][i].y; a[i].z += pp[sl][i].z; a[i].w += pp[sl][i].w;
        }
      }
    }
  }
  if constexpr (XP) {  // + every rank's partial slots, in rank and slot order
    for (int s0 = 0; s0 < nslots; s0 += DR_NS) {
      float4 pp[DR_NS][4];
#pragma unroll
      for (int sl = 0; sl < DR_NS; ++sl)
#pragma unroll
        for (int i = 0; i < 4; ++i)
          pp[sl][i] = s0 + sl < nslots
                          ? __ldcg(reinterpret_cast<const float4*>(slots + (int64_t)(s0 + sl) * P.H + k0) + i)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int sl = 0; sl < DR_NS; ++sl) {
        if (s0 + sl < nslots) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            a[i].x += pp[sl][i].x; a[i].y += pp[sl][i].y; a[i].z += pp[sl][i].z; a[i].w += pp[sl][i].w;
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[4 * i] = a[i].x; v[4 * i + 1] = a[i].y; v[4 * i + 2] = a[i].z; v[4 * i + 3] = a[i].w;
  }
  }
}

// Stages the H inputs of an RMSNorm'd GEMV phase (q|k|v, gate|up, lm_head) as
// digits: the norm weights read first, then the wait for the previous phase
// of the grid (target arrivals; 0: none) or, with xc, for `xtarget` arrivals
// of all ranks on that exchange counter; then x (dr_load16), x = nw * x /
// sqrt(mean(x^2) + eps) (one 16-value item per thread); with wb, this CTA's
// slice of the raw x is written back (the residual).  One inlined copy of
// this code serves every such phase (the instruction cache holds little of
// the step).
template <bool XP>
__device__ __forceinline__ void dr_stage_rms(const DrParams& P, int ph, unsigned int target, const unsigned long long* xc,
                                          unsigned long long xtarget, bool embed, const float* src, const float* slots,
                                          int nslots, const uint16_t* nw, float* wb, uint8_t* xq, float4* fcol,
                                          float* scr) {
  const int K = P.H;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, sq = lane & 3;
  const int nitem = K / 16;  // quarter-groups
  const bool valid = tid < nitem;
  const int k0 = tid * 16;
  uint4 w0 = make_uint4(0, 0, 0, 0), w1 = w0;
  if (valid) {
    w0 = __ldg(reinterpret_cast<const uint4*>(nw + k0));
    w1 = __ldg(reinterpret_cast<const uint4*>(nw + k0 + 8));
  }
  if (xc) dr_xwait(P, xc, xtarget);
  else if (target) dr_grid_wait(P, target);
  dr_mark(P, ph, 0);
  float v[16];
  float ss = 0.f;
  if (valid) {
    dr_load16<XP>(P, embed, src, slots, nslots, k0, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) ss = fmaf(v[i], v[i], ss);
    if (wb) {
      const int G = gridDim.x, c = blockIdx.x;
      const int s0 = (int)((long long)K * c / G), s1 = (int)((long long)K * (c + 1) / G);
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (k0 + i >= s0 && k0 + i < s1) wb[k0 + i] = v[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = 0.f;
  }
  ss = warp_sum(ss);
  if (lane == 0) scr[warp] = ss;
  dr_csync();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < DR_CW; ++w) tot += scr[w];
  const float inv = 1.0f / sqrtf(tot / (float)K + P.eps);
  if (valid) {
    const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[2 * i] = __uint_as_float(ww[i] << 16) * v[2 * i] * inv;
      v[2 * i + 1] = __uint_as_float(ww[i] & 0xFFFF0000u) * v[2 * i + 1] * inv;
    }
  }
  dr_digits16(v, valid, valid ? tid >> 2 : 0, sq, xq, fcol);
  dr_csync();
}

// Stages the K inputs of o_proj / down_proj (plain f32 rows, zero digits up
// to the padded Kd) after the previous phase of the grid.
template <bool XP>
__device__ __forceinline__ void dr_stage_plain(const DrParams& P, int ph, unsigned int target, int Kd, int K,
                                            const float* src, uint8_t* xq, float4* fcol) {
  constexpr int NT = DR_CW * 32;
  const int tid = threadIdx.x, lane = tid & 31, sq = lane & 3;
  const int nitem = K / 16;
  dr_grid_wait(P, target);
  dr_mark(P, ph, 0);
  constexpr int R = 2;  // rounds whose loads are in flight together
  const int nitem_d = Kd / 16;  // with the zero padding
  for (int base = 0; base < nitem_d; base += R * NT) {
    float v[R][16];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int item = base + r * NT + tid;
      if (item < nitem) dr_load16<XP>(P, false, src, nullptr, 0, item * 16, v[r]);
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int item = base + r * NT + tid;
      if (base + r * NT < nitem_d) {
        const bool valid = item < nitem_d;
        if (!valid || item >= nitem) {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[r][i] = 0.f;
        }
        dr_digits16(v[r], valid, valid ? item >> 2 : 0, sq, xq, fcol);
      }
    }
  }
  dr_csync();
}

// ------------------------------------------------------------------ GEMV consumer
// A warp's sums of local tile lt: row g = digit columns 0 + 1 (lane t = 0)
// + 2 (lane t = 1), in column order; the same for row g + 8.
__device__ __forceinline__ void dr_flush(float* red, int lt, int warp, int g, int t, const float (&acc)[4]) {
  const float x0 = __shfl_sync(0xffffffffu, acc[0], g * 4 + 1);
  const float x2 = __shfl_sync(0xffffffffu, acc[2], g * 4 + 1);
  if (t == 0) {
    float* rw = red + (lt * DR_CW + warp) * 16;
    rw[g] = acc[0] + acc[1] + x0;
    rw[g + 8] = acc[2] + acc[3] + x2;
  }
}

// Warp `warp` drains its run of the CTA's stages; per-tile sums into red
// [local tile][warp][16 rows].
__device__ __forceinline__ void dr_gemv_run(const DrParams& P, const DrG& d, uint8_t* ring, uint64_t* full,
                                            uint64_t* empty, const uint8_t* xq, const float4* fcol, float* red, int& u,
                                            int warp, int lane) {
  const int n = d.s1 - d.s0;
  const int a = d.s0 + (int)((long long)n * warp / DR_CW), b = d.s0 + (int)((long long)n * (warp + 1) / DR_CW);
  const int t_lo = d.s0 / d.C;
  const int g = lane >> 2, t = lane & 3;
  // ldmatrix x4: lane l addresses row rr + 8 (l >> 3 & 1) of the 16 rows and
  // 16-byte chunk (l >> 4) of the k32 half; a box row holds 8 chunks stored
  // at chunk ^ (row & 7) (128 B swizzle)
  const int mat = lane >> 3, rr = lane & 7;
  const int lrow = rr + 8 * (mat & 1), mh = mat >> 1;
  const uint32_t lofs = (uint32_t)(lrow * 128);
  const bool has_col = g < 3;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  int cur = -1;
  for (int st = a; st < b; ++st) {
    const int tile = st / d.C, ch = st % d.C;
    if (tile != cur) {
      if (cur >= 0) dr_flush(red, cur - t_lo, warp, g, t, acc);
      cur = tile;
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
    }
    const int slot = 2 * warp + (u & 1);
    dr_mwait(&full[slot], (uint32_t)((u >> 1) & 1), P.status);
    const uint8_t* sb = ring + slot * DR_SLOT_BYTES;
    const uint32_t sbase = smem_u32(sb) + lofs;
    const uint4 sA = *reinterpret_cast<const uint4*>(sb + 16 * DR_CK + g * 16);
    const uint4 sB = *reinterpret_cast<const uint4*>(sb + 16 * DR_CK + (g + 8) * 16);
#pragma unroll
    for (int grp = 0; grp < 8; ++grp) {
      const int gi = ch * 8 + grp;
      const int c0 = 4 * (grp & 1) + mh;
      const uint32_t bx0 = sbase + (grp >> 1) * 2048;
      uint32_t a0, a1, a2, a3, a4, a5, a6, a7;
      dr_ldsm_x4(bx0 + ((c0 ^ rr) << 4), a0, a1, a2, a3);
      dr_ldsm_x4(bx0 + (((c0 + 2) ^ rr) << 4), a4, a5, a6, a7);
      uint4 bx = make_uint4(0, 0, 0, 0);
      if (has_col) bx = *reinterpret_cast<const uint4*>(xq + (int64_t)gi * 192 + g * 64 + t * 16);
      int dd[4] = {0, 0, 0, 0};
      dr_imma(dd, a0, a1, a2, a3, bx.x, bx.y);
      dr_imma(dd, a4, a5, a6, a7, bx.z, bx.w);
      const float4 f = fcol[gi];
      const float fc0 = t == 0 ? f.x : (t == 1 ? f.z : 0.f);
      const float fc1 = t == 0 ? f.y : 0.f;
      const uint32_t wa = (grp >> 1) == 0 ? sA.x : ((grp >> 1) == 1 ? sA.y : ((grp >> 1) == 2 ? sA.z : sA.w));
      const uint32_t wb = (grp >> 1) == 0 ? sB.x : ((grp >> 1) == 1 ? sB.y : ((grp >> 1) == 2 ? sB.z : sB.w));
      const float sa = __half2float(__ushort_as_half((unsigned short)((grp & 1) ? (wa >> 16) : (wa & 0xFFFFu))));
      const float sc = __half2float(__ushort_as_half((unsigned short)((grp & 1) ? (wb >> 16) : (wb & 0xFFFFu))));
      acc[0] = fmaf(__int2float_rn(dd[0]), sa * fc0, acc[0]);
      acc[1] = fmaf(__int2float_rn(dd[1]), sa * fc1, acc[1]);
      acc[2] = fmaf(__int2float_rn(dd[2]), sc * fc0, acc[2]);
      acc[3] = fmaf(__int2float_rn(dd[3]), sc * fc1, acc[3]);
    }
    __syncwarp();
    if (lane == 0) dr_arrive(&empty[slot]);
    ++u;
  }
  if (cur >= 0) dr_flush(red, cur - t_lo, warp, g, t, acc);
}

// Sum of row r (0..15) of local tile lt over the warps whose runs cover it.
__device__ __forceinline__ float dr_tile_sum(const DrG& d, const float* red, int lt, int r) {
  const int n = d.s1 - d.s0, tile = d.s0 / d.C + lt;
  const int ta = max(d.s0, tile * d.C), tb = min(d.s1, (tile + 1) * d.C);
  float v = 0.f;
#pragma unroll
  for (int w = 0; w < DR_CW; ++w) {
    const int a = d.s0 + (int)((long long)n * w / DR_CW), b = d.s0 + (int)((long long)n * (w + 1) / DR_CW);
    if (a < b && a < tb && b > ta) v += red[(lt * DR_CW + w) * 16 + r];
  }
  return v;
}

__device__ __forceinline__ unsigned long long dr_key(float v, int idx) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (uint32_t)(~(uint32_t)idx);
}

// splits whose partials one thread of the merging CTA has in flight together
constexpr int DR_MRG = 10;

// ------------------------------------------------------------------ attention consumer

template <int HD>
__device__ void dr_attn(const DrParams& P, int L, uint8_t* ring, uint64_t* full, uint64_t* empty, int& u, float* sQ,
                        float* sP, float* sKn, float* sVn, float* sX, float (*sm_m)[DR_GMAX],
                        float (*sm_l)[DR_GMAX], int* s_last, const float* sRope, int ph) {
  constexpr int E = HD / 32, CH = HD / 4, J = HD / 32;
  const int c = blockIdx.x, ns = P.nsplit;
  if (c >= P.nkv * ns) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = c / ns, sp = c % ns, G = P.nh / P.nkv;
  const int p = P.pos[0], kv_end = p + 1, nb = (kv_end + 15) / 16;
  const int bl0 = (int)((long long)sp * nb / ns), bl1 = (int)((long long)(sp + 1) * nb / ns);
  const int nblk = bl1 - bl0;
  const int32_t* btr = P.bt + (int64_t)P.seq[0] * P.max_pages;
  const DrLayer* ly = P.layers + L;
  const bool own_new = p >= bl0 * 16 && p < bl1 * 16;

  // prologue: the G q heads (QK-norm, RoPE, scaled) into sQ; the split that
  // holds position p rotates the new k, appends k and v to the cache and keeps
  // them in sKn / sVn for its own block
  {
    const float qscale = 1.4426950408889634f / sqrtf((float)HD);
    const int ntask = G + (own_new ? 1 : 0);
    const int tsk = warp;  // one task per warp (G + 1 <= DR_CW)
    if (tsk < ntask) {
      float v[J], vv[J];
      const float* src = P.qkv + (tsk < G ? (int64_t)(kvh * G + tsk) * HD : (int64_t)(P.nh + kvh) * HD);
#pragma unroll
      for (int j = 0; j < J; ++j) v[j] = __ldcg(src + lane + 32 * j);
      if (tsk == G) {
        const float* vsrc = P.qkv + (int64_t)(P.nh + P.nkv + kvh) * HD;
#pragma unroll
        for (int j = 0; j < J; ++j) vv[j] = __ldcg(vsrc + lane + 32 * j);
      }
      const uint16_t* nw = tsk < G ? ly->q_norm : ly->k_norm;
      if (nw) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < J; ++j) ss = fmaf(v[j], v[j], ss);
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)HD + P.eps);
#pragma unroll
        for (int j = 0; j < J; ++j) v[j] = bf16_bits_to_f32(nw[lane + 32 * j]) * v[j] * inv;
      }
#pragma unroll
      for (int j = 0; j < J / 2; ++j) {
        float sn, cs;
        cs = sRope[lane + 32 * j];  // cos / sin of the step's position, made at launch
        sn = sRope[64 + lane + 32 * j];
        const float x0 = v[j], x1 = v[j + J / 2];
        v[j] = x0 * cs - x1 * sn;
        v[j + J / 2] = x1 * cs + x0 * sn;
      }
      if (tsk < G) {
#pragma unroll
        for (int j = 0; j < J; ++j) sQ[tsk * HD + lane + 32 * j] = v[j] * qscale;
      } else {
        const int64_t off = (((int64_t)btr[p / P.page] * P.nkv + kvh) * P.page + (p % P.page)) * HD;
#pragma unroll
        for (int j = 0; j < J; ++j) {
          ly->kp[off + lane + 32 * j] = v[j];
          ly->vp[off + lane + 32 * j] = vv[j];
          sKn[lane + 32 * j] = v[j];
          sVn[lane + 32 * j] = vv[j];
        }
      }
    }
    dr_csync();
  }

  dr_mark(P, ph, 1);  // prologue done
  float m[DR_GMAX], l[DR_GMAX], o[DR_GMAX][E];
#pragma unroll
  for (int g = 0; g < DR_GMAX; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) o[g][e] = 0.f;
  }
  float* pw = sP + warp * DR_GMAX * 16;
  const int jr = lane >> 1, hh = 4 * (lane & 1);
  const bool lead = (lane & 1) == 0;
  for (int i = warp; i < nblk; i += DR_CW) {
    const int sk = 2 * warp + (u & 1), uk = u >> 1;
    const int sv = 2 * warp + ((u + 1) & 1), uv = (u + 1) >> 1;
    const int key0 = (bl0 + i) * 16;
    const int nv = min(16, kv_end - key0);
    float* kb = reinterpret_cast<float*>(ring + sk * DR_SLOT_BYTES);
    float* vb = reinterpret_cast<float*>(ring + sv * DR_SLOT_BYTES);
    dr_mwait(&full[sk], (uint32_t)(uk & 1), P.status);
    dr_mwait(&full[sv], (uint32_t)(uv & 1), P.status);
    if (own_new && p >= key0 && p < key0 + 16) {  // the appended row, from the prologue
      for (int c4 = lane; c4 < CH; c4 += 32) {
        *reinterpret_cast<float4*>(kb + (p - key0) * HD + 4 * c4) = *reinterpret_cast<const float4*>(sKn + 4 * c4);
        *reinterpret_cast<float4*>(vb + (p - key0) * HD + 4 * c4) = *reinterpret_cast<const float4*>(sVn + 4 * c4);
      }
      // these generic writes land before the bulk copy that later refills the slots
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
    }
    float s[DR_GMAX];
    {
      float s0[DR_GMAX], s1[DR_GMAX];
#pragma unroll
      for (int g = 0; g < DR_GMAX; ++g) s0[g] = s1[g] = 0.f;
      const float4* q4 = reinterpret_cast<const float4*>(sQ);
#pragma unroll 2
      for (int cc = 0; cc < CH / 2; cc += 2) {
        // this lane's half of the chunks (hh), in an order rotated by the
        // position: the 4 positions x 2 halves of an 8-lane phase read 8
        // different bank groups of the plain K rows (and of q)
        const int grp8 = (cc >> 2) << 3;
        const int c0 = grp8 + hh + ((cc + jr) & 3), c1 = grp8 + hh + ((cc + 1 + jr) & 3);
        const float4 k0 = *reinterpret_cast<const float4*>(kb + jr * HD + 4 * c0);
        const float4 k1 = *reinterpret_cast<const float4*>(kb + jr * HD + 4 * c1);
#pragma unroll
        for (int g = 0; g < DR_GMAX; ++g) {
          if (g < G) {
            const float4 qa = q4[g * CH + c0], qb = q4[g * CH + c1];
            s0[g] = fmaf(qa.w, k0.w, fmaf(qa.z, k0.z, fmaf(qa.y, k0.y, fmaf(qa.x, k0.x, s0[g]))));
            s1[g] = fmaf(qb.w, k1.w, fmaf(qb.z, k1.z, fmaf(qb.y, k1.y, fmaf(qb.x, k1.x, s1[g]))));
          }
        }
      }
#pragma unroll
      for (int g = 0; g < DR_GMAX; ++g) {
        const float part = s0[g] + s1[g];
        const float other = __shfl_xor_sync(0xffffffffu, part, 1);
        s[g] = (lane & 1) ? other + part : part + other;
      }
    }
    // the K rows are read: the producer may refill that slot during the PV
    // product (the next block's K then loads while this block's V is used)
    __syncwarp();
    if (lane == 0) dr_arrive(&empty[sk]);
#pragma unroll
    for (int g = 0; g < DR_GMAX; ++g) {
      if (g >= G) break;
      const float sc = jr < nv ? s[g] : -INFINITY;
      const float mn = fmaxf(m[g], warp_max(sc));
      const float corr = exp2f(m[g] - mn);
      const float pz = jr < nv ? exp2f(sc - mn) : 0.f;
      l[g] = fmaf(l[g], corr, lead ? pz : 0.f);
#pragma unroll
      for (int e = 0; e < E; ++e) o[g][e] *= corr;
      m[g] = mn;
      if (lead) pw[g * 16 + jr] = pz;
    }
    __syncwarp();
    for (int j0 = 0; j0 < nv; j0 += 4) {
      float4 pp[DR_GMAX];
#pragma unroll
      for (int g = 0; g < DR_GMAX; ++g)
        if (g < G) pp[g] = *reinterpret_cast<const float4*>(pw + g * 16 + j0);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (j0 + q < nv) {
          float x[E];
          const float* vr = vb + (j0 + q) * HD + lane * E;
          if constexpr (E == 4) {
            const float4 tt = *reinterpret_cast<const float4*>(vr);
            x[0] = tt.x; x[1] = tt.y; x[2] = tt.z; x[3] = tt.w;
          } else {
            const float2 tt = *reinterpret_cast<const float2*>(vr);
            x[0] = tt.x; x[1] = tt.y;
          }
#pragma unroll
          for (int g = 0; g < DR_GMAX; ++g) {
            if (g < G) {
              const float pg = q == 0 ? pp[g].x : (q == 1 ? pp[g].y : (q == 2 ? pp[g].z : pp[g].w));
#pragma unroll
              for (int e = 0; e < E; ++e) o[g][e] = fmaf(pg, x[e], o[g][e]);
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) dr_arrive(&empty[sv]);
    u += 2;
  }
#pragma unroll
  for (int g = 0; g < DR_GMAX; ++g) l[g] = warp_sum(l[g]);
  dr_mark(P, ph, 2);  // this warp's blocks done (marks come from warp 0)

  // merge the consumer warps: (m, l, o) per head, o staged in sX
  float* sO = sX;  // [DR_CW][DR_GMAX][HD]
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < DR_GMAX; ++g) {
      sm_m[warp][g] = m[g];
      sm_l[warp][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < DR_GMAX; ++g) {
    if (g >= G) break;
#pragma unroll
    for (int e = 0; e < E; ++e) sO[(warp * DR_GMAX + g) * HD + lane * E + e] = o[g][e];
  }
  dr_csync();
  const int WS = G * HD + ((2 * G + 3) & ~3);
  constexpr int NT = DR_CW * 32;
  float* mypart = P.apart + ((int64_t)kvh * ns + sp) * WS;
  for (int i = threadIdx.x; i < G * HD; i += NT) {
    const int g = i / HD, dd = i % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < DR_CW; ++w) M = fmaxf(M, sm_m[w][g]);
    float Ls = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < DR_CW; ++w) {
        if (sm_m[w][g] == -INFINITY) continue;
        const float f = exp2f(sm_m[w][g] - M);
        Ls = fmaf(sm_l[w][g], f, Ls);
        O = fmaf(sO[(w * DR_GMAX + g) * HD + dd], f, O);
      }
    }
    if (ns == 1) {
      P.ao[(int64_t)(kvh * G + g) * HD + dd] = Ls > 0.f ? O / Ls : 0.f;
    } else {
      mypart[i] = O;
      if (dd == 0) {
        mypart[G * HD + g] = M;
        mypart[G * HD + G + g] = Ls;
      }
    }
  }
  if (ns == 1) return;
  dr_csync();
  if (threadIdx.x == 0) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                 : "=r"(old)
                 : "l"(P.aticket + kvh)
                 : "memory");
    *s_last = old == ns - 1;
  }
  dr_csync();
  if (!*s_last) return;

  // last split CTA of this kv head: fold the splits in split order (runs of
  // splits per thread, then the runs in order), write the heads' outputs
  const float* base = P.apart + (int64_t)kvh * ns * WS;
  const int nchunk = G * HD / 4;
  const int nrun = max(1, min(ns, NT / nchunk));
  float4* sred = reinterpret_cast<float4*>(sX + DR_CW * DR_GMAX * HD);
  float2* sml = reinterpret_cast<float2*>(sred + nrun * nchunk);
  for (int tt = threadIdx.x; tt < nrun * nchunk; tt += NT) {
    const int i4 = tt % nchunk, run = tt / nchunk;
    const int g = (4 * i4) / HD;
    const int r0 = run * ns / nrun, r1 = (run + 1) * ns / nrun;
    float M = -INFINITY, Ls = 0.f;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = r0; s0 < r1; s0 += DR_MRG) {
      float4 v[DR_MRG];
      float ms[DR_MRG], ls[DR_MRG];
#pragma unroll
      for (int q = 0; q < DR_MRG; ++q) {
        const bool ok = s0 + q < r1;
        const float* ps = base + (int64_t)(s0 + q) * WS;
        v[q] = ok ? __ldcg(reinterpret_cast<const float4*>(ps) + i4) : make_float4(0.f, 0.f, 0.f, 0.f);
        ms[q] = ok ? __ldcg(ps + G * HD + g) : -INFINITY;
        ls[q] = ok ? __ldcg(ps + G * HD + G + g) : 0.f;
      }
#pragma unroll
      for (int q = 0; q < DR_MRG; ++q) {
        if (ms[q] == -INFINITY) continue;
        const float mn = fmaxf(M, ms[q]);
        const float cf = exp2f(M - mn), f = exp2f(ms[q] - mn);
        O.x = fmaf(v[q].x, f, O.x * cf);
        O.y = fmaf(v[q].y, f, O.y * cf);
        O.z = fmaf(v[q].z, f, O.z * cf);
        O.w = fmaf(v[q].w, f, O.w * cf);
        Ls = fmaf(ls[q], f, Ls * cf);
        M = mn;
      }
    }
    sred[run * nchunk + i4] = O;
    sml[run * nchunk + i4] = make_float2(M, Ls);
  }
  dr_csync();
  for (int i4 = threadIdx.x; i4 < nchunk; i4 += NT) {
    float4 O = sred[i4];
    float M = sml[i4].x, Ls = sml[i4].y;
    for (int run = 1; run < nrun; ++run) {
      const float2 ml = sml[run * nchunk + i4];
      if (ml.x == -INFINITY) continue;
      const float4 x = sred[run * nchunk + i4];
      const float mn = fmaxf(M, ml.x);
      const float cf = exp2f(M - mn), f = exp2f(ml.x - mn);
      O.x = fmaf(x.x, f, O.x * cf);
      O.y = fmaf(x.y, f, O.y * cf);
      O.z = fmaf(x.z, f, O.z * cf);
      O.w = fmaf(x.w, f, O.w * cf);
      Ls = fmaf(ml.y, f, Ls * cf);
      M = mn;
    }
    float* dst = P.ao + (int64_t)kvh * G * HD + 4 * i4;
    dst[0] = Ls > 0.f ? O.x / Ls : 0.f;
    dst[1] = Ls > 0.f ? O.y / Ls : 0.f;
    dst[2] = Ls > 0.f ? O.z / Ls : 0.f;
    dst[3] = Ls > 0.f ? O.w / Ls : 0.f;
  }
  if (threadIdx.x == 0) P.aticket[kvh] = 0;  // ready for the next layer
}

// ------------------------------------------------------------------ the step
template <int HD, bool XP>
__global__ void __launch_bounds__(DR_THREADS, 1) k_decode_ring(const DrParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* xq = ring + DR_RING;
  float4* fcol = reinterpret_cast<float4*>(xq + DR_XQ_BYTES);
  float* sQ = reinterpret_cast<float*>(xq + DR_XQ_BYTES + DR_FCOL_BYTES);
  float* sP = sQ + DR_GMAX * 128;
  float* sKn = sP + DR_CW * DR_GMAX * 16;
  float* sVn = sKn + 128;
  uint64_t* full = reinterpret_cast<uint64_t*>(sVn + 128);
  uint64_t* empty = full + DR_SLOTS;
  __shared__ float scr[DR_CW];
  __shared__ float sm_m[DR_CW][DR_GMAX], sm_l[DR_CW][DR_GMAX];
  __shared__ int s_last;
  __shared__ unsigned long long s_key[DR_CW];
  __shared__ unsigned long long s_epoch;  // completed steps of this rank (tensor parallel)
  __shared__ float s_rope[128];           // cos | sin of the step's position x inv_freq (RoPE)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == DR_CW * 32) {
    for (int s = 0; s < DR_SLOTS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == DR_CW) {
    dr_producer<HD>(P, ring, full, empty);
    return;
  }

  // ---------------------------------------------------------------- consumers
  const int G = gridDim.x, c = blockIdx.x;
  constexpr bool tp = XP;  // tensor-parallel instantiation
  // exchange targets grow across steps: the counters are never reset (a rank
  // may already count into a peer's counter for its next step before that
  // peer's launch begins)
  if constexpr (XP) {
    if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile unsigned long long*>(P.xstep);
  }
  if (threadIdx.x < HD / 2) {  // the same position for every layer of the step
    float sn, cs;
    sincosf((float)P.pos[0] * P.inv_freq[threadIdx.x], &sn, &cs);
    s_rope[threadIdx.x] = cs;
    s_rope[64 + threadIdx.x] = sn;
  }
  dr_csync();
  int u = 0;
  unsigned int target = 0;
  const int nphase = 5 * P.L + 1;
  for (int ph = 0; ph < nphase; ++ph) {
    const int kind = dr_kind(P, ph), L = ph / 5;
    if (ph > 0) target += (unsigned int)G;
    if (kind == DP_ATTN) {
      dr_grid_wait(P, target);
      dr_mark(P, ph, 0);
      dr_attn<HD>(P, L, ring, full, empty, u, sQ, sP, sKn, sVn, reinterpret_cast<float*>(xq), sm_m, sm_l, &s_last,
                  s_rope, ph);
      dr_grid_arrive(P);
      dr_mark(P, ph, 3);
      continue;
    }
    const DrG d = dr_gemv_desc(P, kind, L);
    const DrLayer* ly = P.layers + (kind == DP_LM ? 0 : L);
    float* hc = (L & 1) ? P.h1 : P.h0;  // this layer's residual
    // the stagings wait for the previous phase (after their static loads);
    // mark 0 is then the end of the wait.  Folds: the residual + the previous
    // down_proj's partials (this GPU's slots, or every rank's, in rank order);
    // under tensor parallelism gate|up's input also folds every rank's
    // o_proj partial and keeps the sum as the mid residual
    if (kind == DP_O || kind == DP_DOWN) {
      dr_stage_plain<XP>(P, ph, target, kind == DP_O ? P.qdp : P.Fp, kind == DP_O ? P.qd : P.F,
                         kind == DP_O ? P.ao : P.act, xq, fcol);
    } else {
      const int Lp = (kind == DP_LM ? P.L : L) - 1;  // layer of the down_proj folded in
      const unsigned long long* xc = nullptr;
      unsigned long long xt = 0;
      const float* src = tp ? P.hm : ((Lp & 1) ? P.h1 : P.h0);
      const float* slots = tp ? P.xin_me + dr_xin_region(Lp & 1, 1, P.tp, P.H) : P.pres;
      int nsl = tp ? P.tp * P.nsf : P.nsf;
      const uint16_t* nw = kind == DP_QKV ? ly->in_norm : (kind == DP_GU ? ly->post_norm : P.final_norm);
      float* wb = kind == DP_QKV ? hc : nullptr;
      if (tp && kind != DP_GU) {
        xc = P.xcnt_me + 1;
        xt = (s_epoch * (unsigned long long)P.L + (unsigned long long)Lp + 1) * (unsigned long long)P.gsum;
      }
      if (kind == DP_GU) {
        src = hc;
        if (tp) {
          xc = P.xcnt_me + 0;
          xt = (s_epoch * (unsigned long long)P.L + (unsigned long long)L + 1) * (unsigned long long)P.gsum;
          slots = P.xin_me + dr_xin_region(L & 1, 0, P.tp, P.H);
          nsl = P.tp;
          wb = P.hm;
        } else {
          nsl = 0;
        }
      }
      dr_stage_rms<XP>(P, ph, target, xc, xt, kind == DP_QKV && L == 0, src, slots, nsl, nw, wb, xq, fcol, scr);
    }
    float* red = reinterpret_cast<float*>(xq + (((size_t)d.K * 3 + 15) & ~(size_t)15));
    const int n = d.s1 - d.s0;
    const int t_lo = d.s0 / d.C;
    const int ntile = n > 0 ? (d.s1 - 1) / d.C - t_lo + 1 : 0;
    constexpr int NT = DR_CW * 32;
    // o_proj adds into the residual: its rows (at most 16 tiles, one per
    // thread) are read before the product so that the epilogue does not wait
    float hres = 0.f;
    if (!tp && kind == DP_O && threadIdx.x < ntile * 16) hres = __ldcg(hc + t_lo * 16 + threadIdx.x);
    dr_mark(P, ph, 1);
    dr_gemv_run(P, d, ring, full, empty, xq, fcol, red, u, warp, lane);
    dr_csync();
    dr_mark(P, ph, 2);

    // epilogue over the CTA's tiles
    if (kind == DP_GU) {
      for (int i = threadIdx.x; i < ntile * 8; i += NT) {
        const int lt = i >> 3, r = i & 7;
        const float gv = dr_tile_sum(d, red, lt, r), uv = dr_tile_sum(d, red, lt, r + 8);
        P.act[(int64_t)(t_lo + lt) * 8 + r] = silu_mul(gv, uv);
      }
    } else if (kind == DP_LM) {
      unsigned long long best = 0;
      for (int i = threadIdx.x; i < ntile * 16; i += NT) {
        const int lt = i >> 4, r = i & 15;
        const int row = (t_lo + lt) * 16 + r;
        const float v = dr_tile_sum(d, red, lt, r);
        P.logits[row] = v;
        const unsigned long long k = dr_key(v, P.V_off + row);
        best = k > best ? k : best;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long ok = __shfl_xor_sync(0xffffffffu, best, o);
        best = ok > best ? ok : best;
      }
      if (lane == 0) s_key[warp] = best;
      dr_csync();
      if (threadIdx.x == 0) {
        unsigned long long b = 0;
        for (int w = 0; w < DR_CW; ++w) b = s_key[w] > b ? s_key[w] : b;
        if (b) atomicMax(P.amax, b);
        int old;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                     : "=r"(old)
                     : "l"(P.lm_ticket)
                     : "memory");
        if (old == G - 1) {  // every CTA's maximum is in: the step's token
          unsigned long long k = atomicAdd(P.amax, 0ull);
          if (tp) {  // the ranks' maxima: into every rank's slot of this step, then count
            const unsigned long long epoch = s_epoch;
            const int sl = (int)(epoch & 1ull);
#pragma unroll
            for (int r = 0; r < DR_MAXTP; ++r)
              if (r < P.tp) atomicMax_system(P.xamax[r] + sl, k);
            __threadfence_system();
#pragma unroll
            for (int r = 0; r < DR_MAXTP; ++r)
              if (r < P.tp) asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(P.xcnt[r] + 2) : "memory");
            dr_xwait1(P, P.xcnt_me + 2, (epoch + 1ull) * (unsigned long long)P.tp);
            k = dr_ld_acquire_sys(P.xamax_me + sl);
            // every rank's key of this step is in: the slot is free for step + 2
            P.xamax_me[sl] = 0ull;
            *reinterpret_cast<volatile unsigned long long*>(P.xstep) = epoch + 1ull;
          }
          const int32_t tok = (int32_t)(~(uint32_t)(k & 0xFFFFFFFFull));
          P.argmax[0] = tok;
          if (P.gen) {
            const int step = *P.ctr;
            P.ids[0] = tok;
            P.pos[0] += 1;
            if (step < P.hist_cap) P.hist[step] = tok;
            *P.ctr = step + 1;
          }
          *P.amax = 0ull;
          *P.lm_ticket = 0;
        }
      }
      dr_mark(P, ph, 3);
      continue;  // the last phase: no arrival
    } else {
      for (int i = threadIdx.x; i < ntile * 16; i += NT) {
        const int lt = i >> 4, r = i & 15;
        const int tile = t_lo + lt, row = tile * 16 + r;
        const float v = dr_tile_sum(d, red, lt, r);
        if (kind == DP_QKV) {
          P.qkv[row] = v;
        } else if (kind == DP_O) {
          if (tp) {  // this rank's partial row into every rank's inbox
            const int64_t off = dr_xin_region(L & 1, 0, P.tp, P.H) + (int64_t)P.rank * P.H + row;
#pragma unroll
            for (int rk = 0; rk < DR_MAXTP; ++rk)
              if (rk < P.tp) P.xin[rk][off] = v;
          } else {
            hc[row] = (i == (int)threadIdx.x ? hres : __ldcg(hc + row)) + v;
          }
        } else {  // DP_DOWN: this CTA's partial of the tile into its slot;
                  // the tile's last CTA zeroes the slots no CTA fills
          const long long S = (long long)d.T * d.C;
          const int c0 = d.split ? dr_cta_of((long long)tile * d.C, S, d.C) : c;
          const int c1 = d.split ? dr_cta_of((long long)(tile + 1) * d.C - 1, S, d.C) : c;
          if (tp) {
            const int64_t base = dr_xin_region(L & 1, 1, P.tp, P.H) + (int64_t)P.rank * P.nsf * P.H + row;
#pragma unroll
            for (int rk = 0; rk < DR_MAXTP; ++rk) {
              if (rk >= P.tp) break;
              float* dst = P.xin[rk] + base;
              dst[(int64_t)(c - c0) * P.H] = v;
              if (c == c1)
                for (int sl = c1 - c0 + 1; sl < P.nsf; ++sl) dst[(int64_t)sl * P.H] = 0.f;
            }
          } else {
            P.pres[(int64_t)(c - c0) * P.H + row] = v;
            if (c == c1)
              for (int sl = c1 - c0 + 1; sl < P.nsf; ++sl) P.pres[(int64_t)sl * P.H + row] = 0.f;
          }
        }
      }
      if (tp && (kind == DP_O || kind == DP_DOWN)) dr_xarrive(P, kind == DP_O ? 0 : 1);
    }
    dr_grid_arrive(P);
    dr_mark(P, ph, 3);
  }
}

// ------------------------------------------------------------------ ring layout
// 16 bytes of a packed row.  Rows are 16-byte aligned only when K is a
// multiple of 512 (K * 33/32 bytes per row); for other K (multiples of 64)
// every row, scale and code offset is even, so the bytes are read as u16.
__device__ __forceinline__ uint4 dr_ld16_row(const uint8_t* p) {
  if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) return *reinterpret_cast<const uint4*>(p);
  const uint16_t* h = reinterpret_cast<const uint16_t*>(p);
  return make_uint4(h[0] | (uint32_t)h[1] << 16, h[2] | (uint32_t)h[3] << 16, h[4] | (uint32_t)h[5] << 16,
                    h[6] | (uint32_t)h[7] << 16);
}

// One thread per 16-byte chunk of the output: block (t, c) = 16 rows x 512
// codes in swizzled boxes, then the rows' 8 group scales of chunk c.  Codes
// and scales past K (a last chunk of fewer than 512 codes) are zero.
__global__ void k_ring_pack(const uint8_t* __restrict__ W, int64_t nchunk16, int K, int C, int f2,
                            uint8_t* __restrict__ dst) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= nchunk16) return;
  const int64_t blk = e / (DR_BLOCK / 16);
  const int q = (int)(e % (DR_BLOCK / 16));
  const int64_t t = blk / C;
  const int c = (int)(blk % C);
  const int64_t rb = (int64_t)K + K / 32;
  int r;
  int64_t srcoff;
  if (q < 512) {  // code chunk: box j, row r, stored chunk pc -> logical chunk pc ^ (r & 7)
    const int j = q >> 7, within = q & 127;
    r = within >> 3;
    const int lc = (within & 7) ^ (r & 7);
    srcoff = K / 32 + (int64_t)c * DR_CK + j * 128 + lc * 16;
  } else {  // scales of row r
    r = q - 512;
    srcoff = (int64_t)c * 16;
  }
  const int64_t row = f2 ? (r < 8 ? t * 8 + r : (int64_t)f2 + t * 8 + (r - 8)) : t * 16 + r;
  const uint8_t* src = W + row * rb + srcoff;
  uint4 v = make_uint4(0, 0, 0, 0);
  if (q < 512) {
    if (srcoff - K / 32 < K) v = dr_ld16_row(src);  // K is a multiple of 64
  } else {
    const int ng = K / 64, g0 = c * 8;
    if (g0 + 8 <= ng) {
      v = dr_ld16_row(src);
    } else if (g0 < ng) {  // scales of the groups that exist; zero scales after them
      uint16_t h[8];
      for (int i = 0; i < 8; ++i) h[i] = g0 + i < ng ? reinterpret_cast<const uint16_t*>(src)[i] : 0;
      v = make_uint4(h[0] | (uint32_t)h[1] << 16, h[2] | (uint32_t)h[3] << 16, h[4] | (uint32_t)h[5] << 16,
                     h[6] | (uint32_t)h[7] << 16);
    }
  }
  *reinterpret_cast<uint4*>(dst + e * 16) = v;
}

int dr_repack(const uint8_t* W, int64_t rows, int K, int f2, uint8_t* dst, cudaStream_t st) {
  Q8_CHECK_ARG(K % 64 == 0 && rows % 16 == 0 && (f2 == 0 || 2 * (int64_t)f2 == rows),
               "ring layout: unsupported matrix %lld x %d", (long long)rows, K);
  const int C = dr_kpad(K) / DR_CK;
  const int64_t n = rows / 16 * C * (DR_BLOCK / 16);
  k_ring_pack<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(W, n, K, C, f2, dst);
  return launch_check("k_ring_pack");
}

// ------------------------------------------------------------------ host side
size_t dr_rx_bytes(int tp, int H) {
  const size_t inbox = (size_t)dr_xin_region(2, 0, tp, H) * 4;
  return ((inbox + 255) & ~(size_t)255) + 256;
}

size_t dr_apart_floats(int nkv, int nsplit, int hd) {
  return (size_t)nkv * nsplit * (DR_GMAX * hd + 2 * DR_GMAX + 4);
}

// Partial slots per down-projection tile: a tile of C stages meets at most
// ceil((C - 1) / per) + 1 of the split ranges (each >= per stages).
int dr_down_nsf(int H, int F, int G) {
  if (!dr_down_split(F)) return 1;
  const int C = F / DR_CK;
  const long long S = (long long)(H / 16) * C;
  const long long per = S / dr_split_ctas(S, C, G);
  return (int)((C - 2 + per) / per + 1);
}

// Context splits per kv head: enough CTAs to cover the SMs, but no more than
// give each split one 16-position block per consumer warp at the longest
// context (more splits only lengthen the merge, which every layer waits for).
int dr_nsplit(int G, int nkv, int maxlen) {
  const int by_ctx = ((maxlen + 15) / 16 + DR_CW - 1) / DR_CW;
  return std::max(1, std::min({DR_MAXSPLIT, G / std::max(1, nkv), by_ctx}));
}

bool dr_supported(int H, int nh, int nkv, int hd, int F, int V, int page, const char** why) {
  auto no = [&](const char* w) {
    if (why) *why = w;
    return false;
  };
  if (hd != 64 && hd != 128) return no("head_dim must be 64 or 128");
  if (nkv < 1 || nh % nkv != 0 || nh / nkv > DR_GMAX) return no("more than 4 q heads per kv head");
  const int qd = nh * hd, nqkv = qd + 2 * nkv * hd;
  if (H % DR_CK) return no("hidden must be a multiple of 512");
  if (qd % 64 || F % 64) return no("q width and FFN width must be multiples of 64");
  if (nqkv % 16 || H % 16 || V % 16) return no("output widths must be multiples of 16");
  if (std::max({H, dr_kpad(qd), dr_kpad(F)}) > 16384 || H > 8192) return no("inputs too wide for the staging");
  if (page % 16) return no("KV page must be a multiple of 16 positions");
  const int G = num_sms();
  if (nkv > G) return no("more kv heads than SMs");
  // digits + per-warp tile sums fit the staging area in every phase
  auto fits = [&](int K, int T, bool split) {
    const int C = K / DR_CK;
    const int tiles = split ? ((int)((long long)T * C / G) + C - 1) / C + 2 : (T + G - 1) / G + 1;
    return (size_t)K * 3 + 16 + (size_t)tiles * DR_CW * 16 * 4 <= (size_t)DR_XQ_BYTES;
  };
  const int qdp = dr_kpad(qd), Fp = dr_kpad(F);
  if (!fits(H, nqkv / 16, false) || !fits(qdp, H / 16, false) || !fits(H, F / 8, false) ||
      !fits(Fp, H / 16, true) || !fits(H, V / 16, false))
    return no("staging area too small");
  if (H > 16 * DR_CW * 32) return no("hidden wider than the one-item-per-thread RMSNorm staging");
  if (dr_down_nsf(H, Fp, G) > DR_NS) return no("down tiles would span too many CTAs");
  return true;
}

template <int HD>
static int dr_attr(int* per_sm) {
  Q8_CUDA(cudaFuncSetAttribute(k_decode_ring<HD, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, DR_SMEM));
  Q8_CUDA(cudaFuncSetAttribute(k_decode_ring<HD, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, DR_SMEM));
  int a = 0, b = 0;
  Q8_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&a, k_decode_ring<HD, false>, DR_THREADS, DR_SMEM));
  Q8_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k_decode_ring<HD, true>, DR_THREADS, DR_SMEM));
  *per_sm = std::min(a, b);
  return Q8_OK;
}

int dr_prepare(int hd, int* grid) {
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  int dev = 0, coop = 0, per_sm = 0;
  Q8_CUDA(cudaGetDevice(&dev));
  Q8_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
  if (hd == 128) Q8_TRY(dr_attr<128>(&per_sm));
  else Q8_TRY(dr_attr<64>(&per_sm));
  *grid = (coop && per_sm >= 1) ? num_sms() : 0;
  return Q8_OK;
}

int dr_launch(const DrParams& p, int grid, cudaStream_t st) {
  Q8_CHECK_ARG(grid > 0, "decode ring: not prepared");
  Q8_CUDA(cudaMemsetAsync(p.bar, 0, sizeof(unsigned int), st));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(DR_THREADS);
  cfg.dynamicSmemBytes = DR_SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const bool xp = p.tp > 1;
  cudaError_t e = p.hd == 128 ? (xp ? cudaLaunchKernelEx(&cfg, k_decode_ring<128, true>, p)
                                    : cudaLaunchKernelEx(&cfg, k_decode_ring<128, false>, p))
                              : (xp ? cudaLaunchKernelEx(&cfg, k_decode_ring<64, true>, p)
                                    : cudaLaunchKernelEx(&cfg, k_decode_ring<64, false>, p));
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("launch k_decode_ring: %s", cudaGetErrorString(e));
    return Q8_ERR_CUDA;
  }
  return Q8_OK;
}

}  // namespace q8
