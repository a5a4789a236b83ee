// Temperature + nucleus (top-p) sampling on the device: sample()
// (src/sample.mojo:15-59), with the uniform draw supplied per row.
//
// The reference, per logits row:
//   temp <= 0: greedy argmax (first maximum);
//   candidates: logits >= max - 16 in index order, p = exp((l - max) / temp),
//   total = their f32 sum in index order; no candidate: argmax;
//   nucleus: while cum < total * top_p, pick the largest remaining p (the
//   first one in list order), append it, move the list's last entry into its
//   place (swap-remove);
//   r = u * cum; the first nucleus entry whose running sum reaches r.
// Every f32 sum above is sequential, so the result depends on the order of
// the additions; this file keeps each order and each rounding:
//   k_sample_prep   one CTA per row: max / first argmax, candidates compacted
//                   in index order (contiguous range per warp, read 32 at a
//                   time, order kept by ballots), p, and total summed in index
//                   order by one warp
//                   (256 values per round, the next round's loads in flight);
//   sort            candidates by p, descending (CUB segmented sort, one
//                   segment per row);
//   k_sample_walk   one warp per row: the running sums of the sorted p (the
//                   reference's cum after each pick, and also its second
//                   loop's acc: the same additions in the same order); the
//                   nucleus ends at the first sum >= target, r = u * cum, and
//                   the pick is the first sum >= r (binary searches: the sums
//                   never decrease, p >= 0).
//   k_sample_ties   only when the chosen entry's p is shared by other
//                   candidates: which of them the reference picks at that
//                   point depends on their list positions after every earlier
//                   swap-remove, so one thread replays the list up to the
//                   chosen entry, O(1) per removal (rare: equal p needs equal
//                   or nearly equal logits).
// Values of exp() come from CUDA's expf; the reference uses Mojo's exp.
#include "q8_kernels.h"

#include <cub/device/device_segmented_sort.cuh>

#include <float.h>
#include <math.h>

namespace q8 {

constexpr int SP_THREADS = 1024;

struct SampleWs {
  int* cidx;      // [R][n] candidate -> token index, index order
  float* key_in;  // [R][n] candidate p, index order; then the running sums
  int* val_in;    // [R][n] candidate number; then the replay's candidate -> list position
  float* key_out; // [R][n] p, descending
  int* val_out;   // [R][n] candidate number, in key_out's order
  int* beg;       // [R] segment offsets for the sort
  int* end;       // [R]
  int* cnt;       // [R] candidates (0: out already written)
  float* target;  // [R]
  int* tie;       // [R] -1, or the nucleus entry whose equal-p group needs the replay
  int* aux;       // [R][2n] replay: group tags per candidate, then a bitmap of list positions
};

// 256 consecutive values b0.. of a[0, C) for a warp: lane l holds b0 + 32 k + l
// (0 past C: adding +0 leaves a sum of non-negative values unchanged)
__device__ __forceinline__ void sp_ld8(float (&v)[8], const float* a, int b0, int C) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int e = b0 + 32 * k + lane;
    v[k] = e < C ? a[e] : 0.f;
  }
}

// Sequential f32 sum of a[0, C) by one warp: the lanes stage 256 values per
// round in shared memory (coalesced loads, the next round's already in
// flight), lane 0 adds them one by one.  RUN: the running sums also go to
// run[0, C).  Returns the sum on every lane.
template <bool RUN>
__device__ __forceinline__ float sp_seq_sum(const float* a, int C, float* run, float* sbuf) {
  const int lane = threadIdx.x & 31;
  float s = 0.f;
  float cur[8], nxt[8];
  sp_ld8(cur, a, 0, C);
  for (int b0 = 0; b0 < C; b0 += 256) {
    sp_ld8(nxt, a, b0 + 256, C);
#pragma unroll
    for (int k = 0; k < 8; ++k) sbuf[32 * k + lane] = cur[k];
    __syncwarp();
    if (lane == 0) {
      float4* s4 = reinterpret_cast<float4*>(sbuf);
#pragma unroll 16
      for (int j = 0; j < 64; ++j) {  // zeros past C leave the sum unchanged
        float4 v = s4[j];
        s += v.x;
        if (RUN) v.x = s;
        s += v.y;
        if (RUN) v.y = s;
        s += v.z;
        if (RUN) v.z = s;
        s += v.w;
        if (RUN) v.w = s;
        if (RUN) s4[j] = v;
      }
    }
    __syncwarp();
    if (RUN) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int e = b0 + 32 * k + lane;
        if (e < C) run[e] = sbuf[32 * k + lane];
      }
      __syncwarp();  // read before the next round overwrites the stage
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) cur[k] = nxt[k];
  }
  return __shfl_sync(0xffffffffu, s, 0);
}

__device__ __forceinline__ void sp_merge(float& bv, int& bi, float ov, int oi) {
  if (ov > bv || (ov == bv && oi < bi)) {
    bv = ov;
    bi = oi;
  }
}

__global__ void __launch_bounds__(SP_THREADS) k_sample_prep(const float* __restrict__ logits, int n, int64_t ld,
                                                            float temp, float top_p, SampleWs ws,
                                                            int32_t* __restrict__ out) {
  __shared__ float s_v[SP_THREADS / 32];
  __shared__ int s_i[SP_THREADS / 32];
  const int r = blockIdx.x, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const float* x = logits + (int64_t)r * ld;
  const int64_t base = (int64_t)r * n;

  // max and its first index (NaN never wins, as in the greedy argmax kernels)
  // (eight loads in flight per thread: one CTA streams the whole row)
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i0 = threadIdx.x; i0 < n; i0 += 8 * SP_THREADS) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = i0 + k * SP_THREADS;
      v[k] = i < n ? x[i] : -INFINITY;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (i0 + k * SP_THREADS < n) sp_merge(bv, bi, v[k], i0 + k * SP_THREADS);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    sp_merge(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
  if (lane == 0) {
    s_v[w] = bv;
    s_i[w] = bi;
  }
  __syncthreads();
  bv = s_v[0];
  bi = s_i[0];
  for (int k = 1; k < SP_THREADS / 32; ++k) sp_merge(bv, bi, s_v[k], s_i[k]);
  const int am = bi == 0x7fffffff ? 0 : bi;
  const float mx = x[am];
  if (!(temp > 0.f)) {  // greedy
    if (threadIdx.x == 0) {
      out[r] = am;
      ws.cnt[r] = 0;
      ws.beg[r] = (int)base;
      ws.end[r] = (int)base;
      ws.tie[r] = -1;
    }
    return;
  }

  // candidates (not below max - 16) in index order: warp w owns the
  // contiguous range [w L, (w + 1) L), read 32 coalesced values at a time
  __shared__ int s_cnt[SP_THREADS / 32];
  const float cutoff = mx - 16.0f;
  constexpr int NW = SP_THREADS / 32;
  const int L = (n + NW - 1) / NW;
  const int i0 = min(n, w * L), i1 = min(n, i0 + L);
  int mine = 0;
  for (int b = i0 + lane; b < i1; b += 8 * 32) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = b + 32 * k < i1 ? x[b + 32 * k] : -INFINITY;
#pragma unroll
    for (int k = 0; k < 8; ++k) mine += b + 32 * k < i1 && !(v[k] < cutoff);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
  if (lane == 0) s_cnt[w] = mine;
  __syncthreads();
  int off = 0, C = 0;
  for (int k = 0; k < NW; ++k) {  // the warps' offsets, in warp order
    const int v = s_cnt[k];
    if (k < w) off += v;
    C += v;
  }
  for (int b0 = i0; b0 < i1; b0 += 8 * 32) {  // uniform per warp: every lane takes part in the ballots
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = b0 + 32 * k + lane;
      v[k] = i < i1 ? x[i] : -INFINITY;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = b0 + 32 * k + lane;
      const bool take = i < i1 && !(v[k] < cutoff);
      const unsigned m = __ballot_sync(0xffffffffu, take);
      if (take) {
        const int o = off + __popc(m & ((1u << lane) - 1u));
        ws.cidx[base + o] = i;
        ws.key_in[base + o] = expf(__fdiv_rn(v[k] - mx, temp));
        ws.val_in[base + o] = o;
      }
      off += __popc(m);
    }
  }
  __syncthreads();  // the CTA's global stores are visible to the CTA after the barrier

  // total in index order: one warp adds the values one by one
  if (w == 0) {
    __shared__ __align__(16) float sbuf[256];
    const float total = sp_seq_sum<false>(ws.key_in + base, C, nullptr, sbuf);
    if (lane == 0) {
      ws.target[r] = total * top_p;
      ws.cnt[r] = C;
      ws.beg[r] = (int)base;
      ws.end[r] = (int)(base + C);
      ws.tie[r] = -1;
      if (C == 0) out[r] = am;
    }
  }
}

__global__ void __launch_bounds__(32) k_sample_walk(const float* __restrict__ u, int n, SampleWs ws,
                                                    int32_t* __restrict__ out) {
  const int r = blockIdx.x, lane = threadIdx.x;
  const int C = ws.cnt[r];
  if (C == 0) return;
  const int64_t base = (int64_t)r * n;
  const float* ks = ws.key_out + base;
  float* run = ws.key_in + base;  // running sums (the index-order p are no longer needed)
  __shared__ __align__(16) float sbuf[256];
  sp_seq_sum<true>(ks, C, run, sbuf);
  __syncwarp();  // the lanes' running sums, visible to lane 0
  if (lane != 0) return;
  // the reference picks entry i while the sum before it is < target: the
  // nucleus is [0, K), K - 1 the first entry whose sum reaches the target
  const float target = ws.target[r];
  int lo = 0, hi = C - 1;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (run[mid] >= target) hi = mid;
    else lo = mid + 1;
  }
  const int K = lo + 1;
  const float rr = u[r] * run[K - 1];
  lo = 0;
  hi = K - 1;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (rr <= run[mid]) hi = mid;
    else lo = mid + 1;
  }
  const int pick = lo;  // no sum reaches r (u > 1): the last entry, as the reference
  const float pp = ks[pick];
  const bool shared = (pick > 0 && ks[pick - 1] == pp) || (pick + 1 < C && ks[pick + 1] == pp);
  if (!shared) {
    out[r] = ws.cidx[base + ws.val_out[base + pick]];
  } else {
    ws.tie[r] = pick;
  }
}

// The reference's list, replayed up to nucleus entry `pick`.  Entries leave
// in descending p; among equal p the one at the lowest list position goes
// first; a removal moves the list's last entry into the freed position.
// Within a group of equal p: the members' positions are bits of a bitmap,
// taken in ascending order; when a removal moves a member from the list's
// end into the freed position (lower than every other member's), that member
// goes next.  Every step is O(1) apart from the bitmap scan, which only moves
// forward within a group.
__global__ void __launch_bounds__(256) k_sample_ties(int n, SampleWs ws, int32_t* __restrict__ out) {
  const int r = blockIdx.x;
  const int pick = ws.tie[r];
  if (pick < 0) return;
  const int C = ws.cnt[r];
  const int64_t base = (int64_t)r * n;
  int* at = reinterpret_cast<int*>(ws.key_in + base);  // list position -> candidate
  int* pos = ws.val_in + base;                         // candidate -> list position
  int* tag = ws.aux + 2 * base;                        // candidate -> group tag (group start + 1)
  uint32_t* bits = reinterpret_cast<uint32_t*>(tag + n);  // list positions of the group's members
  const int nw = (C + 31) / 32;
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    at[i] = i;
    pos[i] = i;
    tag[i] = 0;
  }
  for (int i = threadIdx.x; i < nw; i += blockDim.x) bits[i] = 0u;
  __syncthreads();
  if (threadIdx.x != 0) return;
  const float* ks = ws.key_out + base;
  const int* vs = ws.val_out + base;
  int len = C, sel = 0, s = 0;
  while (s < C) {
    const float p = ks[s];
    int e = s + 1;
    while (e < C && ks[e] == p) ++e;
    if (e == s + 1) {  // a lone value: no choice to replay
      const int c = vs[s];
      if (sel == pick) {  // cannot happen: the pick's group has several members
        out[r] = ws.cidx[base + c];
        ws.tie[r] = -1;
        return;
      }
      const int b = pos[c], last = at[len - 1];
      at[b] = last;
      pos[last] = b;
      --len;
      ++sel;
      s = e;
      continue;
    }
    const int tg = s + 1;
    int minp = 0x7fffffff;
    for (int q = s; q < e; ++q) {
      const int c = vs[q];
      tag[c] = tg;
      bits[pos[c] >> 5] |= 1u << (pos[c] & 31);
      minp = min(minp, pos[c]);
    }
    int wcur = minp >> 5, carry = -1;
    for (int k = s; k < e; ++k) {
      int c = carry;
      carry = -1;
      if (c < 0) {  // the lowest marked position
        while (wcur < nw && bits[wcur] == 0u) ++wcur;
        if (wcur == nw) {  // cannot happen: the group's members are marked or carried
          out[r] = ws.cidx[base + vs[pick]];
          return;
        }
        const int bpos = wcur * 32 + __ffs(bits[wcur]) - 1;
        bits[wcur] &= bits[wcur] - 1u;
        c = at[bpos];
      }
      if (sel == pick) {
        out[r] = ws.cidx[base + c];
        ws.tie[r] = -1;
        return;
      }
      const int b = pos[c], last = at[len - 1];
      if (last != c) {
        at[b] = last;
        pos[last] = b;
        if (tag[last] == tg) {  // a member leaves the end: it is now the lowest
          bits[(len - 1) >> 5] &= ~(1u << ((len - 1) & 31));
          carry = last;
        }
      }
      --len;
      ++sel;
    }
    s = e;
  }
}

// scratch bytes for R rows of n logits, CUB's temporary storage included
static int sample_ws_bytes(int R, int n, size_t* cub_bytes, size_t* total) {
  size_t cb = 0;
  Q8_CUDA(cub::DeviceSegmentedSort::SortPairsDescending(nullptr, cb, (const float*)nullptr, (float*)nullptr,
                                                        (const int*)nullptr, (int*)nullptr, R * n, R,
                                                        (const int*)nullptr, (const int*)nullptr, (cudaStream_t)0));
  const size_t arr = ((size_t)R * n * 4 + 255) & ~(size_t)255;
  const size_t rows = ((size_t)R * 4 + 255) & ~(size_t)255;
  *cub_bytes = cb;
  *total = 7 * arr + 5 * rows + ((cb + 255) & ~(size_t)255);
  return Q8_OK;
}

static SampleWs sample_ws_carve(void* p, int R, int n, void** cub_tmp) {
  const size_t arr = ((size_t)R * n * 4 + 255) & ~(size_t)255;
  const size_t rows = ((size_t)R * 4 + 255) & ~(size_t)255;
  uint8_t* q = static_cast<uint8_t*>(p);
  SampleWs ws{};
  ws.cidx = (int*)q; q += arr;
  ws.key_in = (float*)q; q += arr;
  ws.val_in = (int*)q; q += arr;
  ws.key_out = (float*)q; q += arr;
  ws.val_out = (int*)q; q += arr;
  ws.beg = (int*)q; q += rows;
  ws.end = (int*)q; q += rows;
  ws.cnt = (int*)q; q += rows;
  ws.target = (float*)q; q += rows;
  ws.tie = (int*)q; q += rows;
  ws.aux = (int*)q; q += 2 * arr;
  *cub_tmp = q;
  return ws;
}

size_t sample_scratch_bytes(int rows, int n) {
  size_t cb = 0, tot = 0;
  if (sample_ws_bytes(rows, n, &cb, &tot) != Q8_OK) return 0;
  return tot;
}

int sample_launch(const float* logits, int rows, int n, int64_t ld, float temp, float top_p, const float* u,
                  int32_t* out, void* scratch, size_t scratch_bytes, cudaStream_t st) {
  Q8_CHECK_ARG(rows >= 0 && n >= 1 && ld >= n && (int64_t)rows * n < ((int64_t)1 << 31),
               "sample: bad shape rows=%d n=%d ld=%lld", rows, n, (long long)ld);
  if (rows == 0) return Q8_OK;
  size_t cb = 0, tot = 0;
  Q8_TRY(sample_ws_bytes(rows, n, &cb, &tot));
  Q8_CHECK_ARG(scratch && scratch_bytes >= tot, "sample: scratch of %zu bytes, %zu needed", scratch_bytes, tot);
  void* cub_tmp = nullptr;
  const SampleWs ws = sample_ws_carve(scratch, rows, n, &cub_tmp);
  k_sample_prep<<<rows, SP_THREADS, 0, st>>>(logits, n, ld, temp, top_p, ws, out);
  Q8_TRY(launch_check("k_sample_prep"));
  if (!(temp > 0.f)) return Q8_OK;
  Q8_CUDA(cub::DeviceSegmentedSort::SortPairsDescending(cub_tmp, cb, ws.key_in, ws.key_out, ws.val_in, ws.val_out,
                                                        rows * n, rows, ws.beg, ws.end, st));
  k_sample_walk<<<rows, 32, 0, st>>>(u, n, ws, out);
  Q8_TRY(launch_check("k_sample_walk"));
  k_sample_ties<<<rows, 256, 0, st>>>(n, ws, out);
  return launch_check("k_sample_ties");
}

}  // namespace q8

using namespace q8;

extern "C" int q8op_sample(const float* logits, int64_t rows, int64_t n, int64_t ld, float temp, float top_p,
                           const float* u, int32_t* out, void* stream) {
  Q8_CHECK_ARG(logits && out && (u || !(temp > 0.f)), "q8op_sample: null pointer");
  // temp NaN would sample with NaN weights; top_p <= 0 leaves the reference's
  // nucleus empty (it then indexes an empty list)
  Q8_CHECK_ARG(!isnan(temp) && (!(temp > 0.f) || top_p > 0.f), "q8op_sample: temp must not be NaN, top_p must be > 0");
  Q8_CHECK_ARG(rows >= 0 && n >= 1 && ld >= n && rows * n < ((int64_t)1 << 31), "q8op_sample: bad shape");
  if (rows == 0) return Q8_OK;
  const size_t need = sample_scratch_bytes((int)rows, (int)n);
  Q8_CHECK_ARG(need > 0, "q8op_sample: scratch size query failed");
  void* scr = nullptr;
  Q8_TRY(op_scratch(need, &scr));
  return sample_launch(logits, (int)rows, (int)n, ld, temp, top_p, u, out, scr, need, (cudaStream_t)stream);
}
