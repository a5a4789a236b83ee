// Layer ops around the Q8 matmuls: embedding gather, (residual +) RMSNorm,
// (QK-norm +) RoPE + paged KV append, causal GQA attention, argmax.
//
// Each kernel cites the reference kernel it replaces.  All arithmetic is f32,
// as in the reference (activations, KV cache and math are f32; W8A32).
#include "q8_kernels.h"
#include <algorithm>
#include <math.h>
#include <mutex>

namespace q8 {

// ------------------------------------------------------------------ embedding
// k_embed_gather_q8 (src/llama_q8.mojo:96-109): y = f32(int8) * f32(f16 scale).
__global__ void k_embed_q8(const uint8_t* __restrict__ emb, int64_t d, const int32_t* __restrict__ ids,
                           int64_t s, float* __restrict__ y) {
  pdl_trigger();
  pdl_wait();
  const int64_t rb = q8_row_bytes(d);
  const int64_t total = s * d;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / d, c = i % d;
    const uint8_t* row = emb + (int64_t)ids[r] * rb;
    const float sc = __half2float(reinterpret_cast<const __half*>(row)[c / Q8_QG]);
    y[i] = (float)(int8_t)row[d / 32 + c] * sc;
  }
}

int embed_launch(const void* emb, int64_t d, const int32_t* ids, int64_t s, float* y, cudaStream_t st) {
  const int64_t total = s * d;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 8);
  return launch_pdl("k_embed_q8", k_embed_q8, dim3(blocks), dim3(256), 0, st, (const uint8_t*)emb, d, ids, s, y);
}

// ------------------------------------------------------------------ RMSNorm
// k_rmsnorm_w (src/llama_common.mojo:197-225): y = w * x * (1/sqrt(sum(x^2)/d + eps));
// with resid: x += resid first (k_res_add_rmsnorm, :361-393; k_res_add :354-358).
// One CTA per row; outputs f32 and/or split-f16 (XS) for the next GEMV.
__global__ void __launch_bounds__(256) k_rmsnorm(float* __restrict__ x, const float* __restrict__ resid,
                                                 const uint16_t* __restrict__ w, int64_t d, float eps,
                                                 float* __restrict__ y32, __half* __restrict__ yxs,
                                                 __half* __restrict__ y16, int64_t y16lo) {
  __shared__ float wsum[8];
  pdl_trigger();
  pdl_wait();
  const int64_t r = blockIdx.x;
  float* xr = x + r * d;
  const float* rr = resid ? resid + r * d : nullptr;
  float ss = 0.f;
  for (int64_t k = threadIdx.x; k < d; k += blockDim.x) {
    float v = xr[k];
    if (rr) {
      v += rr[k];
      xr[k] = v;
    }
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += wsum[i];
  const float inv = 1.0f / sqrtf(tot / (float)d + eps);
  for (int64_t k = threadIdx.x; k < d; k += blockDim.x) {
    const float v = bf16_bits_to_f32(w[k]) * xr[k] * inv;
    if (y32) y32[r * d + k] = v;
    if (yxs) {
      __half hi, lo;
      split_f16(v, hi, lo);
      yxs[xs_index(r, k, d, 0)] = hi;
      yxs[xs_index(r, k, d, 1)] = lo;
    }
    if (y16) {
      const __half hv = __float2half_rn(v);
      y16[r * d + k] = hv;
      if (y16lo) y16[y16lo + r * d + k] = __float2half_rn(v - __half2float(hv));
    }
  }
}

int rmsnorm_launch(float* x, const float* resid, const uint16_t* w, int64_t rows, int64_t d, float eps,
                   float* y32, __half* yxs, __half* y16, cudaStream_t st, int64_t y16lo) {
  if (rows <= 0) return Q8_OK;
  return launch_pdl("k_rmsnorm", k_rmsnorm, dim3((unsigned)rows), dim3(256), 0, st, x, resid, w, d, eps, y32, yxs,
                    y16, y16lo);
}

// Per-head RMSNorm (Qwen3 QK-norm) — k_rmsnorm2_w (src/llama_common.mojo:228-270); warp per row.
__global__ void k_rmsnorm_heads(const float* __restrict__ x, const uint16_t* __restrict__ w, int64_t rows,
                                int hd, float eps, float* __restrict__ y) {
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  float ss = 0.f;
  for (int k = lane; k < hd; k += 32) ss = fmaf(x[r * hd + k], x[r * hd + k], ss);
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / (float)hd + eps);
  for (int k = lane; k < hd; k += 32) y[r * hd + k] = bf16_bits_to_f32(w[k]) * x[r * hd + k] * inv;
}

int rmsnorm_heads_launch(const float* x, const uint16_t* w, int64_t rows, int64_t hd, float eps, float* y,
                         cudaStream_t st) {
  if (rows <= 0) return Q8_OK;
  k_rmsnorm_heads<<<ceil_div(rows, 8), 256, 0, st>>>(x, w, rows, (int)hd, eps, y);
  return launch_check("k_rmsnorm_heads");
}

// ------------------------------------------------------------------ RoPE + KV append
// k_rope_qk_copy2 (src/llama_common.mojo:299-342) with the Qwen3 QK-norm of
// k_rmsnorm2_w fused in front (src/llama_q8.mojo:171-181).  One warp per
// (token, head); lane l holds dims l + 32j, so every rotate-half pair
// (d, d + hd/2) lives in one lane.  freq = f32(pos) * inv_freq[d] and accurate
// sincosf, as the reference's cos/sin of the f32 product.  k heads are written
// to their page slot, and the kv-head warp also copies v.
template <int HD>
__global__ void __launch_bounds__(256) k_rope_kv(float* __restrict__ qkv, int64_t ld, int64_t T,
                                                 const int32_t* __restrict__ pos, const int32_t* __restrict__ seq,
                                                 int nh, int nkv, const float* __restrict__ inv_freq,
                                                 const uint16_t* __restrict__ qn, const uint16_t* __restrict__ kn,
                                                 float eps, float* __restrict__ kp, float* __restrict__ vp,
                                                 int page, const int32_t* __restrict__ bt, int max_pages) {
  constexpr int J = HD / 32;
  pdl_trigger();
  pdl_wait();
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int nall = nh + nkv;
  if (wid >= T * nall) return;
  const int64_t t = wid / nall;
  const int h = (int)(wid % nall);
  const bool is_q = h < nh;
  float* base = qkv + t * ld + (int64_t)h * HD;  // k heads follow q heads contiguously
  float v[J];
#pragma unroll
  for (int j = 0; j < J; ++j) v[j] = base[lane + 32 * j];
  const uint16_t* nw = is_q ? qn : kn;
  if (nw) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) ss = fmaf(v[j], v[j], ss);
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)HD + eps);
#pragma unroll
    for (int j = 0; j < J; ++j) v[j] = bf16_bits_to_f32(nw[lane + 32 * j]) * v[j] * inv;
  }
  const int p = pos[t];
  const float fp = (float)p;
#pragma unroll
  for (int j = 0; j < J / 2; ++j) {
    const int d = lane + 32 * j;
    float sn, cs;
    sincosf(fp * inv_freq[d], &sn, &cs);
    const float x0 = v[j], x1 = v[j + J / 2];
    v[j] = x0 * cs - x1 * sn;
    v[j + J / 2] = x1 * cs + x0 * sn;
  }
  if (is_q) {
#pragma unroll
    for (int j = 0; j < J; ++j) base[lane + 32 * j] = v[j];
    return;
  }
  const int kvh = h - nh;
  const int pg = bt[(int64_t)seq[t] * max_pages + p / page];
  const int64_t off = (((int64_t)pg * nkv + kvh) * page + (p % page)) * HD;
  const float* vsrc = qkv + t * ld + (int64_t)(nh + nkv) * HD + (int64_t)kvh * HD;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    base[lane + 32 * j] = v[j];
    kp[off + lane + 32 * j] = v[j];
    vp[off + lane + 32 * j] = vsrc[lane + 32 * j];
  }
}

int rope_kv_launch(float* qkv, int64_t ld, int64_t T, const int32_t* pos, const int32_t* seq, int nh,
                   int nkv, int hd, const float* inv_freq, const uint16_t* qn, const uint16_t* kn,
                   float eps, float* kp, float* vp, int page, const int32_t* bt, int max_pages,
                   cudaStream_t st) {
  if (T <= 0) return Q8_OK;
  const int64_t warps = T * (nh + nkv);
  const int blocks = ceil_div(warps, 8);
  switch (hd) {
    case 64:
      return launch_pdl("k_rope_kv", k_rope_kv<64>, dim3(blocks), dim3(256), 0, st, qkv, ld, T, pos, seq, nh, nkv,
                        inv_freq, qn, kn, eps, kp, vp, page, bt, max_pages);
    case 128:
      return launch_pdl("k_rope_kv", k_rope_kv<128>, dim3(blocks), dim3(256), 0, st, qkv, ld, T, pos, seq, nh, nkv,
                        inv_freq, qn, kn, eps, kp, vp, page, bt, max_pages);
    case 256:
      return launch_pdl("k_rope_kv", k_rope_kv<256>, dim3(blocks), dim3(256), 0, st, qkv, ld, T, pos, seq, nh, nkv,
                        inv_freq, qn, kn, eps, kp, vp, page, bt, max_pages);
    default:
      set_error("rope: head_dim %d unsupported (64/128/256)", hd);
      return Q8_ERR_ARG;
  }
  return launch_check("k_rope_kv");
}

// ------------------------------------------------------------------ attention
// Replaces k_scores / k_softmax_rows / k_att_out (src/llama_common.mojo:402-473):
// S = q.k / sqrt(hd) with causal mask, row softmax, O = P.V, without the
// materialized [heads, s, nctx] score buffer.  One CTA per (query block, kv
// head, context split); rows = queries x the GQA group sharing that kv head.
// Keys stream through shared memory in tiles of 32 with an online softmax;
// splits write (o, m, l) partials that k_attn_combine merges.
constexpr int ATT_TK = 32;

template <int HD, int RMAX>
struct AttnSmem {
  float q[RMAX][HD + 1];
  float k[ATT_TK][HD + 1];
  float v[ATT_TK][HD];
  float s[RMAX][ATT_TK + 1];
  float o[RMAX][HD];
  float m[RMAX], l[RMAX], corr[RMAX];
  int qpos[RMAX];
};

__device__ __forceinline__ void write_out(const AttnArgs& a, int tok, int col, float v) {
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

__device__ __forceinline__ void write_out_tok(float* out32, int64_t ldo, __half* outxs, int K, int tok, int col,
                                              float v) {
  if (out32) out32[(int64_t)tok * ldo + col] = v;
  if (outxs) {
    __half hi, lo;
    split_f16(v, hi, lo);
    outxs[xs_index(tok, col, K, 0)] = hi;
    outxs[xs_index(tok, col, K, 1)] = lo;
  }
}

template <int HD, int RMAX>
__global__ void __launch_bounds__(128) k_attn(AttnArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  AttnSmem<HD, RMAX>& S = *reinterpret_cast<AttnSmem<HD, RMAX>*>(smem_raw);
  const int qb = blockIdx.x, kvh = blockIdx.y, sp = blockIdx.z;
  const int G = a.nh / a.nkv;
  const int tok0 = a.qb_tok0 ? a.qb_tok0[qb] : qb;
  const int qlen = a.qb_tok0 ? a.qb_len[qb] : 1;
  const int R = qlen * G;
  const int sq = a.seq[tok0];
  const int kv_end = a.pos[tok0 + qlen - 1] + 1;
  const int ntile = (kv_end + ATT_TK - 1) / ATT_TK;
  const int per = (ntile + a.nsplit - 1) / a.nsplit;
  const int k_lo = sp * per * ATT_TK;
  const int k_hi = min(kv_end, (sp + 1) * per * ATT_TK);
  const float rs = sqrtf((float)HD);
  const int tid = threadIdx.x;

  for (int i = tid; i < R * HD; i += blockDim.x) {
    const int r = i / HD, d = i % HD;
    const int qi = r / G, gi = r % G;
    S.q[r][d] = a.q[(int64_t)(tok0 + qi) * a.ldq + (int64_t)(kvh * G + gi) * HD + d];
    S.o[r][d] = 0.f;
  }
  for (int r = tid; r < R; r += blockDim.x) {
    S.m[r] = -INFINITY;
    S.l[r] = 0.f;
    S.qpos[r] = a.pos[tok0 + r / G];
  }
  __syncthreads();

  const int32_t* btr = a.bt + (int64_t)sq * a.max_pages;
  for (int j0 = k_lo; j0 < k_hi; j0 += ATT_TK) {
    for (int i = tid; i < ATT_TK * (HD / 4); i += blockDim.x) {
      const int jj = i / (HD / 4), d4 = (i % (HD / 4)) * 4;
      const int j = j0 + jj;
      float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = kv4;
      if (j < k_hi) {
        const int pg = btr[j / a.page];
        const int64_t off = (((int64_t)pg * a.nkv + kvh) * a.page + (j % a.page)) * HD + d4;
        kv4 = *reinterpret_cast<const float4*>(a.kp + off);
        vv4 = *reinterpret_cast<const float4*>(a.vp + off);
      }
      S.k[jj][d4] = kv4.x; S.k[jj][d4 + 1] = kv4.y; S.k[jj][d4 + 2] = kv4.z; S.k[jj][d4 + 3] = kv4.w;
      *reinterpret_cast<float4*>(&S.v[jj][d4]) = vv4;
    }
    __syncthreads();
    for (int i = tid; i < R * ATT_TK; i += blockDim.x) {
      const int r = i / ATT_TK, jj = i % ATT_TK;
      const int j = j0 + jj;
      float sc = -INFINITY;
      if (j < k_hi && j <= S.qpos[r]) {
        float acc = 0.f;
#pragma unroll 8
        for (int d = 0; d < HD; ++d) acc = fmaf(S.q[r][d], S.k[jj][d], acc);
        sc = acc / rs;
      }
      S.s[r][jj] = sc;
    }
    __syncthreads();
    for (int r = tid; r < R; r += blockDim.x) {
      float mx = -INFINITY;
      for (int jj = 0; jj < ATT_TK; ++jj) mx = fmaxf(mx, S.s[r][jj]);
      const float m_old = S.m[r];
      const float m_new = fmaxf(m_old, mx);
      float corr = 1.f, sum = 0.f;
      if (m_new != -INFINITY) {
        corr = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
        for (int jj = 0; jj < ATT_TK; ++jj) {
          const float pz = (S.s[r][jj] == -INFINITY) ? 0.f : expf(S.s[r][jj] - m_new);
          S.s[r][jj] = pz;
          sum += pz;
        }
      } else {
        for (int jj = 0; jj < ATT_TK; ++jj) S.s[r][jj] = 0.f;
      }
      S.l[r] = S.l[r] * corr + sum;
      S.m[r] = m_new;
      S.corr[r] = corr;
    }
    __syncthreads();
    for (int i = tid; i < R * HD; i += blockDim.x) {
      const int r = i / HD, d = i % HD;
      float o = S.o[r][d] * S.corr[r];
#pragma unroll 8
      for (int jj = 0; jj < ATT_TK; ++jj) o = fmaf(S.s[r][jj], S.v[jj][d], o);
      S.o[r][d] = o;
    }
    __syncthreads();
  }

  if (a.nsplit == 1) {
    for (int i = tid; i < R * HD; i += blockDim.x) {
      const int r = i / HD, d = i % HD;
      const int qi = r / G, gi = r % G;
      const float l = S.l[r];
      write_out(a, tok0 + qi, (kvh * G + gi) * HD + d, l > 0.f ? S.o[r][d] / l : 0.f);
    }
    return;
  }
  // partial layout: item = (qb*nkv + kvh)*nsplit + sp; per item RMAX*HD o, RMAX m, RMAX l
  const int64_t item = ((int64_t)qb * a.nkv + kvh) * a.nsplit + sp;
  float* po = a.part + item * (int64_t)(RMAX * HD + 2 * RMAX);
  for (int i = tid; i < R * HD; i += blockDim.x) po[i] = S.o[i / HD][i % HD];
  for (int r = tid; r < R; r += blockDim.x) {
    po[RMAX * HD + r] = S.m[r];
    po[RMAX * HD + RMAX + r] = S.l[r];
  }
}

template <int HD, int RMAX>
__global__ void __launch_bounds__(128) k_attn_combine(AttnArgs a) {
  const int qb = blockIdx.x, kvh = blockIdx.y;
  const int G = a.nh / a.nkv;
  const int tok0 = a.qb_tok0 ? a.qb_tok0[qb] : qb;
  const int qlen = a.qb_tok0 ? a.qb_len[qb] : 1;
  const int R = qlen * G;
  const int64_t stride = RMAX * HD + 2 * RMAX;
  const float* base = a.part + ((int64_t)qb * a.nkv + kvh) * a.nsplit * stride;
  for (int i = threadIdx.x; i < R * HD; i += blockDim.x) {
    const int r = i / HD, d = i % HD;
    float mx = -INFINITY;
    for (int s = 0; s < a.nsplit; ++s) mx = fmaxf(mx, base[s * stride + RMAX * HD + r]);
    float l = 0.f, o = 0.f;
    if (mx != -INFINITY) {
      for (int s = 0; s < a.nsplit; ++s) {
        const float ms = base[s * stride + RMAX * HD + r];
        if (ms == -INFINITY) continue;
        const float w = expf(ms - mx);
        l = fmaf(base[s * stride + RMAX * HD + RMAX + r], w, l);
        o = fmaf(base[s * stride + i], w, o);
      }
    }
    const int qi = r / G, gi = r % G;
    write_out(a, tok0 + qi, (kvh * G + gi) * HD + d, l > 0.f ? o / l : 0.f);
  }
}

static int attn_rmax(int qb_max, int G) { return qb_max * G <= 8 ? 8 : 64; }

size_t attention_part_floats(int nqb, int nkv, int nsplit, int qb_max, int group, int hd) {
  const int rmax = attn_rmax(qb_max, group);
  return (size_t)nqb * nkv * nsplit * (size_t)(rmax * hd + 2 * rmax);
}

template <int HD, int RMAX>
static int attn_set_smem() {
  Q8_CUDA(cudaFuncSetAttribute(k_attn<HD, RMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)sizeof(AttnSmem<HD, RMAX>)));
  return Q8_OK;
}

// Opts the attention kernels into >48 KB dynamic shared memory on the current
// device.  Called once per device before any launch (never inside a capture).
int attention_init() {
  static bool done[64] = {false};
  int dev = 0;
  Q8_CUDA(cudaGetDevice(&dev));
  if (done[dev & 63]) return Q8_OK;
  Q8_TRY((attn_set_smem<64, 8>()));
  Q8_TRY((attn_set_smem<64, 64>()));
  Q8_TRY((attn_set_smem<128, 8>()));
  Q8_TRY((attn_set_smem<128, 64>()));
  done[dev & 63] = true;
  return Q8_OK;
}

template <int HD, int RMAX>
static int attn_run(const AttnArgs& a, cudaStream_t st) {
  const size_t sm = sizeof(AttnSmem<HD, RMAX>);
  dim3 grid(a.nqb, a.nkv, a.nsplit);
  k_attn<HD, RMAX><<<grid, 128, sm, st>>>(a);
  Q8_TRY(launch_check("k_attn"));
  if (a.nsplit > 1) {
    k_attn_combine<HD, RMAX><<<dim3(a.nqb, a.nkv), 128, 0, st>>>(a);
    Q8_TRY(launch_check("k_attn_combine"));
  }
  return Q8_OK;
}

int attention_launch(const AttnArgs& a, cudaStream_t st) {
  Q8_CHECK_ARG(a.nkv > 0 && a.nh % a.nkv == 0, "attention: n_heads %% n_kv != 0");
  const int G = a.nh / a.nkv;
  Q8_CHECK_ARG(a.qb_max * G <= 64, "attention: query block x group must be <= 64");
  Q8_CHECK_ARG(a.nsplit >= 1 && (a.nsplit == 1 || a.part), "attention: split needs scratch");
  if (a.nqb <= 0) return Q8_OK;
  if (attention_tc_supported(a)) {
    Q8_TRY(attention_tc_launch(a, st));
    if (a.nsplit > 1) {
      if (a.hd == 128) k_attn_combine<128, 64><<<dim3(a.nqb, a.nkv), 128, 0, st>>>(a);
      else k_attn_combine<64, 64><<<dim3(a.nqb, a.nkv), 128, 0, st>>>(a);
      Q8_TRY(launch_check("k_attn_combine"));
    }
    return Q8_OK;
  }
  const bool small = a.qb_max * G <= 8;
  switch (a.hd) {
    case 64: return small ? attn_run<64, 8>(a, st) : attn_run<64, 64>(a, st);
    case 128: return small ? attn_run<128, 8>(a, st) : attn_run<128, 64>(a, st);
    default:
      set_error("attention: head_dim %d unsupported (64/128)", a.hd);
      return Q8_ERR_ARG;
  }
}

// ------------------------------------------------------------------ argmax
// k_argmax (src/llama_common.mojo:493-519): one CTA per row; lowest index wins
// ties (numpy.argmax), where the reference's 32-lane tree keeps the lower lane.
__global__ void __launch_bounds__(1024) k_argmax(const float* __restrict__ x, int64_t n, int64_t ld,
                                                 int32_t* __restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_trigger();
  pdl_wait();
  const float* row = x + (int64_t)blockIdx.x * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = row[i];
    if (v > bv) {
      bv = v;
      bi = (int)i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    bv = threadIdx.x < nw ? sv[threadIdx.x] : -INFINITY;
    bi = threadIdx.x < nw ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (threadIdx.x == 0) out[blockIdx.x] = (bi == 0x7fffffff) ? 0 : bi;
  }
}

// Wide rows (vocabulary logits): blocks reduce chunks of the row; the last
// block to finish (ticket counter) merges the chunk winners in chunk order, so
// the result is the lowest index of the maximum, as in k_argmax.
constexpr int ARGMAX_MAXB = 64;
constexpr int ARGMAX_MAXROWS = 4096;

__device__ __forceinline__ void amax_merge(float& bv, int& bi, float ov, int oi) {
  if (ov > bv || (ov == bv && oi < bi)) {
    bv = ov;
    bi = oi;
  }
}

__global__ void __launch_bounds__(256) k_argmax_mb(const float* __restrict__ x, int64_t n, int64_t ld,
                                                   int32_t* __restrict__ out, float* pv, int* pi, int* ticket) {
  __shared__ float sv[8];
  __shared__ int si[8];
  __shared__ int s_last;
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.y, nb = gridDim.x, b = blockIdx.x;
  const int64_t chunk = ((n + nb - 1) / nb + 3) & ~(int64_t)3;
  const int64_t lo = (int64_t)b * chunk, hi = min(n, lo + chunk);
  const float* row = x + (int64_t)r * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  // lo is a multiple of 4: with a 16-byte aligned row the chunk reads as float4
  const int64_t n4 = ((((uintptr_t)row) & 15) == 0 && hi > lo) ? (hi - lo) / 4 : 0;
  for (int64_t q = threadIdx.x; q < n4; q += blockDim.x) {
    const int64_t i = lo + 4 * q;
    const float4 v = *reinterpret_cast<const float4*>(row + i);
    amax_merge(bv, bi, v.x, (int)i);
    amax_merge(bv, bi, v.y, (int)i + 1);
    amax_merge(bv, bi, v.z, (int)i + 2);
    amax_merge(bv, bi, v.w, (int)i + 3);
  }
  for (int64_t j = lo + 4 * n4 + threadIdx.x; j < hi; j += blockDim.x) amax_merge(bv, bi, row[j], (int)j);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax_merge(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k) amax_merge(bv, bi, sv[k], si[k]);
    pv[r * ARGMAX_MAXB + b] = bv;
    pi[r * ARGMAX_MAXB + b] = bi;
    __threadfence();
    s_last = atomicAdd(ticket + r, 1) == nb - 1;
    __threadfence();
  }
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;
  float v = -INFINITY;
  int ix = 0x7fffffff;
  for (int k = 0; k < nb; ++k) amax_merge(v, ix, __ldcg(pv + r * ARGMAX_MAXB + k), __ldcg(pi + r * ARGMAX_MAXB + k));
  out[r] = (ix == 0x7fffffff) ? 0 : ix;
  ticket[r] = 0;  // ready for the next launch
}

struct ArgmaxScratch {
  float* pv = nullptr;
  int* pi = nullptr;
  int* ticket = nullptr;
};
static ArgmaxScratch g_amax[64];
static std::mutex g_amax_mu;

// Allocated once per device, outside stream capture (model creation calls it).
int argmax_prepare() {
  int dev = 0;
  Q8_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_amax_mu);
  ArgmaxScratch& s = g_amax[dev & 63];
  if (s.pv) return Q8_OK;
  if (cudaMalloc(&s.pv, (size_t)ARGMAX_MAXROWS * ARGMAX_MAXB * 4) != cudaSuccess ||
      cudaMalloc(&s.pi, (size_t)ARGMAX_MAXROWS * ARGMAX_MAXB * 4) != cudaSuccess ||
      cudaMalloc(&s.ticket, (size_t)ARGMAX_MAXROWS * 4) != cudaSuccess ||
      cudaMemset(s.ticket, 0, (size_t)ARGMAX_MAXROWS * 4) != cudaSuccess) {
    cudaGetLastError();
    set_error("argmax scratch allocation failed");
    return Q8_ERR_OOM;
  }
  return Q8_OK;
}

int argmax_launch(const float* logits, int64_t rows, int64_t n, int64_t ld, int32_t* out, cudaStream_t st) {
  if (rows <= 0) return Q8_OK;
  if (n >= 16384 && rows <= ARGMAX_MAXROWS) {
    Q8_TRY(argmax_prepare());
    int dev = 0;
    Q8_CUDA(cudaGetDevice(&dev));
    const ArgmaxScratch& s = g_amax[dev & 63];
    const int nb = (int)std::min<int64_t>(ARGMAX_MAXB, (n + 4095) / 4096);
    return launch_pdl("k_argmax_mb", k_argmax_mb, dim3(nb, (unsigned)rows), dim3(256), 0, st, logits, n, ld, out,
                      s.pv, s.pi, s.ticket);
  }
  return launch_pdl("k_argmax", k_argmax, dim3((unsigned)rows), dim3(1024), 0, st, logits, n, ld, out);
}

}  // namespace q8

using namespace q8;

// ------------------------------------------------------------------ op-level C ABI
extern "C" int q8op_embed(const void* packed_emb, int64_t vocab, int64_t d, const int32_t* ids, int64_t s,
                          float* y, void* stream) {
  Q8_CHECK_ARG(packed_emb && ids && y && vocab > 0 && d > 0 && d % Q8_QG == 0 && s >= 0,
               "q8op_embed: bad argument");
  return embed_launch(packed_emb, d, ids, s, y, (cudaStream_t)stream);
}

extern "C" int q8op_rmsnorm(float* x, const float* resid, const uint16_t* w_bf16, int64_t rows, int64_t d,
                            float eps, float* y, void* stream) {
  Q8_CHECK_ARG(x && w_bf16 && y && rows >= 0 && d > 0, "q8op_rmsnorm: bad argument");
  Q8_CHECK_ARG(!(resid && x == y), "q8op_rmsnorm: y may alias x only without resid");
  return rmsnorm_launch(x, resid, w_bf16, rows, d, eps, y, nullptr, nullptr, (cudaStream_t)stream);
}

extern "C" int q8op_rmsnorm_heads(const float* x, const uint16_t* w_bf16, int64_t rows, int64_t hd, float eps,
                                  float* y, void* stream) {
  Q8_CHECK_ARG(x && w_bf16 && y && rows >= 0 && hd > 0, "q8op_rmsnorm_heads: bad argument");
  return rmsnorm_heads_launch(x, w_bf16, rows, hd, eps, y, (cudaStream_t)stream);
}

extern "C" int q8op_rope_kv_append(float* qkv, int64_t ldqkv, int64_t T, const int32_t* pos, const int32_t* seq,
                                   int n_heads, int n_kv, int hd, const float* inv_freq, const uint16_t* q_norm,
                                   const uint16_t* k_norm, float eps, float* k_pages, float* v_pages, int page,
                                   const int32_t* block_table, int max_pages, void* stream) {
  Q8_CHECK_ARG(qkv && pos && seq && inv_freq && k_pages && v_pages && block_table, "q8op_rope_kv_append: null");
  Q8_CHECK_ARG(n_heads > 0 && n_kv > 0 && page > 0 && max_pages > 0 && ldqkv >= (int64_t)(n_heads + 2 * n_kv) * hd,
               "q8op_rope_kv_append: bad shape");
  return rope_kv_launch(qkv, ldqkv, T, pos, seq, n_heads, n_kv, hd, inv_freq, q_norm, k_norm, eps, k_pages,
                        v_pages, page, block_table, max_pages, (cudaStream_t)stream);
}

extern "C" int q8op_attention(const float* q, int64_t ldq, int64_t T, const int32_t* pos, const int32_t* seq,
                              int n_heads, int n_kv, int hd, const float* k_pages, const float* v_pages,
                              int page, const int32_t* block_table, int max_pages, float* out, int64_t ldo,
                              void* stream) {
  Q8_CHECK_ARG(q && pos && seq && k_pages && v_pages && block_table && out, "q8op_attention: null");
  Q8_CHECK_ARG(T >= 0 && T < (1 << 24) && n_kv > 0 && n_heads % n_kv == 0 && page > 0,
               "q8op_attention: bad shape");
  if (T == 0) return Q8_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const int G = n_heads / n_kv;
  const int items = (int)T * n_kv;
  // every token is an independent query (one per item); split the context so
  // that the grid covers the GPU
  const int nsplit = attention_decode_nsplit(items, (int)std::min<int64_t>((int64_t)max_pages * page, 1 << 30));
  float* part = nullptr;
  int* ticket = nullptr;
  if (nsplit > 1) {
    const size_t pf = attention_decode_part_floats((int)T, n_kv, nsplit, G, hd);
    void* scr = nullptr;
    const size_t pbytes = (pf * 4 + 255) & ~(size_t)255;
    Q8_TRY(op_scratch(pbytes + (size_t)items * 4, &scr));
    part = (float*)scr;
    ticket = (int*)((char*)scr + pbytes);
    Q8_CUDA(cudaMemsetAsync(ticket, 0, (size_t)items * 4, st));
  }
  return attention_decode_launch(q, ldq, (int)T, pos, seq, n_heads, n_kv, hd, k_pages, v_pages, page, block_table,
                                 max_pages, nsplit, part, ticket, out, ldo, nullptr, st);
}

extern "C" int q8op_argmax(const float* logits, int64_t rows, int64_t n, int64_t ld, int32_t* out, void* stream) {
  Q8_CHECK_ARG(logits && out && rows >= 0 && n > 0 && ld >= n, "q8op_argmax: bad argument");
  return argmax_launch(logits, rows, n, ld, out, (cudaStream_t)stream);
}
