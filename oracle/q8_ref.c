/*
 * CPU restatement of the reference Q8 decode path — TEST INFRASTRUCTURE
 * (checker and timed CPU baseline; never linked into libq8cuda).
 *
 * The reference (plutonium-guy/lama32_mojo) has no CPU build: its kernels are
 * Mojo for Apple Metal.  This file restates those kernels in C (multithreaded) so
 * the host cores can run the same algorithm:
 *
 *   q8r_gemv      k_mm_q8        src/llama_q8.mojo:54-93  (32-lane group loop,
 *                 16-wide chunks, per-group f16 scale, 4-wide final sum)
 *   q8r_embed     k_embed_gather_q8  src/llama_q8.mojo:96-109
 *   q8r_rmsnorm   k_rmsnorm_w    src/llama_common.mojo:197-225
 *   q8r_rope_kv   k_rope_qk_copy2 src/llama_common.mojo:299-342 (contiguous cache)
 *   q8r_attend    k_scores / k_softmax_rows / k_att_out  src/llama_common.mojo:402-473
 *   q8r_swiglu    k_swiglu_mul   src/llama_common.mojo:476-481
 *   q8r_argmax    k_argmax       src/llama_common.mojo:493-519 (lowest index on ties)
 *   q8r_layer     run_layer_q8   src/llama_q8.mojo:144-230 (one decode token)
 *   q8r_sample    sample         src/sample.mojo:15-59 (temperature + nucleus, the
 *                 selection loop literally: repeated first-maximum pick with
 *                 swap-remove), the uniform draw supplied by the caller
 *
 * Build: oracle/Makefile (gcc -O3 -shared -pthread).  Parallel loops use a
 * small pthread fork/join over rows (no OpenMP runtime in this toolchain).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#include <pthread.h>
#include <unistd.h>

#define QG 64

static inline float f16_to_f32(uint16_t h) {
  const uint32_t s = (uint32_t)(h >> 15) << 31;
  uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff, bits;
  if (e == 0) {
    if (m == 0) {
      bits = s;
    } else { /* subnormal */
      e = 127 - 15 + 1;
      while (!(m & 0x400)) { m <<= 1; --e; }
      m &= 0x3ff;
      bits = s | (e << 23) | (m << 13);
    }
  } else if (e == 31) {
    bits = s | 0x7f800000u | (m << 13);
  } else {
    bits = s | ((e + 127 - 15) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static inline float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static int g_threads = 0;

int q8r_threads(void) {
  if (g_threads <= 0) {
    const char* e = getenv("Q8REF_THREADS");
    long n = e ? atol(e) : sysconf(_SC_NPROCESSORS_ONLN);
    g_threads = n > 0 ? (int)(n > 256 ? 256 : n) : 1;
  }
  return g_threads;
}

void q8r_set_threads(int n) { g_threads = n; }

typedef void (*range_fn)(void* arg, int64_t lo, int64_t hi);
typedef struct { range_fn fn; void* arg; int64_t lo, hi; } range_job;

static void* range_tramp(void* p) {
  range_job* j = (range_job*)p;
  j->fn(j->arg, j->lo, j->hi);
  return NULL;
}

/* fork/join: split [0, n) into contiguous chunks, one per thread */
static void parallel_for(int64_t n, range_fn fn, void* arg) {
  int t = q8r_threads();
  if (t > n) t = (int)n;
  if (t <= 1) {
    fn(arg, 0, n);
    return;
  }
  pthread_t th[256];
  range_job jobs[256];
  for (int i = 0; i < t; ++i) {
    jobs[i].fn = fn;
    jobs[i].arg = arg;
    jobs[i].lo = n * i / t;
    jobs[i].hi = n * (i + 1) / t;
    if (i > 0) pthread_create(&th[i], NULL, range_tramp, &jobs[i]);
  }
  range_tramp(&jobs[0]);
  for (int i = 1; i < t; ++i) pthread_join(th[i], NULL);
}

typedef struct { const float* x; int s, m; const uint8_t* W; int n; float* y; } gemv_args;

/* one output y[i, j] in the reference's accumulation order (k_mm_q8):
 * lane t walks groups t, t+32, ...; per group a 16-wide FMA over 4 chunks,
 * lane-sum, times the f16 scale; the 32 lane partials are summed 4-wide. */
static void gemv_range(void* p, int64_t lo, int64_t hi) {
  const gemv_args* a = (const gemv_args*)p;
  const int m = a->m;
  const int64_t rb = m / 32 + m;
  const int ng = m / QG;
  for (int64_t idx = lo; idx < hi; ++idx) {
    const int64_t i = idx / a->n, j = idx % a->n;
    const uint8_t* row = a->W + j * rb;
    const uint16_t* sc = (const uint16_t*)row;
    const int8_t* q = (const int8_t*)(row + m / 32);
    const float* xr = a->x + i * m;
    float part[32];
    for (int t = 0; t < 32; ++t) {
      float acc = 0.f;
      for (int g = t; g < ng; g += 32) {
        const int k = g * QG;
        float gacc[16] = {0};
        for (int c = 0; c < 4; ++c)
          for (int l = 0; l < 16; ++l) gacc[l] = fmaf(xr[k + 16 * c + l], (float)q[k + 16 * c + l], gacc[l]);
        float r = 0.f;
        for (int l = 0; l < 16; ++l) r += gacc[l];
        acc += f16_to_f32(sc[g]) * r;
      }
      part[t] = acc;
    }
    float tot[4] = {0, 0, 0, 0};
    for (int qq = 0; qq < 32; qq += 4)
      for (int l = 0; l < 4; ++l) tot[l] += part[qq + l];
    a->y[i * a->n + j] = tot[0] + tot[1] + tot[2] + tot[3];
  }
}

/* y[s, n] = x[s, m] . W[n, m]^T, W packed [n][m/64 f16 | m int8] */
void q8r_gemv(const float* x, int s, int m, const uint8_t* W, int n, float* y) {
  gemv_args a = {x, s, m, W, n, y};
  parallel_for((int64_t)s * n, gemv_range, &a);
}

void q8r_embed(const uint8_t* E, int d, const int32_t* ids, int s, float* y) {
  const int64_t rb = d / 32 + d;
  for (int i = 0; i < s; ++i) {
    const uint8_t* row = E + (int64_t)ids[i] * rb;
    const uint16_t* sc = (const uint16_t*)row;
    const int8_t* q = (const int8_t*)(row + d / 32);
    for (int c = 0; c < d; ++c) y[(int64_t)i * d + c] = (float)q[c] * f16_to_f32(sc[c / QG]);
  }
}

void q8r_rmsnorm(const float* x, const uint16_t* w, int rows, int d, float eps, float* y) {
  for (int r = 0; r < rows; ++r) {
    const float* xr = x + (int64_t)r * d;
    float ss = 0.f;
    for (int k = 0; k < d; ++k) ss = fmaf(xr[k], xr[k], ss);
    const float inv = 1.0f / sqrtf(ss / (float)d + eps);
    for (int k = 0; k < d; ++k) y[(int64_t)r * d + k] = bf16_to_f32(w[k]) * xr[k] * inv;
  }
}

static void rmsnorm_inplace_heads(float* x, const uint16_t* w, int rows, int hd, float eps) {
  for (int r = 0; r < rows; ++r) q8r_rmsnorm(x + (int64_t)r * hd, w, 1, hd, eps, x + (int64_t)r * hd);
}

/* rotate-half RoPE of q and k at position pos; append k, v to the caches [maxlen, kvd] */
void q8r_rope_kv(float* q, float* k, const float* v, int nh, int nkv, int hd, int pos, const float* inv,
                 float* kc, float* vc) {
  const int half = hd / 2;
  for (int h = 0; h < nh + nkv; ++h) {
    float* base = h < nh ? q + h * hd : k + (h - nh) * hd;
    for (int d = 0; d < half; ++d) {
      const float f = (float)pos * inv[d];
      const float c = cosf(f), s = sinf(f);
      const float x0 = base[d], x1 = base[half + d];
      base[d] = x0 * c - x1 * s;
      base[half + d] = x1 * c + x0 * s;
    }
  }
  memcpy(kc + (int64_t)pos * nkv * hd, k, sizeof(float) * nkv * hd);
  memcpy(vc + (int64_t)pos * nkv * hd, v, sizeof(float) * nkv * hd);
}

typedef struct { const float *q, *kc, *vc; int nh, nkv, hd, pos; float* out; } attend_args;

static void attend_range(void* p, int64_t lo, int64_t hi) {
  const attend_args* a = (const attend_args*)p;
  const int group = a->nh / a->nkv, kvd = a->nkv * a->hd, n = a->pos + 1, hd = a->hd;
  float* pr = (float*)malloc(sizeof(float) * n);
  for (int64_t h = lo; h < hi; ++h) {
    const float* qh = a->q + h * hd;
    const int kvh = (int)h / group;
    float mx = -3.0e38f;
    for (int j = 0; j < n; ++j) {
      const float* kr = a->kc + (int64_t)j * kvd + kvh * hd;
      float acc = 0.f;
      for (int d = 0; d < hd; ++d) acc = fmaf(qh[d], kr[d], acc);
      pr[j] = acc / sqrtf((float)hd);
      if (pr[j] > mx) mx = pr[j];
    }
    float sm = 0.f;
    for (int j = 0; j < n; ++j) {
      pr[j] = expf(pr[j] - mx);
      sm += pr[j];
    }
    for (int j = 0; j < n; ++j) pr[j] /= sm;
    for (int d = 0; d < hd; ++d) {
      float acc = 0.f;
      for (int j = 0; j < n; ++j) acc = fmaf(pr[j], a->vc[(int64_t)j * kvd + kvh * hd + d], acc);
      a->out[h * hd + d] = acc;
    }
  }
  free(pr);
}

/* one query token at position pos over cache rows 0..pos (scores, max-subtracted
 * softmax, P.V; heads in parallel) */
void q8r_attend(const float* q, const float* kc, const float* vc, int nh, int nkv, int hd, int pos, float* out) {
  attend_args a = {q, kc, vc, nh, nkv, hd, pos, out};
  parallel_for(nh, attend_range, &a);
}

void q8r_swiglu(float* g, const float* u, int n) {
  for (int i = 0; i < n; ++i) g[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
}

int q8r_argmax(const float* x, int n) {
  int b = 0;
  for (int i = 1; i < n; ++i)
    if (x[i] > x[b]) b = i;
  return b;
}

/* Layer weights of one decode layer (packed rows; q|k|v and gate|up contiguous
 * as in the reference's s==1 fused dispatch, src/llama_q8.mojo:163-166, 215-217). */
typedef struct {
  const uint8_t *qkv, *o, *gu, *down;
  const uint16_t *in_norm, *post_norm, *q_norm, *k_norm; /* q_norm/k_norm NULL for Llama */
} q8r_layer_w;

/* run_layer_q8 for one token at position pos (s == 1); h [H] updated in place.
 * scratch: >= 2*H + 2*QD + 2*KVD + 2*F floats. */
void q8r_layer(const q8r_layer_w* w, float* h, int H, int nh, int nkv, int hd, int F, float eps, int pos,
               const float* inv, float* kc, float* vc, float* scratch) {
  const int QD = nh * hd, KVD = nkv * hd;
  float* xn = scratch;
  float* qkv = xn + H;
  float* ao = qkv + QD + 2 * KVD;
  float* o = ao + QD;
  float* gu = o + H;
  q8r_rmsnorm(h, w->in_norm, 1, H, eps, xn);
  q8r_gemv(xn, 1, H, w->qkv, QD + 2 * KVD, qkv);
  if (w->q_norm) {
    rmsnorm_inplace_heads(qkv, w->q_norm, nh, hd, eps);
    rmsnorm_inplace_heads(qkv + QD, w->k_norm, nkv, hd, eps);
  }
  q8r_rope_kv(qkv, qkv + QD, qkv + QD + KVD, nh, nkv, hd, pos, inv, kc, vc);
  q8r_attend(qkv, kc, vc, nh, nkv, hd, pos, ao);
  q8r_gemv(ao, 1, QD, w->o, H, o);
  for (int i = 0; i < H; ++i) h[i] += o[i];
  q8r_rmsnorm(h, w->post_norm, 1, H, eps, xn);
  q8r_gemv(xn, 1, H, w->gu, 2 * F, gu);
  q8r_swiglu(gu, gu + F, F);
  q8r_gemv(gu, 1, F, w->down, H, o);
  for (int i = 0; i < H; ++i) h[i] += o[i];
}

/* sample (src/sample.mojo:15-59), step by step:
 *   temp <= 0: greedy argmax (:21-22, first maximum, :7-12);
 *   candidates: logits >= max - 16, in index order, p = exp((l - max) / temp),
 *   total = their f32 sum in index order (:23-35); none: argmax (:36-37);
 *   target = total * top_p; the nucleus is built by picking the largest
 *   remaining p (first in list order), appending it and moving the list's last
 *   entry into its place, while cum < target (:38-53);
 *   r = f32(u) * cum and the first nucleus entry whose running sum reaches r
 *   (:54-59).  u is the caller's uniform draw (the reference draws
 *   random_float64()).
 * margin (may be NULL) receives the smallest relative gap of a decision that
 * one ulp of exp() could flip: cum against target at the stop, r against the
 * running sums around the returned entry, and the returned p against the
 * nearest different candidate p.  A checker whose exp() differs in the last
 * place may disagree only when that gap is about 1e-6 or less. */
static double rel_gap(double a, double b) {
  const double d = fabs(a - b), m = fmax(fabs(a), fabs(b));
  return m > 0 ? d / m : 0.0;
}

int q8r_sample(const float* logits, int n, float temp, float top_p, float u, double* margin) {
  if (margin) *margin = INFINITY;
  const int am = q8r_argmax(logits, n);
  if (temp <= 0.0f) return am;
  const float mx = logits[am];
  const float cutoff = mx - 16.0f;
  int* ci = (int*)malloc((size_t)n * sizeof(int));
  float* cp = (float*)malloc((size_t)n * sizeof(float));
  int* ni = (int*)malloc((size_t)n * sizeof(int));
  float* np_ = (float*)malloc((size_t)n * sizeof(float));
  float* all = (float*)malloc((size_t)n * sizeof(float));
  int c = 0;
  float total = 0.0f;
  for (int i = 0; i < n; ++i) {
    if (logits[i] < cutoff) continue;
    const float pr = expf((logits[i] - mx) / temp);
    ci[c] = i;
    cp[c] = pr;
    all[c] = pr;
    ++c;
    total += pr;
  }
  const int nc = c;
  int tok = am;
  if (c > 0) {
    const float target = total * top_p;
    int k = 0;
    float cum = 0.0f, prev = 0.0f;
    while (cum < target && c > 0) {
      int b = 0;
      for (int i = 1; i < c; ++i)
        if (cp[i] > cp[b]) b = i;
      prev = cum;
      cum += cp[b];
      ni[k] = ci[b];
      np_[k] = cp[b];
      ++k;
      ci[b] = ci[c - 1];
      cp[b] = cp[c - 1];
      --c;
    }
    double mg = INFINITY;
    if (margin) {
      mg = fmin(rel_gap(cum, target), k > 1 ? rel_gap(prev, target) : INFINITY);
    }
    const float r = u * cum;
    float acc = 0.0f, before = 0.0f;
    int pick = k - 1;
    for (int i = 0; i < k; ++i) {
      before = acc;
      acc += np_[i];
      if (r <= acc) {
        pick = i;
        break;
      }
    }
    tok = ni[pick];
    if (margin) {
      mg = fmin(mg, rel_gap(r, acc));
      if (pick > 0) mg = fmin(mg, rel_gap(r, before));
      const float pp = np_[pick];
      for (int i = 0; i < nc; ++i)
        if (all[i] != pp) mg = fmin(mg, rel_gap(all[i], pp));
      *margin = mg;
    }
  }
  free(ci);
  free(cp);
  free(ni);
  free(np_);
  free(all);
  return tok;
}
