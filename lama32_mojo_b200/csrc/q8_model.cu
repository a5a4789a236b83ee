// Model runtime behind the C ABI: context, weight arena (with tensor-parallel
// slicing at load), paged f32 KV cache, forward / batched decode / on-device
// greedy generation (CUDA graphs), NCCL all-reduce for tensor parallelism.
//
// Reference structure being replaced (paths in plutonium-guy/lama32_mojo):
//   QwenQ8 / Llama shells      qwen3_mojo/src/qwen_q8.mojo:55-177, src/llama_gpu.mojo:52-170
//   run_layer_q8               src/llama_q8.mojo:144-230
//   Weights arena, upload_all  src/resident.mojo:15-60
//   Acts bump arena            src/llama_common.mojo:578-606
//   SafeTensors                src/safetensors.mojo:17-96
#include "q8_allreduce.h"
#include "q8_decode_ring.h"
#include "q8_kernels.h"
#include "safetensors.h"

#include <array>
#include <cmath>
#include <fcntl.h>
#include <nccl.h>
#include <stdarg.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <map>
#include <set>
#include <string>
#include <vector>

namespace q8 {

static thread_local std::string t_err;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
}
const char* get_error() { return t_err.c_str(); }

bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("Q8_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// --------------------------------------------------------------------------- TP helper kernels
__global__ void k_argmax_local(const float* __restrict__ x, int64_t n, int64_t ld, float* __restrict__ val,
                               int32_t* __restrict__ idx) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const float* row = x + (int64_t)blockIdx.x * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = row[i];
    if (v > bv) { bv = v; bi = (int)i; }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    bv = threadIdx.x < nw ? sv[threadIdx.x] : -INFINITY;
    bi = threadIdx.x < nw ? si[threadIdx.x] : 0x7fffffff;
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (threadIdx.x == 0) { val[blockIdx.x] = bv; idx[blockIdx.x] = bi; }
  }
}

// gathered [tp][rows] (val, local idx) -> global argmax, lowest global index on ties
__global__ void k_argmax_pick(const float* __restrict__ val, const int32_t* __restrict__ idx, int tp, int rows,
                              int64_t vloc, int32_t* __restrict__ out) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float bv = -INFINITY;
  int64_t bi = 0;
  bool any = false;
  for (int k = 0; k < tp; ++k) {
    const float v = val[k * rows + r];
    const int li = idx[k * rows + r];
    if (li == 0x7fffffff) continue;
    const int64_t gi = k * vloc + li;
    if (!any || v > bv || (v == bv && gi < bi)) { bv = v; bi = gi; any = true; }
  }
  out[r] = (int32_t)bi;
}

// generation step epilogue: feed argmax back as next ids, advance positions,
// append to the on-device token history.
// Uniform draw of a sampled row: SplitMix64's finalizer (Steele, Lea, Flood
// 2014) over seed + (key + 1) * golden gamma, key = sequence << 32 | position
// of the fed token; the top 24 bits give u in [0, 1) exactly.
__host__ __device__ inline float q8_draw(unsigned long long seed, int seq, int pos) {
  const unsigned long long key = ((unsigned long long)(unsigned)seq << 32) | (unsigned)pos;
  unsigned long long z = seed + (key + 1ull) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(z >> 40) * (1.0f / 16777216.0f);
}

__global__ void k_sample_draws(const int32_t* __restrict__ pos, const int32_t* __restrict__ seq, int rows,
                               unsigned long long seed, float* __restrict__ u) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < rows) u[b] = q8_draw(seed, seq[b], pos[b]);
}

__global__ void k_step_end(const int32_t* __restrict__ amax, int32_t* __restrict__ ids, int32_t* __restrict__ pos,
                           int32_t* __restrict__ hist, int32_t* __restrict__ ctr, int B, int cap) {
  const int b = threadIdx.x;
  const int step = *ctr;
  if (b < B) {
    const int32_t t = amax[b];
    ids[b] = t;
    pos[b] += 1;
    if (step < cap) hist[(int64_t)step * B + b] = t;
  }
  __syncthreads();
  if (b == 0) *ctr = step + 1;
}

}  // namespace q8

using namespace q8;

// --------------------------------------------------------------------------- context
struct LayerW {
  uint8_t *qkv = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;
  uint16_t *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
};

struct ProfEvent {
  std::string name;
  cudaEvent_t a, b;
  double bytes;
};

struct q8_ctx {
  q8_config cfg{};
  int dev = 0, tp_rank = 0, tp_size = 1;
  int max_seqs = 1, maxlen = 0, max_tokens = 0;
  int page = 64, max_pages = 0;
  int H = 0, hd = 0, nh = 0, nkv = 0, G = 0, qd = 0, kvd = 0, F = 0, V = 0, V_loc = 0, V_off = 0;
  int qb_max = 1;
  cudaStream_t st = nullptr;
  ncclComm_t comm = nullptr;
  int tc_dmin = 16;        // decode batches from this size run the tensor-core pipeline
  ArState ar;             // one-shot P2P allreduce for decode (TP > 1)
  int* ar_status_pin = nullptr;
  // error words of the files whose kernels have bounded waits (tensor-core
  // GEMM, decode attention), copied after every call into dev_err_pin
  int* dev_err[2] = {nullptr, nullptr};
  int* dev_err_pin = nullptr;
  std::string err;

  uint8_t* warena = nullptr;
  size_t wbytes = 0;
  uint8_t *embed = nullptr, *lm_head = nullptr;
  uint16_t* final_norm = nullptr;
  std::vector<LayerW> layers;
  std::set<std::string> loaded;
  std::vector<std::string> required;
  bool ready = false;

  float *kpool = nullptr, *vpool = nullptr;
  size_t layer_kv = 0;  // floats per layer per pool
  int32_t* bt_d = nullptr;
  std::vector<int> n_cached;
  float* inv_freq_d = nullptr;

  int32_t *ids_d = nullptr, *pos_d = nullptr, *seq_d = nullptr, *qb_tok0_d = nullptr, *qb_len_d = nullptr;
  int32_t *argmax_d = nullptr, *hist_d = nullptr, *ctr_d = nullptr;
  int* ticket_d = nullptr;  // attention split tickets, zero at rest
  int hist_cap = 0;
  int32_t* pin = nullptr;  // pinned staging: 5 * max_tokens int32
  float *h = nullptr, *qkv = nullptr, *ypart = nullptr, *logits = nullptr, *part = nullptr;
  size_t part_floats = 0;
  __half *xs_in = nullptr, *xs_ao = nullptr, *xs_act = nullptr;
  bool tc = false;  // tensor-core GEMM for prefill batches (every K a multiple of 512)
  bool bf16 = false;  // linear weights kept as bf16 rows (q8_config.weight_dtype == Q8_BF16)
  // weight-ring decode step (one GPU, one sequence): q8_decode_ring.cu
  bool dr = false;
  int dr_grid = 0, dr_nsplit = 1;
  DrLayer* dr_layers = nullptr;
  float *dr_h1 = nullptr, *dr_pres = nullptr, *dr_apart = nullptr;
  int *dr_aticket = nullptr, *dr_lm_ticket = nullptr, *dr_status = nullptr, *dr_status_pin = nullptr;
  unsigned long long* dr_amax = nullptr;
  unsigned int* dr_bar = nullptr;
  uint8_t* dr_wring = nullptr;  // the matrices again, in ring layout (q8_decode_ring.cu)
  std::vector<std::array<uint8_t*, 4>> dr_rw;  // per layer: q|k|v, o, gate|up, down in dr_wring
  uint8_t* dr_rlm = nullptr;                   // lm_head rows of this rank in dr_wring
  float* dr_hm = nullptr;                      // residual after o_proj (tensor parallel)
  bool dr_packed = false;       // dr_wring matches the loaded weights
  unsigned long long* dr_trace = nullptr;  // CTA 0's phase marks of the last profiled ring step
  bool dr_traced = false;
  double dr_wbytes = 0;  // weight bytes one step streams
  double dr_kv_bytes = 0;
  float *xn32 = nullptr, *ao32 = nullptr, *act32 = nullptr;  // f32 copies of the GEMV inputs
  float *am_val = nullptr, *am_gval = nullptr, *lg_gather = nullptr;
  int32_t *am_idx = nullptr, *am_gidx = nullptr;
  float* logits_host_pin = nullptr;
  // sampling (q8_set_sampling): temp > 0 replaces the greedy argmax
  float samp_temp = 0.f, samp_top_p = 1.f;
  unsigned long long samp_seed = 0;
  void* samp_ws = nullptr;
  size_t samp_ws_bytes = 0;
  float* samp_u = nullptr;       // [rows] uniform draws of the step
  float* samp_logits = nullptr;  // [rows][V] vocabulary-ordered rows (TP > 1)

  std::map<int, cudaGraphExec_t> g_decode, g_gen;

  bool profiling = false;
  std::vector<ProfEvent> prof;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev_pool;
  size_t ev_used = 0;
  int prof_depth_guard = 0;
};

// Bytes of one stored weight row of K inputs: packed Q8, or plain bf16.
static int64_t wrow_bytes(const q8_ctx* c, int64_t K) { return c->bf16 ? 2 * K : q8_row_bytes(K); }

static int fail_ctx(q8_ctx* c, int s) {
  if (s != Q8_OK && c) c->err = get_error();
  return s;
}

// --------------------------------------------------------------------------- profiling
static int prof_begin(q8_ctx* c, cudaEvent_t* b_out) {
  if (!c->profiling) return Q8_OK;
  if (c->ev_used == c->ev_pool.size()) {
    cudaEvent_t a, b;
    Q8_CUDA(cudaEventCreate(&a));
    Q8_CUDA(cudaEventCreate(&b));
    c->ev_pool.push_back({a, b});
  }
  auto& pr = c->ev_pool[c->ev_used];
  Q8_CUDA(cudaEventRecord(pr.first, c->st));
  *b_out = pr.first;
  return Q8_OK;
}
static int prof_end(q8_ctx* c, const char* name, double bytes) {
  if (!c->profiling) return Q8_OK;
  auto& pr = c->ev_pool[c->ev_used++];
  Q8_CUDA(cudaEventRecord(pr.second, c->st));
  c->prof.push_back({name, pr.first, pr.second, bytes});
  return Q8_OK;
}
#define PROF(c, name, bytes, expr)                 \
  do {                                             \
    cudaEvent_t _pe;                               \
    Q8_TRY(prof_begin((c), &_pe));                 \
    Q8_TRY(expr);                                  \
    Q8_TRY(prof_end((c), (name), (bytes)));        \
  } while (0)

static double gemv_bytes(int64_t M, int64_t K, int64_t N) {
  return (double)N * q8_row_bytes(K) + (double)M * K * 4.0 + (double)M * N * 4.0;
}

// --------------------------------------------------------------------------- forward core
static int allreduce(q8_ctx* c, float* buf, size_t n) {
  if (c->tp_size == 1) return Q8_OK;
  ncclResult_t r = ncclAllReduce(buf, buf, n, ncclFloat, ncclSum, c->comm, c->st);
  if (r != ncclSuccess) {
    set_error("ncclAllReduce: %s", ncclGetErrorString(r));
    return Q8_ERR_COMM;
  }
  return Q8_OK;
}

// Decode-sized row-parallel sums: h += sum over ranks of part on the P2P path
// (the next RMSNorm then runs in the GEMV prologue); returns false when the
// batch is too large for it, so the caller keeps NCCL + the RMSNorm kernel.
static bool p2p_fits(q8_ctx* c, int T) { return c->ar.ok && (int64_t)T * c->H <= c->ar.slot; }

// Ring-layout copy of every matrix the ring step streams, made once after
// the weights are loaded (and again after a reload), outside graph capture.
static int ring_prepare(q8_ctx* c) {
  if (!c->dr || c->dr_packed) return Q8_OK;
  const int H = c->H, nqkv = c->qd + 2 * c->kvd;
  for (int L = 0; L < c->cfg.layers; ++L) {
    const LayerW& w = c->layers[L];
    Q8_TRY(dr_repack(w.qkv, nqkv, H, 0, c->dr_rw[L][0], c->st));
    Q8_TRY(dr_repack(w.o, H, c->qd, 0, c->dr_rw[L][1], c->st));
    Q8_TRY(dr_repack(w.gu, 2 * (int64_t)c->F, H, c->F, c->dr_rw[L][2], c->st));
    Q8_TRY(dr_repack(w.down, H, c->F, 0, c->dr_rw[L][3], c->st));
  }
  Q8_TRY(dr_repack(c->lm_head, c->V_loc, H, 0, c->dr_rlm, c->st));
  Q8_CUDA(cudaStreamSynchronize(c->st));
  c->dr_packed = true;
  return Q8_OK;
}

// Whether a step of T tokens runs as one weight-ring launch (one decode
// token, greedy, the whole vocabulary on this GPU).
static bool ring_ok(q8_ctx* c, int T, bool blocks, int lrow0, int lrows) {
  return c->dr && T == 1 && !blocks && lrow0 == 0 && lrows == 1 && !(c->samp_temp > 0.f);
}

// One weight-ring decode step for the token in ids_d / pos_d / seq_d; with
// gen, the launch also feeds its argmax back (k_step_end's work).
static int ring_step(q8_ctx* c, bool gen) {
  DrParams p{};
  p.H = c->H; p.nh = c->nh; p.nkv = c->nkv; p.hd = c->hd; p.qd = c->qd; p.nqkv = c->qd + 2 * c->kvd;
  p.F = c->F; p.V = c->V_loc; p.L = c->cfg.layers; p.eps = c->cfg.eps;
  p.layers = c->dr_layers; p.embed = c->embed; p.lm_head = c->dr_rlm;
  p.final_norm = c->final_norm;
  p.ids = c->ids_d; p.pos = c->pos_d; p.seq = c->seq_d; p.inv_freq = c->inv_freq_d;
  p.page = c->page; p.bt = c->bt_d; p.max_pages = c->max_pages;
  p.qdp = dr_kpad(c->qd); p.Fp = dr_kpad(c->F);
  p.h0 = c->h; p.h1 = c->dr_h1; p.pres = c->dr_pres; p.nsf = dr_down_nsf(c->H, p.Fp, c->dr_grid);
  p.qkv = c->qkv; p.ao = c->ao32; p.act = c->act32;
  p.logits = c->logits; p.apart = c->dr_apart; p.aticket = c->dr_aticket; p.nsplit = c->dr_nsplit;
  p.amax = c->dr_amax; p.lm_ticket = c->dr_lm_ticket; p.argmax = c->argmax_d;
  p.gen = gen ? 1 : 0; p.hist = c->hist_d; p.ctr = c->ctr_d; p.hist_cap = c->hist_cap;
  p.bar = c->dr_bar; p.status = c->dr_status;
  p.trace = c->profiling ? c->dr_trace : nullptr;
  c->dr_traced = c->profiling;
  p.tp = c->tp_size; p.rank = c->tp_rank; p.V_off = c->V_off; p.gsum = c->tp_size * c->dr_grid;
  if (c->tp_size > 1) {
    const size_t xo = (size_t)dr_xin_region(2, 0, c->tp_size, c->H) * 4;
    const size_t co = (xo + 255) & ~(size_t)255;  // counters after the inbox (dr_rx_bytes)
    for (int k = 0; k < c->tp_size; ++k) {
      uint8_t* b = c->ar.peers.rx[k];
      p.xin[k] = reinterpret_cast<float*>(b);
      p.xcnt[k] = reinterpret_cast<unsigned long long*>(b + co);
      p.xamax[k] = reinterpret_cast<unsigned long long*>(b + co + 64);
    }
    p.xstep = reinterpret_cast<unsigned long long*>(c->ar.rx + co + 128);
    p.xin_me = p.xin[c->tp_rank];
    p.xcnt_me = p.xcnt[c->tp_rank];
    p.xamax_me = p.xamax[c->tp_rank];
    p.hm = c->dr_hm;
  }
  return dr_launch(p, c->dr_grid, c->st);
}

// Next tokens of logit rows [lrow0, lrow0 + lrows) into argmax_d: sampled
// (q8_set_sampling) or greedy (k_argmax, src/llama_common.mojo:493-519).
static int select_tokens(q8_ctx* c, int lrow0, int lrows) {
  cudaStream_t st = c->st;
  const bool tp = c->tp_size > 1;
  if (c->samp_temp > 0.f) {  // sampled tokens into argmax_d
    cudaEvent_t pe;
    Q8_TRY(prof_begin(c, &pe));
    const float* lg = c->logits;
    if (tp) {  // every rank samples the whole vocabulary with the same draws
      ncclResult_t r = ncclAllGather(c->logits, c->lg_gather, (size_t)lrows * c->V_loc, ncclFloat, c->comm, st);
      if (r != ncclSuccess) {
        set_error("logits allgather: %s", ncclGetErrorString(r));
        return Q8_ERR_COMM;
      }
      for (int k = 0; k < c->tp_size; ++k)  // [tp][rows][V_loc] -> [rows][V]
        Q8_CUDA(cudaMemcpy2DAsync(c->samp_logits + (size_t)k * c->V_loc, (size_t)c->V * 4,
                                  c->lg_gather + (size_t)k * lrows * c->V_loc, (size_t)c->V_loc * 4,
                                  (size_t)c->V_loc * 4, lrows, cudaMemcpyDeviceToDevice, st));
      lg = c->samp_logits;
    }
    k_sample_draws<<<ceil_div(lrows, 128), 128, 0, st>>>(c->pos_d + lrow0, c->seq_d + lrow0, lrows, c->samp_seed,
                                                         c->samp_u);
    Q8_TRY(launch_check("k_sample_draws"));
    Q8_TRY(sample_launch(lg, lrows, c->V, c->V, c->samp_temp, c->samp_top_p, c->samp_u, c->argmax_d, c->samp_ws,
                         c->samp_ws_bytes, st));
    Q8_TRY(prof_end(c, "sample", (double)lrows * c->V * 4.0));
  } else if (!tp) {
    PROF(c, "argmax", (double)lrows * c->V * 4.0,
         argmax_launch(c->logits, lrows, c->V, c->V, c->argmax_d, st));
  } else {
    cudaEvent_t pe;
    Q8_TRY(prof_begin(c, &pe));
    k_argmax_local<<<lrows, 1024, 0, st>>>(c->logits, c->V_loc, c->V_loc, c->am_val, c->am_idx);
    Q8_TRY(launch_check("k_argmax_local"));
    ncclGroupStart();
    ncclAllGather(c->am_val, c->am_gval, lrows, ncclFloat, c->comm, st);
    ncclAllGather(c->am_idx, c->am_gidx, lrows, ncclInt32, c->comm, st);
    ncclResult_t r = ncclGroupEnd();
    if (r != ncclSuccess) {
      set_error("argmax allgather: %s", ncclGetErrorString(r));
      return Q8_ERR_COMM;
    }
    k_argmax_pick<<<ceil_div(lrows, 128), 128, 0, st>>>(c->am_gval, c->am_gidx, c->tp_size, lrows, c->V_loc,
                                                         c->argmax_d);
    Q8_TRY(launch_check("k_argmax_pick"));
    Q8_TRY(prof_end(c, "argmax", (double)lrows * c->V_loc * 4.0));
  }
  return Q8_OK;
}

// bf16-weight layers: the reference's non-Q8 run_layer
// (src/llama_common.mojo:697-780) behind mm_op (:636-684).  Standalone
// RMSNorm into f32 rows, bf16 products with the residual add and SwiGLU fused
// into their epilogues, the Q8 path's RoPE / KV-append / attention kernels, and
// a bf16 lm_head (tied: the embedding rows).
static int run_tokens_bf16(q8_ctx* c, int T, bool blocks, int nqb, int qb_max, int nsplit, int lrow0, int lrows,
                           double kv_bytes_hint) {
  const int H = c->H;
  const int nqkv = c->qd + 2 * c->kvd;
  cudaStream_t st = c->st;
  const bool tp = c->tp_size > 1;
  const float eps = c->cfg.eps;
  auto bw = [](const uint8_t* p) { return reinterpret_cast<const uint16_t*>(p); };
  auto bytes = [](int64_t M, int64_t K, int64_t N) { return (double)N * K * 2.0 + (double)M * (K + N) * 4.0; };
  PROF(c, "embed", (double)T * H * 6.0, embed_bf16_launch(bw(c->embed), H, c->ids_d, T, c->h, st));
  const float* pending = nullptr;  // row-parallel sum not yet added to h (TP prefill)
  // row-parallel output (o_proj, down): added into h, or summed over ranks
  auto rowpar = [&](const char* name, const float* x, int K, const uint8_t* W) -> int {
    if (!tp) {
      PROF(c, name, bytes(T, K, H), gemm_bf16_launch(EPI_ADD, x, K, T, K, bw(W), H, c->h, H, st));
      return Q8_OK;
    }
    PROF(c, name, bytes(T, K, H), gemm_bf16_launch(EPI_STORE, x, K, T, K, bw(W), H, c->ypart, H, st));
    if (!blocks && p2p_fits(c, T)) {
      PROF(c, "allreduce", (double)T * H * 4.0 * c->tp_size, ar_launch(c->ar, c->ypart, c->h, T * H, st));
    } else {
      PROF(c, "allreduce", (double)T * H * 4.0, allreduce(c, c->ypart, (size_t)T * H));
      pending = c->ypart;
    }
    return Q8_OK;
  };
  for (int L = 0; L < c->cfg.layers; ++L) {
    const LayerW& w = c->layers[L];
    PROF(c, "rmsnorm", (double)T * H * (pending ? 16.0 : 8.0),
         rmsnorm_launch(c->h, pending, w.in_norm, T, H, eps, c->xn32, nullptr, nullptr, st));
    pending = nullptr;
    PROF(c, "gemm_qkv", bytes(T, H, nqkv), gemm_bf16_launch(EPI_STORE, c->xn32, H, T, H, bw(w.qkv), nqkv, c->qkv,
                                                            nqkv, st));
    float* kp = c->kpool + (size_t)L * c->layer_kv;
    float* vp = c->vpool + (size_t)L * c->layer_kv;
    if (blocks) {
      PROF(c, "rope_kv", (double)T * (c->qd + 3.0 * c->kvd) * 8.0,
           rope_kv_launch(c->qkv, nqkv, T, c->pos_d, c->seq_d, c->nh, c->nkv, c->hd, c->inv_freq_d, w.q_norm,
                          w.k_norm, eps, kp, vp, c->page, c->bt_d, c->max_pages, st));
      AttnArgs a{};
      a.q = c->qkv; a.ldq = nqkv; a.T = T; a.pos = c->pos_d; a.seq = c->seq_d;
      a.nh = c->nh; a.nkv = c->nkv; a.hd = c->hd;
      a.kp = kp; a.vp = vp;
      a.page = c->page; a.bt = c->bt_d; a.max_pages = c->max_pages;
      a.qb_tok0 = c->qb_tok0_d; a.qb_len = c->qb_len_d;
      a.nqb = nqb; a.qb_max = qb_max; a.nsplit = nsplit; a.part = c->part;
      a.out32 = c->ao32; a.ldo = c->qd; a.outxs = nullptr;
      PROF(c, "attention", kv_bytes_hint / c->cfg.layers + (double)T * c->qd * 8.0, attention_launch(a, st));
    } else {
      const AttnRope rope{c->inv_freq_d, w.q_norm, w.k_norm, eps, kp, vp};
      PROF(c, "attention", kv_bytes_hint / c->cfg.layers + (double)T * c->qd * 8.0,
           attention_decode_launch(c->qkv, nqkv, T, c->pos_d, c->seq_d, c->nh, c->nkv, c->hd, kp, vp, c->page,
                                   c->bt_d, c->max_pages, nsplit, c->part, c->ticket_d, c->ao32, c->qd, nullptr, st,
                                   &rope, (int64_t)(c->layer_kv / c->hd)));
    }
    Q8_TRY(rowpar("gemm_o", c->ao32, c->qd, w.o));
    PROF(c, "rmsnorm", (double)T * H * (pending ? 16.0 : 8.0),
         rmsnorm_launch(c->h, pending, w.post_norm, T, H, eps, c->xn32, nullptr, nullptr, st));
    pending = nullptr;
    PROF(c, "gemm_gateup", bytes(T, H, 2 * c->F),
         gemm_bf16_launch(EPI_SWIGLU, c->xn32, H, T, H, bw(w.gu), c->F, c->act32, c->F, st));
    Q8_TRY(rowpar("gemm_down", c->act32, c->F, w.down));
  }
  if (lrows <= 0) return Q8_OK;
  float* hrow = c->h + (size_t)lrow0 * H;
  const float* prow = pending ? pending + (size_t)lrow0 * H : nullptr;
  PROF(c, "rmsnorm", (double)lrows * H * 8.0,
       rmsnorm_launch(hrow, prow, c->final_norm, lrows, H, eps, c->xn32, nullptr, nullptr, st));
  PROF(c, "gemm_lmhead", bytes(lrows, H, c->V_loc),
       gemm_bf16_launch(EPI_STORE, c->xn32, H, lrows, H, bw(c->lm_head), c->V_loc, c->logits, c->V_loc, st));
  return select_tokens(c, lrow0, lrows);
}

// Runs T tokens whose ids/pos/seq (and query blocks, when qb_tok0 != null) are
// already in the device buffers.  Produces logits + argmax for token rows
// [lrow0, lrow0 + lrows).  kv_ctx_hint bounds the context for split sizing.
static int run_tokens(q8_ctx* c, int T, bool blocks, int nqb, int qb_max, int nsplit, int lrow0, int lrows,
                      double kv_bytes_hint) {
  const int H = c->H;
  const int nqkv = c->qd + 2 * c->kvd;
  cudaStream_t st = c->st;
  const bool tp = c->tp_size > 1;
  if (ring_ok(c, T, blocks, lrow0, lrows)) {
    PROF(c, "decode_step", c->dr_wbytes + kv_bytes_hint, ring_step(c, false));
    return Q8_OK;
  }
  if (c->bf16) return run_tokens_bf16(c, T, blocks, nqb, qb_max, nsplit, lrow0, lrows, kv_bytes_hint);
  PROF(c, "embed", (double)T * (q8_row_bytes(H) + H * 4.0),
       embed_launch(c->embed, H, c->ids_d, T, c->h, st));
  const float* pending = nullptr;  // row-parallel partial sum not yet added to h
  // small token batches fuse RMSNorm into the GEMV prologue (K = hidden fits
  // the shared-memory staging); large batches keep the standalone kernel
  const bool fuse_norm = H <= 6144 && T <= 64;
  // prefill-sized batches, and decode batches of at least c->tc_dmin
  // sequences, run the tensor-core GEMM on f16 activation rows; the XS
  // buffers double as those rows (they hold twice the elements)
  const bool tc = c->tc && T >= (blocks ? kTcMinTokens : c->tc_dmin);
  __half* xn16 = c->xs_in;
  __half* ao16 = c->xs_ao;
  __half* act16 = c->xs_act;
  // split activations: lo planes half a buffer further (each XS buffer holds
  // max_tokens x 2K halves)
  const bool tcx = tc && gemm_tc_exact();
  const int64_t loH = tcx ? (int64_t)c->max_tokens * H : 0, loQ = tcx ? (int64_t)c->max_tokens * c->qd : 0,
                loF = tcx ? (int64_t)c->max_tokens * c->F : 0;
  for (int L = 0; L < c->cfg.layers; ++L) {
    const LayerW& w = c->layers[L];
    if (tc) {
      PROF(c, "rmsnorm", (double)T * H * (pending ? 14.0 : 10.0),
           rmsnorm_launch(c->h, pending, w.in_norm, T, H, c->cfg.eps, nullptr, nullptr, xn16, st, loH));
      PROF(c, "gemm_qkv", gemv_bytes(T, H, nqkv),
           gemm_tc_launch(EPI_STORE, xn16, H, loH, T, H, w.qkv, nqkv, c->qkv, nqkv, nullptr, 0, 0, st));
    } else if (!pending && fuse_norm) {  // RMSNorm fused into the GEMV prologue
      PROF(c, "gemv_qkv", gemv_bytes(T, H, nqkv),
           gemv_rms_launch(EPI_STORE, c->h, H, w.in_norm, c->cfg.eps, T, H, w.qkv, nqkv, c->qkv, nqkv, nullptr, st));
    } else {
      PROF(c, "rmsnorm", (double)T * H * (pending ? 16.0 : 8.0),
           rmsnorm_launch(c->h, pending, w.in_norm, T, H, c->cfg.eps, c->xn32, c->xs_in, nullptr, st));
      PROF(c, "gemv_qkv", gemv_bytes(T, H, nqkv),
           gemm_dispatch(EPI_STORE, c->xn32, H, c->xs_in, T, H, w.qkv, nqkv, c->qkv, nqkv, nullptr, st));
    }
    // decode: RoPE, QK-norm and the KV append run inside the attention kernel
    if (blocks)
      PROF(c, "rope_kv", (double)T * (c->qd + 3.0 * c->kvd) * 8.0,
           rope_kv_launch(c->qkv, nqkv, T, c->pos_d, c->seq_d, c->nh, c->nkv, c->hd, c->inv_freq_d, w.q_norm,
                          w.k_norm, c->cfg.eps, c->kpool + (size_t)L * c->layer_kv,
                          c->vpool + (size_t)L * c->layer_kv, c->page, c->bt_d, c->max_pages, st));
    AttnArgs a{};
    a.q = c->qkv; a.ldq = nqkv; a.T = T; a.pos = c->pos_d; a.seq = c->seq_d;
    a.nh = c->nh; a.nkv = c->nkv; a.hd = c->hd;
    a.kp = c->kpool + (size_t)L * c->layer_kv; a.vp = c->vpool + (size_t)L * c->layer_kv;
    a.page = c->page; a.bt = c->bt_d; a.max_pages = c->max_pages;
    a.qb_tok0 = blocks ? c->qb_tok0_d : nullptr; a.qb_len = blocks ? c->qb_len_d : nullptr;
    a.nqb = nqb; a.qb_max = qb_max; a.nsplit = nsplit; a.part = c->part;
    a.out32 = c->ao32; a.ldo = c->qd; a.outxs = c->xs_ao;
    if (tc) {
      a.out32 = nullptr;
      a.outxs = nullptr;
      a.out16 = ao16;
      a.out16lo = loQ;
    }
    if (blocks) {
      PROF(c, "attention", kv_bytes_hint / c->cfg.layers + (double)T * c->qd * 8.0, attention_launch(a, st));
    } else {
      const AttnRope rope{c->inv_freq_d, w.q_norm, w.k_norm, c->cfg.eps, const_cast<float*>(a.kp),
                          const_cast<float*>(a.vp)};
      PROF(c, "attention", kv_bytes_hint / c->cfg.layers + (double)T * c->qd * 8.0,
           attention_decode_launch(c->qkv, nqkv, T, c->pos_d, c->seq_d, c->nh, c->nkv, c->hd, a.kp, a.vp, c->page,
                                   c->bt_d, c->max_pages, nsplit, c->part, c->ticket_d, tc ? nullptr : c->ao32,
                                   c->qd, tc ? nullptr : c->xs_ao, st, &rope, (int64_t)(c->layer_kv / c->hd),
                                   tc ? ao16 : nullptr, tc ? loQ : 0));
    }
    if (tc) {
      PROF(c, "gemm_o", gemv_bytes(T, c->qd, H),
           gemm_tc_launch(tp ? EPI_STORE : EPI_ADD, ao16, c->qd, loQ, T, c->qd, w.o, H, tp ? c->ypart : c->h, H,
                          nullptr, 0, 0, st));
      if (tp) {
        PROF(c, "allreduce", (double)T * H * 4.0, allreduce(c, c->ypart, (size_t)T * H));
        pending = c->ypart;
      }
    } else if (!tp) {
      PROF(c, "gemv_o", gemv_bytes(T, c->qd, H),
           gemm_dispatch(EPI_ADD, c->ao32, c->qd, c->xs_ao, T, c->qd, w.o, H, c->h, H, nullptr, st));
    } else {
      PROF(c, "gemv_o", gemv_bytes(T, c->qd, H),
           gemm_dispatch(EPI_STORE, c->ao32, c->qd, c->xs_ao, T, c->qd, w.o, H, c->ypart, H, nullptr, st));
      if (!blocks && p2p_fits(c, T)) {
        PROF(c, "allreduce", (double)T * H * 4.0 * c->tp_size, ar_launch(c->ar, c->ypart, c->h, T * H, st));
      } else {
        PROF(c, "allreduce", (double)T * H * 4.0, allreduce(c, c->ypart, (size_t)T * H));
        pending = c->ypart;
      }
    }
    if (tc) {
      PROF(c, "rmsnorm", (double)T * H * (pending ? 14.0 : 10.0),
           rmsnorm_launch(c->h, pending, w.post_norm, T, H, c->cfg.eps, nullptr, nullptr, xn16, st, loH));
      PROF(c, "gemm_gateup", gemv_bytes(T, H, 2 * c->F),
           gemm_tc_launch(EPI_SWIGLU, xn16, H, loH, T, H, w.gu, c->F, nullptr, 0, act16, c->F, loF, st));
      pending = nullptr;
      PROF(c, "gemm_down", gemv_bytes(T, c->F, H),
           gemm_tc_launch(tp ? EPI_STORE : EPI_ADD, act16, c->F, loF, T, c->F, w.down, H, tp ? c->ypart : c->h, H,
                          nullptr, 0, 0, st));
      if (tp) {
        PROF(c, "allreduce", (double)T * H * 4.0, allreduce(c, c->ypart, (size_t)T * H));
        pending = c->ypart;
      }
      continue;
    }
    if (!pending && fuse_norm) {
      PROF(c, "gemv_gateup", gemv_bytes(T, H, 2 * c->F),
           gemv_rms_launch(EPI_SWIGLU, c->h, H, w.post_norm, c->cfg.eps, T, H, w.gu, c->F, c->act32, c->F,
                           c->xs_act, st));
    } else {
      PROF(c, "rmsnorm", (double)T * H * (pending ? 16.0 : 8.0),
           rmsnorm_launch(c->h, pending, w.post_norm, T, H, c->cfg.eps, c->xn32, c->xs_in, nullptr, st));
      PROF(c, "gemv_gateup", gemv_bytes(T, H, 2 * c->F),
           gemm_dispatch(EPI_SWIGLU, c->xn32, H, c->xs_in, T, H, w.gu, c->F, c->act32, c->F, c->xs_act, st));
    }
    pending = nullptr;
    if (!tp) {
      PROF(c, "gemv_down", gemv_bytes(T, c->F, H),
           gemm_dispatch(EPI_ADD, c->act32, c->F, c->xs_act, T, c->F, w.down, H, c->h, H, nullptr, st));
    } else {
      PROF(c, "gemv_down", gemv_bytes(T, c->F, H),
           gemm_dispatch(EPI_STORE, c->act32, c->F, c->xs_act, T, c->F, w.down, H, c->ypart, H, nullptr, st));
      if (!blocks && p2p_fits(c, T)) {
        PROF(c, "allreduce", (double)T * H * 4.0 * c->tp_size, ar_launch(c->ar, c->ypart, c->h, T * H, st));
      } else {
        PROF(c, "allreduce", (double)T * H * 4.0, allreduce(c, c->ypart, (size_t)T * H));
        pending = c->ypart;
      }
    }
  }
  if (lrows <= 0) return Q8_OK;
  float* hrow = c->h + (size_t)lrow0 * H;
  const float* prow = pending ? pending + (size_t)lrow0 * H : nullptr;
  if (tc && lrows >= c->tc_dmin) {
    PROF(c, "rmsnorm", (double)lrows * H * 10.0,
         rmsnorm_launch(hrow, prow, c->final_norm, lrows, H, c->cfg.eps, nullptr, nullptr, xn16, st, loH));
    PROF(c, "gemv_lmhead", gemv_bytes(lrows, H, c->V_loc),
         gemm_tc_launch(EPI_STORE, xn16, H, loH, lrows, H, c->lm_head, c->V_loc, c->logits, c->V_loc, nullptr, 0, 0,
                        st));
  } else if (!prow && fuse_norm) {
    PROF(c, "gemv_lmhead", gemv_bytes(lrows, H, c->V_loc),
         gemv_rms_launch(EPI_STORE, hrow, H, c->final_norm, c->cfg.eps, lrows, H, c->lm_head, c->V_loc, c->logits,
                         c->V_loc, nullptr, st));
  } else {
    PROF(c, "rmsnorm", (double)lrows * H * 8.0,
         rmsnorm_launch(hrow, prow, c->final_norm, lrows, H, c->cfg.eps, c->xn32, c->xs_in, nullptr, st));
    PROF(c, "gemv_lmhead", gemv_bytes(lrows, H, c->V_loc),
         gemm_dispatch(EPI_STORE, c->xn32, H, c->xs_in, lrows, H, c->lm_head, c->V_loc, c->logits, c->V_loc, nullptr,
                       st));
  }
  return select_tokens(c, lrow0, lrows);
}

// Device status words (bounded waits of the ring step, the tensor-core GEMM,
// the decode attention and the P2P exchange): queued copies to pinned memory
// with the call's other results, checked after the call's synchronize.
static int status_copy(q8_ctx* c) {
  for (int i = 0; i < 2; ++i)
    Q8_CUDA(cudaMemcpyAsync(c->dev_err_pin + i, c->dev_err[i], 4, cudaMemcpyDeviceToHost, c->st));
  if (c->dr) Q8_CUDA(cudaMemcpyAsync(c->dr_status_pin, c->dr_status, 4, cudaMemcpyDeviceToHost, c->st));
  if (c->ar.ok) Q8_CUDA(cudaMemcpyAsync(c->ar_status_pin, c->ar.status, 4, cudaMemcpyDeviceToHost, c->st));
  return Q8_OK;
}

static int status_check(q8_ctx* c) {
  if (c->dev_err_pin[0] != 0 || c->dev_err_pin[1] != 0) {
    // a bounded wait gave up: the call's results are not trusted.  Clear the
    // words so that later waits in those kernels run to their full bound.
    const int v0 = c->dev_err_pin[0], v1 = c->dev_err_pin[1];
    c->dev_err_pin[0] = c->dev_err_pin[1] = 0;
    for (int i = 0; i < 2; ++i) Q8_CUDA(cudaMemsetAsync(c->dev_err[i], 0, 4, c->st));
    Q8_CUDA(cudaStreamSynchronize(c->st));
    set_error("%s: a bounded device wait timed out (device status %d)",
              v0 ? "tensor-core GEMM" : "decode attention", v0 ? v0 : v1);
    return Q8_ERR_TIMEOUT;
  }
  if (c->ar.ok && *c->ar_status_pin != 0) {
    const int v = *c->ar_status_pin;
    *c->ar_status_pin = 0;
    Q8_CUDA(cudaMemsetAsync(c->ar.status, 0, 4, c->st));
    Q8_CUDA(cudaStreamSynchronize(c->st));
    set_error("tensor-parallel allreduce: a peer flag wait timed out (device status %d)", v);
    return Q8_ERR_COMM;
  }
  if (!c->dr || *c->dr_status_pin == 0) return Q8_OK;
  const int v = *c->dr_status_pin;
  *c->dr_status_pin = 0;
  // the grid drained early: clear the status word and the step's tickets
  Q8_CUDA(cudaMemsetAsync(c->dr_status, 0, 4, c->st));
  Q8_CUDA(cudaMemsetAsync(c->dr_aticket, 0, (size_t)c->nkv * 4, c->st));
  Q8_CUDA(cudaMemsetAsync(c->dr_lm_ticket, 0, 4, c->st));
  Q8_CUDA(cudaMemsetAsync(c->dr_amax, 0, 8, c->st));
  Q8_CUDA(cudaStreamSynchronize(c->st));
  if (v == Q8_ERR_COMM) {
    set_error("decode step: a tensor-parallel exchange wait timed out (a peer rank did not arrive)");
    return Q8_ERR_COMM;
  }
  set_error("decode step: a bounded device wait timed out (device status %d)", v);
  return Q8_ERR_TIMEOUT;
}

static int gather_logits(q8_ctx* c, int rows, float* host) {
  if (c->tp_size == 1) {
    Q8_CUDA(cudaMemcpyAsync(host, c->logits, (size_t)rows * c->V * 4, cudaMemcpyDeviceToHost, c->st));
    return Q8_OK;
  }
  ncclResult_t r = ncclAllGather(c->logits, c->lg_gather, (size_t)rows * c->V_loc, ncclFloat, c->comm, c->st);
  if (r != ncclSuccess) {
    set_error("logits allgather: %s", ncclGetErrorString(r));
    return Q8_ERR_COMM;
  }
  // [tp][rows][V_loc] -> host [rows][V]
  for (int k = 0; k < c->tp_size; ++k) {
    Q8_CUDA(cudaMemcpy2DAsync(host + (size_t)k * c->V_loc, (size_t)c->V * 4,
                              c->lg_gather + (size_t)k * rows * c->V_loc, (size_t)c->V_loc * 4,
                              (size_t)c->V_loc * 4, rows, cudaMemcpyDeviceToHost, c->st));
  }
  return Q8_OK;
}

static int check_ready(q8_ctx* c) {
  if (c->ready) return Q8_OK;
  for (auto& n : c->required) {
    if (!c->loaded.count(n)) {
      set_error("weights not loaded: missing tensor %s", n.c_str());
      return Q8_ERR_STATE;
    }
  }
  c->ready = true;
  return Q8_OK;
}

static int decode_nsplit(q8_ctx* c, int B) {
  const int items = B * c->nkv;
  return std::max(1, std::min(attention_decode_nsplit(items, c->maxlen), 1024 / items));
}

static double kv_read_bytes(q8_ctx* c, const std::vector<int>& ctxlens) {
  double b = 0;
  for (int n : ctxlens) b += (double)n * 2.0 * c->kvd * 4.0;
  return b * c->cfg.layers;
}

// --------------------------------------------------------------------------- C ABI: model
extern "C" {

const char* q8_last_error(const q8_ctx* ctx) {
  if (ctx && !ctx->err.empty()) return ctx->err.c_str();
  return get_error();
}

const char* q8_status_string(int s) {
  switch (s) {
    case Q8_OK: return "ok";
    case Q8_ERR_ARG: return "invalid argument";
    case Q8_ERR_CUDA: return "CUDA error";
    case Q8_ERR_OOM: return "out of device memory";
    case Q8_ERR_KV_FULL: return "KV cache full";
    case Q8_ERR_IO: return "I/O error";
    case Q8_ERR_FORMAT: return "bad checkpoint format";
    case Q8_ERR_COMM: return "communication error";
    case Q8_ERR_TIMEOUT: return "device wait timed out";
    case Q8_ERR_STATE: return "invalid state";
    default: return "unknown status";
  }
}

const char* q8_version(void) { return "libq8cuda 0.1 sm_100a (W8A32 group-64)"; }

int q8_rope_inv_freq(const q8_config* cfg, float* out) {
  Q8_CHECK_ARG(cfg && out && cfg->head_dim > 0 && cfg->head_dim % 2 == 0, "q8_rope_inv_freq: bad argument");
  const int hd = cfg->head_dim;
  for (int d = 0; d < hd / 2; ++d) {
    const double inv = 1.0 / pow(cfg->theta, (double)(2 * d) / (double)hd);
    double v = inv;
    if (cfg->rope_type == Q8_ROPE_LLAMA3) {
      const double wavelen = 2.0 * 3.14159265358979323846 / inv;
      if (wavelen >= cfg->orig_ctx / cfg->high_ff) {
        if (wavelen > cfg->orig_ctx / cfg->low_ff) {
          v = inv / cfg->rope_factor;
        } else {
          const double smooth = (cfg->orig_ctx / wavelen - cfg->low_ff) / (cfg->high_ff - cfg->low_ff);
          v = (1.0 - smooth) * inv / cfg->rope_factor + smooth * inv;
        }
      }
    }
    out[d] = (float)v;
  }
  return Q8_OK;
}

int q8_nccl_unique_id(void* out128) {
  Q8_CHECK_ARG(out128, "q8_nccl_unique_id: null");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) {
    set_error("ncclGetUniqueId: %s", ncclGetErrorString(r));
    return Q8_ERR_COMM;
  }
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
  memcpy(out128, &id, 128);
  return Q8_OK;
}

static int destroy_impl(q8_ctx* c) {
  if (!c) return Q8_OK;
  cudaSetDevice(c->dev);
  if (c->st) cudaStreamSynchronize(c->st);
  for (auto& kv : c->g_decode) cudaGraphExecDestroy(kv.second);
  for (auto& kv : c->g_gen) cudaGraphExecDestroy(kv.second);
  for (auto& e : c->ev_pool) { cudaEventDestroy(e.first); cudaEventDestroy(e.second); }
  ar_teardown(&c->ar);
  if (c->ar_status_pin) cudaFreeHost(c->ar_status_pin);
  if (c->comm) ncclCommDestroy(c->comm);
  void* ptrs[] = {c->warena, c->kpool, c->vpool, c->bt_d, c->inv_freq_d, c->ids_d, c->pos_d, c->seq_d,
                  c->qb_tok0_d, c->qb_len_d, c->argmax_d, c->hist_d, c->ctr_d, c->ticket_d, c->h, c->qkv, c->ypart,
                  c->logits, c->part, c->xs_in, c->xs_ao, c->xs_act, c->xn32, c->ao32, c->act32, c->am_val, c->am_gval, c->lg_gather,
                  c->am_idx, c->am_gidx, c->dr_layers, c->dr_h1, c->dr_pres, c->dr_apart, c->dr_aticket,
                  c->dr_lm_ticket, c->dr_status, c->dr_amax, c->dr_bar, c->dr_trace, c->dr_wring,
                  c->dr_hm, c->samp_ws, c->samp_u, c->samp_logits};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  if (c->pin) cudaFreeHost(c->pin);
  if (c->dev_err_pin) cudaFreeHost(c->dev_err_pin);
  if (c->dr_status_pin) cudaFreeHost(c->dr_status_pin);
  if (c->st) cudaStreamDestroy(c->st);
  delete c;
  return Q8_OK;
}

int q8_destroy(q8_ctx* ctx) { return destroy_impl(ctx); }

static int dmalloc(void** p, size_t bytes) {
  if (cudaMalloc(p, std::max<size_t>(bytes, 256)) != cudaSuccess) {
    cudaGetLastError();
    set_error("cudaMalloc(%zu bytes) failed", bytes);
    return Q8_ERR_OOM;
  }
  return Q8_OK;
}

static std::vector<std::string> required_names(const q8_config& c) {
  std::vector<std::string> n = {"model.embed_tokens.weight", "model.norm.weight"};
  for (int L = 0; L < c.layers; ++L) {
    const std::string p = "model.layers." + std::to_string(L) + ".";
    for (const char* s : {"input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight",
                          "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight",
                          "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"})
      n.push_back(p + s);
    if (c.qk_norm) {
      n.push_back(p + "self_attn.q_norm.weight");
      n.push_back(p + "self_attn.k_norm.weight");
    }
  }
  if (!c.tied) n.push_back("lm_head.weight");
  return n;
}

static int create_impl(const q8_config* cfg, int device, int max_seqs, int maxlen, int max_tokens, int tp_rank,
                       int tp_size, const void* nccl_id, q8_ctx** out) {
  Q8_CHECK_ARG(cfg && out, "q8_create: null argument");
  const q8_config& C = *cfg;
  Q8_CHECK_ARG(C.hidden > 0 && C.layers > 0 && C.n_heads > 0 && C.n_kv > 0 && C.head_dim > 0 && C.inter > 0 &&
                   C.vocab > 0,
               "q8_create: non-positive dimension");
  Q8_CHECK_ARG(C.hidden % 64 == 0 && C.inter % 64 == 0, "q8_create: hidden and inter must be multiples of 64");
  Q8_CHECK_ARG(C.head_dim == 64 || C.head_dim == 128, "q8_create: head_dim must be 64 or 128");
  Q8_CHECK_ARG(C.n_heads % C.n_kv == 0, "q8_create: n_heads %% n_kv != 0");
  Q8_CHECK_ARG(tp_size >= 1 && tp_rank >= 0 && tp_rank < tp_size, "q8_create: bad tp rank/size");
  Q8_CHECK_ARG(C.n_kv % tp_size == 0 && C.n_heads % tp_size == 0 && C.vocab % tp_size == 0,
               "q8_create: heads and vocab must divide by tp_size");
  Q8_CHECK_ARG((C.inter / tp_size) % 64 == 0 && ((C.n_heads / tp_size) * C.head_dim) % 64 == 0,
               "q8_create: row-parallel K shards must be multiples of 64");
  Q8_CHECK_ARG(max_seqs >= 1 && maxlen >= 1 && max_tokens >= 1, "q8_create: bad capacities");
  Q8_CHECK_ARG(tp_size == 1 || nccl_id, "q8_create: tp_size > 1 needs an NCCL id");
  Q8_CHECK_ARG(C.n_heads / C.n_kv <= 64, "q8_create: GQA group > 64 unsupported");
  Q8_CHECK_ARG(C.weight_dtype == 0 || C.weight_dtype == Q8_PACKED || C.weight_dtype == Q8_BF16,
               "q8_create: weight_dtype must be Q8_PACKED (or 0) or Q8_BF16");

  q8_ctx* c = new q8_ctx();
  c->cfg = C;
  c->dev = device;
  c->tp_rank = tp_rank;
  c->tp_size = tp_size;
  c->max_seqs = max_seqs;
  c->maxlen = maxlen;
  c->max_tokens = std::max(max_tokens, max_seqs);
  c->H = C.hidden;
  c->hd = C.head_dim;
  c->nh = C.n_heads / tp_size;
  c->nkv = C.n_kv / tp_size;
  c->G = c->nh / c->nkv;
  c->qd = c->nh * c->hd;
  c->kvd = c->nkv * c->hd;
  c->F = C.inter / tp_size;
  c->bf16 = C.weight_dtype == Q8_BF16;
  {
    // Q8_TC=0 keeps prefill on the GEMV kernels (A/B comparisons); the
    // tensor-core GEMM reads packed Q8 rows only
    const char* e = getenv("Q8_TC");
    c->tc = !c->bf16 && C.hidden % 512 == 0 && c->qd % 512 == 0 && c->F % 512 == 0 && !(e && e[0] == '0');
    // Q8_TC_DECODE_MIN: decode batches from this many sequences use the
    // tensor-core pipeline (default 16; the GEMV kernels below it)
    const char* d = getenv("Q8_TC_DECODE_MIN");
    c->tc_dmin = d ? std::max(1, atoi(d)) : 16;
  }
  c->V = C.vocab;
  c->V_loc = C.vocab / tp_size;
  c->V_off = tp_rank * c->V_loc;
  c->qb_max = std::max(1, 64 / c->G);
  c->max_pages = ceil_div(maxlen, c->page);
  c->required = required_names(C);
  c->n_cached.assign(max_seqs, 0);

  auto bail = [&](int s) {
    std::string e = get_error();
    destroy_impl(c);
    set_error("%s", e.c_str());
    return s;
  };
  if (cudaSetDevice(device) != cudaSuccess) {
    cudaGetLastError();
    set_error("cudaSetDevice(%d) failed", device);
    delete c;
    return Q8_ERR_CUDA;
  }
  if (attention_init() != Q8_OK || gemv_init() != Q8_OK) {
    delete c;
    return Q8_ERR_CUDA;
  }
  if (cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking) != cudaSuccess) {
    set_error("cudaStreamCreate failed");
    delete c;
    return Q8_ERR_CUDA;
  }

  // ---- weight arena layout
  const int H = c->H;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    off = align256(off);
    size_t o = off;
    off += bytes;
    return o;
  };
  const size_t o_embed = take((size_t)C.vocab * wrow_bytes(c, H));
  const size_t o_head = C.tied ? 0 : take((size_t)c->V_loc * wrow_bytes(c, H));
  const size_t o_fnorm = take((size_t)H * 2);
  struct LOff { size_t qkv, o, gu, down, inn, post, qn, kn; };
  std::vector<LOff> lo(C.layers);
  for (int L = 0; L < C.layers; ++L) {
    lo[L].qkv = take((size_t)(c->qd + 2 * c->kvd) * wrow_bytes(c, H));
    lo[L].o = take((size_t)H * wrow_bytes(c, c->qd));
    lo[L].gu = take((size_t)2 * c->F * wrow_bytes(c, H));
    lo[L].down = take((size_t)H * wrow_bytes(c, c->F));
    lo[L].inn = take((size_t)H * 2);
    lo[L].post = take((size_t)H * 2);
    lo[L].qn = C.qk_norm ? take((size_t)c->hd * 2) : 0;
    lo[L].kn = C.qk_norm ? take((size_t)c->hd * 2) : 0;
  }
  c->wbytes = align256(off);
  int s;
  if ((s = dmalloc((void**)&c->warena, c->wbytes))) return bail(s);
  c->embed = c->warena + o_embed;
  c->lm_head = C.tied ? c->embed + (size_t)c->V_off * wrow_bytes(c, H) : c->warena + o_head;
  c->final_norm = (uint16_t*)(c->warena + o_fnorm);
  c->layers.resize(C.layers);
  for (int L = 0; L < C.layers; ++L) {
    LayerW& w = c->layers[L];
    w.qkv = c->warena + lo[L].qkv;
    w.o = c->warena + lo[L].o;
    w.gu = c->warena + lo[L].gu;
    w.down = c->warena + lo[L].down;
    w.in_norm = (uint16_t*)(c->warena + lo[L].inn);
    w.post_norm = (uint16_t*)(c->warena + lo[L].post);
    w.q_norm = C.qk_norm ? (uint16_t*)(c->warena + lo[L].qn) : nullptr;
    w.k_norm = C.qk_norm ? (uint16_t*)(c->warena + lo[L].kn) : nullptr;
  }

  // ---- paged KV cache: every sequence owns max_pages pages (static map)
  const size_t num_pages = (size_t)max_seqs * c->max_pages;
  c->layer_kv = num_pages * c->nkv * c->page * c->hd;
  if ((s = dmalloc((void**)&c->kpool, c->layer_kv * C.layers * 4))) return bail(s);
  if ((s = dmalloc((void**)&c->vpool, c->layer_kv * C.layers * 4))) return bail(s);
  {
    std::vector<int32_t> bt((size_t)max_seqs * c->max_pages);
    for (size_t i = 0; i < bt.size(); ++i) bt[i] = (int32_t)i;
    if ((s = dmalloc((void**)&c->bt_d, bt.size() * 4))) return bail(s);
    if (cudaMemcpy(c->bt_d, bt.data(), bt.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
      return bail((set_error("block table upload failed"), Q8_ERR_CUDA));
  }
  {
    std::vector<float> inv(c->hd / 2);
    q8_rope_inv_freq(&C, inv.data());
    if ((s = dmalloc((void**)&c->inv_freq_d, inv.size() * 4))) return bail(s);
    if (cudaMemcpy(c->inv_freq_d, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
      return bail((set_error("inv_freq upload failed"), Q8_ERR_CUDA));
  }

  // ---- activations
  const int T = c->max_tokens;
  const int Kmax = std::max(std::max(H, c->qd), c->F);
  const int rows_out = std::max(max_seqs, 1);
  c->hist_cap = 4096;
  if ((s = dmalloc((void**)&c->ids_d, (size_t)T * 4))) return bail(s);
  if ((s = dmalloc((void**)&c->pos_d, (size_t)T * 4))) return bail(s);
  if ((s = dmalloc((void**)&c->seq_d, (size_t)T * 4))) return bail(s);
  if ((s = dmalloc((void**)&c->qb_tok0_d, (size_t)T * 4))) return bail(s);
  if ((s = dmalloc((void**)&c->qb_len_d, (size_t)T * 4))) return bail(s);
  if ((s = dmalloc((void**)&c->argmax_d, (size_t)rows_out * 4))) return bail(s);
  if ((s = dmalloc((void**)&c->hist_d, (size_t)c->hist_cap * rows_out * 4))) return bail(s);
  if ((s = dmalloc((void**)&c->ctr_d, 4))) return bail(s);
  if ((s = dmalloc((void**)&c->ticket_d, (size_t)T * c->nkv * 4))) return bail(s);
  if (cudaMemset(c->ticket_d, 0, (size_t)T * c->nkv * 4) != cudaSuccess)
    return bail((set_error("ticket clear failed"), Q8_ERR_CUDA));
  if ((s = dmalloc((void**)&c->h, (size_t)T * H * 4))) return bail(s);
  if ((s = dmalloc((void**)&c->qkv, (size_t)T * (c->qd + 2 * c->kvd) * 4))) return bail(s);
  if (tp_size > 1 && (s = dmalloc((void**)&c->ypart, (size_t)T * H * 4))) return bail(s);
  if ((s = dmalloc((void**)&c->logits, (size_t)rows_out * c->V_loc * 4))) return bail(s);
  c->part_floats = (size_t)1024 * (64 * c->hd + 128);
  if ((s = dmalloc((void**)&c->part, c->part_floats * 4))) return bail(s);
  (void)Kmax;
  if ((s = dmalloc((void**)&c->xs_in, (size_t)T * 2 * H * 2))) return bail(s);
  if ((s = dmalloc((void**)&c->xs_ao, (size_t)T * 2 * c->qd * 2))) return bail(s);
  if ((s = dmalloc((void**)&c->xs_act, (size_t)T * 2 * c->F * 2))) return bail(s);
  if ((s = dmalloc((void**)&c->xn32, (size_t)T * H * 4))) return bail(s);
  if ((s = dmalloc((void**)&c->ao32, (size_t)T * c->qd * 4))) return bail(s);
  if ((s = dmalloc((void**)&c->act32, (size_t)T * c->F * 4))) return bail(s);
  if (tp_size > 1) {
    if ((s = dmalloc((void**)&c->am_val, (size_t)rows_out * 4))) return bail(s);
    if ((s = dmalloc((void**)&c->am_idx, (size_t)rows_out * 4))) return bail(s);
    if ((s = dmalloc((void**)&c->am_gval, (size_t)rows_out * tp_size * 4))) return bail(s);
    if ((s = dmalloc((void**)&c->am_gidx, (size_t)rows_out * tp_size * 4))) return bail(s);
    if ((s = dmalloc((void**)&c->lg_gather, (size_t)rows_out * C.vocab * 4))) return bail(s);
  }
  if (cudaMallocHost((void**)&c->pin, (size_t)T * 5 * 4) != cudaSuccess)
    return bail((set_error("cudaMallocHost failed"), Q8_ERR_OOM));
  if (cudaMallocHost((void**)&c->dev_err_pin, 2 * 4) != cudaSuccess)
    return bail((set_error("cudaMallocHost failed"), Q8_ERR_OOM));
  c->dev_err_pin[0] = c->dev_err_pin[1] = 0;
  if ((s = gemm_tc_error_word(&c->dev_err[0]))) return bail(s);
  if ((s = attn_dec_error_word(&c->dev_err[1]))) return bail(s);

  if ((s = argmax_prepare())) return bail(s);
  // the tensor-core GEMM's kernel attributes and split-K workspace, before
  // any decode step is captured into a graph (no allocation during capture)
  if (c->tc && (s = gemm_tc_prepare())) return bail(s);
  // digit GEMV scratch (split-tile partials, tickets): sized here, outside any
  // stream capture
  if ((s = gemv_d_prepare(std::max({ceil_div(c->qd + 2 * c->kvd, 16), ceil_div(H, 16), ceil_div(c->F, 8),
                                    ceil_div(c->V_loc, 16)})))) return bail(s);

  if (tp_size > 1) {
    ncclUniqueId id;
    memcpy(&id, nccl_id, 128);
    ncclResult_t r = ncclCommInitRank(&c->comm, tp_size, id, tp_rank);
    if (r != ncclSuccess) return bail((set_error("ncclCommInitRank: %s", ncclGetErrorString(r)), Q8_ERR_COMM));
    // decode-sized row-parallel sums over P2P, and the one-launch step's
    // exchange block (every rank takes this step)
    if ((s = ar_setup(&c->ar, c->comm, tp_size, tp_rank, (int64_t)std::max(1, max_seqs) * H,
                      dr_rx_bytes(tp_size, H), c->st)))
      return bail(s);
    if (c->ar.ok) {
      if (cudaMallocHost((void**)&c->ar_status_pin, 4) != cudaSuccess)
        return bail((set_error("pinned status allocation failed"), Q8_ERR_OOM));
      *c->ar_status_pin = 0;
    }
  }

  // ---- weight-ring decode step for one-sequence greedy decode
  // (default; Q8_RING=0 keeps those steps on the per-operation kernels)
  {
    const char* e = getenv("Q8_RING");
    const char* why = nullptr;
    if (!(e && e[0] == '0') && (tp_size == 1 || c->ar.ok) && !c->bf16 &&
        dr_supported(H, c->nh, c->nkv, c->hd, c->F, c->V_loc, c->page, &why)) {
      if ((s = dr_prepare(c->hd, &c->dr_grid))) return bail(s);
    }
    if (tp_size > 1) {  // every rank runs the ring step, with the same grid, or none does
      int* d = nullptr;
      if ((s = dmalloc((void**)&d, 8))) return bail(s);
      int v[2] = {c->dr_grid, -c->dr_grid}, o[2] = {0, 0};
      bool ok = cudaMemcpyAsync(d, v, 8, cudaMemcpyHostToDevice, c->st) == cudaSuccess &&
                ncclAllReduce(d, d, 2, ncclInt32, ncclMin, c->comm, c->st) == ncclSuccess &&
                cudaMemcpyAsync(o, d, 8, cudaMemcpyDeviceToHost, c->st) == cudaSuccess &&
                cudaStreamSynchronize(c->st) == cudaSuccess;
      cudaFree(d);
      if (!ok) return bail((set_error("decode step: rank agreement failed"), Q8_ERR_COMM));
      if (o[0] != -o[1]) c->dr_grid = 0;  // some rank cannot (or has another grid)
    }
    if (c->dr_grid > 0) {
      const int nqkv = c->qd + 2 * c->kvd;
      c->dr_nsplit = dr_nsplit(c->dr_grid, c->nkv, maxlen);
      if ((s = dmalloc((void**)&c->dr_h1, (size_t)H * 4))) return bail(s);
      if ((s = dmalloc((void**)&c->dr_pres, (size_t)DR_NS * H * 4))) return bail(s);
      if ((s = dmalloc((void**)&c->dr_apart, dr_apart_floats(c->nkv, c->dr_nsplit, c->hd) * 4))) return bail(s);
      if ((s = dmalloc((void**)&c->dr_aticket, (size_t)c->nkv * 4))) return bail(s);
      if ((s = dmalloc((void**)&c->dr_lm_ticket, 4))) return bail(s);
      if ((s = dmalloc((void**)&c->dr_status, 4))) return bail(s);
      if ((s = dmalloc((void**)&c->dr_amax, 8))) return bail(s);
      if ((s = dmalloc((void**)&c->dr_bar, 4))) return bail(s);
      if ((s = dmalloc((void**)&c->dr_layers, sizeof(DrLayer) * C.layers))) return bail(s);
      if (cudaMemset(c->dr_aticket, 0, (size_t)c->nkv * 4) != cudaSuccess ||
          cudaMemset(c->dr_lm_ticket, 0, 4) != cudaSuccess || cudaMemset(c->dr_status, 0, 4) != cudaSuccess ||
          cudaMemset(c->dr_amax, 0, 8) != cudaSuccess)
        return bail((set_error("decode step state clear failed"), Q8_ERR_CUDA));
      if (cudaMallocHost((void**)&c->dr_status_pin, 4) != cudaSuccess)
        return bail((set_error("cudaMallocHost failed"), Q8_ERR_OOM));
      *c->dr_status_pin = 0;
      // ring-layout copies: o_proj and down_proj inputs padded to whole
      // 512-code chunks (tensor-parallel K slices need not be)
      size_t rofs = 0;
      std::vector<std::array<size_t, 4>> ro(C.layers);
      auto rtake = [&](size_t b) {
        const size_t o = rofs;
        rofs += (b + 255) & ~(size_t)255;
        return o;
      };
      for (int L = 0; L < C.layers; ++L)
        ro[L] = {rtake(dr_ring_bytes(nqkv, H)), rtake(dr_ring_bytes(H, c->qd)), rtake(dr_ring_bytes(2 * c->F, H)),
                 rtake(dr_ring_bytes(H, c->F))};
      const size_t rlm = rtake(dr_ring_bytes(c->V_loc, H));
      if ((s = dmalloc((void**)&c->dr_wring, rofs))) return bail(s);
      if (tp_size > 1 && (s = dmalloc((void**)&c->dr_hm, (size_t)H * 4))) return bail(s);
      c->dr_rlm = c->dr_wring + rlm;
      c->dr_rw.resize(C.layers);
      std::vector<DrLayer> dl(C.layers);
      for (int L = 0; L < C.layers; ++L) {
        const LayerW& w = c->layers[L];
        for (int j = 0; j < 4; ++j) c->dr_rw[L][j] = c->dr_wring + ro[L][j];
        dl[L] = DrLayer{c->dr_rw[L][0], c->dr_rw[L][1], c->dr_rw[L][2], c->dr_rw[L][3], w.in_norm, w.post_norm,
                        w.q_norm, w.k_norm, c->kpool + (size_t)L * c->layer_kv, c->vpool + (size_t)L * c->layer_kv};
      }
      if (cudaMemcpy(c->dr_layers, dl.data(), sizeof(DrLayer) * C.layers, cudaMemcpyHostToDevice) != cudaSuccess)
        return bail((set_error("decode step layer table upload failed"), Q8_ERR_CUDA));
      if ((s = dmalloc((void**)&c->dr_trace, sizeof(unsigned long long) * 4 * (5 * C.layers + 1)))) return bail(s);
      // algorithmic bytes: the packed rows of this rank's matrices (the
      // zero padding of the ring layout is not counted)
      c->dr_wbytes = (double)C.layers * ((double)nqkv * q8_row_bytes(H) + (double)H * q8_row_bytes(c->qd) +
                                         2.0 * c->F * q8_row_bytes(H) + (double)H * q8_row_bytes(c->F)) +
                     (double)c->V_loc * q8_row_bytes(H);
      c->dr = true;
    }
  }

  *out = c;
  return Q8_OK;
}

int q8_create(const q8_config* cfg, int device, int max_seqs, int maxlen, int max_tokens, int tp_rank,
              int tp_size, const void* nccl_id, q8_ctx** out) {
  return create_impl(cfg, device, max_seqs, maxlen, max_tokens, tp_rank, tp_size, nccl_id, out);
}

// ---- weight loading
static int put_packed(q8_ctx* c, uint8_t* dst, const uint8_t* src, int64_t src_K, int64_t row0, int64_t nrows,
                      int64_t k0, int64_t Kl, int dtype, bool on_dev) {
  const cudaMemcpyKind kind = on_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  if (dtype == Q8_PACKED) {
    const int64_t srb = q8_row_bytes(src_K), drb = q8_row_bytes(Kl);
    if (Kl == src_K) {
      Q8_CUDA(cudaMemcpyAsync(dst, src + row0 * srb, (size_t)(nrows * srb), kind, c->st));
    } else {
      Q8_CUDA(cudaMemcpy2DAsync(dst, drb, src + row0 * srb + (k0 / 64) * 2, srb, Kl / 32, nrows, kind, c->st));
      Q8_CUDA(cudaMemcpy2DAsync(dst + Kl / 32, drb, src + row0 * srb + src_K / 32 + k0, srb, Kl, nrows, kind,
                                c->st));
    }
    Q8_CUDA(cudaStreamSynchronize(c->st));
    return Q8_OK;
  }
  // bf16 source: copy the slice to a device temp, quantize with the GPU packer
  void* tmp = nullptr;
  Q8_TRY(dmalloc(&tmp, (size_t)nrows * Kl * 2));
  int s = Q8_OK;
  if (cudaMemcpy2DAsync(tmp, Kl * 2, src + (row0 * src_K + k0) * 2, src_K * 2, Kl * 2, nrows, kind, c->st) !=
      cudaSuccess) {
    set_error("bf16 slice copy failed");
    s = Q8_ERR_CUDA;
  }
  if (s == Q8_OK) s = pack_launch(tmp, nrows, Kl, dst, c->st);
  if (s == Q8_OK && cudaStreamSynchronize(c->st) != cudaSuccess) {
    set_error("pack sync failed");
    s = Q8_ERR_CUDA;
  }
  cudaFree(tmp);
  return s;
}

struct ShardPlan {
  std::string slot;
  int64_t n = 0, m = 0;           // expected logical shape (m = 1 for vectors)
  int64_t row0 = 0, nrows = 0;    // source rows
  int64_t k0 = 0, kl = 0;         // source K slice
  int64_t dst_row = 0;            // first destination row in the slot
};

// Single source of truth for tensor-parallel placement (column-parallel
// q/k/v/gate/up, row-parallel o/down, vocab-parallel untied lm_head).
static int shard_plan(const q8_config& C, int r, int t, const std::string& name, ShardPlan& p) {
  const int64_t H = C.hidden, hd = C.head_dim;
  const int64_t QD = (int64_t)C.n_heads * hd, KVD = (int64_t)C.n_kv * hd, F = C.inter;
  const int64_t qd = QD / t, kvd = KVD / t, f = F / t, vloc = C.vocab / t;
  auto rows = [&](const char* slot, int64_t n, int64_t m, int64_t row0, int64_t nrows, int64_t dst) {
    p.slot = slot; p.n = n; p.m = m; p.row0 = row0; p.nrows = nrows; p.k0 = 0; p.kl = m; p.dst_row = dst;
  };
  auto kslice = [&](const char* slot, int64_t n, int64_t m, int64_t k0, int64_t kl) {
    p.slot = slot; p.n = n; p.m = m; p.row0 = 0; p.nrows = n; p.k0 = k0; p.kl = kl; p.dst_row = 0;
  };
  auto vec = [&](const char* slot, int64_t n) { rows(slot, n, 1, 0, n, 0); };
  p = ShardPlan();
  if (name == "model.embed_tokens.weight") { rows("embed", C.vocab, H, 0, C.vocab, 0); return Q8_OK; }
  if (name == "lm_head.weight") {
    if (!C.tied) rows("lm_head", C.vocab, H, (int64_t)r * vloc, vloc, 0);
    return Q8_OK;
  }
  if (name == "model.norm.weight") { vec("final_norm", H); return Q8_OK; }
  if (name.rfind("model.layers.", 0) != 0) return Q8_OK;
  const size_t dot = name.find('.', 13);
  if (dot == std::string::npos) return Q8_OK;
  const int L = atoi(name.substr(13, dot - 13).c_str());
  if (L < 0 || L >= C.layers) return Q8_OK;
  const std::string sfx = name.substr(dot + 1);
  if (sfx == "self_attn.q_proj.weight") rows("qkv", QD, H, r * qd, qd, 0);
  else if (sfx == "self_attn.k_proj.weight") rows("qkv", KVD, H, r * kvd, kvd, qd);
  else if (sfx == "self_attn.v_proj.weight") rows("qkv", KVD, H, r * kvd, kvd, qd + kvd);
  else if (sfx == "self_attn.o_proj.weight") kslice("o", H, QD, r * qd, qd);
  else if (sfx == "mlp.gate_proj.weight") rows("gu", F, H, r * f, f, 0);
  else if (sfx == "mlp.up_proj.weight") rows("gu", F, H, r * f, f, f);
  else if (sfx == "mlp.down_proj.weight") kslice("down", H, F, r * f, f);
  else if (sfx == "input_layernorm.weight") vec("in_norm", H);
  else if (sfx == "post_attention_layernorm.weight") vec("post_norm", H);
  else if (sfx == "self_attn.q_norm.weight" && C.qk_norm) vec("q_norm", hd);
  else if (sfx == "self_attn.k_norm.weight" && C.qk_norm) vec("k_norm", hd);
  return Q8_OK;
}

static int load_tensor_impl(q8_ctx* c, const char* cname, int dtype, int64_t rows, int64_t cols, const void* data,
                            int on_dev) {
  Q8_CHECK_ARG(c && cname && data, "q8_load_tensor: null argument");
  Q8_CHECK_ARG(dtype == Q8_PACKED || dtype == Q8_BF16, "q8_load_tensor: dtype must be Q8_PACKED or Q8_BF16");
  Q8_CUDA(cudaSetDevice(c->dev));
  const std::string name(cname);
  ShardPlan p;
  Q8_TRY(shard_plan(c->cfg, c->tp_rank, c->tp_size, name, p));
  if (p.slot.empty()) return Q8_OK;  // not used by the Q8 path (or a tied lm_head)
  c->dr_packed = false;  // the ring-layout copy is remade before the next ring step
  const int64_t gotm = (cols == 0) ? 1 : cols;
  if (rows != p.n || gotm != p.m) {
    set_error("tensor %s: expected logical shape [%lld, %lld], got [%lld, %lld]", cname, (long long)p.n,
              (long long)p.m, (long long)rows, (long long)gotm);
    return Q8_ERR_FORMAT;
  }
  const uint8_t* src = (const uint8_t*)data;
  // device data may come from another stream of the caller (e.g. a framework's
  // default stream): the library stream does not order against it, so wait
  // for the whole device before reading
  if (on_dev) Q8_CUDA(cudaDeviceSynchronize());
  c->ready = false;
  int s = Q8_OK;
  if (p.m == 1) {  // 1-D norm weights stay bf16 (quantize.py:55-57)
    if (dtype != Q8_BF16) {
      set_error("tensor %s: 1-D weights must be bf16", cname);
      return Q8_ERR_FORMAT;
    }
    uint16_t* dst = nullptr;
    const int dot = (int)name.find('.', 13);
    const int L = name.rfind("model.layers.", 0) == 0 ? atoi(name.substr(13, dot - 13).c_str()) : -1;
    if (p.slot == "final_norm") dst = c->final_norm;
    else if (p.slot == "in_norm") dst = c->layers[L].in_norm;
    else if (p.slot == "post_norm") dst = c->layers[L].post_norm;
    else if (p.slot == "q_norm") dst = c->layers[L].q_norm;
    else if (p.slot == "k_norm") dst = c->layers[L].k_norm;
    Q8_CUDA(cudaMemcpyAsync(dst, src, (size_t)p.n * 2, on_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                            c->st));
    Q8_CUDA(cudaStreamSynchronize(c->st));
  } else {
    uint8_t* base = nullptr;
    if (p.slot == "embed") base = c->embed;
    else if (p.slot == "lm_head") base = c->lm_head;
    else {
      const int dot = (int)name.find('.', 13);
      const LayerW& w = c->layers[atoi(name.substr(13, dot - 13).c_str())];
      if (p.slot == "qkv") base = w.qkv;
      else if (p.slot == "o") base = w.o;
      else if (p.slot == "gu") base = w.gu;
      else if (p.slot == "down") base = w.down;
    }
    if (c->bf16) {  // bf16 rows stored as given (the slice of this rank)
      if (dtype != Q8_BF16) {
        set_error("tensor %s: a bf16-weight model (weight_dtype Q8_BF16) loads bf16 matrices, not packed Q8", cname);
        return Q8_ERR_FORMAT;
      }
      uint8_t* dst = base + p.dst_row * p.kl * 2;
      Q8_CUDA(cudaMemcpy2DAsync(dst, p.kl * 2, src + (p.row0 * p.m + p.k0) * 2, p.m * 2, p.kl * 2, p.nrows,
                                on_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, c->st));
      Q8_CUDA(cudaStreamSynchronize(c->st));
    } else {
      uint8_t* dst = base + p.dst_row * q8_row_bytes(p.kl);
      s = put_packed(c, dst, src, p.m, p.row0, p.nrows, p.k0, p.kl, dtype, on_dev);
    }
  }
  if (s == Q8_OK) c->loaded.insert(name);
  return s;
}

int q8_shard_plan(const q8_config* cfg, int tp_rank, int tp_size, const char* name, int64_t* n_expect,
                  int64_t* m_expect, int64_t* row0, int64_t* nrows, int64_t* k0, int64_t* kl, int64_t* dst_row,
                  char* slot, int slot_cap) {
  Q8_CHECK_ARG(cfg && name && tp_size >= 1 && tp_rank >= 0 && tp_rank < tp_size, "q8_shard_plan: bad argument");
  ShardPlan p;
  Q8_TRY(shard_plan(*cfg, tp_rank, tp_size, name, p));
  if (n_expect) *n_expect = p.n;
  if (m_expect) *m_expect = p.m;
  if (row0) *row0 = p.row0;
  if (nrows) *nrows = p.nrows;
  if (k0) *k0 = p.k0;
  if (kl) *kl = p.kl;
  if (dst_row) *dst_row = p.dst_row;
  if (slot && slot_cap > 0) {
    strncpy(slot, p.slot.c_str(), (size_t)slot_cap - 1);
    slot[slot_cap - 1] = 0;
  }
  return Q8_OK;
}

int q8_inspect_checkpoint(const char* dir, char* buf, size_t cap, int* n) {
  Q8_CHECK_ARG(dir, "q8_inspect_checkpoint: null dir");
  std::map<std::string, TensorInfo> infos;
  std::string err;
  if (!safetensors_scan(dir, infos, err)) {
    set_error("%s", err.c_str());
    return Q8_ERR_FORMAT;
  }
  std::string out;
  for (auto& kv : infos) {
    const TensorInfo& t = kv.second;
    out += t.name + " " + t.dtype + " ";
    for (size_t i = 0; i < t.shape.size(); ++i) out += (i ? "," : "") + std::to_string(t.shape[i]);
    out += " " + std::to_string(t.begin) + " " + std::to_string(t.end) + "\n";
  }
  if (buf && cap > 0) {
    const size_t k = std::min(cap - 1, out.size());
    memcpy(buf, out.data(), k);
    buf[k] = 0;
  }
  if (n) *n = (int)infos.size();
  return Q8_OK;
}

int q8_load_tensor(q8_ctx* ctx, const char* name, int dtype, int64_t rows, int64_t cols, const void* data,
                   int data_on_device) {
  return fail_ctx(ctx, load_tensor_impl(ctx, name, dtype, rows, cols, data, data_on_device));
}

static int load_st_impl(q8_ctx* c, const char* dir) {
  Q8_CHECK_ARG(c && dir, "q8_load_safetensors: null argument");
  std::map<std::string, TensorInfo> infos;
  std::string err;
  if (!safetensors_scan(dir, infos, err)) {
    set_error("%s", err.c_str());
    return Q8_ERR_FORMAT;
  }
  std::map<std::string, std::pair<void*, size_t>> maps;
  int s = Q8_OK;
  for (const auto& name : c->required) {
    auto it = infos.find(name);
    if (it == infos.end()) {
      set_error("checkpoint %s has no tensor %s", dir, name.c_str());
      s = Q8_ERR_FORMAT;
      break;
    }
    const TensorInfo& ti = it->second;
    if (!maps.count(ti.path)) {
      int fd = open(ti.path.c_str(), O_RDONLY);
      if (fd < 0) {
        set_error("cannot open %s", ti.path.c_str());
        s = Q8_ERR_IO;
        break;
      }
      struct stat stt;
      fstat(fd, &stt);
      void* m = mmap(nullptr, (size_t)stt.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
      close(fd);
      if (m == MAP_FAILED) {
        set_error("mmap failed for %s", ti.path.c_str());
        s = Q8_ERR_IO;
        break;
      }
      maps[ti.path] = {m, (size_t)stt.st_size};
    }
    const uint8_t* base = (const uint8_t*)maps[ti.path].first + ti.begin;
    int dtype;
    int64_t rows, cols;
    if (ti.shape.size() == 1) {
      if (ti.dtype != "BF16") {
        set_error("tensor %s: 1-D dtype %s (want BF16)", name.c_str(), ti.dtype.c_str());
        s = Q8_ERR_FORMAT;
        break;
      }
      dtype = Q8_BF16;
      rows = ti.shape[0];
      cols = 1;
    } else if (ti.shape.size() == 2 && ti.dtype == "F16") {
      // packed Q8 rows stored as F16 [n, m/64 + m/2] (quantize.py:41-43)
      const int64_t u = ti.shape[1];
      if ((u * 64) % 33 != 0) {
        set_error("tensor %s: F16 width %lld is not a packed Q8 row", name.c_str(), (long long)u);
        s = Q8_ERR_FORMAT;
        break;
      }
      dtype = Q8_PACKED;
      rows = ti.shape[0];
      cols = u * 64 / 33;
    } else if (ti.shape.size() == 2 && ti.dtype == "BF16") {
      dtype = Q8_BF16;
      rows = ti.shape[0];
      cols = ti.shape[1];
    } else {
      set_error("tensor %s: unsupported dtype/shape %s", name.c_str(), ti.dtype.c_str());
      s = Q8_ERR_FORMAT;
      break;
    }
    const int64_t expect_bytes = dtype == Q8_PACKED ? rows * q8_row_bytes(cols) : rows * cols * 2;
    if (ti.end - ti.begin != expect_bytes) {
      set_error("tensor %s: byte size %lld does not match its shape", name.c_str(), (long long)(ti.end - ti.begin));
      s = Q8_ERR_FORMAT;
      break;
    }
    s = load_tensor_impl(c, name.c_str(), dtype, rows, cols, base, 0);
    if (s) break;
  }
  for (auto& kv : maps) munmap(kv.second.first, kv.second.second);
  return s;
}

int q8_load_safetensors(q8_ctx* ctx, const char* dir) { return fail_ctx(ctx, load_st_impl(ctx, dir)); }

// ---- forward
static int forward_impl(q8_ctx* c, const int32_t* ids, int s, int seq, float* logits, int32_t* argmax) {
  Q8_CHECK_ARG(c && ids && s > 0, "q8_forward: bad argument");
  Q8_CHECK_ARG(seq >= 0 && seq < c->max_seqs, "q8_forward: seq %d out of range", seq);
  Q8_CUDA(cudaSetDevice(c->dev));
  Q8_TRY(check_ready(c));
  Q8_TRY(ring_prepare(c));
  if (c->n_cached[seq] + s > c->maxlen) {
    set_error("KV cache full: seq %d has %d cached, +%d > maxlen %d", seq, c->n_cached[seq], s, c->maxlen);
    return Q8_ERR_KV_FULL;
  }
  for (int i = 0; i < s; ++i)
    if (ids[i] < 0 || ids[i] >= c->V) {
      set_error("token id %d out of range [0, %d)", ids[i], c->V);
      return Q8_ERR_ARG;
    }
  c->prof.clear();
  c->ev_used = 0;
  int done = 0;
  while (done < s) {
    const int T = std::min(s - done, c->max_tokens);
    const int pos0 = c->n_cached[seq];
    int32_t* pin = c->pin;
    // ids | pos | seq | qb_tok0 | qb_len
    int nqb = 0;
    for (int i = 0; i < T; ++i) {
      pin[i] = ids[done + i];
      pin[T + i] = pos0 + i;
      pin[2 * T + i] = seq;
    }
    for (int i = 0; i < T; i += c->qb_max) {
      pin[3 * T + nqb] = i;
      pin[4 * T + nqb] = std::min(c->qb_max, T - i);
      ++nqb;
    }
    Q8_CUDA(cudaMemcpyAsync(c->ids_d, pin, (size_t)T * 4, cudaMemcpyHostToDevice, c->st));
    Q8_CUDA(cudaMemcpyAsync(c->pos_d, pin + T, (size_t)T * 4, cudaMemcpyHostToDevice, c->st));
    Q8_CUDA(cudaMemcpyAsync(c->seq_d, pin + 2 * T, (size_t)T * 4, cudaMemcpyHostToDevice, c->st));
    Q8_CUDA(cudaMemcpyAsync(c->qb_tok0_d, pin + 3 * T, (size_t)nqb * 4, cudaMemcpyHostToDevice, c->st));
    Q8_CUDA(cudaMemcpyAsync(c->qb_len_d, pin + 4 * T, (size_t)nqb * 4, cudaMemcpyHostToDevice, c->st));
    const int kv_end = pos0 + T;
    const int items = nqb * c->nkv;
    int nsplit = std::max(1, std::min(ceil_div(2 * num_sms(), items), ceil_div(kv_end, 128)));
    nsplit = std::max(1, std::min(nsplit, 1024 / std::max(1, items)));
    if ((size_t)items * nsplit * (64 * c->hd + 128) > c->part_floats) nsplit = 1;
    const bool last = done + T == s;
    std::vector<int> lens;
    for (int i = 0; i < T; ++i) lens.push_back(pos0 + i + 1);
    if (T == 1) nsplit = decode_nsplit(c, 1);
    Q8_TRY(run_tokens(c, T, T > 1, nqb, c->qb_max, nsplit, T - 1, last ? 1 : 0, kv_read_bytes(c, lens)));
    // the pinned staging is rewritten next chunk: wait for the copies
    Q8_CUDA(cudaStreamSynchronize(c->st));
    c->n_cached[seq] += T;
    done += T;
  }
  if (logits) Q8_TRY(gather_logits(c, 1, logits));
  if (argmax) Q8_CUDA(cudaMemcpyAsync(argmax, c->argmax_d, 4, cudaMemcpyDeviceToHost, c->st));
  Q8_TRY(status_copy(c));
  Q8_CUDA(cudaStreamSynchronize(c->st));
  Q8_TRY(status_check(c));
  return Q8_OK;
}

int q8_forward(q8_ctx* ctx, const int32_t* ids, int s, int seq, float* logits, int32_t* argmax) {
  return fail_ctx(ctx, forward_impl(ctx, ids, s, seq, logits, argmax));
}

static int forward_hidden_impl(q8_ctx* c, const int32_t* ids, int s, int seq, int layer, float* out) {
  Q8_CHECK_ARG(c && ids && out && s > 0 && s <= c->max_tokens, "q8_forward_hidden: bad argument (s <= max_tokens)");
  Q8_CHECK_ARG(seq >= 0 && seq < c->max_seqs && layer >= 0 && layer < c->cfg.layers, "q8_forward_hidden: bad seq/layer");
  Q8_CUDA(cudaSetDevice(c->dev));
  Q8_TRY(check_ready(c));
  Q8_TRY(ring_prepare(c));
  if (c->n_cached[seq] + s > c->maxlen) {
    set_error("KV cache full");
    return Q8_ERR_KV_FULL;
  }
  const int T = s, pos0 = c->n_cached[seq];
  int32_t* pin = c->pin;
  int nqb = 0;
  for (int i = 0; i < T; ++i) { pin[i] = ids[i]; pin[T + i] = pos0 + i; pin[2 * T + i] = seq; }
  for (int i = 0; i < T; i += c->qb_max) { pin[3 * T + nqb] = i; pin[4 * T + nqb] = std::min(c->qb_max, T - i); ++nqb; }
  Q8_CUDA(cudaMemcpyAsync(c->ids_d, pin, (size_t)T * 4, cudaMemcpyHostToDevice, c->st));
  Q8_CUDA(cudaMemcpyAsync(c->pos_d, pin + T, (size_t)T * 4, cudaMemcpyHostToDevice, c->st));
  Q8_CUDA(cudaMemcpyAsync(c->seq_d, pin + 2 * T, (size_t)T * 4, cudaMemcpyHostToDevice, c->st));
  Q8_CUDA(cudaMemcpyAsync(c->qb_tok0_d, pin + 3 * T, (size_t)nqb * 4, cudaMemcpyHostToDevice, c->st));
  Q8_CUDA(cudaMemcpyAsync(c->qb_len_d, pin + 4 * T, (size_t)nqb * 4, cudaMemcpyHostToDevice, c->st));
  const int saved = c->cfg.layers;
  c->cfg.layers = layer + 1;  // run layers [0, layer]
  c->prof.clear();
  c->ev_used = 0;
  int items = nqb * c->nkv;
  int nsplit = std::max(1, std::min(ceil_div(2 * num_sms(), items), ceil_div(pos0 + T, 128)));
  nsplit = std::max(1, std::min(nsplit, 1024 / std::max(1, items)));
  int st = run_tokens(c, T, true, nqb, c->qb_max, nsplit, 0, 0, 0.0);
  c->cfg.layers = saved;
  Q8_TRY(st);
  if (c->tp_size > 1) {  // fold the last row-parallel partial into the residual
    Q8_TRY(rmsnorm_launch(c->h, c->ypart, c->final_norm, T, c->H, c->cfg.eps, nullptr, nullptr, nullptr, c->st));
  }
  Q8_CUDA(cudaMemcpyAsync(out, c->h, (size_t)T * c->H * 4, cudaMemcpyDeviceToHost, c->st));
  Q8_TRY(status_copy(c));
  Q8_CUDA(cudaStreamSynchronize(c->st));
  Q8_TRY(status_check(c));
  return Q8_OK;
}

int q8_forward_hidden(q8_ctx* ctx, const int32_t* ids, int s, int seq, int layer, float* out) {
  return fail_ctx(ctx, forward_hidden_impl(ctx, ids, s, seq, layer, out));
}

// Records the decode step for B sequences (one token each) on the stream.
static int decode_body(q8_ctx* c, int B, bool gen_epilogue, double kvb) {
  if (ring_ok(c, B, false, 0, B)) {  // one launch, argmax fed back inside it
    PROF(c, "decode_step", c->dr_wbytes + kvb, ring_step(c, gen_epilogue));
    return Q8_OK;
  }
  Q8_TRY(run_tokens(c, B, false, B, 1, decode_nsplit(c, B), 0, B, kvb));
  if (gen_epilogue) {
    k_step_end<<<1, std::max(32, ((B + 31) / 32) * 32), 0, c->st>>>(c->argmax_d, c->ids_d, c->pos_d, c->hist_d,
                                                                    c->ctr_d, B, c->hist_cap);
    Q8_TRY(launch_check("k_step_end"));
  }
  return Q8_OK;
}

static int get_graph(q8_ctx* c, int B, bool gen, cudaGraphExec_t* out) {
  auto& m = gen ? c->g_gen : c->g_decode;
  auto it = m.find(B);
  if (it != m.end()) {
    *out = it->second;
    return Q8_OK;
  }
  cudaGraph_t g;
  Q8_CUDA(cudaStreamBeginCapture(c->st, cudaStreamCaptureModeThreadLocal));
  int s = decode_body(c, B, gen, 0.0);
  cudaError_t e = cudaStreamEndCapture(c->st, &g);
  if (s != Q8_OK) {
    if (e == cudaSuccess) cudaGraphDestroy(g);
    return s;
  }
  if (e != cudaSuccess) {
    set_error("graph capture failed: %s", cudaGetErrorString(e));
    return Q8_ERR_CUDA;
  }
  cudaGraphExec_t ge;
  e = cudaGraphInstantiate(&ge, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    set_error("graph instantiate failed: %s", cudaGetErrorString(e));
    return Q8_ERR_CUDA;
  }
  m[B] = ge;
  *out = ge;
  return Q8_OK;
}

static int stage_decode(q8_ctx* c, const int32_t* ids, const int32_t* seqs, int B, std::vector<int>& lens) {
  Q8_CHECK_ARG(B >= 1 && B <= c->max_seqs && B <= c->max_tokens, "decode: B=%d exceeds capacity", B);
  std::vector<char> seen(c->max_seqs, 0);
  for (int b = 0; b < B; ++b) {
    const int sq = seqs[b];
    Q8_CHECK_ARG(sq >= 0 && sq < c->max_seqs, "decode: seq %d out of range", sq);
    Q8_CHECK_ARG(!seen[sq], "decode: seq %d appears twice", sq);
    seen[sq] = 1;
    Q8_CHECK_ARG(ids[b] >= 0 && ids[b] < c->V, "decode: token id %d out of range", ids[b]);
    if (c->n_cached[sq] + 1 > c->maxlen) {
      set_error("KV cache full: seq %d has %d cached (maxlen %d)", sq, c->n_cached[sq], c->maxlen);
      return Q8_ERR_KV_FULL;
    }
  }
  int32_t* pin = c->pin;
  lens.clear();
  for (int b = 0; b < B; ++b) {
    pin[b] = ids[b];
    pin[B + b] = c->n_cached[seqs[b]];
    pin[2 * B + b] = seqs[b];
    lens.push_back(c->n_cached[seqs[b]] + 1);
  }
  Q8_CUDA(cudaMemcpyAsync(c->ids_d, pin, (size_t)B * 4, cudaMemcpyHostToDevice, c->st));
  Q8_CUDA(cudaMemcpyAsync(c->pos_d, pin + B, (size_t)B * 4, cudaMemcpyHostToDevice, c->st));
  Q8_CUDA(cudaMemcpyAsync(c->seq_d, pin + 2 * B, (size_t)B * 4, cudaMemcpyHostToDevice, c->st));
  return Q8_OK;
}

static int decode_impl(q8_ctx* c, const int32_t* ids, const int32_t* seqs, int B, float* logits, int32_t* argmax) {
  Q8_CHECK_ARG(c && ids && seqs, "q8_decode: null argument");
  Q8_CUDA(cudaSetDevice(c->dev));
  Q8_TRY(check_ready(c));
  Q8_TRY(ring_prepare(c));
  std::vector<int> lens;
  Q8_TRY(stage_decode(c, ids, seqs, B, lens));
  c->prof.clear();
  c->ev_used = 0;
  if (c->profiling) {
    Q8_TRY(decode_body(c, B, false, kv_read_bytes(c, lens)));
  } else {
    cudaGraphExec_t ge;
    Q8_TRY(get_graph(c, B, false, &ge));
    Q8_CUDA(cudaGraphLaunch(ge, c->st));
  }
  if (logits) Q8_TRY(gather_logits(c, B, logits));
  if (argmax) Q8_CUDA(cudaMemcpyAsync(argmax, c->argmax_d, (size_t)B * 4, cudaMemcpyDeviceToHost, c->st));
  Q8_TRY(status_copy(c));
  Q8_CUDA(cudaStreamSynchronize(c->st));
  Q8_TRY(status_check(c));
  for (int b = 0; b < B; ++b) c->n_cached[seqs[b]] += 1;
  return Q8_OK;
}

int q8_decode(q8_ctx* ctx, const int32_t* ids, const int32_t* seqs, int B, float* logits, int32_t* argmax) {
  return fail_ctx(ctx, decode_impl(ctx, ids, seqs, B, logits, argmax));
}

static int generate_impl(q8_ctx* c, const int32_t* first, const int32_t* seqs, int B, int steps, int32_t* out) {
  Q8_CHECK_ARG(c && first && seqs && steps >= 0, "q8_generate: bad argument");
  Q8_CHECK_ARG(steps <= c->hist_cap, "q8_generate: steps %d > %d per call", steps, c->hist_cap);
  Q8_CUDA(cudaSetDevice(c->dev));
  Q8_TRY(check_ready(c));
  Q8_TRY(ring_prepare(c));
  if (steps == 0) return Q8_OK;
  for (int b = 0; b < B; ++b) {
    Q8_CHECK_ARG(seqs[b] >= 0 && seqs[b] < c->max_seqs, "q8_generate: bad seq");
    if (c->n_cached[seqs[b]] + steps > c->maxlen) {
      set_error("KV cache full: seq %d has %d cached, +%d steps > maxlen %d", seqs[b], c->n_cached[seqs[b]], steps,
                c->maxlen);
      return Q8_ERR_KV_FULL;
    }
  }
  std::vector<int> lens;
  Q8_TRY(stage_decode(c, first, seqs, B, lens));
  Q8_CUDA(cudaMemsetAsync(c->ctr_d, 0, 4, c->st));
  cudaGraphExec_t ge;
  Q8_TRY(get_graph(c, B, true, &ge));
  for (int i = 0; i < steps; ++i) Q8_CUDA(cudaGraphLaunch(ge, c->st));
  if (out) Q8_CUDA(cudaMemcpyAsync(out, c->hist_d, (size_t)steps * B * 4, cudaMemcpyDeviceToHost, c->st));
  Q8_TRY(status_copy(c));
  Q8_CUDA(cudaStreamSynchronize(c->st));
  Q8_TRY(status_check(c));
  for (int b = 0; b < B; ++b) c->n_cached[seqs[b]] += steps;
  return Q8_OK;
}

int q8_generate(q8_ctx* ctx, const int32_t* first_ids, const int32_t* seqs, int B, int steps, int32_t* out_tokens) {
  return fail_ctx(ctx, generate_impl(ctx, first_ids, seqs, B, steps, out_tokens));
}

int q8_reset(q8_ctx* ctx, int seq) {
  Q8_CHECK_ARG(ctx && seq >= 0 && seq < ctx->max_seqs, "q8_reset: bad seq");
  ctx->n_cached[seq] = 0;
  return Q8_OK;
}

int q8_n_cached(const q8_ctx* ctx, int seq, int* out) {
  Q8_CHECK_ARG(ctx && out && seq >= 0 && seq < ctx->max_seqs, "q8_n_cached: bad argument");
  *out = ctx->n_cached[seq];
  return Q8_OK;
}

int q8_set_n_cached(q8_ctx* ctx, int seq, int n) {
  Q8_CHECK_ARG(ctx && seq >= 0 && seq < ctx->max_seqs, "q8_set_n_cached: bad seq");
  Q8_CHECK_ARG(n >= 0 && n <= ctx->n_cached[seq], "q8_set_n_cached: can only shrink (have %d, asked %d)",
               ctx->n_cached[seq], n);
  ctx->n_cached[seq] = n;
  return Q8_OK;
}

int q8_debug_set_device_status(int unit, int value) {
  Q8_CHECK_ARG(unit == 0 || unit == 1, "q8_debug_set_device_status: unit must be 0 or 1");
  int* w = nullptr;
  Q8_TRY(unit == 0 ? gemm_tc_error_word(&w) : attn_dec_error_word(&w));
  Q8_CUDA(cudaDeviceSynchronize());
  Q8_CUDA(cudaMemcpy(w, &value, 4, cudaMemcpyHostToDevice));
  return Q8_OK;
}

int q8_stream(const q8_ctx* ctx, void** stream) {
  Q8_CHECK_ARG(ctx && stream, "q8_stream: null");
  *stream = (void*)ctx->st;
  return Q8_OK;
}

static int set_sampling_impl(q8_ctx* c, float temp, float top_p, unsigned long long seed) {
  Q8_CHECK_ARG(c, "q8_set_sampling: null");
  Q8_CHECK_ARG(!std::isnan(temp) && (!(temp > 0.f) || top_p > 0.f),
               "q8_set_sampling: temp must not be NaN, top_p must be > 0");
  Q8_CHECK_ARG((int64_t)c->V_loc * c->tp_size == c->V, "q8_set_sampling: vocabulary shards must tile the vocabulary");
  Q8_CUDA(cudaSetDevice(c->dev));
  Q8_CUDA(cudaStreamSynchronize(c->st));
  // the captured decode steps hold the previous mode and parameters
  for (auto& kv : c->g_decode) cudaGraphExecDestroy(kv.second);
  for (auto& kv : c->g_gen) cudaGraphExecDestroy(kv.second);
  c->g_decode.clear();
  c->g_gen.clear();
  if (temp > 0.f && !c->samp_ws) {
    const int rows = std::max(c->max_seqs, 1);
    const size_t bytes = sample_scratch_bytes(rows, c->V);
    Q8_CHECK_ARG(bytes > 0, "q8_set_sampling: scratch size query failed");
    Q8_TRY(dmalloc(&c->samp_ws, bytes));
    c->samp_ws_bytes = bytes;
    Q8_TRY(dmalloc((void**)&c->samp_u, (size_t)rows * 4));
    if (c->tp_size > 1) Q8_TRY(dmalloc((void**)&c->samp_logits, (size_t)rows * c->V * 4));
  }
  c->samp_temp = temp > 0.f ? temp : 0.f;
  c->samp_top_p = top_p;
  c->samp_seed = seed;
  return Q8_OK;
}

int q8_set_sampling(q8_ctx* ctx, float temp, float top_p, unsigned long long seed) {
  return fail_ctx(ctx, set_sampling_impl(ctx, temp, top_p, seed));
}

int q8_set_profiling(q8_ctx* ctx, int on) {
  Q8_CHECK_ARG(ctx, "q8_set_profiling: null");
  ctx->profiling = on != 0;
  return Q8_OK;
}

int q8_profile(const q8_ctx* ctx, int cap, const char** names, double* ms, double* bytes, int* launches, int* n) {
  Q8_CHECK_ARG(ctx && n, "q8_profile: null");
  std::vector<std::string> order;
  std::map<std::string, double> tms, tb;
  std::map<std::string, int> cnt;
  for (const auto& e : ctx->prof) {
    float t = 0.f;
    if (cudaEventElapsedTime(&t, e.a, e.b) != cudaSuccess) {
      cudaGetLastError();
      set_error("q8_profile: events not complete");
      return Q8_ERR_STATE;
    }
    if (!tms.count(e.name)) order.push_back(e.name);
    tms[e.name] += t;
    tb[e.name] += e.bytes;
    cnt[e.name] += 1;
  }
  // phases of the last profiled ring step as CTA 0 saw them, summed over the
  // layers: wait (for the previous phase of the whole grid), stage (the
  // activation vector; the whole attention for attention phases), stream
  // (the CTA's ring stages), epi (epilogue stores and arrival)
  if (ctx->dr_traced && ctx->dr_trace) {
    const int L = ctx->cfg.layers, nph = 5 * L + 1;
    std::vector<unsigned long long> t((size_t)4 * nph);
    if (cudaMemcpy(t.data(), ctx->dr_trace, t.size() * 8, cudaMemcpyDeviceToHost) == cudaSuccess) {
      const char* kn[6] = {"qkv", "attn", "o", "gateup", "down", "lmhead"};
      const char* pn[4] = {"wait", "stage", "stream", "epi"};
      double acc[6][4] = {};
      for (int ph = 0; ph < nph; ++ph) {
        const int k = ph == 5 * L ? 5 : ph % 5;
        const unsigned long long* m = t.data() + 4 * ph;
        if (ph > 0) acc[k][0] += (double)(m[0] - t[4 * (ph - 1) + 3]) * 1e-6;
        for (int j = 1; j < 4; ++j) acc[k][j] += (double)(m[j] - m[j - 1]) * 1e-6;
      }
      for (int k = 0; k < 6; ++k)
        for (int j = 0; j < 4; ++j) {
          const std::string nm = std::string("phase:") + kn[k] + "." + pn[j];
          order.push_back(nm);
          tms[nm] = acc[k][j];
          tb[nm] = 0;
          cnt[nm] = 0;
        }
    } else {
      cudaGetLastError();
    }
  }
  int k = 0;
  static thread_local std::vector<std::string> keep;
  keep = order;
  for (const auto& nm : keep) {
    if (k >= cap) break;
    if (names) names[k] = nm.c_str();
    if (ms) ms[k] = tms[nm];
    if (bytes) bytes[k] = tb[nm];
    if (launches) launches[k] = cnt[nm];
    ++k;
  }
  *n = k;
  return Q8_OK;
}

}  // extern "C"
