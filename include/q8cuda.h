/*
 * libq8cuda — C ABI of the B200 (sm_100a) INT8 group-quantized (W8A32, group 64)
 * transformer decode/prefill path.
 *
 * Drop-in boundary for plutonium-guy/lama32_mojo's Q8 path.  Each entry point
 * names the reference interface it replaces (paths relative to that repo).
 * The reference is Mojo-internal (no FFI); its host code would bind these
 * symbols through `DLHandle` / `external_call`.
 *
 * Conventions
 *   - Every function returns an int status (Q8_OK = 0).  On error the message
 *     is available from q8_last_error(ctx) (ctx may be NULL for op-level calls;
 *     the message is then per host thread).  No C++ exception crosses the ABI.
 *   - Op-level functions (q8op_*) take DEVICE pointers and a cudaStream_t passed
 *     as `void*` (NULL = legacy default stream); they allocate nothing except
 *     where documented (scratch for split reductions is taken from a caller
 *     buffer or from a per-device cache).
 *   - Model-level functions (q8_*) own all device memory of a context; host
 *     buffers passed to them belong to the caller.  A context is bound to one
 *     GPU and is not thread-safe.
 *   - Per-device scratch (the decode GEMV's split-tile partials and tickets,
 *     the tensor-core GEMM's split-K workspace and tickets, the op scratch) is
 *     shared by every context and op-level call on a device.  Calls whose
 *     kernels could overlap on the GPU (two contexts on one device driven from
 *     different threads, op-level calls on several streams) must be
 *     serialized by the caller.  Scratch that grows is never freed while the
 *     process runs, so captured decode graphs keep valid pointers.
 *   - Packed Q8 weight rows keep the reference layout
 *     (qwen3_mojo/scripts/quantize.py:31-43, src/llama_q8.mojo:26-42):
 *     row of K inputs = [K/64 f16 scales | K int8 codes] = K/64 + K/2 uint16.
 */
#ifndef Q8CUDA_H_
#define Q8CUDA_H_

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
enum {
  Q8_OK = 0,
  Q8_ERR_ARG = 1,       /* bad argument / shape (reference: assert in pack_q8, quantize.py:33) */
  Q8_ERR_CUDA = 2,      /* CUDA runtime error */
  Q8_ERR_OOM = 3,       /* device allocation failed (reference: "acts arena overflow", llama_common.mojo:599) */
  Q8_ERR_KV_FULL = 4,   /* sequence would exceed maxlen (reference: "KV cache full", qwen_q8.mojo:128-129) */
  Q8_ERR_IO = 5,        /* file read failed (reference: resident.mojo:42-54) */
  Q8_ERR_FORMAT = 6,    /* malformed safetensors / missing or mis-shaped tensor */
  Q8_ERR_COMM = 7,      /* NCCL / peer communication failure */
  Q8_ERR_TIMEOUT = 8,   /* a bounded device-side wait expired */
  Q8_ERR_STATE = 9      /* call not valid in the current state (e.g. weights not loaded) */
};

/* activation / tensor dtypes */
enum { Q8_F32 = 0, Q8_BF16 = 1, Q8_F16 = 2, Q8_PACKED = 3 };

/* RoPE frequency schedule */
enum { Q8_ROPE_DEFAULT = 0, /* rope_inv_freq, src/llama_common.mojo:609-615 */
       Q8_ROPE_LLAMA3 = 1   /* llama3_inv_freq, src/llama_common.mojo:618-633 */ };

/* Model dimensions.  Mirrors `Config` (src/llama_common.mojo:26-52) plus the
 * model-family switches the reference encodes in its shells:
 * qk_norm  <- LayerOffs.q_norm >= 0 (src/llama_common.mojo:67, src/llama_q8.mojo:171)
 * tied     <- lm_head = embed_tokens (qwen3_mojo/src/qwen_q8.mojo:143-145) vs
 *             untied lm_head.weight (llama31_mojo/src/llama_gpu.mojo:150)        */
typedef struct q8_config {
  int32_t hidden, layers, n_heads, n_kv, head_dim, inter, vocab;
  float eps;
  double theta, rope_factor, low_ff, high_ff, orig_ctx;
  int32_t rope_type;
  int32_t qk_norm;
  int32_t tied;
  /* Q8_BF16: keep the linear weights as bf16 (the reference's non-Q8 path,
   * run_layer, src/llama_common.mojo:697-780); anything else (0 or
   * Q8_PACKED): Q8 group-64 weights. */
  int32_t weight_dtype;
} q8_config;

typedef struct q8_ctx q8_ctx;

/* Last error message of `ctx` (or of this host thread when ctx is NULL). */
const char* q8_last_error(const q8_ctx* ctx);
const char* q8_status_string(int status);
/* Library build string (arch, version). */
const char* q8_version(void);
/* Synchronizes the current device, then reports and clears a timeout that a
   bounded barrier wait inside a tensor-core GEMM or the decode attention
   recorded (Q8_ERR_TIMEOUT), else Q8_OK.  The model entry points (q8_forward,
   q8_forward_hidden, q8_decode, q8_generate) read both words after every call,
   with the call's other results, and fail with Q8_ERR_TIMEOUT when one is set;
   op-level callers poll this when they synchronize.  No counterpart in the
   reference (its kernels have no device-side waits). */
int q8_device_status(void);
/* Test aid (no counterpart in the reference): writes `value` into the device
   error word of one kernel family on the current device, as a bounded wait
   that gave up would (unit 0: tensor-core GEMM, unit 1: decode attention).
   The next model call then reports Q8_ERR_TIMEOUT and clears the word; the
   kernels themselves run unchanged unless a wait actually exceeds 2^20
   cycles.  Synchronizes the device. */
int q8_debug_set_device_status(int unit, int value);

/* =================================================================== op level */

/* GPU quantizer/packer, bit-exact with pack_q8 (qwen3_mojo/scripts/quantize.py:31-43):
 * w_bf16 [n, m] row-major bf16 -> packed [n, m/64 + m/2] uint16.  m % 64 == 0. */
int q8op_pack(const void* w_bf16, int64_t n, int64_t m, void* packed, void* stream);

/* Inverse of the packing for checks: packed -> f32 dequantized weights
 * w = int8 * f16 scale (src/llama_q8.mojo:9). */
int q8op_dequant(const void* packed, int64_t n, int64_t m, float* w, void* stream);

/* y[M, N] = x[M, K] . W[N, K]^T with W packed Q8 — replaces k_mm_q8 / mm_q8_op
 * (src/llama_q8.mojo:54-93, :124-141).  x_dtype in {Q8_F32, Q8_BF16, Q8_F16};
 * ldx / ldy in elements.  Needs K % 64 == 0 and 2-byte aligned packed rows. */
int q8op_gemm(const void* x, int x_dtype, int64_t ldx, int64_t M, int64_t K,
              const void* packed_w, int64_t N, float* y, int64_t ldy, void* stream);

/* Allocation-free variant of q8op_gemm (no counterpart in the reference).
 * Some callers cannot call cudaMalloc: a host that owns a fixed device-memory
 * budget handed out by its own pool (a Mojo DeviceContext arena, an inference
 * server that reserves all memory at start-up), or code on a path where an
 * allocation's implicit device synchronization or failure is not acceptable.
 * This entry point stages x in a file-scope __device__ array of
 * Q8_NOALLOC_MAX_ELEMS split-f16 elements (8 MiB, held by every GPU that loads
 * the library until the process exits) instead of a cudaMalloc'd buffer.
 * It rejects M*K > Q8_NOALLOC_MAX_ELEMS with Q8_ERR_ARG.  The array's device
 * address is looked up on the first call on each device (that call should come
 * before any stream capture on the device).  Every call shares the array:
 * calls whose executions overlap on the GPU (other streams, other threads)
 * race; serialize them.  Caller still owns x and y. */
#define Q8_NOALLOC_MAX_ELEMS (2 * 1024 * 1024)
int q8op_gemm_noalloc(const void* x, int x_dtype, int64_t ldx, int64_t M, int64_t K,
                      const void* packed_w, int64_t N, float* y, int64_t ldy, void* stream);

/* bf16-weight product y[M, N] = x[M, K] . W[N, K]^T, x f32 rows, W plain bf16
 * rows (no quantization), f32 accumulation — the reference's non-Q8 matmul
 * k_mm_w / k_mm_tile behind mm_op (src/llama_common.mojo:89-162, :636-684).
 * K % 8 == 0; x, W 16-byte aligned, ldx % 4 == 0. */
int q8op_gemm_bf16(const float* x, int64_t ldx, int64_t M, int64_t K, const void* w_bf16, int64_t N,
                   float* y, int64_t ldy, void* stream);

/* Fused gate|up GEMV + SwiGLU: act[M, F] = silu(x.Wg^T) * (x.Wu^T) where
 * packed_gu holds the F gate rows followed by the F up rows — replaces the
 * s==1 fused gate|up mm_q8_op + k_swiglu_mul (src/llama_q8.mojo:215-224,
 * src/llama_common.mojo:476-481). */
int q8op_gemm_swiglu(const void* x, int x_dtype, int64_t ldx, int64_t M, int64_t K,
                     const void* packed_gu, int64_t F, float* act, int64_t ld_act,
                     void* stream);

/* Q8 embedding gather y[s, d] = f32(int8) * f16 scale — k_embed_gather_q8
 * (src/llama_q8.mojo:96-109). */
int q8op_embed(const void* packed_emb, int64_t vocab, int64_t d, const int32_t* ids,
               int64_t s, float* y, void* stream);

/* RMSNorm with bf16 weight — k_rmsnorm_w / rmsnorm_op (src/llama_common.mojo:197-225,
 * :687-694).  If `resid` is non-NULL, first x += resid in place (k_res_add_rmsnorm,
 * :361-393).  x may alias y only when resid is NULL. */
int q8op_rmsnorm(float* x, const float* resid, const uint16_t* w_bf16, int64_t rows,
                 int64_t d, float eps, float* y, void* stream);

/* Per-head Q/K RMSNorm (Qwen3) — k_rmsnorm2_w (src/llama_common.mojo:228-270). */
int q8op_rmsnorm_heads(const float* x, const uint16_t* w_bf16, int64_t rows, int64_t hd,
                       float eps, float* y, void* stream);

/* RoPE inverse frequencies (f64 math -> f32): rope_inv_freq / llama3_inv_freq
 * (src/llama_common.mojo:609-633).  Host function; out has head_dim/2 floats. */
int q8_rope_inv_freq(const q8_config* cfg, float* out);

/* Fused (QK-norm +) RoPE + paged KV append — k_rope_qk_copy2
 * (src/llama_common.mojo:299-342) with the page table of a paged cache.
 * qkv [T, ldqkv] f32 holds q | k | v per token; q (and k) are rotated in place.
 * k_pages / v_pages: [num_pages, n_kv, page, hd] f32.  pos[T], seq[T] int32;
 * block_table [n_seq, max_pages] int32.  q_norm / k_norm may be NULL. */
int q8op_rope_kv_append(float* qkv, int64_t ldqkv, int64_t T, const int32_t* pos,
                        const int32_t* seq, int n_heads, int n_kv, int hd,
                        const float* inv_freq, const uint16_t* q_norm,
                        const uint16_t* k_norm, float eps, float* k_pages,
                        float* v_pages, int page, const int32_t* block_table,
                        int max_pages, void* stream);

/* Causal GQA attention over the paged cache — k_scores + k_softmax_rows +
 * k_att_out (src/llama_common.mojo:402-473), flash-style (no materialized
 * scores).  q [T, ldq] f32 (roped), token t of sequence seq[t] at position
 * pos[t] attends to cache positions 0..pos[t].  out [T, ldo] f32.
 * Uses a per-device scratch buffer for split-context partials. */
int q8op_attention(const float* q, int64_t ldq, int64_t T, const int32_t* pos,
                   const int32_t* seq, int n_heads, int n_kv, int hd,
                   const float* k_pages, const float* v_pages, int page,
                   const int32_t* block_table, int max_pages, float* out, int64_t ldo,
                   void* stream);

/* Greedy argmax per row (lowest index on ties) — k_argmax / argmax_op
 * (src/llama_common.mojo:493-519, :783-789). */
int q8op_argmax(const float* logits, int64_t rows, int64_t n, int64_t ld, int32_t* out,
                void* stream);

/* Temperature + nucleus (top-p) sampling per row — sample()
 * (src/sample.mojo:15-59) on the device, with the reference's arithmetic
 * order: candidates are the logits >= max - 16, p = exp((l - max) / temp),
 * total summed in index order, the nucleus taken largest p first (equal p in
 * the order of the reference's swap-remove list) while the running sum is
 * below total * top_p, then the first nucleus entry whose running sum reaches
 * u * sum.  logits [rows, ld] f32 with n used columns; u [rows] f32 uniform
 * draws in [0, 1), device memory (the reference draws random_float64(),
 * src/sample.mojo:55); out [rows] int32.  temp <= 0 is greedy (first
 * maximum; u may then be NULL).  top_p must be > 0 when temp > 0.  Uses the
 * per-device op scratch (28 bytes per logit).  exp() is CUDA's expf. */
int q8op_sample(const float* logits, int64_t rows, int64_t n, int64_t ld, float temp, float top_p,
                const float* u, int32_t* out, void* stream);

/* ================================================================ model level */

/* Create a context on `device`.  Mirrors QwenQ8/Llama.__init__ + Acts/Weights
 * (qwen3_mojo/src/qwen_q8.mojo:71-108, src/resident.mojo:15-28,
 * src/llama_common.mojo:578-606).
 *   max_seqs  independent sequences (the reference has one: n_cached)
 *   maxlen    KV capacity per sequence (reference `maxlen`)
 *   max_tokens  largest token batch one forward processes (prefill is chunked)
 *   tp_rank/tp_size  tensor-parallel position (1 = single GPU)
 *   nccl_id   128-byte ncclUniqueId from q8_nccl_unique_id() (NULL if tp_size==1)
 * Collective when tp_size > 1: every rank calls it.  The ranks map each
 * other's exchange buffers (CUDA IPC) and agree on whether one-sequence greedy
 * decode steps run as one launch with the row-parallel sums exchanged inside
 * it (every rank or none).  After a model call returned Q8_ERR_COMM or
 * Q8_ERR_TIMEOUT the ranks' exchange state no longer agrees: destroy and
 * recreate the contexts. */
int q8_create(const q8_config* cfg, int device, int max_seqs, int maxlen, int max_tokens,
              int tp_rank, int tp_size, const void* nccl_id, q8_ctx** out);
int q8_destroy(q8_ctx* ctx);

/* 128-byte NCCL unique id for q8_create on rank 0 (broadcast it to the ranks). */
int q8_nccl_unique_id(void* out128);

/* Weight upload of one named tensor — Weights.upload_all per tensor
 * (src/resident.mojo:30-60).  dtype Q8_PACKED: data is the packed rows [n, m/64+m/2]
 * of a [n, m] weight (quantize.py output); Q8_BF16: bf16 [n, m] (2-D tensors are
 * quantized on the GPU by the packer, 1-D norm weights are stored as bf16).
 * rows/cols are the LOGICAL [n, m] shape.  data_on_device selects host/device
 * source; device data may still be in flight on any of the caller's streams
 * (the call synchronizes the device before reading it).  Tensor-parallel
 * slicing (column/row/vocab parallel) happens here. */
int q8_load_tensor(q8_ctx* ctx, const char* name, int dtype, int64_t rows, int64_t cols,
                   const void* data, int data_on_device);

/* Tensor-parallel placement of one named tensor (pure host function, used by
 * q8_load_tensor).  Column-parallel q/k/v/gate/up rows, row-parallel o/down K
 * slices, vocab-parallel untied lm_head rows, replicated embedding and norms.
 * Source rows [*row0, *row0 + *nrows) and inputs [*k0, *k0 + *kl) of the
 * logical [n, m] tensor land at rows [*dst_row, ...) of destination `slot`
 * ("embed", "lm_head", "final_norm", "qkv", "o", "gu", "down", "in_norm",
 * "post_norm", "q_norm", "k_norm"; "" = not used by the Q8 path).
 * *n_expect/*m_expect give the logical shape the tensor must have. */
int q8_shard_plan(const q8_config* cfg, int tp_rank, int tp_size, const char* name, int64_t* n_expect,
                  int64_t* m_expect, int64_t* row0, int64_t* nrows, int64_t* k0, int64_t* kl,
                  int64_t* dst_row, char* slot, int slot_cap);

/* Host-only checkpoint scan (SafeTensors.__init__, src/safetensors.mojo:40-87):
 * writes one line per tensor "name dtype d0,d1,... begin end\n" into buf
 * (truncated to cap bytes) and the tensor count into *n. */
int q8_inspect_checkpoint(const char* dir, char* buf, size_t cap, int* n);

/* Load every tensor the model needs from a safetensors checkpoint directory
 * (single file or model.safetensors.index.json shards) — SafeTensors + upload_all
 * (src/safetensors.mojo:40-96, src/resident.mojo:30-60).  Accepts the packed Q8
 * files written by quantize.py (F16-typed [n, m/64+m/2]) and plain BF16 files. */
int q8_load_safetensors(q8_ctx* ctx, const char* dir);

/* Prefill/decode `s` tokens of sequence `seq` — _run_forward / forward /
 * forward_argmax (qwen3_mojo/src/qwen_q8.mojo:126-162).  Host buffers;
 * logits (vocab floats, last token) and/or argmax (1 int32) may be NULL. */
int q8_forward(q8_ctx* ctx, const int32_t* ids, int s, int seq, float* logits,
               int32_t* argmax);

/* Residual stream after layer `layer` for the `s` tokens of a prefill at the
 * sequence's current position (the reference oracle's after_layer{L} dumps,
 * scripts/gen_oracle.py:120-123).  Writes KV for layers <= layer but does not
 * advance n_cached.  out: host [s, hidden] f32. */
int q8_forward_hidden(q8_ctx* ctx, const int32_t* ids, int s, int seq, int layer, float* out);

/* One decode token for each of B sequences (batched forward_argmax).  Host
 * buffers: ids[B], seqs[B]; logits [B, vocab] and/or argmax[B] may be NULL. */
int q8_decode(q8_ctx* ctx, const int32_t* ids, const int32_t* seqs, int B, float* logits,
              int32_t* argmax);

/* Greedy generation fully on the device: `steps` decode steps for B sequences,
 * each step feeding back its argmax.  first_ids[B] (host) are the inputs of the
 * first step; out_tokens [steps, B] (host) receives every step's argmax. */
int q8_generate(q8_ctx* ctx, const int32_t* first_ids, const int32_t* seqs, int B, int steps,
                int32_t* out_tokens);

/* Temperature + nucleus sampling of every token the context picks — the chat
 * REPLs' sample(logits, temp, top_p) (src/sample.mojo:15-59) run on the device
 * right after lm_head, so a chat step needs no logits copy to the host.
 * temp > 0: q8_forward's argmax output, q8_decode's argmax[] and every
 * q8_generate step are sampled as q8op_sample does; temp <= 0 (the default)
 * restores the greedy argmax.  The draw of a row is
 *   z = seed + (key + 1) * 0x9E3779B97F4A7C15, key = seq << 32 | pos
 *   z = (z ^ z >> 30) * 0xBF58476D1CE4E5B9; z = (z ^ z >> 27) * 0x94D049BB133111EB;
 *   z ^= z >> 31;  u = (z >> 40) / 2^24
 * (SplitMix64's finalizer; pos is the position of the token fed in that row),
 * so a run is reproducible from the seed.  Synchronizes the context's stream
 * and drops its captured decode graphs; allocates the sampling scratch (about
 * 28 bytes per vocabulary entry per sequence) on first use.  top_p must be > 0
 * when temp > 0.  No counterpart in the reference's GPU path (its sampler runs
 * on the host over the logits). */
int q8_set_sampling(q8_ctx* ctx, float temp, float top_p, unsigned long long seed);

/* KV cache state — n_cached (qwen_q8.mojo:69; chat /reset sets it to 0,
 * src/chat.mojo:133-136).  q8_set_n_cached can only shrink. */
int q8_reset(q8_ctx* ctx, int seq);
int q8_n_cached(const q8_ctx* ctx, int seq, int* out);
int q8_set_n_cached(q8_ctx* ctx, int seq, int n);

/* Stream the context runs on (cudaStream_t as void*). */
int q8_stream(const q8_ctx* ctx, void** stream);

/* Per-kernel-class device time of the last q8_decode/q8_generate step run with
 * profiling on (q8_set_profiling): fills names/ms/bytes arrays of `cap` entries,
 * returns the count in *n. */
int q8_set_profiling(q8_ctx* ctx, int on);
int q8_profile(const q8_ctx* ctx, int cap, const char** names, double* ms, double* bytes,
               int* launches, int* n);

#ifdef __cplusplus
}
#endif

#endif /* Q8CUDA_H_ */
