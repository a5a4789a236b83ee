// Internal launcher declarations shared by the op-level ABI and the model runtime.
#pragma once
#include "q8_common.cuh"

#include <cuda.h>

namespace q8 {

enum { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2 };

int pack_launch(const void* w_bf16, int64_t n, int64_t m, void* packed, cudaStream_t st);
int to_xs_launch(const void* x, int dtype, int64_t ldx, int M, int K, __half* xs, cudaStream_t st);
int gemv_init();
int gemv_rms_launch(int epi, const float* h, int64_t ldh, const uint16_t* nw, float eps, int M, int K,
                    const void* W, int N, float* y, int64_t ldy, __half* ys, cudaStream_t st);
// Activations come as f32 rows (x32, used by the int8-digit kernel) and/or the
// split-f16 XS rows (xs, used by the general kernel); either may be null when
// the other covers the shape.
int gemv_launch(int epi, const float* x32, int64_t ldx32, const __half* xs, int M, int K, const void* W, int N,
                float* y, int64_t ldy, __half* ys, cudaStream_t st);
// Digit GEMV (int8 tensor cores, 1-2 tokens, K % 256 == 0): x f32 rows, or
// x = RMSNorm(h) * nw when rms.  gemv_d_prepare sizes its per-device scratch
// outside stream capture.
bool gemv_d_supported(int M, int K, int N, bool rms, const void* W);
int gemv_d_prepare(int max_tiles);
int gemv_d_launch(int epi, bool rms, const float* x, int64_t ldx, const float* h, int64_t ldh, const uint16_t* nw,
                  float eps, int M, int K, const void* W, int N, float* y, int64_t ldy, __half* ys, cudaStream_t st);
bool gemv_d_enabled();
// Decode-shaped GEMMs (the GEMV kernels above); prefill-sized batches go to
// gemm_tc_launch.
int gemm_dispatch(int epi, const float* x32, int64_t ldx32, const __half* xs, int M, int K, const void* W, int N,
                  float* y, int64_t ldy, __half* ys, cudaStream_t st);
int op_scratch(size_t bytes, void** out);

// Tensor-core GEMM (tcgen05/TMEM) for prefill batches: x16 plain f16 rows
// [M][ld16]; K a multiple of 512.  STORE/ADD write y (f32); SWIGLU (N = F
// pairs, W = 2F rows gate|up) writes y and/or y16 (f16 rows [M][ldy16]).
// x16lo > 0: the activations are split, lo = f16(x - f16(x)) at x16 + x16lo,
// and the GEMM runs on split operands (exact to f32 accumulation); y16lo > 0
// writes the SwiGLU output split the same way.  gemm_tc_exact(): whether
// callers should produce split activations (Q8_TC_FAST=1 turns it off).
bool gemm_tc_supported(int K, const void* W, const __half* x16, int64_t ld16);
bool gemm_tc_exact();
int gemm_tc_launch(int epi, const __half* x16, int64_t ld16, int64_t x16lo, int M, int K, const void* W, int N,
                   float* y, int64_t ldy, __half* y16, int64_t ldy16, int64_t y16lo, cudaStream_t st);
// After a synchronize: Q8_OK, or the timeout a pipeline wait recorded (cleared).
int gemm_tc_poll_error();
// 2-D tensor map (cuTensorMapEncodeTiled) over `rows` rows of `inner`
// elements (dtype 0: u8, 1: u16, 2: f32) `row_bytes` apart.
int tensor_map_2d(CUtensorMap* m, int dtype, const void* base, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                  uint32_t box_inner, uint32_t box_rows, bool swizzle128);
// Device address of the error word of the tensor-core GEMM file (read
// asynchronously by the model calls together with their results).
int gemm_tc_error_word(int** out);
// Kernel attributes and the per-device split-K workspace (outside stream capture).
int gemm_tc_prepare();
// Smallest token batch the model runtime sends to the tensor-core GEMM.
constexpr int kTcMinTokens = 128;
// Token count from which op-level GEMMs and decode steps take the tensor-core GEMM.
constexpr int kTcDecodeMinTokens = 16;
// token count from which op-level GEMMs use the tensor-core GEMM (Q8_TC_MIN, default kTcDecodeMinTokens)
int tc_min_tokens();
// x (Q8_F32 / Q8_BF16 / Q8_F16 rows) -> plain f16 rows [M][K].
int to_f16_launch(const void* x, int dtype, int64_t ldx, int M, int K, __half* y, cudaStream_t st,
                  int64_t ylo = 0);

// bf16-weight products (q8_bf16.cu): y = x . W^T with f32 x rows, epilogue
// STORE / ADD / SWIGLU (W = gate rows then up rows); bf16 embedding gather.
int gemm_bf16_launch(int epi, const float* x, int64_t ldx, int M, int K, const uint16_t* W, int N, float* y,
                     int64_t ldy, cudaStream_t st);
int embed_bf16_launch(const uint16_t* E, int64_t d, const int32_t* ids, int64_t s, float* y, cudaStream_t st);

int embed_launch(const void* packed_emb, int64_t d, const int32_t* ids, int64_t s, float* y,
                 cudaStream_t st);
// y32 / yxs / y16 (plain f16 rows, the tensor-core GEMM input) may be null;
// resid may be null.
int rmsnorm_launch(float* x, const float* resid, const uint16_t* w, int64_t rows, int64_t d,
                   float eps, float* y32, __half* yxs, __half* y16, cudaStream_t st, int64_t y16lo = 0);
int rmsnorm_heads_launch(const float* x, const uint16_t* w, int64_t rows, int64_t hd, float eps,
                         float* y, cudaStream_t st);
int rope_kv_launch(float* qkv, int64_t ldqkv, int64_t T, const int32_t* pos, const int32_t* seq,
                   int nh, int nkv, int hd, const float* inv_freq, const uint16_t* qn,
                   const uint16_t* kn, float eps, float* kp, float* vp, int page,
                   const int32_t* bt, int max_pages, cudaStream_t st);

struct AttnArgs {
  const float* q; int64_t ldq;
  int T;
  const int32_t* pos; const int32_t* seq;
  int nh, nkv, hd;
  const float* kp; const float* vp; int page;
  const int32_t* bt; int max_pages;
  // query blocks: token range [qb_tok0[i], qb_tok0[i]+qb_len[i]) of one sequence
  // with consecutive positions; null => one block per token.
  const int32_t* qb_tok0; const int32_t* qb_len; int nqb; int qb_max;
  int nsplit;
  float* part;                 // scratch: nqb*nkv*nsplit*(rmax*hd + 2*rmax) floats
  float* out32; int64_t ldo;   // nullable
  __half* outxs;               // nullable, XS over K = nh*hd
  __half* out16;               // nullable, plain f16 rows [T][nh*hd]
  int64_t out16lo;             // > 0: f16 remainder rows at out16 + out16lo
};
int attention_init();
int attention_launch(const AttnArgs& a, cudaStream_t st);
// tensor-core prefill attention (q8_attn_tc.cu) for query blocks of 9..64 rows
bool attention_tc_supported(const AttnArgs& a);
int attention_tc_launch(const AttnArgs& a, cudaStream_t st);
size_t attention_part_floats(int nqb, int nkv, int nsplit, int qb_max, int group, int hd);

size_t attention_decode_part_floats(int T, int nkv, int nsplit, int group, int hd);
// context splits for `items` (token, kv head) pairs: about one CTA per SM
int attention_decode_nsplit(int items, int maxlen);
int attn_dec_poll_error();
int attn_dec_error_word(int** out);
// Fused RoPE / QK-norm / KV append for the decode attention: q and the new
// k, v are read un-rotated from the q|k|v rows; kw / vw are the (same) pools.
struct AttnRope {
  const float* inv_freq;
  const uint16_t* qn;
  const uint16_t* kn;
  float eps;
  float* kw;
  float* vw;
};
int attention_decode_launch(const float* q, int64_t ldq, int T, const int32_t* pos, const int32_t* seq, int nh,
                            int nkv, int hd, const float* kp, const float* vp, int page, const int32_t* bt,
                            int max_pages, int nsplit, float* part, int* ticket, float* out32, int64_t ldo,
                            __half* outxs, cudaStream_t st, const AttnRope* rope = nullptr,
                            int64_t pool_rows = 0,  // rows of each pool (0: unknown)
                            __half* out16 = nullptr, int64_t out16lo = 0);

int argmax_prepare();  // per-device scratch of the wide-row argmax (outside capture)
int argmax_launch(const float* logits, int64_t rows, int64_t n, int64_t ld, int32_t* out,
                  cudaStream_t st);
// Temperature + nucleus sampling of rows of logits (q8_sample.cu); u [rows]
// uniform draws on the device; scratch of sample_scratch_bytes(rows, n).
size_t sample_scratch_bytes(int rows, int n);
int sample_launch(const float* logits, int rows, int n, int64_t ld, float temp, float top_p, const float* u,
                  int32_t* out, void* scratch, size_t scratch_bytes, cudaStream_t st);

}  // namespace q8
