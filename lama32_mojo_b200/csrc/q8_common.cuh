// Shared device/host helpers for libq8cuda (B200, sm_100a).
//
// Packed Q8 row layout (src/llama_q8.mojo:3-9, 26-42; qwen3_mojo/scripts/quantize.py:31-43):
//   one weight row of K inputs = [K/64 f16 group scales | K int8 codes]
//   = K/64 + K/2 u16 elements = K*33/32 bytes; rows are contiguous.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <string>

#include "../../include/q8cuda.h"

#define Q8_QG 64

namespace q8 {

// ------------------------------------------------------------------ error state
void set_error(const char* fmt, ...);
const char* get_error();

#define Q8_CUDA(call)                                                              \
  do {                                                                             \
    cudaError_t _e = (call);                                                       \
    if (_e != cudaSuccess) {                                                       \
      ::q8::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call,                   \
                      cudaGetErrorString(_e));                                     \
      return Q8_ERR_CUDA;                                                          \
    }                                                                              \
  } while (0)

#define Q8_CHECK_ARG(cond, ...)                                                    \
  do {                                                                             \
    if (!(cond)) {                                                                 \
      ::q8::set_error(__VA_ARGS__);                                                \
      return Q8_ERR_ARG;                                                           \
    }                                                                              \
  } while (0)

#define Q8_TRY(expr)                                                               \
  do {                                                                             \
    int _s = (expr);                                                               \
    if (_s != Q8_OK) return _s;                                                    \
  } while (0)

static inline int launch_check(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("launch %s: %s", what, cudaGetErrorString(e));
    return Q8_ERR_CUDA;
  }
  return Q8_OK;
}

// ------------------------------------------------------------------ layout helpers
__host__ __device__ inline int64_t q8_row_bytes(int64_t k) { return k / 32 + k; }
__host__ __device__ inline int64_t q8_row_u16(int64_t k) { return k / Q8_QG + k / 2; }

// Split-f16 activation layout ("XS"): token row m of K values is K/16 chunks,
// each chunk = 16 f16 "hi" values then 16 f16 "lo" values, hi = f16(x),
// lo = f16(x - hi).  hi + lo carries ~22 bits of x, so the tensor-core GEMV
// reproduces the f32 activations of the reference (W8A32) to ~1e-6.
__host__ __device__ inline int64_t xs_row_halves(int64_t k) { return 2 * k; }
__device__ __forceinline__ int64_t xs_index(int64_t m, int64_t k, int64_t K, int lo) {
  return (m * (K >> 4) + (k >> 4)) * 32 + (lo ? 16 : 0) + (k & 15);
}

__device__ __forceinline__ void split_f16(float v, __half& hi, __half& lo) {
  v = fminf(fmaxf(v, -65504.f), 65504.f);
  hi = __float2half_rn(v);
  lo = __float2half_rn(v - __half2float(hi));
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(((uint32_t)b) << 16);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

int num_sms();

}  // namespace q8
