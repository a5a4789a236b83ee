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

// SwiGLU activation silu(g) * u — k_swiglu_mul (src/llama_common.mojo:476).
__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

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

// Programmatic dependent launch.  A kernel launched with the programmatic
// stream-serialization attribute may start while its predecessor in the
// stream is still running; it must call pdl_wait() before touching anything
// the predecessor writes (weights and other read-only inputs may be read
// before).  pdl_trigger() lets the successor launch early.  Both are no-ops
// for ordinary launches.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- shared-memory barriers + bulk async copies (TMA engine, no tensor map)
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// make barrier initialization visible to the async (TMA) proxy
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Device-side error word (one per translation unit): a bounded wait that
// gives up records its code here.
static __device__ int g_q8_device_error;

// Bounded wait on a barrier phase: gives up after ~2^31 cycles (about a
// second), records Q8_ERR_TIMEOUT in g_q8_device_error and returns false, so
// a lost completion never hangs the GPU.  The error word (another wait gave
// up: return so the grid drains) is read every 2^20 cycles of waiting, not
// on entry: a global load there would add its latency to every wait.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  long long next = t0 + (1ll << 20);
  while (!mbar_try_wait(bar, parity)) {
    const long long t = clock64();
    if (t > next) {
      if (*reinterpret_cast<volatile int*>(&g_q8_device_error)) return false;
      if (t - t0 > (1ll << 31)) {
        atomicExch(&g_q8_device_error, Q8_ERR_TIMEOUT);
        return false;
      }
      next = t + (1ll << 20);
    }
  }
  return true;
}

// 1-D bulk copy global -> this CTA's shared memory; completion counts bytes on bar.
// src, dst 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Whether decode-path launches use programmatic dependent launch (env Q8_PDL=0 disables).
bool pdl_enabled();

// cudaLaunchKernelEx with the programmatic stream-serialization attribute.
template <typename... KArgs, typename... Args>
inline int launch_pdl(const char* what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t st, Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  if (e != cudaSuccess) {
    set_error("launch %s: %s", what, cudaGetErrorString(e));
    return Q8_ERR_CUDA;
  }
  return Q8_OK;
}

int num_sms();

}  // namespace q8
