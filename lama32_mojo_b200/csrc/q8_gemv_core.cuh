// Register-level building blocks of the Q8 GEMV (shared by the standalone
// decode GEMV kernels and the persistent decode step):
//  * int8 codes -> exact f16 integers by byte permutation into 1024.0h,
//  * m16n8k16 f16 tensor-core MMA with f32 accumulation,
//  * 16-byte code loads with a no-L1-allocate, 256 B L2 prefetch hint.
#pragma once
#include "q8_common.cuh"

namespace q8 {

// 64-wide groups whose codes one lane loads before computing them
constexpr int GEMV_BATCH = 8;

__device__ __forceinline__ uint32_t cvt_s8x2_to_f16x2(uint32_t w_biased, uint32_t sel) {
  // w_biased = 4 int8 codes XOR 0x80 (offset binary).  Place two of them in
  // the low mantissa byte of f16 1024.0 (0x6400) -> 1024 + b + 128, then
  // subtract 1152: exact integer b in f16.
  uint32_t r = __byte_perm(w_biased, 0x64646464u, sel);
  __half2 h = *reinterpret_cast<__half2*>(&r);
  const uint32_t k1152 = 0x64806480u;
  h = __hsub2(h, *reinterpret_cast<const __half2*>(&k1152));
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void mma16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int VEC>
__device__ __forceinline__ void load_codes16(const uint8_t* p, uint32_t c[4]) {
  if constexpr (VEC == 16) {
    // weights are read once: no L1 allocation, 256 B L2 prefetch granule
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
                 : "l"(p));
  } else if constexpr (VEC == 8) {
    uint2 v0 = __ldg(reinterpret_cast<const uint2*>(p));
    uint2 v1 = __ldg(reinterpret_cast<const uint2*>(p + 8));
    c[0] = v0.x; c[1] = v0.y; c[2] = v1.x; c[3] = v1.y;
  } else if constexpr (VEC == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) c[i] = __ldg(reinterpret_cast<const uint32_t*>(p + 4 * i));
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t lo = __ldg(reinterpret_cast<const uint16_t*>(p + 4 * i));
      uint32_t hi = __ldg(reinterpret_cast<const uint16_t*>(p + 4 * i + 2));
      c[i] = lo | (hi << 16);
    }
  }
}

// Row addresses of lane (g, t) for a row tile: rows g and g+8 (SWIGLU: gate
// pair p and its up row F + p).

}  // namespace q8
