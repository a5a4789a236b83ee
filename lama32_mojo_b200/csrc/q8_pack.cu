// GPU quantizer/packer, bit-exact with the reference packer
// pack_q8 (qwen3_mojo/scripts/quantize.py:31-43):
//
//   scale_g = f16( max( f32(absmax_g) / 127 , 1e-8 ) )      (:36-37, IEEE f32 divide, RNE to f16)
//   q       = clip( rint( x / f32(scale_g) ), -127, 127 )   (:38-39, round-half-even)
//   row     = [ scales (m/64 f16) | codes (m int8) ]         (:41-43)
//
// Edge cases reproduced: a scale that underflows to 0 in f16 gives x/0 ->
// +-inf -> +-127, and 0/0 = NaN -> 0 (numpy's NaN->int8 on x86); an f16 scale
// that overflows to inf gives x/inf = 0.
//
// One warp per 64-wide group; each lane owns two adjacent elements, so the
// loads (4 B per lane) and the code stores (2 B per lane) are coalesced.
#include "q8_common.cuh"

namespace q8 {

__global__ void __launch_bounds__(256) k_pack_q8(const uint16_t* __restrict__ w, int64_t n,
                                                 int64_t m, uint8_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t gpr = m / Q8_QG;  // groups per row
  const int64_t total = n * gpr;
  const int64_t rb = q8_row_bytes(m);
  for (int64_t gid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); gid < total;
       gid += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int64_t row = gid / gpr, g = gid % gpr;
    const uint32_t pair = *reinterpret_cast<const uint32_t*>(w + row * m + g * Q8_QG + 2 * lane);
    const float x0 = __uint_as_float(pair << 16);
    const float x1 = __uint_as_float(pair & 0xffff0000u);
    const float amax = warp_max(fmaxf(fabsf(x0), fabsf(x1)));
    float s = __fdiv_rn(amax, 127.0f);
    s = fmaxf(s, 1e-8f);
    const __half sh = __float2half_rn(s);
    const float sf = __half2float(sh);
    float q0 = rintf(__fdiv_rn(x0, sf));
    float q1 = rintf(__fdiv_rn(x1, sf));
    q0 = (q0 != q0) ? 0.f : fminf(fmaxf(q0, -127.f), 127.f);
    q1 = (q1 != q1) ? 0.f : fminf(fmaxf(q1, -127.f), 127.f);
    uint8_t* orow = out + row * rb;
    if (lane == 0) reinterpret_cast<__half*>(orow)[g] = sh;
    const uint16_t codes = (uint16_t)(uint8_t)(int8_t)(int)q0 | ((uint16_t)(uint8_t)(int8_t)(int)q1 << 8);
    *reinterpret_cast<uint16_t*>(orow + m / 32 + g * Q8_QG + 2 * lane) = codes;
  }
}

__global__ void k_dequant_q8(const uint8_t* __restrict__ packed, int64_t n, int64_t m,
                             float* __restrict__ w) {
  const int64_t total = n * m;
  const int64_t rb = q8_row_bytes(m);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / m, c = i % m;
    const uint8_t* row = packed + r * rb;
    const float s = __half2float(reinterpret_cast<const __half*>(row)[c / Q8_QG]);
    w[i] = (float)(int8_t)row[m / 32 + c] * s;
  }
}

int pack_launch(const void* w_bf16, int64_t n, int64_t m, void* packed, cudaStream_t st) {
  Q8_CHECK_ARG(w_bf16 && packed, "q8op_pack: null pointer");
  Q8_CHECK_ARG(n > 0 && m > 0 && m % Q8_QG == 0, "q8op_pack: need m %% 64 == 0 (n=%lld m=%lld)",
               (long long)n, (long long)m);
  Q8_CHECK_ARG(((uintptr_t)w_bf16 & 3) == 0 && ((uintptr_t)packed & 1) == 0,
               "q8op_pack: misaligned pointer");
  const int64_t groups = n * (m / Q8_QG);
  const int blocks = (int)std::min<int64_t>((groups + 7) / 8, (int64_t)num_sms() * 16);
  k_pack_q8<<<blocks, 256, 0, st>>>((const uint16_t*)w_bf16, n, m, (uint8_t*)packed);
  return launch_check("k_pack_q8");
}

}  // namespace q8

extern "C" int q8op_pack(const void* w_bf16, int64_t n, int64_t m, void* packed, void* stream) {
  return q8::pack_launch(w_bf16, n, m, packed, (cudaStream_t)stream);
}

extern "C" int q8op_dequant(const void* packed, int64_t n, int64_t m, float* w, void* stream) {
  Q8_CHECK_ARG(packed && w, "q8op_dequant: null pointer");
  Q8_CHECK_ARG(n > 0 && m > 0 && m % Q8_QG == 0, "q8op_dequant: need m %% 64 == 0");
  const int64_t total = n * m;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)q8::num_sms() * 32);
  q8::k_dequant_q8<<<blocks, 256, 0, (cudaStream_t)stream>>>((const uint8_t*)packed, n, m, w);
  return q8::launch_check("k_dequant_q8");
}
