// Parameters of the persistent decode step (q8_decode_mk.cu) shared with the
// model runtime that fills them.
#pragma once
#include "q8_common.cuh"

namespace q8 {

constexpr int MK_THREADS = 256;              // 8 warps per CTA, one CTA per SM
constexpr int MK_WARPS = MK_THREADS / 32;
constexpr int MK_BMAX = 8;                   // token stride of the work buffers
constexpr int MK_GMAX = 4;                   // q heads per kv head
constexpr int MK_XS_BYTES = 128 * 1024;      // staged split-f16 activations
constexpr int MK_RED_BYTES = MK_WARPS * 2 * 16 * MK_BMAX * 4;  // warp partials of split tiles
constexpr int MK_SMEM = MK_XS_BYTES + MK_RED_BYTES + 1024;
constexpr int MK_MAXSPLIT = 128;             // attention context splits per (token, kv head)

struct MkLayer {
  const uint8_t* qkv;  // packed [nq*hd + 2*nkv*hd rows][H]
  const uint8_t* o;    // [H rows][nq*hd]
  const uint8_t* gu;   // [2F rows][H]: F gate rows then F up rows
  const uint8_t* down; // [H rows][F]
  const uint16_t* in_norm;
  const uint16_t* post_norm;
  const uint16_t* q_norm;  // Qwen3 QK-norm (null otherwise)
  const uint16_t* k_norm;
  float* kp;           // this layer's paged K / V pools
  float* vp;
};

struct MkParams {
  int B, H, nh, nkv, hd, qd, nqkv, F, V, L;
  float eps;
  const MkLayer* layers;       // device array [L]
  const uint8_t* embed;        // packed [V][H]
  const uint8_t* lm_head;      // packed [V][H]
  const uint16_t* final_norm;
  const int32_t* ids;          // [B]
  const int32_t* pos;          // [B] position of each step token
  const int32_t* seq;          // [B] KV sequence slot
  const float* inv_freq;       // [hd/2]
  int page;
  const int32_t* bt;           // block table [max_seqs][max_pages]
  int max_pages;
  // work buffers (all written inside the launch: read with L2-coherent loads)
  float* hA;                   // residual ping-pong [MK_BMAX][H]
  float* hB;
  float* pqkv;                 // cross-CTA partial slots [SL][MK_BMAX][nqkv]
  float* pres;                 // cross-CTA partial slots [SL][MK_BMAX][H] (o_proj, down)
  float* ao;                   // attention output [MK_BMAX][qd]
  float* act;                  // SwiGLU output f32 [MK_BMAX][F]
  float* logits;               // [B][V]
  unsigned long long* amax_key;// [MK_BMAX] packed (ordered value, ~index)
  int32_t* argmax;             // [B]
  float* apart;                // attention split partials
  int* ticket;                 // [MK_BMAX * nkv], zero at rest
  int nsplit;
  unsigned int* bar;           // grid barrier arrivals (zeroed before each launch)
  int* status;                 // device status word (zero at rest)
  int pf_bytes;                // L2 prefetch budget per CTA per phase
  unsigned long long* ts;      // optional phase trace: [0] start, [i] barrier i done (ns)
  unsigned long long* ts2;     // optional sub-phase trace of CTA 0: [phase * 4 + j]
};

// Host helpers (q8_decode_mk.cu).
// Largest number of CTAs sharing one output tile in a GEMV of N rows
// (pairs when swiglu) over K on G CTAs with unit-balanced ranges.
int mk_slots(int K, int N, bool swiglu, bool aligned, int G);
size_t mk_attn_part_floats(int nkv, int nsplit, int hd);
int mk_smem_bytes();
// Step batch limit (0, 1 or 2) set by the shared-memory staging of the
// widest GEMV input.
int mk_max_batch(int H, int qd, int F);
// Whether a co-resident grid of G CTAs of the step kernel fits this device.
int mk_check_residency(int hd, int vec, int G, bool* ok);
int mk_launch(const MkParams& p, int vec, int G, cudaStream_t st);

}  // namespace q8
