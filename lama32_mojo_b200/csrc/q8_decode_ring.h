// Parameters of the weight-ring decode step (q8_decode_ring.cu) shared with
// the model runtime that fills them.
#pragma once
#include "q8_common.cuh"

#include <cuda.h>

namespace q8 {

constexpr int DR_CW = 8;                         // consumer warps
constexpr int DR_THREADS = (DR_CW + 1) * 32;     // + one producer warp
constexpr int DR_SLOTS = 2 * DR_CW;              // ring slots, two per consumer warp
constexpr int DR_CK = 512;                       // code bytes of one row in a GEMV stage
// A ring block: 16 rows x 512 codes as four 16 x 128 B boxes (16-byte chunk c
// of row r stored at chunk c ^ (r & 7)), then the rows' 16 x 8 f16 group
// scales.  Weights are copied once into this block order ("ring layout"), so
// that every stage is one bulk copy.
constexpr int DR_BLOCK = 16 * DR_CK + 16 * 16;   // 8448 bytes
constexpr int DR_SLOT_BYTES = DR_BLOCK;
constexpr int DR_XQ_BYTES = 48 * 1024;           // activation digits + per-warp tile sums
constexpr int DR_NS = 3;                         // partial slots of a down tile shared by CTAs
constexpr int DR_GMAX = 4;                       // q heads per kv head
constexpr int DR_MAXSPLIT = 128;                 // attention context splits per kv head
constexpr int DR_MAXTP = 8;                      // tensor-parallel ranks

struct DrLayer {
  // each matrix in ring layout: block (t, c) of 16-row tile t and 512-code
  // chunk c at (t * K/512 + c) * DR_BLOCK (gate|up tiles: 8 gate + 8 up rows)
  const uint8_t* qkv;  // [nq*hd + 2*nkv*hd rows][H]
  const uint8_t* o;    // [H rows][nq*hd]
  const uint8_t* gu;   // [2F rows][H]: tile t = gate rows t*8.. and up rows t*8..
  const uint8_t* down; // [H rows][F]
  const uint16_t* in_norm;
  const uint16_t* post_norm;
  const uint16_t* q_norm;  // Qwen3 QK-norm (null otherwise)
  const uint16_t* k_norm;
  float* kp;           // this layer's paged K / V pools [pages][nkv][page][hd]
  float* vp;
};

struct DrParams {
  int H, nh, nkv, hd, qd, nqkv, F, V, L;
  float eps;
  const DrLayer* layers;       // device array [L]
  const uint8_t* embed;        // packed [vocab][H]
  const uint8_t* lm_head;      // [V][H] in ring layout
  const uint16_t* final_norm;
  int32_t* ids;                // [1] token of the step (the generate epilogue writes the next one)
  int32_t* pos;                // [1] its position
  const int32_t* seq;          // [1] its KV sequence slot
  const float* inv_freq;       // [hd/2]
  int page;
  const int32_t* bt;           // block table [max_seqs][max_pages]
  int max_pages;
  // work buffers, written inside the launch and read by other CTAs with
  // L2-coherent loads
  float* h0;                   // residual of even layers [H]
  float* h1;                   // residual of odd layers [H]
  float* pres;                 // down-projection partial slots [nsf][H]
  int nsf;                     // slots per down tile (every one written each step)
  float* qkv;                  // [nqkv]
  float* ao;                   // attention output [qd]
  float* act;                  // SwiGLU output [F]
  float* logits;               // [V]
  float* apart;                // attention split partials [nkv][nsplit][GMAX*hd + 2*GMAX]
  int* aticket;                // [nkv], zero at rest
  int nsplit;
  unsigned long long* amax;    // packed (ordered value, ~index) of the step's argmax, zero at rest
  int* lm_ticket;              // zero at rest
  int32_t* argmax;             // [1]
  int gen;                     // generate epilogue: ids = argmax, pos += 1, hist[ctr] = argmax, ctr += 1
  int32_t* hist;
  int32_t* ctr;
  int hist_cap;
  unsigned int* bar;           // grid barrier arrivals (zeroed before each launch)
  int* status;                 // device status word (zero at rest)
  unsigned long long* trace;   // optional: CTA 0's globaltimer marks [phase][4] (wait done, staged,
                               // streamed, arrived)
  int qdp, Fp;                 // o_proj / down_proj inputs rounded up to 512 (zero-padded ring blocks)
  // tensor parallelism (tp > 1): q|k|v, gate|up and the vocabulary rows are
  // this rank's shard; o_proj and down_proj are row-parallel: every CTA stores
  // its partial rows into every rank's inbox (plain stores over NVLink), fences
  // at system scope and counts itself in every rank's arrival counter; the
  // next phase waits for the CTAs of all ranks and adds the partials in rank
  // order, so every rank holds the same residual
  int tp, rank;
  int V_off;                   // first vocabulary row of this rank (argmax keys are global rows)
  int gsum;                    // CTAs of all ranks (arrivals per exchange)
  float* xin[DR_MAXTP];        // every rank's inbox, mapped here: [parity][o | down][tp][slots][H]
  unsigned long long* xcnt[DR_MAXTP];   // every rank's monotonic arrival counters [o, down, lm_head]
  unsigned long long* xamax[DR_MAXTP];  // every rank's argmax keys [step parity]
  unsigned long long* xstep;   // this rank's completed steps
  float* xin_me;               // xin[rank]
  unsigned long long* xcnt_me; // xcnt[rank]
  unsigned long long* xamax_me;// xamax[rank]
  float* hm;                   // residual after o_proj [H]
};

// Inbox of the row-parallel exchange: floats from region (parity, kind) on
// (kind 0: o_proj, one slot per rank; kind 1: down_proj, nsf slots per rank).
__host__ __device__ inline int64_t dr_xin_region(int par, int kind, int tp, int H) {
  return (int64_t)(par * 2 + kind) * tp * DR_NS * H;
}
// Bytes of one rank's exchange block: the inbox, then 256 bytes of counters
// (xcnt [4] at +0, xamax [2] at +64, xstep at +128).
size_t dr_rx_bytes(int tp, int H);

// Host side (q8_decode_ring.cu).
// Whether the ring step supports these model dimensions on this device
// (one sequence, one GPU); *why gets the reason when it does not.
// Dimensions are this rank's (tensor-parallel shards).
bool dr_supported(int H, int nh, int nkv, int hd, int F, int V, int page, const char** why);
// K rounded up to whole 512-code ring chunks.
inline int dr_kpad(int K) { return (K + DR_CK - 1) / DR_CK * DR_CK; }
int dr_prepare(int hd, int* grid);  // kernel attributes, residency check; grid = CTAs (one per SM)
size_t dr_apart_floats(int nkv, int nsplit, int hd);
int dr_nsplit(int G, int nkv, int maxlen);
// down_proj tiles are split over CTAs (partial rows into slots) when they are
// at least 8 chunks deep; shallower ones (tensor-parallel slices) stay whole,
// so that each rank sends one partial row per output
__host__ __device__ inline bool dr_down_split(int Fp) { return Fp / DR_CK >= 8; }
int dr_down_nsf(int H, int F, int G);
int dr_launch(const DrParams& p, int grid, cudaStream_t st);
// Copies a packed-row matrix (rows x K, SwiGLU: 2 F rows with f2 = F) into
// ring layout at dst (dr_ring_bytes(rows, K) bytes; codes and scales past K
// are zero).
int dr_repack(const uint8_t* W, int64_t rows, int K, int f2, uint8_t* dst, cudaStream_t st);
inline size_t dr_ring_bytes(int64_t rows, int K) { return (size_t)(rows / 16) * (dr_kpad(K) / DR_CK) * DR_BLOCK; }

}  // namespace q8
