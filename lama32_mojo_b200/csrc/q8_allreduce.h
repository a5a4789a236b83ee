// One-shot P2P allreduce for the tensor-parallel decode step (see q8_allreduce.cu).
#pragma once
#include "q8_kernels.h"

#include <nccl.h>
#include <vector>

namespace q8 {

constexpr int AR_MAXTP = 8;
constexpr int AR_NB = 32;  // CTAs per call (flags per source rank and parity)

struct ArPeers {
  float* land[AR_MAXTP];  // every rank's landing buffer, mapped in this process
  int* flag[AR_MAXTP];    // every rank's flags
  uint8_t* rx[AR_MAXTP];  // every rank's block for the one-launch step's exchange (rx_bytes)
};

struct ArState {
  bool ok = false;        // P2P path usable (else NCCL carries decode too)
  int tp = 0, rank = 0;
  int64_t slot = 0;       // floats per (parity, source rank) slot
  void* block = nullptr;  // this rank's exported buffer
  size_t bytes = 0;
  float* land = nullptr;
  int* flag = nullptr;
  int* seq = nullptr;
  int* ticket = nullptr;
  int* status = nullptr;  // device: Q8_ERR_TIMEOUT after a spin gave up
  uint8_t* rx = nullptr;  // this rank's block for the one-launch step's exchange (zeroed at setup)
  size_t rx_bytes = 0;
  void* opened[AR_MAXTP] = {};
  ArPeers peers{};
};

// Collective over `comm` (every rank calls it at the same point): allocates
// and exports this rank's landing buffer for up to max_floats per call, plus
// rx_bytes for the decode step's exchange, and maps the peers'.  s->ok stays
// false (and Q8_OK is returned) when IPC is not available, so callers fall
// back to NCCL.
int ar_setup(ArState* s, ncclComm_t comm, int tp, int rank, int64_t max_floats, size_t rx_bytes, cudaStream_t st);
void ar_teardown(ArState* s);
// h[0..n) += sum over ranks of part[0..n); every rank calls it with the same n.
int ar_launch(const ArState& s, const float* part, float* h, int n, cudaStream_t st);

}  // namespace q8
