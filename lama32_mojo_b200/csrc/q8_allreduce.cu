// One-shot P2P allreduce for the tensor-parallel decode step.
//
// After each row-parallel projection (o_proj, down_proj) every rank holds a
// partial [T, H] that must be summed over ranks and added to the residual
// stream (run_layer_q8's `k_res_add`, src/llama_common.mojo:354-358; the
// reference itself is single-device).  Decode messages are small (T * H
// floats, 16 KB at T = 1 for H = 4096), so the exchange is latency-bound and
// is done in one kernel:
//   1. each CTA stores its chunk of the local partial into slot [parity][rank]
//      of EVERY rank's landing buffer (plain stores over NVLink into the
//      peer's own memory: no remote reads, no TMA, no multicast);
//   2. a system-scope fence, then a release store of the call's sequence
//      number into each rank's flag for (parity, rank, CTA);
//   3. a bounded acquire spin on this rank's flags of every source rank for
//      the same CTA index;
//   4. residual += sum of the slots in rank order from local memory, so every
//      rank computes bit-identical values;
//   5. the last CTA (ticket) advances the rank's sequence number.
// Slots and flags are double-buffered by the parity of the sequence number: a
// rank can be at most one call ahead of another (it cannot pass step 3 of call
// s+1 before every rank has started call s+1, i.e. finished reading call s).
// The RMSNorm that follows runs in the next GEMV's prologue, as at TP = 1.
// Buffers are exported with CUDA IPC; the handles travel over NCCL at setup.
#include "q8_allreduce.h"

#include <string.h>

namespace q8 {

constexpr long long AR_SPIN_LIMIT = 1ll << 25;  // x ~64 ns sleeps: about two seconds

__device__ __forceinline__ void ar_st_release(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ar_ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct ArArgs {
  ArPeers peers;
  const float* part;   // [n] this rank's partial
  float* h;            // [n] residual, += sum of the partials
  int n;               // floats, multiple of 4
  float* land;         // this rank's landing buffer [2][tp][slot]
  int* flag;           // this rank's flags [2][tp][AR_NB]
  int* seq;            // sequence number of the last completed call
  int* ticket;         // zero at rest
  int* status;         // Q8_ERR_TIMEOUT when a spin gave up
  int tp, rank;
  int64_t slot;        // floats per (parity, source) slot
};

__global__ void __launch_bounds__(256) k_ar_p2p(ArArgs a) {
  __shared__ int s_seq;
  pdl_trigger();
  pdl_wait();  // the partial is written by the previous kernel
  if (threadIdx.x == 0) s_seq = *reinterpret_cast<volatile int*>(a.seq) + 1;
  __syncthreads();
  const int sq = s_seq, par = sq & 1, b = blockIdx.x, nb = gridDim.x;
  const int n4 = a.n / 4, per = (n4 + nb - 1) / nb;
  const int i0 = min(n4, b * per), i1 = min(n4, i0 + per);
  const float4* src = reinterpret_cast<const float4*>(a.part);
  for (int r = 0; r < a.tp; ++r) {
    float4* dst = reinterpret_cast<float4*>(a.peers.land[r] + ((int64_t)par * a.tp + a.rank) * a.slot);
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) dst[i] = src[i];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < a.tp) ar_st_release(a.peers.flag[threadIdx.x] + (par * a.tp + a.rank) * AR_NB + b, sq);
  if (threadIdx.x < a.tp) {
    const int* f = a.flag + (par * a.tp + threadIdx.x) * AR_NB + b;
    long long it = 0;
    while (ar_ld_acquire(f) < sq) {
      if (++it > AR_SPIN_LIMIT) {
        atomicExch(a.status, Q8_ERR_TIMEOUT);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  float4* h4 = reinterpret_cast<float4*>(a.h);
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    float4 acc = h4[i];
    for (int r = 0; r < a.tp; ++r) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(a.land + ((int64_t)par * a.tp + r) * a.slot) + i);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    h4[i] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.ticket, 1) == nb - 1) {
      *a.ticket = 0;
      *reinterpret_cast<volatile int*>(a.seq) = sq;
    }
  }
}

// ------------------------------------------------------------------ host side
// block: [land 2*tp*slot floats][flag 2*tp*AR_NB ints][seq][ticket][status] (256 B)[rx]
static size_t ar_land_bytes(int tp, int64_t slot) { return ((size_t)2 * tp * slot * 4 + 255) & ~(size_t)255; }

// Two collectives, taken by every rank whatever happens locally: an
// all-gather of (IPC handle, usable) records, then an all-reduce (min) of
// "mapped every peer", so all ranks agree on P2P versus NCCL.
struct ArHandleRec {
  cudaIpcMemHandle_t h;
  int valid;
  int pad[15];
};

int ar_setup(ArState* s, ncclComm_t comm, int tp, int rank, int64_t max_floats, size_t rx_bytes, cudaStream_t st) {
  *s = ArState{};
  if (tp < 2 || tp > AR_MAXTP) return Q8_OK;
  s->tp = tp;
  s->rank = rank;
  s->slot = (max_floats + 63) & ~(int64_t)63;
  const size_t lb = ar_land_bytes(tp, s->slot);
  const size_t fb = (size_t)2 * tp * AR_NB * 4;
  const size_t rxo = lb + fb + 256;  // the exchange block of the decode step, 256-byte aligned
  s->bytes = rxo + ((rx_bytes + 255) & ~(size_t)255);
  ArHandleRec mine{};
  // zeroed on `st`, ahead of this rank's contribution to the exchange below
  if (cudaMalloc(&s->block, s->bytes) == cudaSuccess && cudaMemsetAsync(s->block, 0, s->bytes, st) == cudaSuccess &&
      cudaIpcGetMemHandle(&mine.h, s->block) == cudaSuccess)
    mine.valid = 1;
  cudaGetLastError();
  // exchange the records (each rank's zeroing precedes its contribution)
  void* dbuf = nullptr;
  Q8_CUDA(cudaMalloc(&dbuf, (size_t)(tp + 2) * sizeof(ArHandleRec)));
  ArHandleRec* drec = static_cast<ArHandleRec*>(dbuf);
  std::vector<ArHandleRec> all(tp);
  int ok_local = 0, ok_all = 0;
  cudaError_t ce = cudaMemcpyAsync(drec, &mine, sizeof(mine), cudaMemcpyHostToDevice, st);
  ncclResult_t r = ncclAllGather(drec, drec + 1, sizeof(ArHandleRec), ncclChar, comm, st);
  if (ce == cudaSuccess) ce = cudaMemcpyAsync(all.data(), drec + 1, (size_t)tp * sizeof(ArHandleRec),
                                              cudaMemcpyDeviceToHost, st);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
  bool every = r == ncclSuccess && ce == cudaSuccess;
  for (int k = 0; k < tp && every; ++k) every = all[k].valid == 1;
  if (every) {
    uint8_t* base = static_cast<uint8_t*>(s->block);
    ok_local = 1;
    for (int k = 0; k < tp; ++k) {
      uint8_t* p = base;
      if (k != rank) {
        void* q = nullptr;
        if (cudaIpcOpenMemHandle(&q, all[k].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
          cudaGetLastError();
          ok_local = 0;
          break;
        }
        s->opened[k] = q;
        p = static_cast<uint8_t*>(q);
      }
      s->peers.land[k] = reinterpret_cast<float*>(p);
      s->peers.flag[k] = reinterpret_cast<int*>(p + lb);
      s->peers.rx[k] = rx_bytes ? p + rxo : nullptr;
    }
  }
  // agree: P2P only if every rank mapped every peer
  int* dok = reinterpret_cast<int*>(drec + tp + 1);
  ce = cudaMemcpyAsync(dok, &ok_local, 4, cudaMemcpyHostToDevice, st);
  ncclResult_t r2 = ncclAllReduce(dok, dok, 1, ncclInt32, ncclMin, comm, st);
  if (ce == cudaSuccess) ce = cudaMemcpyAsync(&ok_all, dok, 4, cudaMemcpyDeviceToHost, st);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
  cudaFree(dbuf);
  if (r != ncclSuccess || r2 != ncclSuccess || ce != cudaSuccess) {
    ar_teardown(s);
    set_error("allreduce: handle exchange failed");
    return Q8_ERR_COMM;
  }
  if (ok_all != 1) {
    ar_teardown(s);  // NCCL carries decode too
    return Q8_OK;
  }
  uint8_t* base = static_cast<uint8_t*>(s->block);
  s->land = reinterpret_cast<float*>(base);
  s->flag = reinterpret_cast<int*>(base + lb);
  s->seq = reinterpret_cast<int*>(base + lb + fb);
  s->ticket = s->seq + 1;
  s->status = s->seq + 2;
  s->rx = rx_bytes ? base + rxo : nullptr;
  s->rx_bytes = rx_bytes;
  s->ok = true;
  return Q8_OK;
}

void ar_teardown(ArState* s) {
  for (int k = 0; k < AR_MAXTP; ++k)
    if (s->opened[k]) cudaIpcCloseMemHandle(s->opened[k]);
  if (s->block) cudaFree(s->block);
  *s = ArState{};
}

int ar_launch(const ArState& s, const float* part, float* h, int n, cudaStream_t st) {
  Q8_CHECK_ARG(s.ok && n > 0 && n % 4 == 0 && n <= s.slot, "allreduce: %d floats do not fit", n);
  ArArgs a{};
  a.peers = s.peers;
  a.part = part;
  a.h = h;
  a.n = n;
  a.land = s.land;
  a.flag = s.flag;
  a.seq = s.seq;
  a.ticket = s.ticket;
  a.status = s.status;
  a.tp = s.tp;
  a.rank = s.rank;
  a.slot = s.slot;
  const int nb = std::max(1, std::min(AR_NB, n / 4 / 64));
  return launch_pdl("k_ar_p2p", k_ar_p2p, dim3(nb), dim3(256), 0, st, a);
}

}  // namespace q8
