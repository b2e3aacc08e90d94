// NVLink peer-memory exchange for Ulysses sequence parallelism.
//
// Every rank allocates the same receive buffers and a small flag array, and
// maps its peers' buffers through CUDA IPC.  A producing kernel (the fused
// norm+RoPE for seq->head, the attention epilogue for head->seq) stores each
// row straight into the owning rank's receive buffer over NVLink; then
//   tm_peer_signal  one thread per peer: a system-scope fence, then a release
//                   store of this rank's next epoch into the peer's flag slot;
//   tm_peer_wait    one thread spins (acquire loads, bounded by 2 s of
//                   %globaltimer) until every rank's flag reached this rank's
//                   next epoch; on timeout it records TM device error 2 and
//                   returns, so a lost peer never hangs the GPU;
//   tm_peer_exchange  both in one launch.
// Epochs are counted on the device (per slot), so the same launches can be
// replayed from a CUDA graph.  Plain peer loads/stores only: no multicast,
// no NVLS.
//
// Reference counterpart: the all_to_all_single calls of _seq_to_head /
// _head_to_seq (taomate/runtime_support/parallel/all_to_all.py:125-173).
#include <atomic>
#include <cstring>

#include "common.cuh"
#include "host_common.h"

namespace tmb {
namespace peer {

constexpr int kMaxRanks = 8;
constexpr int kSlots = 4;
constexpr unsigned long long kPeerWaitNs = 2000000000ull;  // default limit of a wait
constexpr int kDevPeerTimeout = 2;

// Limit of the flag waits launched from now on (a kernel parameter, so a
// captured graph keeps the limit it was captured with).
std::atomic<unsigned long long> g_wait_limit_ns{kPeerWaitNs};

// Flag array of a rank: int64 flags[kSlots][kMaxRanks], then the local
// counters: sent[kSlots], awaited[kSlots].
struct SignalParams {
  unsigned long long* peer_flags[kMaxRanks];  // each rank's flag array, mapped here
  unsigned long long* counters;               // this rank's counters (local)
  int n_ranks, rank, slot;
};

__global__ void signal_kernel(const __grid_constant__ SignalParams p) {
  __shared__ unsigned long long epoch;
  if (threadIdx.x == 0) {
    epoch = ++p.counters[p.slot];
    asm volatile("fence.sc.sys;" ::: "memory");
  }
  __syncthreads();
  const int g = threadIdx.x;
  if (g < p.n_ranks) {
    unsigned long long* f = p.peer_flags[g] + p.slot * kMaxRanks + p.rank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(epoch) : "memory");
  }
}

// Thread 0 waits until every rank's flag of `slot` reached this rank's next
// awaited epoch (bounded; device error kDevPeerTimeout on giving up).
__device__ void wait_flags(const unsigned long long* flags, unsigned long long* counters,
                           int n_ranks, int slot, unsigned long long limit_ns, int* err) {
  const unsigned long long target = ++counters[kSlots + slot];
  const unsigned long long* f = flags + slot * kMaxRanks;
  const unsigned long long t0 = globaltimer_ns();
  for (int g = 0; g < n_ranks; ++g) {
    for (uint32_t i = 0;; ++i) {
      unsigned long long v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(f + g) : "memory");
      if (v >= target) break;
      if ((i & 63u) == 0u && globaltimer_ns() - t0 > limit_ns) {
        atomicCAS(err, 0, kDevPeerTimeout);
        return;
      }
    }
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

__global__ void wait_kernel(const unsigned long long* flags, unsigned long long* counters,
                            int n_ranks, int slot, unsigned long long limit_ns, int* err) {
  if (threadIdx.x == 0) wait_flags(flags, counters, n_ranks, slot, limit_ns, err);
}

// signal_kernel then wait_kernel in one launch: a replayed graph pays one
// node instead of two per exchange.
__global__ void exchange_kernel(const __grid_constant__ SignalParams p,
                                const unsigned long long* flags, unsigned long long limit_ns,
                                int* err) {
  __shared__ unsigned long long epoch;
  if (threadIdx.x == 0) {
    epoch = ++p.counters[p.slot];
    asm volatile("fence.sc.sys;" ::: "memory");
  }
  __syncthreads();
  const int g = threadIdx.x;
  if (g < p.n_ranks) {
    unsigned long long* f = p.peer_flags[g] + p.slot * kMaxRanks + p.rank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(epoch) : "memory");
  }
  if (threadIdx.x == 0) wait_flags(flags, p.counters, p.n_ranks, p.slot, limit_ns, err);
}

}  // namespace peer
}  // namespace tmb

using namespace tmb;

extern "C" int tm_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle) {
  if (bytes <= 0 || !ptr || !ipc_handle)
    return set_error(TM_ERR_INVALID_ARGUMENT, "peer_alloc: bad arguments");
  void* p = nullptr;
  int st = check_cuda(cudaMalloc(&p, static_cast<size_t>(bytes)), "peer_alloc: cudaMalloc");
  if (st) return st;
  st = check_cuda(cudaMemset(p, 0, static_cast<size_t>(bytes)), "peer_alloc: clear");
  if (!st) {
    cudaIpcMemHandle_t h;
    st = check_cuda(cudaIpcGetMemHandle(&h, p), "peer_alloc: IPC handle");
    if (!st) memcpy(ipc_handle, &h, sizeof(h));
  }
  if (st) {
    cudaFree(p);
    return st;
  }
  *ptr = p;
  return TM_OK;
}

extern "C" int tm_peer_free(void* ptr) {
  if (!ptr) return TM_OK;
  return check_cuda(cudaFree(ptr), "peer_free");
}

extern "C" int tm_peer_open(const void* ipc_handle, void** peer_ptr) {
  if (!ipc_handle || !peer_ptr) return set_error(TM_ERR_INVALID_ARGUMENT, "peer_open: null");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return check_cuda(cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess),
                    "peer_open: cudaIpcOpenMemHandle");
}

extern "C" int tm_peer_close(void* peer_ptr) {
  if (!peer_ptr) return TM_OK;
  return check_cuda(cudaIpcCloseMemHandle(peer_ptr), "peer_close");
}

extern "C" int tm_peer_signal(void* const* peer_flags, int n_ranks, int rank, void* counters,
                              int slot, void* stream) {
  using namespace tmb::peer;
  if (n_ranks < 1 || n_ranks > kMaxRanks || rank < 0 || rank >= n_ranks || slot < 0 ||
      slot >= kSlots || !peer_flags || !counters)
    return set_error(TM_ERR_INVALID_ARGUMENT, "peer_signal: bad arguments");
  SignalParams p;
  memset(&p, 0, sizeof(p));
  for (int g = 0; g < n_ranks; ++g) {
    if (!peer_flags[g]) return set_error(TM_ERR_INVALID_ARGUMENT, "peer_signal: null flags");
    p.peer_flags[g] = static_cast<unsigned long long*>(peer_flags[g]);
  }
  p.counters = static_cast<unsigned long long*>(counters);
  p.n_ranks = n_ranks;
  p.rank = rank;
  p.slot = slot;
  signal_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_cuda(cudaGetLastError(), "peer_signal: launch");
}

extern "C" int tm_peer_wait(const void* flags, int n_ranks, void* counters, int slot,
                            void* stream) {
  using namespace tmb::peer;
  if (n_ranks < 1 || n_ranks > kMaxRanks || slot < 0 || slot >= kSlots || !flags || !counters)
    return set_error(TM_ERR_INVALID_ARGUMENT, "peer_wait: bad arguments");
  int* err = device_error_flag();
  if (!err) return set_error(TM_ERR_CUDA, "peer_wait: device error flag unavailable");
  wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const unsigned long long*>(flags), static_cast<unsigned long long*>(counters),
      n_ranks, slot, g_wait_limit_ns.load(), err);
  return check_cuda(cudaGetLastError(), "peer_wait: launch");
}

extern "C" int tm_peer_exchange(void* const* peer_flags, int n_ranks, int rank, const void* flags,
                                void* counters, int slot, void* stream) {
  using namespace tmb::peer;
  if (n_ranks < 1 || n_ranks > kMaxRanks || rank < 0 || rank >= n_ranks || slot < 0 ||
      slot >= kSlots || !peer_flags || !flags || !counters)
    return set_error(TM_ERR_INVALID_ARGUMENT, "peer_exchange: bad arguments");
  int* err = device_error_flag();
  if (!err) return set_error(TM_ERR_CUDA, "peer_exchange: device error flag unavailable");
  SignalParams p;
  memset(&p, 0, sizeof(p));
  for (int g = 0; g < n_ranks; ++g) {
    if (!peer_flags[g]) return set_error(TM_ERR_INVALID_ARGUMENT, "peer_exchange: null flags");
    p.peer_flags[g] = static_cast<unsigned long long*>(peer_flags[g]);
  }
  p.counters = static_cast<unsigned long long*>(counters);
  p.n_ranks = n_ranks;
  p.rank = rank;
  p.slot = slot;
  exchange_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      p, static_cast<const unsigned long long*>(flags), g_wait_limit_ns.load(), err);
  return check_cuda(cudaGetLastError(), "peer_exchange: launch");
}

extern "C" int64_t tm_peer_flag_bytes(void) {
  using namespace tmb::peer;
  return static_cast<int64_t>(sizeof(unsigned long long)) * (kSlots * kMaxRanks + 2 * kSlots);
}

extern "C" int64_t tm_peer_set_wait_limit(int64_t ns) {
  using namespace tmb::peer;
  if (ns <= 0) ns = static_cast<int64_t>(kPeerWaitNs);
  return static_cast<int64_t>(g_wait_limit_ns.exchange(static_cast<unsigned long long>(ns)));
}
