// kvb_peer_barrier: a bounded barrier between the GPUs of a context-parallel
// group, over signal words in peer-mapped memory (plain NVLink stores and
// loads; no NCCL call, no TMA, no multicast).
//
// Rank r owns an array of `world` 32-bit words mapped into every rank.  One
// launch on rank r stores `epoch` into word r of every rank's array (a
// system-scope release after a system-scope fence, so every write this GPU
// made before the launch is visible to a peer that sees the word), then waits
// until every word of its own array has reached `epoch` (system-scope acquire
// loads).  Epochs only grow, so a word left over from an earlier barrier never
// satisfies a later one.  A wait that has not been satisfied after
// `timeout_ns` (%globaltimer) gives up: the kernel ORs KVB_STATUS_PEER_WAIT
// into *status and returns, leaving the context usable; the host reads the
// status word after the launch and treats the collective as failed.

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "kvb_attn.h"

int kvb_detail_fail(int code, const std::string& msg);

namespace {

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void store_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct SignalArgs {
  uint32_t* slot[8];
  int world;
  int rank;
};

// One warp; lane t < world signals rank t and waits for rank t's signal.
__global__ void __launch_bounds__(32) kvb_peer_barrier_kernel(const SignalArgs a, uint32_t epoch,
                                                              int64_t timeout_ns, int* status) {
  const int t = threadIdx.x;
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  if (t < a.world) store_release_sys(a.slot[t] + a.rank, epoch);
  bool ok = true;
  if (t < a.world) {
    const uint32_t* mine = a.slot[a.rank] + t;
    const uint64_t t0 = now_ns();
#pragma unroll 1
    while (static_cast<int32_t>(load_acquire_sys(mine) - epoch) < 0) {
      if (static_cast<int64_t>(now_ns() - t0) > timeout_ns) {
        ok = false;
        break;
      }
      __nanosleep(64);
    }
  }
  if (!ok && status) atomicOr(status, KVB_STATUS_PEER_WAIT);
  __syncwarp();
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

}  // namespace

extern "C" int kvb_peer_barrier(const KvbPeerSignals* sig, uint32_t epoch, int64_t timeout_ns,
                                int* status, void* stream) {
  if (!sig) return kvb_detail_fail(KVB_ERR_INVALID, "kvb_peer_barrier: signals is NULL");
  if (sig->world < 1 || sig->world > 8)
    return kvb_detail_fail(KVB_ERR_UNSUPPORTED, "kvb_peer_barrier: world must be in [1, 8]");
  if (sig->rank < 0 || sig->rank >= sig->world)
    return kvb_detail_fail(KVB_ERR_INVALID, "kvb_peer_barrier: rank must be in [0, world)");
  if (epoch == 0)
    return kvb_detail_fail(KVB_ERR_INVALID, "kvb_peer_barrier: epoch must be >= 1");
  if (timeout_ns <= 0 || timeout_ns > 60ll * 1000000000ll)
    return kvb_detail_fail(KVB_ERR_INVALID, "kvb_peer_barrier: timeout_ns must be in (0, 60 s]");
  SignalArgs a = {};
  for (int r = 0; r < sig->world; ++r) {
    if (!sig->slot[r] || (reinterpret_cast<uintptr_t>(sig->slot[r]) & 3))
      return kvb_detail_fail(KVB_ERR_INVALID,
                             "kvb_peer_barrier: every signal array must be non-null and 4-byte "
                             "aligned");
    a.slot[r] = sig->slot[r];
  }
  a.world = sig->world;
  a.rank = sig->rank;
  kvb_peer_barrier_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a, epoch,
                                                                                timeout_ns, status);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return kvb_detail_fail(KVB_ERR_CUDA, std::string("kvb_peer_barrier: ") + cudaGetErrorString(e));
  return KVB_OK;
}
