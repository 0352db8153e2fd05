// kvb_paged_prefill_fwd_noalloc: the int8 paged reuse prefill with its
// dequantised-prefix workspace in a fixed static device array.
//
// Callers that cannot allocate on the request path use it: a serving loop
// whose device memory is planned up front (every byte reserved before the
// first request, so a per-call cudaMalloc would break the plan or stall
// behind other streams), and code running between a caching allocator's pool
// reservation and its release, where a new allocation would grow the pool.
// Nothing here calls cudaMalloc/cudaFree or an allocating library routine.
//
// The array lives in this library's module.  Under lazy module loading (the
// default since CUDA 12.2, CUDA_MODULE_LOADING=LAZY) a process reserves it on
// a device only once something in the module runs or is looked up there; with
// CUDA_MODULE_LOADING=EAGER every process that loads the library reserves the
// 32 MiB on each device it uses.  The first call on a device looks up its
// address with cudaGetSymbolAddress, which loads the module on that device;
// make that call before any stream capture.  The address is kept per device
// together with the context it belongs to: after a context teardown
// (cudaDeviceReset) the next call looks it up again in the new context, so,
// like the first call, it should come before any stream capture.  Every call
// on a device shares the one array: calls that overlap in time (different
// streams or host threads) race on it.

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "kvb_attn.h"

int64_t kvb_detail_paged_materialize_bytes(const KvbPagedPrefillParams& p);
int kvb_detail_paged_prefill_scratch(const KvbPagedPrefillParams& p, void* scratch,
                                     int64_t scratch_bytes, cudaStream_t s);
int kvb_detail_fail(int code, const std::string& msg);

// Dequantised K/V of the prefix plus the fresh suffix, [2][batch][kv_heads][kv_pad][D].
static __device__ __align__(256) unsigned char g_noalloc_scratch[KVB_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};

using CtxGetCurrent = CUresult (*)(CUcontext*);

// cuCtxGetCurrent through the runtime's driver entry point (no link to libcuda).
CtxGetCurrent ctx_get_current() {
  static CtxGetCurrent fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrent>(p);
  });
  return fn;
}

// Address of this device's copy of the scratch, looked up with that device
// current once per device and context.
int scratch_for_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return kvb_detail_fail(KVB_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return kvb_detail_fail(KVB_ERR_UNSUPPORTED, "device ordinal " + std::to_string(dev) +
                                                    " is beyond the scratch table");
  CtxGetCurrent get_ctx = ctx_get_current();
  CUcontext ctx = nullptr;
  if (get_ctx == nullptr || get_ctx(&ctx) != CUDA_SUCCESS)
    return kvb_detail_fail(KVB_ERR_CUDA, "cuCtxGetCurrent is not available");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr || g_scratch_ctx[dev] != ctx) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return kvb_detail_fail(KVB_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") +
                                               cudaGetErrorString(e));
    g_scratch_ptr[dev] = ptr;
    g_scratch_ctx[dev] = ctx;
  }
  *out = g_scratch_ptr[dev];
  return KVB_OK;
}

}  // namespace

extern "C" int kvb_paged_prefill_fwd_noalloc(const KvbPagedPrefillParams* params, void* stream) {
  if (!params) return kvb_detail_fail(KVB_ERR_INVALID, "params is NULL");
  const int64_t need = kvb_detail_paged_materialize_bytes(*params);
  if (need < 0) return (int)(-need);
  if (need > KVB_NOALLOC_SCRATCH_BYTES)
    return kvb_detail_fail(
        KVB_ERR_UNSUPPORTED,
        "kvb_paged_prefill_fwd_noalloc: these params need " + std::to_string(need) +
            " bytes of scratch (2 * batch * num_kv_heads * round_up(prefix_len + q_len, 128) * "
            "head_dim * 2); the static scratch holds " +
            std::to_string((long long)KVB_NOALLOC_SCRATCH_BYTES) + " bytes (32 MiB)");
  if (need == 0) return KVB_OK;   // q_len == 0: nothing to compute
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != KVB_OK) return rc;
  return kvb_detail_paged_prefill_scratch(*params, scratch, KVB_NOALLOC_SCRATCH_BYTES,
                                          reinterpret_cast<cudaStream_t>(stream));
}
