// Store-side K/V kernels of the chunk cache, sm_100a:
//
//  * kvb_quantize_store: a freshly encoded chunk's K/V, read straight from the
//    model's per-layer cache tensors, KIVI-quantised to int8 and written into
//    its 16-token blocks of the int8 pool with the float16 / float32 scales --
//    the reference's store path (engine.py:846-850 -> cache_manager.py:164-175
//    -> kv_quantize.py:73-100 -> cpu_paged/chunk_to_blocks.py:57-101) in one
//    launch over all layers.
//  * kvb_cacheblend_fwd: CacheBlend's repair of stitched chunk K/V
//    (cacheblend.py:141-197): per-position cosine deviation between cached and
//    full-context K averaged over layers, the top-k deviated positions above a
//    threshold chosen on the device (radix select, one CTA), and the fresh K/V
//    rows copied over the cached ones there.
//
// Both are HBM-bound byte work: one read of each operand, coalesced, grids
// of many small CTAs.  The per-layer pointer tables travel as __grid_constant__
// kernel parameters (up to 128 layers: ~8 KB, within sm_100's 32 KB limit), so a
// launch needs no host-to-device copy of pointers.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <type_traits>

#include "kvb_attn.h"

int kvb_detail_fail(int code, const std::string& msg);

namespace kvb_store {

// ---- arithmetic in the source dtype ---------------------------------------------------
template <typename T>
struct Num;

template <>
struct Num<__nv_bfloat16> {
  static __device__ __forceinline__ float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ float2 pair(uint32_t u) {
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
  }
};

template <>
struct Num<__half> {
  static __device__ __forceinline__ float round(float x) { return __half2float(__float2half_rn(x)); }
  static __device__ __forceinline__ float load(const __half* p) { return __half2float(*p); }
  static __device__ __forceinline__ float2 pair(uint32_t u) {
    __half2 h;
    memcpy(&h, &u, 4);
    return __half22float2(h);
  }
};

// scale = round(round(max(amax, 1e-8)) / 127): torch evaluates each step of
// kv_quantize.py:84-86 in float32 and rounds the result to the tensor's dtype.
template <typename T>
__device__ __forceinline__ float kivi_scale(float amax) {
  const float m = Num<T>::round(fmaxf(amax, 1e-8f));
  return Num<T>::round(__fdiv_rn(m, 127.0f));
}

// q = clamp(rint(round(x / scale)), -128, 127); NaN (0 / 0 on an all-zero
// float16 row) becomes 0, as the reference's float-to-int8 cast gives on its CPU.
template <typename T>
__device__ __forceinline__ int8_t kivi_q(float x, float scale) {
  const float r = Num<T>::round(__fdiv_rn(x, scale));
  if (isnan(r)) return 0;
  const float q = fminf(fmaxf(rintf(r), -128.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(q));
}

// ---- quantise-on-store ----------------------------------------------------------------
struct QStoreArgs {
  const void* src_k[KVB_MAX_LAYERS];
  const void* src_v[KVB_MAX_LAYERS];
  int8_t* pool[KVB_MAX_LAYERS];
  __half* ks16[KVB_MAX_LAYERS];
  __half* vs16[KVB_MAX_LAYERS];
  float* ks32[KVB_MAX_LAYERS];
  float* vs32[KVB_MAX_LAYERS];
  int32_t block_ids[KVB_MAX_CHUNK_BLOCKS];
  int64_t src_head_stride, src_row_stride;
  int32_t L, H, S, nblk;
};

constexpr int kQThreads = 1024;
constexpr int kQWarps = kQThreads / 32;
constexpr int kQRowsInFlight = 4;   // K rows a warp loads before reducing any of them

__device__ __forceinline__ float2 load_pair(const void* p, bool bf16) {
  const uint32_t u = *static_cast<const uint32_t*>(p);
  if (bf16) return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
  __half2 h;
  memcpy(&h, &u, 4);
  return __half22float2(h);
}

template <typename T>
__device__ __forceinline__ uint16_t kivi_q2(float2 x, float sx, float sy) {
  return static_cast<uint16_t>(static_cast<uint8_t>(kivi_q<T>(x.x, sx)) |
                               (static_cast<uint32_t>(static_cast<uint8_t>(kivi_q<T>(x.y, sy))) << 8));
}

// One launch per chunk, all layers: grid (K|V, kv head, layer), one CTA of 1024
// threads each -- one wave for a 36-layer x 2-head chunk, every CTA's loads in
// flight at once.  K CTA: each warp takes rows w, w + 32, ... (kQRowsInFlight at a
// time, loads first), amax over head_dim by shuffles, one scale per token, slots
// of the last block past the chunk's end zeroed.  V CTA: thread = (column pair,
// token phase); each column's amax over the chunk's tokens is reduced over the
// phases in shared memory, then the CTA quantises the rows (re-read from L1).
// Loads are 4-byte column pairs, coalesced along the row.
template <typename T, int D>
__global__ void __launch_bounds__(kQThreads) kvb_quantize_store_kernel(const __grid_constant__ QStoreArgs a) {
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int kPairs = D / 2;
  const int h = blockIdx.y, layer = blockIdx.z, H = a.H, S = a.S, slots = a.nblk * 16;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int8_t* pool = a.pool[layer];
  if (blockIdx.x == 0) {
    constexpr int kIters = (kPairs + 31) / 32;
    const T* src = static_cast<const T*>(a.src_k[layer]) + h * a.src_head_stride;
    __half* ks16 = a.ks16[layer];
    float* ks32 = a.ks32[layer];
    for (int t0 = warp; t0 < slots; t0 += kQWarps * kQRowsInFlight) {
      float2 x[kQRowsInFlight][kIters];
#pragma unroll
      for (int r = 0; r < kQRowsInFlight; ++r) {
        const int t = t0 + r * kQWarps;
#pragma unroll
        for (int j = 0; j < kIters; ++j) {
          const int pr = lane + 32 * j;
          x[r][j] = (t < S && pr < kPairs) ? load_pair(src + t * a.src_row_stride + 2 * pr, kBf16)
                                           : make_float2(0.0f, 0.0f);
        }
      }
#pragma unroll
      for (int r = 0; r < kQRowsInFlight; ++r) {
        const int t = t0 + r * kQWarps;
        if (t >= slots) break;
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < kIters; ++j) amax = fmaxf(amax, fmaxf(fabsf(x[r][j].x), fabsf(x[r][j].y)));
#pragma unroll
        for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const bool live = t < S;
        const float scale = live ? kivi_scale<T>(amax) : 0.0f;
        const int blk = a.block_ids[t >> 4], slot = t & 15;
        int8_t* dst = pool + ((static_cast<int64_t>(blk) * 2 + 0) * H + h) * 16 * D + slot * D;
#pragma unroll
        for (int j = 0; j < kIters; ++j) {
          const int pr = lane + 32 * j;
          if (pr < kPairs)
            *reinterpret_cast<uint16_t*>(dst + 2 * pr) = live ? kivi_q2<T>(x[r][j], scale, scale) : uint16_t(0);
        }
        if (lane == 0) {
          const __half s16 = __float2half_rn(scale);
          const int64_t si = (static_cast<int64_t>(blk) * H + h) * 16 + slot;
          if (ks16) ks16[si] = s16;
          if (ks32) ks32[si] = __half2float(s16);
        }
      }
    }
    return;
  }
  // ---- V ----
  constexpr int kPhases = kQThreads / kPairs;   // 32 (D 64), 21 (D 96), 16 (D 128)
  __shared__ float part[kPhases][D];
  const int pr = threadIdx.x % kPairs, phase = threadIdx.x / kPairs;
  const bool active = phase < kPhases;
  const int col = 2 * pr;
  const T* src = static_cast<const T*>(a.src_v[layer]) + h * a.src_head_stride + col;
  if (active) {
    float ax = 0.0f, ay = 0.0f;
#pragma unroll 8
    for (int t = phase; t < S; t += kPhases) {
      const float2 x = load_pair(src + t * a.src_row_stride, kBf16);
      ax = fmaxf(ax, fabsf(x.x));
      ay = fmaxf(ay, fabsf(x.y));
    }
    part[phase][col] = ax;
    part[phase][col + 1] = ay;
  }
  __syncthreads();
  if (!active) return;
  float ax = 0.0f, ay = 0.0f;
#pragma unroll
  for (int ph = 0; ph < kPhases; ++ph) {
    ax = fmaxf(ax, part[ph][col]);
    ay = fmaxf(ay, part[ph][col + 1]);
  }
  const float sx = kivi_scale<T>(ax), sy = kivi_scale<T>(ay);
#pragma unroll 4
  for (int t = phase; t < slots; t += kPhases) {
    const uint16_t w = t < S ? kivi_q2<T>(load_pair(src + t * a.src_row_stride, kBf16), sx, sy) : uint16_t(0);
    const int blk = a.block_ids[t >> 4], slot = t & 15;
    *reinterpret_cast<uint16_t*>(pool + ((static_cast<int64_t>(blk) * 2 + 1) * H + h) * 16 * D + slot * D + col) = w;
  }
  const __half2 s16 = __halves2half2(__float2half_rn(sx), __float2half_rn(sy));
  const float2 s32 = __half22float2(s16);
  __half* vs16 = a.vs16[layer];
  float* vs32 = a.vs32[layer];
  for (int b = phase; b < a.nblk; b += kPhases) {
    const int64_t si = (static_cast<int64_t>(a.block_ids[b]) * H + h) * D + col;
    if (vs16) *reinterpret_cast<__half2*>(vs16 + si) = s16;
    if (vs32) *reinterpret_cast<float2*>(vs32 + si) = s32;
  }
}

// ---- CacheBlend -----------------------------------------------------------------------
struct BlendArgs {
  void* ck[KVB_MAX_LAYERS];
  void* cv[KVB_MAX_LAYERS];
  const void* fk[KVB_MAX_LAYERS];
  const void* fv[KVB_MAX_LAYERS];
  int64_t c_hs, c_rs, f_hs, f_rs;
  float* deviation;
  int32_t* selected;
  int32_t* num_selected;
  int32_t L, H, S, k;
};

constexpr int kDevWarps = 8;   // positions per CTA in the deviation kernel
constexpr int kLayerUnroll = 4;

// One warp per cached position: for each layer, dot(c, f), |c|^2, |f|^2 over
// the position's K vectors of every head (16-byte loads, kLayerUnroll layers in
// flight), reduced across the warp; deviation = mean over layers of 1 - cos.
template <typename T, int D>
__global__ void __launch_bounds__(kDevWarps * 32) kvb_blend_deviation_kernel(const __grid_constant__ BlendArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * kDevWarps + warp;
  if (t >= a.S) return;
  constexpr int VPH = D / 8;   // 16-byte vectors per head row
  const int nvec = a.H * VPH;
  float dev_sum = 0.0f;
  for (int l0 = 0; l0 < a.L; l0 += kLayerUnroll) {
    float dot[kLayerUnroll], nc[kLayerUnroll], nf[kLayerUnroll];
#pragma unroll
    for (int u = 0; u < kLayerUnroll; ++u) dot[u] = nc[u] = nf[u] = 0.0f;
    for (int v = lane; v < nvec; v += 32) {
      const int h = v / VPH, dv = (v - h * VPH) * 8;
#pragma unroll
      for (int u = 0; u < kLayerUnroll; ++u) {
        if (l0 + u < a.L) {
          const T* c = static_cast<const T*>(a.ck[l0 + u]) + h * a.c_hs + t * a.c_rs + dv;
          const T* f = static_cast<const T*>(a.fk[l0 + u]) + h * a.f_hs + t * a.f_rs + dv;
          const uint4 cu = *reinterpret_cast<const uint4*>(c);
          const uint4 fu = *reinterpret_cast<const uint4*>(f);
          const uint32_t cw[4] = {cu.x, cu.y, cu.z, cu.w}, fw[4] = {fu.x, fu.y, fu.z, fu.w};
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const float2 x = Num<T>::pair(cw[w]), y = Num<T>::pair(fw[w]);
            dot[u] = fmaf(x.x, y.x, fmaf(x.y, y.y, dot[u]));
            nc[u] = fmaf(x.x, x.x, fmaf(x.y, x.y, nc[u]));
            nf[u] = fmaf(y.x, y.x, fmaf(y.y, y.y, nf[u]));
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kLayerUnroll; ++u) {
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        dot[u] += __shfl_xor_sync(0xffffffffu, dot[u], o);
        nc[u] += __shfl_xor_sync(0xffffffffu, nc[u], o);
        nf[u] += __shfl_xor_sync(0xffffffffu, nf[u], o);
      }
      if (l0 + u < a.L) {
        const float cosv = dot[u] / (fmaxf(sqrtf(nc[u]), 1e-8f) * fmaxf(sqrtf(nf[u]), 1e-8f));
        dev_sum += 1.0f - cosv;
      }
    }
  }
  if (lane == 0) a.deviation[t] = dev_sum / static_cast<float>(a.L);
}

// Total order on float bit patterns (larger float -> larger key).
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kSelThreads = 1024;

// Exclusive prefix sum over the CTA; *total gets the CTA's sum.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* warp_tot, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_tot[lane] = w;
  }
  __syncthreads();
  const uint32_t excl = x - v + (warp ? warp_tot[warp - 1] : 0u);
  *total = warp_tot[31];
  __syncthreads();
  return excl;
}

// One CTA: count the candidates (deviation > min_deviation), find the key of the
// kk-th largest candidate by a 4 x 8-bit radix select, then emit, in position
// order, every candidate above that key and the first `remaining` equal to it.
__global__ void __launch_bounds__(kSelThreads) kvb_blend_select_kernel(const float* __restrict__ dev, int S, int k,
                                                                        float min_dev, int32_t* selected,
                                                                        int32_t* num_selected) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t warp_tot[32];
  __shared__ uint32_t s_prefix, s_remaining;
  const int tid = threadIdx.x;

  uint32_t cnt = 0;
  for (int i = tid; i < S; i += kSelThreads) cnt += dev[i] > min_dev ? 1u : 0u;
  uint32_t total;
  block_exclusive_scan(cnt, warp_tot, &total);
  const uint32_t kk = min(static_cast<uint32_t>(k), total);
  if (kk == 0) {
    for (int j = tid; j < k; j += kSelThreads) selected[j] = -1;
    if (tid == 0) *num_selected = 0;
    return;
  }

  uint32_t prefix = 0, mask = 0, remaining = kk;
  const int lane = tid & 31;
  for (int shift = 24; shift >= 0; shift -= 8) {
    if (tid < 256) hist[tid] = 0;
    __syncthreads();
    for (int i0 = 0; i0 < S; i0 += kSelThreads) {
      const int i = i0 + tid;
      bool in = false;
      uint32_t bin = 0;
      if (i < S) {
        const float x = dev[i];
        const uint32_t key = order_key(x);
        in = x > min_dev && (key & mask) == prefix;
        bin = (key >> shift) & 255u;
      }
      // one shared atomic per distinct bin in the warp (deviations cluster in few bins)
      const uint32_t active = __ballot_sync(0xffffffffu, in);
      if (in) {
        const uint32_t peers = __match_any_sync(active, bin);
        if (lane == __ffs(peers) - 1) atomicAdd(&hist[bin], static_cast<uint32_t>(__popc(peers)));
      }
    }
    __syncthreads();
    if (tid < 32) {
      // lane l owns bins 255 - 8l .. 248 - 8l; find the bin holding the remaining-th
      // largest by a suffix scan over lanes from the top bin down
      uint32_t c[8], sum = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hist[255 - 8 * lane - j];
        sum += c[j];
      }
      uint32_t incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const uint32_t hit = __ballot_sync(0xffffffffu, incl >= remaining);
      const int owner = hit ? __ffs(hit) - 1 : 31;
      if (lane == owner) {
        uint32_t rem = remaining - (incl - sum);
        int b = 255 - 8 * lane;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (c[j] >= rem || j == 7) {
            b = 255 - 8 * lane - j;
            break;
          }
          rem -= c[j];
        }
        s_prefix = prefix | (static_cast<uint32_t>(b) << shift);
        s_remaining = rem;
      }
    }
    __syncthreads();
    prefix = s_prefix;
    remaining = s_remaining;
    mask |= 255u << shift;
  }
  const uint32_t kth = prefix;   // key of the kk-th largest; `remaining` of its equals are taken

  uint32_t base_sel = 0, base_eq = 0;
  for (int start = 0; start < S; start += kSelThreads) {
    const int i = start + tid;
    bool gt = false, eq = false;
    if (i < S) {
      const float x = dev[i];
      const uint32_t key = order_key(x);
      const bool cand = x > min_dev;
      gt = cand && key > kth;
      eq = cand && key == kth;
    }
    uint32_t eq_total, sel_total;
    const uint32_t eq_excl = block_exclusive_scan(eq ? 1u : 0u, warp_tot, &eq_total);
    const bool take = gt || (eq && base_eq + eq_excl < remaining);
    const uint32_t sel_excl = block_exclusive_scan(take ? 1u : 0u, warp_tot, &sel_total);
    const uint32_t out = base_sel + sel_excl;
    if (take && out < kk) selected[out] = i;
    base_sel += sel_total;
    base_eq += eq_total;
  }
  for (int j = static_cast<int>(kk) + tid; j < k; j += kSelThreads) selected[j] = -1;
  if (tid == 0) *num_selected = static_cast<int32_t>(kk);
}

constexpr int kPatchSlots = 16;  // chosen positions per CTA
constexpr int kPatchThreads = 256;

// Grid (chosen-position groups, layer): 16-byte copies of the fresh K and V
// rows of every head over the cached ones; groups past *num_selected exit.
template <typename T, int D>
__global__ void __launch_bounds__(kPatchThreads) kvb_blend_patch_kernel(const __grid_constant__ BlendArgs a) {
  const int n = *a.num_selected;
  const int layer = blockIdx.y;
  if (static_cast<int>(blockIdx.x) * kPatchSlots >= n) return;
  constexpr int VPH = D / 8;
  const int per_kv = a.H * VPH, per_slot = 2 * per_kv;
  for (int idx = threadIdx.x; idx < kPatchSlots * per_slot; idx += kPatchThreads) {
    const int j = blockIdx.x * kPatchSlots + idx / per_slot;
    if (j >= n) break;
    const int r = idx % per_slot;
    const int kv = r / per_kv, hv = r - kv * per_kv;
    const int h = hv / VPH, dv = (hv - h * VPH) * 8;
    const int t = a.selected[j];
    const T* src = static_cast<const T*>(kv ? a.fv[layer] : a.fk[layer]) + h * a.f_hs + t * a.f_rs + dv;
    T* dst = static_cast<T*>(kv ? a.cv[layer] : a.ck[layer]) + h * a.c_hs + t * a.c_rs + dv;
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
  }
}

// ---- host side ------------------------------------------------------------------------
int fail(int code, const std::string& msg) { return kvb_detail_fail(code, msg); }

bool head_dim_ok(int d) { return d == 64 || d == 96 || d == 128; }

template <typename T, int D>
cudaError_t launch_qstore(const QStoreArgs& a, int L, cudaStream_t s) {
  kvb_quantize_store_kernel<T, D><<<dim3(2, a.H, L), kQThreads, 0, s>>>(a);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_qstore_d(const QStoreArgs& a, int L, int D, cudaStream_t s) {
  switch (D) {
    case 64: return launch_qstore<T, 64>(a, L, s);
    case 96: return launch_qstore<T, 96>(a, L, s);
    default: return launch_qstore<T, 128>(a, L, s);
  }
}

template <typename T, int D>
cudaError_t launch_blend(const BlendArgs& a, float min_dev, bool patch, cudaStream_t s) {
  kvb_blend_deviation_kernel<T, D><<<(a.S + kDevWarps - 1) / kDevWarps, kDevWarps * 32, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  kvb_blend_select_kernel<<<1, kSelThreads, 0, s>>>(a.deviation, a.S, a.k, min_dev, a.selected, a.num_selected);
  e = cudaGetLastError();
  if (e != cudaSuccess || !patch) return e;
  kvb_blend_patch_kernel<T, D><<<dim3((a.k + kPatchSlots - 1) / kPatchSlots, a.L), kPatchThreads, 0, s>>>(a);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_blend_d(const BlendArgs& a, int D, float min_dev, bool patch, cudaStream_t s) {
  switch (D) {
    case 64: return launch_blend<T, 64>(a, min_dev, patch, s);
    case 96: return launch_blend<T, 96>(a, min_dev, patch, s);
    default: return launch_blend<T, 128>(a, min_dev, patch, s);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace kvb_store

using namespace kvb_store;

extern "C" int kvb_quantize_store(const KvbQuantizeStoreParams* p, void* stream) {
  if (!p) return fail(KVB_ERR_INVALID, "params is NULL");
  if (p->dtype != KVB_DTYPE_BF16 && p->dtype != KVB_DTYPE_FP16)
    return fail(KVB_ERR_INVALID, "dtype must be KVB_DTYPE_BF16 or KVB_DTYPE_FP16");
  if (!head_dim_ok(p->head_dim)) return fail(KVB_ERR_INVALID, "head_dim must be 64, 96 or 128");
  if (p->num_layers < 1 || p->num_layers > KVB_MAX_LAYERS)
    return fail(KVB_ERR_INVALID, "num_layers must be in [1, " + std::to_string(KVB_MAX_LAYERS) + "]");
  if (p->num_kv_heads < 1 || p->num_kv_heads > 65535) return fail(KVB_ERR_INVALID, "num_kv_heads must be in [1, 65535]");
  if (p->num_tokens < 1) return fail(KVB_ERR_INVALID, "num_tokens must be >= 1");
  const int need = (p->num_tokens + 15) / 16;
  if (p->num_chunk_blocks < need || p->num_chunk_blocks > KVB_MAX_CHUNK_BLOCKS)
    return fail(KVB_ERR_INVALID, "num_chunk_blocks must be in [ceil(num_tokens / 16) = " + std::to_string(need) +
                                     ", " + std::to_string(KVB_MAX_CHUNK_BLOCKS) + "]");
  if (p->src_row_stride < 1 || p->src_head_stride < 0 || (p->src_row_stride | p->src_head_stride) & 1)
    return fail(KVB_ERR_INVALID, "src_row_stride must be >= 1, src_head_stride >= 0, both even");
  if (!p->src_k || !p->src_v || !p->pool) return fail(KVB_ERR_INVALID, "src_k, src_v and pool must be non-null");
  for (int b = 0; b < p->num_chunk_blocks; ++b) {
    const int id = p->block_ids[b];
    if (id < 0 || id >= p->num_pool_blocks)
      return fail(KVB_ERR_INVALID, "block_ids[" + std::to_string(b) + "] = " + std::to_string(id) +
                                       " is outside the pool [0, " + std::to_string(p->num_pool_blocks) + ")");
    for (int c = 0; c < b; ++c)
      if (p->block_ids[c] == id) return fail(KVB_ERR_INVALID, "block_ids repeat block " + std::to_string(id));
  }
  QStoreArgs a{};
  for (int l = 0; l < p->num_layers; ++l) {
    if (!p->src_k[l] || !p->src_v[l] || !p->pool[l])
      return fail(KVB_ERR_INVALID, "layer " + std::to_string(l) + ": src_k, src_v and pool pointers must be non-null");
    if ((reinterpret_cast<uintptr_t>(p->src_k[l]) | reinterpret_cast<uintptr_t>(p->src_v[l])) & 3u)
      return fail(KVB_ERR_INVALID, "layer " + std::to_string(l) + ": source pointers must be 4-byte aligned");
    a.src_k[l] = p->src_k[l];
    a.src_v[l] = p->src_v[l];
    a.pool[l] = static_cast<int8_t*>(p->pool[l]);
    a.ks16[l] = p->k_scale16 ? static_cast<__half*>(p->k_scale16[l]) : nullptr;
    a.vs16[l] = p->v_scale16 ? static_cast<__half*>(p->v_scale16[l]) : nullptr;
    a.ks32[l] = p->k_scale ? static_cast<float*>(p->k_scale[l]) : nullptr;
    a.vs32[l] = p->v_scale ? static_cast<float*>(p->v_scale[l]) : nullptr;
  }
  for (int b = 0; b < p->num_chunk_blocks; ++b) a.block_ids[b] = p->block_ids[b];
  a.src_head_stride = p->src_head_stride;
  a.src_row_stride = p->src_row_stride;
  a.L = p->num_layers;
  a.H = p->num_kv_heads;
  a.S = p->num_tokens;
  a.nblk = p->num_chunk_blocks;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t e = p->dtype == KVB_DTYPE_BF16 ? launch_qstore_d<__nv_bfloat16>(a, p->num_layers, p->head_dim, s)
                                                   : launch_qstore_d<__half>(a, p->num_layers, p->head_dim, s);
  if (e != cudaSuccess) return fail(KVB_ERR_CUDA, std::string("kvb_quantize_store launch: ") + cudaGetErrorString(e));
  return KVB_OK;
}

extern "C" int kvb_cacheblend_fwd(const KvbCacheBlendParams* p, void* stream) {
  if (!p) return fail(KVB_ERR_INVALID, "params is NULL");
  if (p->dtype != KVB_DTYPE_BF16 && p->dtype != KVB_DTYPE_FP16)
    return fail(KVB_ERR_INVALID, "dtype must be KVB_DTYPE_BF16 or KVB_DTYPE_FP16");
  if (!head_dim_ok(p->head_dim)) return fail(KVB_ERR_INVALID, "head_dim must be 64, 96 or 128");
  if (p->num_layers < 1 || p->num_layers > KVB_MAX_LAYERS)
    return fail(KVB_ERR_INVALID, "num_layers must be in [1, " + std::to_string(KVB_MAX_LAYERS) + "]");
  if (p->num_kv_heads < 1) return fail(KVB_ERR_INVALID, "num_kv_heads must be >= 1");
  if (p->num_tokens < 1) return fail(KVB_ERR_INVALID, "num_tokens must be >= 1");
  if (p->num_select < 1) return fail(KVB_ERR_INVALID, "num_select must be >= 1");
  if (p->patch != 0 && p->patch != 1) return fail(KVB_ERR_INVALID, "patch must be 0 or 1");
  if (!p->cached_k || !p->fresh_k || (p->patch && (!p->cached_v || !p->fresh_v)))
    return fail(KVB_ERR_INVALID, "cached_k and fresh_k (and, to patch, cached_v and fresh_v) must be non-null");
  if (!p->deviation || !p->selected || !p->num_selected)
    return fail(KVB_ERR_INVALID, "deviation, selected and num_selected must be non-null");
  const int64_t strides[4] = {p->cached_head_stride, p->cached_row_stride, p->fresh_head_stride, p->fresh_row_stride};
  for (int64_t st : strides)
    if (st < 0 || st % 8) return fail(KVB_ERR_INVALID, "strides must be non-negative multiples of 8 elements");
  if (p->cached_row_stride == 0 || p->fresh_row_stride == 0) return fail(KVB_ERR_INVALID, "row strides must be non-zero");
  BlendArgs a{};
  for (int l = 0; l < p->num_layers; ++l) {
    const void* ptrs[4] = {p->cached_k[l], p->fresh_k[l], p->patch ? p->cached_v[l] : nullptr,
                           p->patch ? p->fresh_v[l] : nullptr};
    for (int i = 0; i < (p->patch ? 4 : 2); ++i)
      if (!ptrs[i] || !aligned16(ptrs[i]))
        return fail(KVB_ERR_INVALID, "layer " + std::to_string(l) + ": K/V pointers must be non-null and 16-byte aligned");
    a.ck[l] = p->cached_k[l];
    a.fk[l] = p->fresh_k[l];
    a.cv[l] = p->patch ? p->cached_v[l] : nullptr;
    a.fv[l] = p->patch ? p->fresh_v[l] : nullptr;
  }
  a.c_hs = p->cached_head_stride;
  a.c_rs = p->cached_row_stride;
  a.f_hs = p->fresh_head_stride;
  a.f_rs = p->fresh_row_stride;
  a.deviation = p->deviation;
  a.selected = p->selected;
  a.num_selected = p->num_selected;
  a.L = p->num_layers;
  a.H = p->num_kv_heads;
  a.S = p->num_tokens;
  a.k = p->num_select;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t e =
      p->dtype == KVB_DTYPE_BF16 ? launch_blend_d<__nv_bfloat16>(a, p->head_dim, p->min_deviation, p->patch, s)
                                 : launch_blend_d<__half>(a, p->head_dim, p->min_deviation, p->patch, s);
  if (e != cudaSuccess) return fail(KVB_ERR_CUDA, std::string("kvb_cacheblend_fwd launch: ") + cudaGetErrorString(e));
  return KVB_OK;
}
