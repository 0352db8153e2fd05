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

// q = clamp(rint(round(x / scale)), -128, 127) for scale > 0 (x finite): the
// reference's kv_quantize.py:86 / :91 with torch's rounding of the quotient to the
// tensor's dtype.  Fast path, no conversion instructions: y = x * (1 / scale) is
// within 3 float32 ulps of the correctly rounded quotient (two roundings of 2^-24
// each against one), i.e. within 6 ulps of y's own binade.  For |y| >= 0.25 both
// are normal in bfloat16 and float16, where rounding float32 to T is
// round-to-nearest-even at bit 16 (bf16) / bit 13 (fp16) of the float32 pattern;
// when y's dropped bits are more than 8 ulps from the halfway point, the quotient
// rounds to the same T value as y, computed here with integer operations.  rint of
// that value (exact in float32, |value| < 2^22) is the low word of value +
// 1.5 * 2^23.  Near a halfway point the quotient is computed exactly.  |y| < 0.25
// gives 0 outright (the quotient is below 0.26).
template <typename T>
struct RoundBits;

template <>
struct RoundBits<__nv_bfloat16> {
  static constexpr uint32_t kDrop = 16;
};

template <>
struct RoundBits<__half> {
  static constexpr uint32_t kDrop = 13;
};

__device__ __forceinline__ int rint_small(float v) {   // round half to even, |v| < 2^22
  return __float_as_int(v + 12582912.0f) - 0x4B400000;
}

template <typename T>
__device__ __forceinline__ int kivi_q_pos(float x, float scale, float rcp) {
  constexpr uint32_t kDrop = RoundBits<T>::kDrop, kHalf = 1u << (kDrop - 1), kMask = (1u << kDrop) - 1;
  const float y = x * rcp;
  if (fabsf(y) < 0.25f) return 0;
  const uint32_t u = __float_as_uint(y);
  int q;
  if (static_cast<uint32_t>(abs(static_cast<int>(u & kMask) - static_cast<int>(kHalf))) > 8u) {
    const uint32_t r = (u + (kHalf - 1) + ((u >> kDrop) & 1u)) & ~kMask;   // round to T, nearest even
    q = rint_small(__uint_as_float(r));
  } else {
    q = __float2int_rn(Num<T>::round(__fdiv_rn(x, scale)));
  }
  return min(max(q, -128), 127);
}

// scale == 0 (an all-zero float16 row, or amax so small that amax / 127 rounds to
// 0 in float16): x / 0 is +-inf -> 127 / -128, and 0 / 0 is NaN, which the
// reference's float-to-int8 cast turns into 0 on its CPU.
__device__ __forceinline__ int kivi_q_zero_scale(float x) { return x > 0.0f ? 127 : (x < 0.0f ? -128 : 0); }

template <typename T>
__device__ __forceinline__ int kivi_q(float x, float scale, float rcp) {
  return scale > 0.0f ? kivi_q_pos<T>(x, scale, rcp) : kivi_q_zero_scale(x);
}

// kivi_q of 8 elements packed as 8 int8 bytes, branch-free on the fast path:
// each element is rounded to T with integer operations, clamped to [-128, 127]
// in float (the same as clamping after rint: T values >= 127.5 are the only ones
// that rint above 127), and t + 1.5 * 2^23 carries rint(t) in its low byte.  If
// any element's quotient lies within 8 ulps of a halfway point, or a scale is 0
// (zero_scale), all 8 are redone by kivi_q (rare).  Rounding y of |y| < 0.25 with
// the float16 rule is inexact in float16's subnormal range, but rint of it is 0
// either way.
// 8 int8 values packed little-endian into two words.
__device__ __forceinline__ uint2 pack8(const int (&q)[8]) {
  uint2 r;
  r.x = __byte_perm(__byte_perm(q[0], q[1], 0x0040), __byte_perm(q[2], q[3], 0x0040), 0x5410);
  r.y = __byte_perm(__byte_perm(q[4], q[5], 0x0040), __byte_perm(q[6], q[7], 0x0040), 0x5410);
  return r;
}

// The exact path for 8 elements, out of line: it runs rarely and its IEEE
// divisions would otherwise raise the fast path's register count.
template <typename T>
__device__ __noinline__ uint2 kivi_q8_exact(const float4 x0, const float4 x1, const float4 s0, const float4 s1,
                                            const float4 r0, const float4 r1) {
  const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
  const float sc[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
  const float rc[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
  int q[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) q[e] = kivi_q<T>(x[e], sc[e], rc[e]);
  return pack8(q);
}

// a * b + c (mod 2^32) as one integer multiply-add.
__device__ __forceinline__ uint32_t imad_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint64_t pack_f2(float lo, float hi) {
  return static_cast<uint64_t>(__float_as_uint(lo)) | (static_cast<uint64_t>(__float_as_uint(hi)) << 32);
}

// The fast path of kivi_q8: the 8 packed results, and `near` ORed with whether
// any element needs the exact path.
template <typename T>
__device__ __forceinline__ uint2 kivi_q8_fast(const float (&x)[8], const float (&rc)[8], bool& near) {
  constexpr uint32_t kDrop = RoundBits<T>::kDrop, kHalf = 1u << (kDrop - 1), kMask = (1u << kDrop) - 1;
  uint32_t w[8];
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    // bfloat16: the rounding of y to T by the conversion unit (round to nearest
    // even, as the integer rule above), two at a time; only the upper clamp,
    // since |y| <= 127.3 (scale = amax / 127 rounded to 8 bits, y within 3
    // float32 ulps of the quotient), so rint(T(y)) >= -128.  The halfway test
    // looks at the dropped 16 bits as the top half of (u - (kHalf - 8)) << 16.
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      uint64_t y2;
      asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(y2) : "l"(pack_f2(x[e], x[e + 1])), "l"(pack_f2(rc[e], rc[e + 1])));
      const float y0 = __uint_as_float(static_cast<uint32_t>(y2));
      const float y1 = __uint_as_float(static_cast<uint32_t>(y2 >> 32));
      uint32_t p;
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(y1), "f"(y0));
      asm("min.bf16x2 %0, %0, %1;" : "+r"(p) : "r"(0x42FE42FEu));   // clamp both to 127
      const float t0 = __uint_as_float(imad_u32(p, 65536u, 0u));
      const float t1 = __uint_as_float(p & 0xffff0000u);
      uint64_t r2;
      asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r2) : "l"(pack_f2(t0, t1)), "l"(pack_f2(12582912.0f, 12582912.0f)));
      w[e] = static_cast<uint32_t>(r2);
      w[e + 1] = static_cast<uint32_t>(r2 >> 32);
      constexpr uint32_t kOff = (0u - (kHalf - 8u)) << 16;          // (u - (kHalf - 8)) << 16
      near |= imad_u32(__float_as_uint(y0), 65536u, kOff) <= (16u << 16 | 0xffffu);
      near |= imad_u32(__float_as_uint(y1), 65536u, kOff) <= (16u << 16 | 0xffffu);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t u = __float_as_uint(x[e] * rc[e]);
      const uint32_t r = (u + (kHalf - 1) + ((u >> kDrop) & 1u)) & ~kMask;
      const float t = fminf(fmaxf(__uint_as_float(r), -128.0f), 127.0f);
      w[e] = __float_as_uint(t + 12582912.0f);
      near |= ((u - (kHalf - 8u)) & kMask) <= 16u;     // low bits within 8 of the halfway point
    }
  }
  uint2 p;
  p.x = __byte_perm(__byte_perm(w[0], w[1], 0x0040), __byte_perm(w[2], w[3], 0x0040), 0x5410);
  p.y = __byte_perm(__byte_perm(w[4], w[5], 0x0040), __byte_perm(w[6], w[7], 0x0040), 0x5410);
  return p;
}

template <typename T>
__device__ __forceinline__ uint2 kivi_q8(const float (&x)[8], const float (&sc)[8], const float (&rc)[8],
                                         bool zero_scale) {
  bool near = zero_scale;
  const uint2 p = kivi_q8_fast<T>(x, rc, near);
  if (near)
    return kivi_q8_exact<T>(make_float4(x[0], x[1], x[2], x[3]), make_float4(x[4], x[5], x[6], x[7]),
                            make_float4(sc[0], sc[1], sc[2], sc[3]), make_float4(sc[4], sc[5], sc[6], sc[7]),
                            make_float4(rc[0], rc[1], rc[2], rc[3]), make_float4(rc[4], rc[5], rc[6], rc[7]));
  return p;
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
  int64_t src_head_stride, src_row_stride, num_pool_blocks;
  int32_t L, H, S, nblk;
};

constexpr int kQThreads = 256;                  // several CTAs per SM overlap their chains
constexpr int kQWarps = kQThreads / 32;
constexpr int kQLanesPerRow = 8;                 // K: 8 lanes per token row, 4 rows per warp
constexpr int kQRowsPerWarp = 32 / kQLanesPerRow;
// K: token rows per thread (all loaded before any is reduced).  One row keeps
// the kernel at 58 registers and 4 CTAs per SM; 2 and 4 rows (74 and 116
// registers) measured 9 % and 36 % slower on the 24-chunk store.
constexpr int kQKRows = 1;
constexpr int kQRowsPerCta = kQWarps * kQRowsPerWarp * kQKRows;   // K: 128 token rows per CTA
constexpr int kQVCols = 32;                      // V: 32 columns per CTA (4 pieces x 64 phases)

template <bool kBf16>
__device__ __forceinline__ void unpack8(const uint4& u, float (&x)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f;
    if (kBf16) {
      f = make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
    } else {
      __half2 h;
      memcpy(&h, &w[i], 4);
      f = __half22float2(h);
    }
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}


// One CTA of quantise-on-store: either 32 token rows of K or 32 columns of V of one
// (KV head, layer, chunk).  Sources are read in 16-byte pieces (8 elements).
//  K: a token row per 8 lanes, 4 rows per warp: amax over head_dim (3 shuffle
//    steps), one scale per token, 8 int8 written per lane per piece; slots of the
//    last block past the chunk's end zeroed.
//  V: thread = (8-column piece, token phase); column amax partials go to shared
//    memory, one thread per column reduces them and computes the column's scale
//    and reciprocal once, then every thread quantises its tokens' pieces.
// Block ids outside [0, num_pool_blocks) are skipped and flagged in *status.
struct QStoreUnit {
  const void* src;          // this layer's K or V, element (h, t, d) at src + h*hs + t*rs + d
  int64_t hs, rs;
  const int32_t* block_ids; // the chunk's blocks
  int nblk, S, H;
  int64_t num_pool_blocks;
  int8_t* pool;
  __half* s16;              // K: [blocks][H][16]; V: [blocks][H][D]
  float* s32;
  int* status;
};

__device__ __forceinline__ bool block_ok(int blk, const QStoreUnit& u) {
  if (blk >= 0 && blk < u.num_pool_blocks) return true;
  if (u.status) atomicOr(u.status, KVB_STATUS_BAD_BLOCK);
  return false;
}

template <typename T, int D>
__device__ __forceinline__ void quantize_store_k(const QStoreUnit& u, int h, int row0) {
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int VPR = D / 8;                                   // 16-byte pieces per row
  constexpr int kPieces = (VPR + kQLanesPerRow - 1) / kQLanesPerRow;
  constexpr int kStride = kQWarps * kQRowsPerWarp;             // 32 rows between a thread's rows
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, slots = u.nblk * 16;
  if (row0 + warp * kQRowsPerWarp >= slots) return;            // warp-uniform
  const T* src = static_cast<const T*>(u.src) + h * u.hs;
  const int sub = lane & (kQLanesPerRow - 1);
  const int tr = row0 + warp * kQRowsPerWarp + (lane >> 3);   // this thread's first row
  // every row's pieces are requested before any is reduced
  uint4 w[kQKRows][kPieces];
#pragma unroll
  for (int r = 0; r < kQKRows; ++r) {
    const int t = tr + r * kStride;
#pragma unroll
    for (int c = 0; c < kPieces; ++c) {
      const int piece = sub + kQLanesPerRow * c;
      w[r][c] = (t < u.S && piece < VPR)
                    ? *reinterpret_cast<const uint4*>(src + t * u.rs + 8 * piece)
                    : make_uint4(0, 0, 0, 0);
    }
  }
  float amax[kQKRows];
#pragma unroll
  for (int r = 0; r < kQKRows; ++r) {
    amax[r] = 0.0f;
#pragma unroll
    for (int c = 0; c < kPieces; ++c) {
      float x[8];
      unpack8<kBf16>(w[r][c], x);
#pragma unroll
      for (int e = 0; e < 8; ++e) amax[r] = fmaxf(amax[r], fabsf(x[e]));
    }
  }
#pragma unroll
  for (int o = 1; o < kQLanesPerRow; o <<= 1)
#pragma unroll
    for (int r = 0; r < kQKRows; ++r)
      amax[r] = fmaxf(amax[r], __shfl_xor_sync(0xffffffffu, amax[r], o));
#pragma unroll
  for (int r = 0; r < kQKRows; ++r) {
    const int t = tr + r * kStride;
    if (t >= slots) break;                                     // rows only grow with r
    const bool live = t < u.S;
    const int blk = u.block_ids[t >> 4], slot = t & 15;
    if (!block_ok(blk, u)) continue;
    const float scale = live ? kivi_scale<T>(amax[r]) : 0.0f;
    const float rcp = __frcp_rn(scale);
    int8_t* dst = u.pool + ((static_cast<int64_t>(blk) * 2 + 0) * u.H + h) * 16 * D + slot * D;
    float sc[8], rc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      sc[e] = scale;
      rc[e] = rcp;
    }
#pragma unroll
    for (int c = 0; c < kPieces; ++c) {
      const int piece = sub + kQLanesPerRow * c;
      if (piece < VPR) {
        float x[8];
        unpack8<kBf16>(w[r][c], x);
        *reinterpret_cast<uint2*>(dst + 8 * piece) =
            live ? kivi_q8<T>(x, sc, rc, !(scale > 0.0f)) : make_uint2(0, 0);
      }
    }
    if (sub == 0) {
      const __half s16 = __float2half_rn(scale);
      const int64_t si = (static_cast<int64_t>(blk) * u.H + h) * 16 + slot;
      if (u.s16) u.s16[si] = s16;
      if (u.s32) u.s32[si] = __half2float(s16);
    }
  }
}

template <typename T, int D>
__device__ __forceinline__ void quantize_store_v(const QStoreUnit& u, int h, int col0) {
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int kG = kQVCols / 8;              // 16-byte pieces per CTA row
  constexpr int kPhases = kQThreads / kG;      // 64 token phases
  constexpr int kWarpsV = kQThreads / 32;
  __shared__ float part[kWarpsV][kQVCols];
  __shared__ float col_scale[kQVCols], col_rcp[kQVCols];
  const int g = threadIdx.x % kG, phase = threadIdx.x / kG, slots = u.nblk * 16;
  const T* src = static_cast<const T*>(u.src) + h * u.hs + col0 + 8 * g;
  float m[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  // A chunk of up to 2 * kPhases tokens (the 128-token chunks) stays in registers
  // between the two passes: both of a thread's pieces are loaded before either is
  // reduced, and the quantise pass reads no memory.
  constexpr int kHeld = 2;
  const bool held = u.S <= kHeld * kPhases;
  uint4 keep[kHeld];
  if (held) {
#pragma unroll
    for (int i = 0; i < kHeld; ++i) {
      const int t = phase + i * kPhases;
      keep[i] = t < u.S ? *reinterpret_cast<const uint4*>(src + t * u.rs) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < kHeld; ++i) {
      float x[8];
      unpack8<kBf16>(keep[i], x);
#pragma unroll
      for (int e = 0; e < 8; ++e) m[e] = fmaxf(m[e], fabsf(x[e]));
    }
  } else {
    for (int t = phase; t < u.S; t += kPhases) {
      float x[8];
      unpack8<kBf16>(*reinterpret_cast<const uint4*>(src + t * u.rs), x);
#pragma unroll
      for (int e = 0; e < 8; ++e) m[e] = fmaxf(m[e], fabsf(x[e]));
    }
  }
  // column maxima: over the warp's 8 token phases (lanes g, g + 4, ...) by
  // shuffles, then over the 8 warps through shared memory
#pragma unroll
  for (int o = kG; o < 32; o <<= 1)
#pragma unroll
    for (int e = 0; e < 8; ++e) m[e] = fmaxf(m[e], __shfl_xor_sync(0xffffffffu, m[e], o));
  if ((threadIdx.x & 31) < kG)
#pragma unroll
    for (int e = 0; e < 8; ++e) part[threadIdx.x >> 5][8 * g + e] = m[e];
  __syncthreads();
  if (threadIdx.x < kQVCols) {
    float mx = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarpsV; ++w) mx = fmaxf(mx, part[w][threadIdx.x]);
    const float sc = kivi_scale<T>(mx);
    col_scale[threadIdx.x] = sc;
    col_rcp[threadIdx.x] = __frcp_rn(sc);
    const __half s16 = __float2half_rn(sc);
    for (int b = 0; b < u.nblk; ++b) {
      const int blk = u.block_ids[b];
      if (!block_ok(blk, u)) continue;
      const int64_t si = (static_cast<int64_t>(blk) * u.H + h) * D + col0 + threadIdx.x;
      if (u.s16) u.s16[si] = s16;
      if (u.s32) u.s32[si] = __half2float(s16);
    }
  }
  __syncthreads();
  float sc[8], rc[8];
  bool zero_scale = false;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    sc[e] = col_scale[8 * g + e];
    rc[e] = col_rcp[8 * g + e];
    zero_scale |= !(sc[e] > 0.0f);
  }
  if (held) {
#pragma unroll
    for (int i = 0; i < kHeld; ++i) {
      const int t = phase + i * kPhases;
      if (t >= slots) break;
      const int blk = u.block_ids[t >> 4], slot = t & 15;
      if (!block_ok(blk, u)) continue;
      uint2 q = make_uint2(0, 0);
      if (t < u.S) {
        float x[8];
        unpack8<kBf16>(keep[i], x);
        q = kivi_q8<T>(x, sc, rc, zero_scale);
      }
      *reinterpret_cast<uint2*>(u.pool + ((static_cast<int64_t>(blk) * 2 + 1) * u.H + h) * 16 * D +
                                slot * D + col0 + 8 * g) = q;
    }
    return;
  }
  for (int t = phase; t < slots; t += kPhases) {
    const int blk = u.block_ids[t >> 4], slot = t & 15;
    if (!block_ok(blk, u)) continue;
    uint2 q = make_uint2(0, 0);
    if (t < u.S) {
      float x[8];
      unpack8<kBf16>(*reinterpret_cast<const uint4*>(src + t * u.rs), x);
      q = kivi_q8<T>(x, sc, rc, zero_scale);
    }
    *reinterpret_cast<uint2*>(u.pool + ((static_cast<int64_t>(blk) * 2 + 1) * u.H + h) * 16 * D + slot * D +
                              col0 + 8 * g) = q;
  }
}

// CTA x of a (head, layer[, chunk]): x < n_k -> K rows [32x, 32x + 32), else V
// columns [32 (x - n_k), +32).
template <typename T, int D>
__device__ __forceinline__ void quantize_store_cta(QStoreUnit& u, const void* src_k, const void* src_v,
                                                   __half* ks16, float* ks32, __half* vs16, float* vs32,
                                                   int n_k) {
  const int x = blockIdx.x;
  if (x < n_k) {
    u.src = src_k;
    u.s16 = ks16;
    u.s32 = ks32;
    quantize_store_k<T, D>(u, blockIdx.y, x * kQRowsPerCta);
  } else {
    u.src = src_v;
    u.s16 = vs16;
    u.s32 = vs32;
    quantize_store_v<T, D>(u, blockIdx.y, (x - n_k) * kQVCols);
  }
}

// One chunk, all layers: grid (K row blocks + V column blocks, KV head, layer); the
// pointer tables travel as kernel parameters (block ids checked on the host).
template <typename T, int D>
__global__ void __launch_bounds__(kQThreads) kvb_quantize_store_kernel(const __grid_constant__ QStoreArgs a) {
  const int layer = blockIdx.z;
  QStoreUnit u;
  u.hs = a.src_head_stride;
  u.rs = a.src_row_stride;
  u.block_ids = a.block_ids;
  u.nblk = a.nblk;
  u.S = a.S;
  u.H = a.H;
  u.num_pool_blocks = a.num_pool_blocks;
  u.pool = a.pool[layer];
  u.status = nullptr;
  quantize_store_cta<T, D>(u, a.src_k[layer], a.src_v[layer], a.ks16[layer], a.ks32[layer], a.vs16[layer],
                           a.vs32[layer], (a.nblk * 16 + kQRowsPerCta - 1) / kQRowsPerCta);
}

// Several chunks, all layers, in one launch: grid (K row blocks of the longest
// chunk + V column blocks, KV head, chunk x layer); the per-(chunk, layer) source
// pointers and strides, the pool's per-layer pointers, token counts and block ids
// come from small device tables.
struct QStoreBatchArgs {
  const void* const* src;        // [chunks][layers][2] (K, V)
  void* const* tables;           // [5][layers]: pool, K scale16, V scale16, K scale32, V scale32
  const int32_t* num_tokens;     // [chunks]
  const int32_t* block_ids;      // [chunks][max_blocks]
  const int64_t* src_strides;    // [chunks][2]: head, row
  int64_t num_pool_blocks;
  int32_t L, H, max_blocks;
  int* status;
};

template <typename T, int D>
__global__ void __launch_bounds__(kQThreads) kvb_quantize_store_batch_kernel(const QStoreBatchArgs a) {
  const int chunk = blockIdx.z / a.L, layer = blockIdx.z - chunk * a.L;
  const int n_k = (a.max_blocks * 16 + kQRowsPerCta - 1) / kQRowsPerCta;
  QStoreUnit u;
  u.S = a.num_tokens[chunk];
  u.nblk = (u.S + 15) / 16;
  const int64_t si = (static_cast<int64_t>(chunk) * a.L + layer) * 2;
  const void* src_k = a.src[si];
  const void* src_v = a.src[si + 1];
  u.hs = a.src_strides[2 * chunk];
  u.rs = a.src_strides[2 * chunk + 1];
  // checked here: the tables are device memory the host did not validate
  if (u.S < 1 || u.nblk > a.max_blocks || u.hs < 0 || u.rs < 1 || ((u.hs | u.rs) & 7) ||
      ((reinterpret_cast<uintptr_t>(src_k) | reinterpret_cast<uintptr_t>(src_v)) & 15)) {
    if (threadIdx.x == 0 && a.status) atomicOr(a.status, KVB_STATUS_BAD_LENGTH);
    return;
  }
  if ((int)blockIdx.x < n_k && (int)blockIdx.x * kQRowsPerCta >= u.nblk * 16) return;   // shorter chunk
  u.block_ids = a.block_ids + static_cast<int64_t>(chunk) * a.max_blocks;
  u.H = a.H;
  u.num_pool_blocks = a.num_pool_blocks;
  u.pool = static_cast<int8_t*>(a.tables[layer]);
  u.status = a.status;
  quantize_store_cta<T, D>(u, src_k, src_v, static_cast<__half*>(a.tables[a.L + layer]),
                           static_cast<float*>(a.tables[3 * a.L + layer]),
                           static_cast<__half*>(a.tables[2 * a.L + layer]),
                           static_cast<float*>(a.tables[4 * a.L + layer]), n_k);
}

// ---- quantise-on-store, staged: one CTA per (chunk, layer, KV head, K or V) -------------
// For chunks of up to 128 tokens at head_dim 128 (the engine's chunks): the CTA
// copies the chunk's K or V tile of one head (128 rows x 256 bytes) into shared
// memory with cp.async (zero-filled past the chunk's tokens), then
//  K: row maxima with 8 lanes per token row (16 elements each, 4 rows per warp
//     and pass, 4 passes), one thread per row for its scale and reciprocal, then
//     the same 8-lanes-per-row walk quantises;
//  V: thread = (8-column group cg, token phase tb): tokens tb, tb + 16, ...; the
//     column maxima reduce over the 16 phases of a half-warp by shuffles, and
//     lanes tb < 8 compute column cg * 8 + tb's scale once.
// Row t's 16-byte piece p sits at t * 256 + ((p ^ (t & 15)) << 4): the copies,
// the K reads (one row per 8 lanes) and the V reads (16 rows, one per lane, per
// column group) all spread over the 32 banks.  Maxima are taken on packed pairs
// (max.xorsign.abs; sign bits cleared at the end).  48 registers and 33 KB of
// shared memory: 5 CTAs per SM.  Output bytes and scales are those of
// quantize_store_k / quantize_store_v.
constexpr int kSTileRows = 128;
constexpr int kSRowBytes = 256;                         // head_dim 128, 16-bit
constexpr int kSTileBytes = kSTileRows * kSRowBytes;    // 32 KB per operand
constexpr int kSThreads = 256;
constexpr int kSSmem = kSTileBytes;                     // one operand per CTA

__device__ __forceinline__ uint32_t s_piece(int t, int p) {
  return static_cast<uint32_t>(t * kSRowBytes + ((p ^ (t & 15)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool live) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(live ? 16 : 0)
               : "memory");
}

// Pairwise max(|m|, |w|) in the pair's 16-bit type; the sign bits of the result
// are not meaningful (clear them with 0x7fff7fff before use).
template <typename T>
__device__ __forceinline__ uint32_t max_abs2(uint32_t m, uint32_t w) {
  uint32_t r;
  if (std::is_same<T, __nv_bfloat16>::value)
    asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(m), "r"(w));
  else
    asm("max.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(r) : "r"(m), "r"(w));
  return r;
}

template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  return Num<T>::pair(w);
}

template <typename T>
__device__ __forceinline__ void unpack8s(const uint4& u, float (&x)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {   // low half by a multiply
      x[2 * i] = __uint_as_float(imad_u32(w[i], 65536u, 0u));
      x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    } else {
      const float2 f = unpack2<T>(w[i]);
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    }
  }
}

// Exact paths of the staged kernels, out of line: the 8 elements at shared address
// `piece`, with one scale (K row) or the 8 columns' scales and reciprocals at
// shared addresses `sc`, `rc` (V).
template <typename T>
__device__ __noinline__ uint2 kivi_q8_exact_row(uint32_t piece, float scale, float rcp) {
  uint4 w;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
               : "r"(piece));
  float x[8];
  unpack8s<T>(w, x);
  int q[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) q[e] = kivi_q<T>(x[e], scale, rcp);
  return pack8(q);
}

template <typename T>
__device__ __noinline__ uint2 kivi_q8_exact_cols(uint32_t piece, const float* sc, const float* rc) {
  uint4 w;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
               : "r"(piece));
  float x[8];
  unpack8s<T>(w, x);
  int q[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) q[e] = kivi_q<T>(x[e], sc[e], rc[e]);
  return pack8(q);
}

template <typename T>
__device__ __forceinline__ void quantize_unit_staged(const QStoreUnit& u0, const void* src_k,
                                                     const void* src_v, __half* ks16, float* ks32,
                                                     __half* vs16, float* vs32, int h, int kv) {
  constexpr int D = 128;
  extern __shared__ __align__(128) uint8_t s_tile[];
  const uint32_t sK = static_cast<uint32_t>(__cvta_generic_to_shared(s_tile));
  const uint32_t sV = sK;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int S = u0.S, slots = u0.nblk * 16;
  // ---- stage this CTA's operand: 2048 pieces, 8 per thread ------------------------------
  {
    const T* src = static_cast<const T*>(kv ? src_v : src_k) + h * u0.hs;
#pragma unroll
    for (int k = 0; k < kSTileBytes / 16 / kSThreads; ++k) {
      const int i = tid + kSThreads * k;
      const int t = i >> 4, pc = i & 15;
      const bool live = t < S;
      cp_async16(sK + s_piece(t, pc), live ? src + t * u0.rs + 8 * pc : src, live);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  // the chunk's block ids, read once while the tile is in flight
  __shared__ int s_blk[kSTileRows / 16];
  if (tid < u0.nblk) s_blk[tid] = u0.block_ids[tid];
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  if (kv == 0) {
    // ---- K: per-token scales ----------------------------------------------------------
    // (a) row maxima, 8 lanes per row; (b) one thread per row computes its scale,
    // reciprocal and stored scales; (c) quantise, 8 lanes per row.
    __shared__ float s_scale[kSTileRows], s_rcp[kSTileRows];
    const int sub = lane & 7;
#pragma unroll 1
    for (int pass = 0; pass < 4; ++pass) {
      const int t = pass * 32 + warp * 4 + (lane >> 3);
      if (t >= slots) break;                          // 4-row groups: warp-uniform
      uint4 w0, w1;
      asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(w0.x), "=r"(w0.y), "=r"(w0.z), "=r"(w0.w)
                   : "r"(sK + s_piece(t, sub)));
      asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(w1.x), "=r"(w1.y), "=r"(w1.z), "=r"(w1.w)
                   : "r"(sK + s_piece(t, sub + 8)));
      uint32_t m2 = max_abs2<T>(max_abs2<T>(max_abs2<T>(w0.x, w0.y), max_abs2<T>(w0.z, w0.w)),
                                max_abs2<T>(max_abs2<T>(w1.x, w1.y), max_abs2<T>(w1.z, w1.w)));
      const float2 mf = unpack2<T>(m2 & 0x7fff7fffu);
      float amax = fmaxf(mf.x, mf.y);
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (sub == 0) s_scale[t] = amax;
    }
    __syncthreads();
    if (tid < slots) {
      const int t = tid;
      const float scale = t < S ? kivi_scale<T>(s_scale[t]) : 0.0f;
      s_scale[t] = scale;
      s_rcp[t] = __frcp_rn(scale);
      const int blk = s_blk[t >> 4];
      if (blk >= 0 && blk < u0.num_pool_blocks) {     // flagged by the row writes below
        const __half s16 = __float2half_rn(scale);
        const int64_t si = (static_cast<int64_t>(blk) * u0.H + h) * 16 + (t & 15);
        if (ks16) ks16[si] = s16;
        if (ks32) ks32[si] = __half2float(s16);
      }
    }
    __syncthreads();
#pragma unroll 1
    for (int pass = 0; pass < 4; ++pass) {
      const int t = pass * 32 + warp * 4 + (lane >> 3);
      if (t >= slots) break;
      const int blk = s_blk[t >> 4], slot = t & 15;
      if (!block_ok(blk, u0)) continue;
      int8_t* dst = u0.pool + ((static_cast<int64_t>(blk) * 2 + 0) * u0.H + h) * 16 * D + slot * D;
      uint2 q0 = make_uint2(0, 0), q1 = make_uint2(0, 0);
      if (t < S) {
        uint4 w0, w1;
        asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(w0.x), "=r"(w0.y), "=r"(w0.z), "=r"(w0.w)
                     : "r"(sK + s_piece(t, sub)));
        asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(w1.x), "=r"(w1.y), "=r"(w1.z), "=r"(w1.w)
                     : "r"(sK + s_piece(t, sub + 8)));
        const float scale = s_scale[t], rcp = s_rcp[t];
        float rc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) rc[e] = rcp;
        float x[8];
        bool n0 = !(scale > 0.0f), n1 = n0;
        unpack8s<T>(w0, x);
        q0 = kivi_q8_fast<T>(x, rc, n0);
        unpack8s<T>(w1, x);
        q1 = kivi_q8_fast<T>(x, rc, n1);
        if (n0) q0 = kivi_q8_exact_row<T>(sK + s_piece(t, sub), scale, rcp);
        if (n1) q1 = kivi_q8_exact_row<T>(sK + s_piece(t, sub + 8), scale, rcp);
      }
      *reinterpret_cast<uint2*>(dst + 8 * sub) = q0;
      *reinterpret_cast<uint2*>(dst + 8 * (sub + 8)) = q1;
    }
  } else {
    // ---- V: per-channel scales over the chunk -------------------------------------------
    const int cg = warp * 2 + (lane >> 4), tb = lane & 15;
    uint32_t m2[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {   // rows past the chunk are zero-filled
      uint4 w;
      asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
                   : "r"(sV + s_piece(tb + 16 * i, cg)));
      m2[0] = max_abs2<T>(m2[0], w.x);
      m2[1] = max_abs2<T>(m2[1], w.y);
      m2[2] = max_abs2<T>(m2[2], w.z);
      m2[3] = max_abs2<T>(m2[3], w.w);
    }
#pragma unroll
    for (int o = 1; o < 16; o <<= 1)
#pragma unroll
      for (int k = 0; k < 4; ++k) m2[k] = max_abs2<T>(m2[k], __shfl_xor_sync(0xffffffffu, m2[k], o));
    // lane tb < 8 owns column cg * 8 + tb
    const uint32_t mine = (tb & 4) ? ((tb & 2) ? m2[3] : m2[2]) : ((tb & 2) ? m2[1] : m2[0]);
    const float2 mf = unpack2<T>(mine & 0x7fff7fffu);
    const float my_sc = kivi_scale<T>((tb & 1) ? mf.y : mf.x);
    const float my_rc = __frcp_rn(my_sc);
    const __half my_s16 = __float2half_rn(my_sc);
    __shared__ float s_vsc[kSTileRows], s_vrc[kSTileRows];   // per column, for the exact path
    if (tb < 8) {
      s_vsc[cg * 8 + tb] = my_sc;
      s_vrc[cg * 8 + tb] = my_rc;
    }
    __syncwarp();
    float rc[8];
    bool zero_scale = false;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      rc[e] = __shfl_sync(0xffffffffu, my_rc, (lane & 16) + e);
      zero_scale |= !(__shfl_sync(0xffffffffu, my_sc, (lane & 16) + e) > 0.0f);
    }
#pragma unroll 1
    for (int i = 0; i < u0.nblk; ++i) {          // token tb + 16 i sits in block i, slot tb
      const int t = tb + 16 * i;
      const int blk = s_blk[i];
      if (!block_ok(blk, u0)) continue;
      if (tb < 8) {                                // the block's copy of the column scales
        const int64_t si = (static_cast<int64_t>(blk) * u0.H + h) * D + cg * 8 + tb;
        if (vs16) vs16[si] = my_s16;
        if (vs32) vs32[si] = __half2float(my_s16);
      }
      uint2 q = make_uint2(0, 0);
      if (t < S) {
        uint4 w;
        asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
                     : "r"(sV + s_piece(t, cg)));
        float x[8];
        unpack8s<T>(w, x);
        bool nr = zero_scale;
        q = kivi_q8_fast<T>(x, rc, nr);
        if (nr) q = kivi_q8_exact_cols<T>(sV + s_piece(t, cg), s_vsc + cg * 8, s_vrc + cg * 8);
      }
      *reinterpret_cast<uint2*>(u0.pool + ((static_cast<int64_t>(blk) * 2 + 1) * u0.H + h) * 16 * D +
                                tb * D + cg * 8) = q;
    }
  }
}

// One chunk (<= 128 tokens), all layers, head_dim 128: grid (KV head, layer, K/V).
template <typename T>
__global__ void __launch_bounds__(kSThreads, 5) kvb_quantize_store_staged_kernel(const __grid_constant__ QStoreArgs a) {
  const int layer = blockIdx.y;
  QStoreUnit u;
  u.hs = a.src_head_stride;
  u.rs = a.src_row_stride;
  u.block_ids = a.block_ids;
  u.nblk = a.nblk;
  u.S = a.S;
  u.H = a.H;
  u.num_pool_blocks = a.num_pool_blocks;
  u.pool = a.pool[layer];
  u.status = nullptr;
  quantize_unit_staged<T>(u, a.src_k[layer], a.src_v[layer], a.ks16[layer], a.ks32[layer], a.vs16[layer],
                          a.vs32[layer], blockIdx.x, blockIdx.z);
}

// Several chunks (each <= 128 tokens), all layers, head_dim 128: grid (KV head,
// chunk x layer, K/V); tables and checks as in kvb_quantize_store_batch_kernel.
template <typename T>
__global__ void __launch_bounds__(kSThreads, 5) kvb_quantize_store_batch_staged_kernel(const QStoreBatchArgs a) {
  const int chunk = blockIdx.y / a.L, layer = blockIdx.y - chunk * a.L;
  QStoreUnit u;
  u.S = a.num_tokens[chunk];
  u.nblk = (u.S + 15) / 16;
  const int64_t si = (static_cast<int64_t>(chunk) * a.L + layer) * 2;
  const void* src_k = a.src[si];
  const void* src_v = a.src[si + 1];
  u.hs = a.src_strides[2 * chunk];
  u.rs = a.src_strides[2 * chunk + 1];
  if (u.S < 1 || u.nblk > a.max_blocks || u.hs < 0 || u.rs < 1 || ((u.hs | u.rs) & 7) ||
      ((reinterpret_cast<uintptr_t>(src_k) | reinterpret_cast<uintptr_t>(src_v)) & 15)) {
    if (threadIdx.x == 0 && a.status) atomicOr(a.status, KVB_STATUS_BAD_LENGTH);
    return;
  }
  u.block_ids = a.block_ids + static_cast<int64_t>(chunk) * a.max_blocks;
  u.H = a.H;
  u.num_pool_blocks = a.num_pool_blocks;
  u.pool = static_cast<int8_t*>(a.tables[layer]);
  u.status = a.status;
  quantize_unit_staged<T>(u, src_k, src_v, static_cast<__half*>(a.tables[a.L + layer]),
                          static_cast<float*>(a.tables[3 * a.L + layer]),
                          static_cast<__half*>(a.tables[2 * a.L + layer]),
                          static_cast<float*>(a.tables[4 * a.L + layer]), blockIdx.x, blockIdx.z);
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

constexpr int kDevWarps = 8;        // warps per CTA; warp w takes layers w, w + 8, ...
constexpr int kDevPositions = 4;    // positions per CTA (8 lanes each, in every warp)
constexpr int kDevLanes = 32 / kDevPositions;
constexpr int kDevVecs = 4;         // 16-byte vectors per lane per operand in flight

// CTA = 4 positions x all layers.  In every warp, lanes 8p..8p+7 own position p
// and split its per-layer K vector (all heads, 16-byte pieces); the warp walks its
// share of the layers, reducing dot(c, f), |c|^2, |f|^2 over the 8 lanes (three
// shuffle steps) and adding 1 - cos per layer; the 8 warps' partial sums are added
// in warp order in shared memory (a fixed order: same inputs, same bits).
template <typename T, int D>
__global__ void __launch_bounds__(kDevWarps * 32) kvb_blend_deviation_kernel(const __grid_constant__ BlendArgs a) {
  __shared__ float part[kDevWarps][kDevPositions];
  constexpr int VPH = D / 8;   // 16-byte vectors per head row
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p = lane / kDevLanes, sub = lane % kDevLanes;
  const int t = blockIdx.x * kDevPositions + p;
  const bool valid = t < a.S;
  const int tt = valid ? t : 0;
  const int nvec = a.H * VPH;
  float acc = 0.0f;
  for (int l = warp; l < a.L; l += kDevWarps) {
    const T* cb = static_cast<const T*>(a.ck[l]) + static_cast<int64_t>(tt) * a.c_rs;
    const T* fb = static_cast<const T*>(a.fk[l]) + static_cast<int64_t>(tt) * a.f_rs;
    float dot = 0.0f, nc = 0.0f, nf = 0.0f;
    for (int v0 = sub; v0 < nvec; v0 += kDevLanes * kDevVecs) {
      uint4 cu[kDevVecs], fu[kDevVecs];
#pragma unroll
      for (int k = 0; k < kDevVecs; ++k) {
        const int v = v0 + kDevLanes * k;
        if (valid && v < nvec) {
          const int h = v / VPH, dv = (v - h * VPH) * 8;
          cu[k] = *reinterpret_cast<const uint4*>(cb + h * a.c_hs + dv);
          fu[k] = *reinterpret_cast<const uint4*>(fb + h * a.f_hs + dv);
        } else {
          cu[k] = fu[k] = make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int k = 0; k < kDevVecs; ++k) {
        const uint32_t cw[4] = {cu[k].x, cu[k].y, cu[k].z, cu[k].w};
        const uint32_t fw[4] = {fu[k].x, fu[k].y, fu[k].z, fu[k].w};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const float2 x = Num<T>::pair(cw[w]), y = Num<T>::pair(fw[w]);
          dot = fmaf(x.x, y.x, fmaf(x.y, y.y, dot));
          nc = fmaf(x.x, x.x, fmaf(x.y, x.y, nc));
          nf = fmaf(y.x, y.x, fmaf(y.y, y.y, nf));
        }
      }
    }
#pragma unroll
    for (int o = 1; o < kDevLanes; o <<= 1) {
      dot += __shfl_xor_sync(0xffffffffu, dot, o);
      nc += __shfl_xor_sync(0xffffffffu, nc, o);
      nf += __shfl_xor_sync(0xffffffffu, nf, o);
    }
    acc += 1.0f - dot / (fmaxf(sqrtf(nc), 1e-8f) * fmaxf(sqrtf(nf), 1e-8f));
  }
  if (sub == 0) part[warp][p] = acc;
  __syncthreads();
  if (threadIdx.x < kDevPositions) {
    const int tp = blockIdx.x * kDevPositions + threadIdx.x;
    if (tp < a.S) {
      float sum = 0.0f;
#pragma unroll
      for (int w = 0; w < kDevWarps; ++w) sum += part[w][threadIdx.x];
      a.deviation[tp] = sum / static_cast<float>(a.L);
    }
  }
}

// Total order on float bit patterns (larger float -> larger key).
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kSelThreads = 1024;
constexpr int kSelBits = 11;                  // radix digit: passes of 11, 11 and 10 bits
constexpr int kSelBins = 1 << kSelBits;
constexpr int kSelCache = 8192;               // deviations kept in shared memory up to this many

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

// One CTA.  Candidates are positions with deviation > min_dev; the key of the
// kk-th largest candidate (kk = min(k, #candidates)) is found by a radix select
// over the float's order-preserving bit pattern (3 digit passes, shared
// histogram with warp-aggregated atomics, the bin found by one warp's suffix scan).
// Then each thread takes a contiguous run of positions: every candidate above that
// key, and the first `remaining` equal to it in position order (two CTA scans give
// each run its offsets), written ascending.
__global__ void __launch_bounds__(kSelThreads) kvb_blend_select_kernel(const float* __restrict__ dev_g, int S, int k,
                                                                        float min_dev, int32_t* selected,
                                                                        int32_t* num_selected) {
  __shared__ uint32_t hist[kSelBins];
  __shared__ uint32_t warp_tot[32];
  __shared__ uint32_t s_prefix, s_remaining;
  extern __shared__ float dev_cache[];   // S floats when S <= kSelCache, else unused
  const int tid = threadIdx.x, lane = tid & 31;
  const bool cached = S <= kSelCache;
  const float* dev = cached ? dev_cache : dev_g;

  uint32_t cnt = 0;
  for (int i = tid; i < S; i += kSelThreads) {
    const float x = dev_g[i];
    if (cached) dev_cache[i] = x;
    cnt += x > min_dev ? 1u : 0u;
  }
  uint32_t total;
  block_exclusive_scan(cnt, warp_tot, &total);
  const uint32_t kk = min(static_cast<uint32_t>(k), total);
  if (kk == 0) {
    for (int j = tid; j < k; j += kSelThreads) selected[j] = -1;
    if (tid == 0) *num_selected = 0;
    return;
  }

  uint32_t prefix = 0, mask = 0, remaining = kk;
#pragma unroll 1
  for (int pass = 0; pass < 3; ++pass) {
    const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
    const uint32_t dmask = pass == 2 ? 1023u : 2047u;
    for (int b = tid; b < kSelBins; b += kSelThreads) hist[b] = 0;
    __syncthreads();
    for (int i0 = 0; i0 < S; i0 += kSelThreads) {
      const int i = i0 + tid;
      bool in = false;
      uint32_t bin = 0;
      if (i < S) {
        const float x = dev[i];
        const uint32_t key = order_key(x);
        in = x > min_dev && (key & mask) == prefix;
        bin = (key >> shift) & dmask;
      }
      const uint32_t active = __ballot_sync(0xffffffffu, in);
      if (in) {
        const uint32_t peers = __match_any_sync(active, bin);
        if (lane == __ffs(peers) - 1) atomicAdd(&hist[bin], static_cast<uint32_t>(__popc(peers)));
      }
    }
    __syncthreads();
    {
      // thread t owns bins dmask - 2t and dmask - 2t - 1 (descending); a CTA scan of
      // the owned counts finds the bin holding the remaining-th largest
      const int b0 = static_cast<int>(dmask) - 2 * tid;
      const uint32_t c0 = b0 >= 0 ? hist[b0] : 0u, c1 = b0 >= 1 ? hist[b0 - 1] : 0u;
      uint32_t tot;
      const uint32_t before = block_exclusive_scan(c0 + c1, warp_tot, &tot);
      if (before < remaining && before + c0 + c1 >= remaining) {
        const uint32_t rem = remaining - before;
        const bool first = c0 >= rem;
        s_prefix = prefix | (static_cast<uint32_t>(first ? b0 : b0 - 1) << shift);
        s_remaining = first ? rem : rem - c0;
      }
    }
    __syncthreads();
    prefix = s_prefix;
    remaining = s_remaining;
    mask |= dmask << shift;
  }
  const uint32_t kth = prefix;   // key of the kk-th largest; `remaining` of its equals are taken

  const int per = (S + kSelThreads - 1) / kSelThreads;
  const int lo = min(tid * per, S), hi = min(lo + per, S);
  uint32_t gt = 0, eq = 0;
  for (int i = lo; i < hi; ++i) {
    const float x = dev[i];
    if (x > min_dev) {
      const uint32_t key = order_key(x);
      gt += key > kth ? 1u : 0u;
      eq += key == kth ? 1u : 0u;
    }
  }
  uint32_t eq_total, sel_total;
  const uint32_t eq_before = block_exclusive_scan(eq, warp_tot, &eq_total);
  const uint32_t take_eq = eq_before >= remaining ? 0u : min(eq, remaining - eq_before);
  uint32_t out = block_exclusive_scan(gt + take_eq, warp_tot, &sel_total);
  uint32_t eq_left = take_eq;
  for (int i = lo; i < hi; ++i) {
    const float x = dev[i];
    if (!(x > min_dev)) continue;
    const uint32_t key = order_key(x);
    bool take = key > kth;
    if (key == kth && eq_left > 0) {
      take = true;
      --eq_left;
    }
    if (take && out < kk) selected[out++] = i;
  }
  for (int j = static_cast<int>(kk) + tid; j < k; j += kSelThreads) selected[j] = -1;
  if (tid == 0) *num_selected = static_cast<int32_t>(kk);
}

constexpr int kPatchSlots = 32;  // chosen positions per CTA (4 per warp)
constexpr int kPatchThreads = 256;

// Grid (chosen-position groups, layer); warp w copies chosen positions 4w .. 4w + 3
// of its group: for each, the fresh K and V rows of every head over the cached
// ones in 16-byte pieces (all loads before the stores).  Groups past
// *num_selected exit.
template <typename T, int D>
__global__ void __launch_bounds__(kPatchThreads) kvb_blend_patch_kernel(const __grid_constant__ BlendArgs a) {
  constexpr int VPH = D / 8;
  constexpr int kPerWarp = kPatchSlots / (kPatchThreads / 32);
  const int n = *a.num_selected;
  const int layer = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j0 = blockIdx.x * kPatchSlots + warp * kPerWarp;
  if (j0 >= n) return;
  const T* fk = static_cast<const T*>(a.fk[layer]);
  const T* fv = static_cast<const T*>(a.fv[layer]);
  T* ck = static_cast<T*>(a.ck[layer]);
  T* cv = static_cast<T*>(a.cv[layer]);
  int t[kPerWarp];
#pragma unroll
  for (int s = 0; s < kPerWarp; ++s) t[s] = j0 + s < n ? a.selected[j0 + s] : -1;
  const int nvec = a.H * VPH;
  for (int e = lane; e < nvec; e += 32) {
    const int h = e / VPH, dv = (e - h * VPH) * 8;
    uint4 kx[kPerWarp], vx[kPerWarp];
#pragma unroll
    for (int s = 0; s < kPerWarp; ++s) {
      if (t[s] >= 0) {
        const int64_t so = h * a.f_hs + static_cast<int64_t>(t[s]) * a.f_rs + dv;
        kx[s] = *reinterpret_cast<const uint4*>(fk + so);
        vx[s] = *reinterpret_cast<const uint4*>(fv + so);
      }
    }
#pragma unroll
    for (int s = 0; s < kPerWarp; ++s) {
      if (t[s] >= 0) {
        const int64_t d = h * a.c_hs + static_cast<int64_t>(t[s]) * a.c_rs + dv;
        *reinterpret_cast<uint4*>(ck + d) = kx[s];
        *reinterpret_cast<uint4*>(cv + d) = vx[s];
      }
    }
  }
}

// ---- host side ------------------------------------------------------------------------
int fail(int code, const std::string& msg) { return kvb_detail_fail(code, msg); }

bool head_dim_ok(int d) { return d == 64 || d == 96 || d == 128; }

// The staged kernels take 32 KB of dynamic shared memory (opted in once per device
// and kernel -- one instantiation per kernel, so each keeps its own flags -- in
// case the default limit is lower).
template <typename T, bool BATCH>
cudaError_t staged_smem_opt_in() {
  static int configured[64] = {};
  const void* kernel = BATCH ? reinterpret_cast<const void*>(kvb_quantize_store_batch_staged_kernel<T>)
                             : reinterpret_cast<const void*>(kvb_quantize_store_staged_kernel<T>);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (configured[dev]) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSSmem);
  if (e == cudaSuccess) configured[dev] = 1;
  return e;
}

template <typename T, int D>
cudaError_t launch_qstore(const QStoreArgs& a, int L, cudaStream_t s) {
  if (D == 128 && a.nblk <= kSTileRows / 16) {
    cudaError_t e = staged_smem_opt_in<T, false>();
    if (e != cudaSuccess) return e;
    kvb_quantize_store_staged_kernel<T><<<dim3(a.H, L, 2), kSThreads, kSSmem, s>>>(a);
    return cudaGetLastError();
  }
  const int n_k = (a.nblk * 16 + kQRowsPerCta - 1) / kQRowsPerCta;
  kvb_quantize_store_kernel<T, D><<<dim3(n_k + D / kQVCols, a.H, L), kQThreads, 0, s>>>(a);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t launch_qstore_batch(const QStoreBatchArgs& a, int chunks, cudaStream_t s) {
  if (D == 128 && a.max_blocks <= kSTileRows / 16) {
    cudaError_t e = staged_smem_opt_in<T, true>();
    if (e != cudaSuccess) return e;
    kvb_quantize_store_batch_staged_kernel<T><<<dim3(a.H, chunks * a.L, 2), kSThreads, kSSmem, s>>>(a);
    return cudaGetLastError();
  }
  const int n_k = (a.max_blocks * 16 + kQRowsPerCta - 1) / kQRowsPerCta;
  kvb_quantize_store_batch_kernel<T, D><<<dim3(n_k + D / kQVCols, a.H, chunks * a.L), kQThreads, 0, s>>>(a);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_qstore_batch_d(const QStoreBatchArgs& a, int chunks, int D, cudaStream_t s) {
  switch (D) {
    case 64: return launch_qstore_batch<T, 64>(a, chunks, s);
    case 96: return launch_qstore_batch<T, 96>(a, chunks, s);
    default: return launch_qstore_batch<T, 128>(a, chunks, s);
  }
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
  kvb_blend_deviation_kernel<T, D><<<(a.S + kDevPositions - 1) / kDevPositions, kDevWarps * 32, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const size_t cache_bytes = a.S <= kSelCache ? static_cast<size_t>(a.S) * sizeof(float) : 0;
  kvb_blend_select_kernel<<<1, kSelThreads, cache_bytes, s>>>(a.deviation, a.S, a.k, min_dev, a.selected,
                                                              a.num_selected);
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
  if (p->src_row_stride < 1 || p->src_head_stride < 0 || (p->src_row_stride | p->src_head_stride) & 7)
    return fail(KVB_ERR_INVALID, "src_row_stride must be >= 1, src_head_stride >= 0, both multiples of 8");
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
    if ((reinterpret_cast<uintptr_t>(p->src_k[l]) | reinterpret_cast<uintptr_t>(p->src_v[l])) & 15u)
      return fail(KVB_ERR_INVALID, "layer " + std::to_string(l) + ": source pointers must be 16-byte aligned");
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
  a.num_pool_blocks = p->num_pool_blocks;
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

extern "C" int kvb_quantize_store_batch(const KvbQuantizeStoreBatch* p, void* stream) {
  if (!p) return fail(KVB_ERR_INVALID, "params is NULL");
  if (p->dtype != KVB_DTYPE_BF16 && p->dtype != KVB_DTYPE_FP16)
    return fail(KVB_ERR_INVALID, "dtype must be KVB_DTYPE_BF16 or KVB_DTYPE_FP16");
  if (!head_dim_ok(p->head_dim)) return fail(KVB_ERR_INVALID, "head_dim must be 64, 96 or 128");
  if (p->num_layers < 1 || p->num_layers > KVB_MAX_LAYERS)
    return fail(KVB_ERR_INVALID, "num_layers must be in [1, " + std::to_string(KVB_MAX_LAYERS) + "]");
  if (p->num_kv_heads < 1 || p->num_kv_heads > 65535) return fail(KVB_ERR_INVALID, "num_kv_heads must be in [1, 65535]");
  if (p->num_chunks < 1 || (int64_t)p->num_chunks * p->num_layers > 65535)
    return fail(KVB_ERR_INVALID, "num_chunks must be >= 1 with num_chunks * num_layers <= 65535");
  if (p->max_chunk_blocks < 1 || p->max_chunk_blocks > KVB_MAX_CHUNK_BLOCKS)
    return fail(KVB_ERR_INVALID, "max_chunk_blocks must be in [1, " + std::to_string(KVB_MAX_CHUNK_BLOCKS) + "]");
  if (p->num_pool_blocks < 1) return fail(KVB_ERR_INVALID, "num_pool_blocks must be >= 1");
  if (!p->src || !p->src_strides || !p->tables || !p->num_tokens || !p->block_ids)
    return fail(KVB_ERR_INVALID, "src, src_strides, tables, num_tokens and block_ids must be non-null device arrays");
  QStoreBatchArgs a{};
  a.src = p->src;
  a.tables = p->tables;
  a.num_tokens = p->num_tokens;
  a.block_ids = p->block_ids;
  a.src_strides = p->src_strides;
  a.num_pool_blocks = p->num_pool_blocks;
  a.L = p->num_layers;
  a.H = p->num_kv_heads;
  a.max_blocks = p->max_chunk_blocks;
  a.status = p->status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t e =
      p->dtype == KVB_DTYPE_BF16 ? launch_qstore_batch_d<__nv_bfloat16>(a, p->num_chunks, p->head_dim, s)
                                 : launch_qstore_batch_d<__half>(a, p->num_chunks, p->head_dim, s);
  if (e != cudaSuccess)
    return fail(KVB_ERR_CUDA, std::string("kvb_quantize_store_batch launch: ") + cudaGetErrorString(e));
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
