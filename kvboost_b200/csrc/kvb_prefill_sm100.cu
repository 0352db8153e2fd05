// Offset-causal prefill attention for B200 (sm_100a).
//
// One CTA (one per SM: 202 KB of shared memory, all 512 TMEM columns) runs two
// 128-row query tiles ("slots") that share a KV head — two query heads of a
// GQA pair, two consecutive tiles of one head, or (split-key mode) packed GQA
// rows — in ping-pong against the visible part of that KV head:
//
//   warps 0-15  softmax / epilogue, two warpgroups per slot.  Thread t of a
//               warpgroup owns query row t = TMEM lane t and one half of the
//               key columns; the two threads of a row agree on the running
//               maximum through 64-thread named-barrier reductions.
//   warp 16     TMA producer: Q once per slot, then K_j / V_j tiles (128 x D,
//               128-byte swizzle) into NS-deep shared-memory rings.
//   warp 17     MMA issuer (one thread) and TMEM owner:
//                 S_j  = Q K_j^T   tcgen05.mma SS, fp32 accumulator in TMEM
//                 O   += P_j V_j   tcgen05.mma TS, P read from TMEM
//               issued PV0(j), S0(j+1), PV1(j), S1(j+1), so one slot's MMAs
//               overlap the other slot's softmax.
//   (paged kernels: one softmax warpgroup per slot, three converter warps that
//   gather int8 blocks through the block table and dequantise into the ring.)
//
// TMEM: S0, S1, O0, O1 at columns 0/128/256/384; each warpgroup writes its P
// as packed 16-bit pairs over the start of its own S columns.
//
// Online softmax runs in the log2 domain against a stale running maximum: a
// tile is exponentiated in one pass, and the maximum is raised (tile maximum,
// O rescale, redo) only when a thread's probability sum shows one could leave
// the P operand's range; the final normalisation uses the same maximum, so
// this is exact up to rounding.
//
// Causality is bottom-right (key j visible to query i iff
// j <= i + kv_len - q_len) or, on request, top-left (j <= i); key tiles
// entirely above the diagonal are never loaded, and only the tiles crossing
// the diagonal or the end of the keys are masked element by element.
//
// Every mbarrier wait is bounded (KVB_WAIT_NS); a wait that gives up sets a
// CTA-wide abort flag and ORs a code into the caller's status word, after
// which every role drains its in-flight copies / MMAs and the CTA frees its
// TMEM and exits.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>
#include <utility>

#include "kvb_attn.h"
#include "kvb_sm100_ptx.cuh"

// Share of exponent pairs computed on the FMA pipe instead of MUFU: pair i of
// each chunk uses the polynomial when (i % 8) < the pairs-of-8 count.  At
// D = 64 a tile's two MMAs take half the cycles of its exponentials, so moving
// a quarter of them to the FMA pipe pays (+4-5 % measured); at D >= 96 the
// MMAs already match the exponentials and it costs 3-5 %.
template <int D>
__host__ __device__ constexpr int poly_pairs_of_8() {
  return D <= 64 ? 2 : 0;
}
// 1: pack bf16 probabilities with integer round-half-up + byte permute
// instead of the cvt.rn.bf16x2.f32 conversion.
#ifndef KVB_PACK_INT
#define KVB_PACK_INT 0
#endif

#ifndef KVB_WAIT_NS
#define KVB_WAIT_NS 2000000000ull  // 2 s: far above any legitimate wait
#endif

namespace kvb {

// Optional per-CTA phase timestamps (SM clock) for pipeline studies; compiled
// only with -DKVB_TRACE, never in the shipped library.
#ifdef KVB_TRACE
__device__ long long* g_kvb_trace;
#define KVB_TRACE_AT(slot)                                 \
  do {                                                     \
    if (kvb_trace_row) kvb_trace_row[(slot)] = clock64();  \
  } while (0)
#define KVB_TRACE_SETUP()                                                                      \
  long long* kvb_trace_row =                                                                   \
      g_kvb_trace ? g_kvb_trace + 512ull * (blockIdx.x +                                       \
                                            gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z)) \
                  : nullptr
// global-timer stamps (ns, comparable across SMs) for launch-level timelines
#define KVB_TRACE_GT(slot)                                                                 \
  do {                                                                                     \
    if (kvb_trace_row) kvb_trace_row[(slot)] = static_cast<long long>(ptx::globaltimer_ns()); \
  } while (0)
#else
#define KVB_TRACE_GT(slot) \
  do {                     \
  } while (0)
#define KVB_TRACE_SETUP() \
  do {                    \
  } while (0)
#define KVB_TRACE_AT(slot) \
  do {                     \
  } while (0)
#endif

constexpr int BM = 128;        // query rows per slot (= TMEM lanes)
constexpr int BN = 128;        // keys per tile
constexpr int kSlots = 2;      // query tiles per CTA, processed in ping-pong
// Warp roles.  Dense: warps 0-15 softmax, two warpgroups per slot (slot s,
// column half h -> warps 4*(2s+h) .. +3; each thread owns one row and half of
// its columns), warp 16 TMA, warp 17 MMA (576 threads).  Paged: warps 0-3 /
// 4-7 softmax of slot 0 / 1 (one warpgroup per slot, whole rows), warps 8-10
// gather + dequantise K/V into shared memory (warp 8 lane 0 also issues the
// Q TMA), warp 11 MMA (384 threads).
template <bool PAGED>
struct Roles {
  static constexpr int kHalves = PAGED ? 1 : 2;                 // softmax warpgroups per slot
  static constexpr int kSoftmaxWarps = 4 * kSlots * kHalves;
  static constexpr int kWarpTma = kSoftmaxWarps;
  static constexpr int kConvWarps = PAGED ? 3 : 0;
  static constexpr int kWarpMma = PAGED ? kWarpTma + kConvWarps : kWarpTma + 1;
  static constexpr int kThreads = (kWarpMma + 1) * 32;
};

template <int D>
struct Geo {
  static constexpr int DP = (D + 63) / 64 * 64;  // head_dim padded to whole 64-element atoms
  static constexpr int NATOM = DP / 64;          // 128-byte swizzle atoms per row
  static constexpr int ATOM_BYTES = 128 * 128;   // 128 rows x 128 bytes
  static constexpr int TILE_BYTES = NATOM * ATOM_BYTES;
  static constexpr int NS = (D <= 64) ? 4 : 2;   // K/V ring depth
  // K ring depth of the split-key dual mode: both slots read slot 0's Q tile,
  // so slot 1's Q buffer is one more K stage when the ring has two.
  static constexpr int KSD = (NS == 2) ? 3 : NS;
  static constexpr int TMEM_COLS = 512;          // S0 S1 O0 O1, 128 columns each
  static constexpr int QK_STEPS = D / 16;        // K-steps of S = Q K^T
  static constexpr int PV_STEPS = BN / 16;       // K-steps of O += P V
  static constexpr int BAR_BYTES = 512;
  // Row-statistic exchange between the two column halves of a slot:
  // running maxima and final row sums, [kSlots][2 halves][128 rows] each.
  static constexpr int XCH_BYTES = 2 * kSlots * 2 * 128 * 4;
  static constexpr int SMEM_BYTES =
      1024 + TILE_BYTES * (kSlots + 2 * NS) + BAR_BYTES + XCH_BYTES;
  __host__ __device__ static constexpr uint32_t s_col(int slot) { return slot * 128; }
  __host__ __device__ static constexpr uint32_t o_col(int slot) { return 256 + slot * 128; }
};

// Barrier slots (per-slot barriers at +slot, ring barriers at +stage)
enum {
  BAR_Q_FULL = 0,
  BAR_S_FULL = 2,
  BAR_P_FULL = 4,
  BAR_O_FULL = 6,
  BAR_DRAIN = 8,
  BAR_K_FULL = 9,
  BAR_K_EMPTY = 13,
  BAR_V_FULL = 17,
  BAR_V_EMPTY = 21,
  BAR_COUNT = 25
};

struct DenseArgs {
  void* o;
  float* lse;
  int64_t o_bs, o_hs, o_rs;
  int64_t lse_bs, lse_hs;
  const int* cu_q;
  const int* cu_k;
  int q_len, kv_len;
  int group;       // num_q_heads / num_kv_heads
  int pair_heads;  // 1: slots are heads 2y, 2y+1 (same KV head) on one query tile;
                   // 0: slots are query tiles 2x, 2x+1 of one head
  int causal;
  float scale_log2;
  int* status;
  // Dense layout with per-sequence key counts: sequence b uses the first
  // kv_prefix[b] + q_len rows of its K/V (the rest may be padding).
  const int* kv_prefix;
};

// Reused-prefix K/V in the int8 paged pool plus the suffix's own fresh K/V.
struct PagedArgs {
  union {
    struct {                  // paged kernels
      const int8_t* pool;     // [num_blocks, 2, num_kv_heads, 16, D] int8 (K then V)
      const float* k_scale;   // [num_blocks, num_kv_heads, 16]  per-token K scale
      const float* v_scale;   // [num_blocks, num_kv_heads, D]   per-channel V scale of the block's chunk
      const int* block_table; // [batch, max_blocks]
      const int* prefix_lens; // [batch] cached tokens, or null -> prefix_len
      const void* k_new;      // suffix K (compute dtype), element (b, h, i, d) at
      const void* v_new;      //   b*bs + h*hs + i*rs + d
      int64_t kn_bs, kn_hs, kn_rs, vn_bs, vn_hs, vn_rs;
    };
    struct {                  // split-key attention: where kvb_split_merge_kernel writes
      void* o_final;          // final O, element (b, head, i, d) at b*bs + head*hs + i*rs + d
      float* lse_final;       // final LSE (b, head, i) at b*bs + head*hs + i, or null
      int64_t of_bs, of_hs, of_rs, lf_bs, lf_hs;
      int group_heads;        // query heads per KV head
      int tile_pairs;         // 256-row pairs of packed tiles per group (grid x = splits * pairs)
      int dual;               // 1: one packed tile; slot s of CTA c takes key split 2c + s
    };
  };
  int max_blocks;
  int num_blocks;
  int num_kv_heads;
  int prefix_len;
  int pool16;             // 1: the pool holds K/V in the compute dtype, no scales
  // Split-key decode (the dense SPLITKV kernels, which read no pool and carry
  // these here: growing DenseArgs measurably slowed every dense launch): query
  // rows are a GQA group's heads packed as (head, row) with rows_per_head rows
  // each; CTA x takes packed tiles 2p, 2p + 1 (p = x / c, c CTAs per tile
  // pair) and key tiles [s * split_tiles, (s + 1) * split_tiles) (s = x % c),
  // and writes its normalised partial O / LSE at o + s * o_split_stride,
  // lse + s * lse_split_stride.  With dual set (all packed rows in one tile),
  // both slots take that tile and slot t takes key split s = 2 (x % c) + t, so
  // that one CTA runs two independent key ranges in ping-pong.
  int rows_per_head;
  int split_tiles;
  int64_t o_split_stride, lse_split_stride;
};

struct SharedCtl {
  uint32_t tmem_base;
  int abort_flag;
};

// Bounded wait: spins on try_wait, then checks the CTA abort flag and the
// global timer.  Returns false if the CTA is aborting or the limit passed.
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                         int* status, int code) {
  if (ptx::mbar_test_wait(bar, parity)) return true;
#pragma unroll 1
  for (int i = 0; i < 128; ++i)
    if (ptx::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = ptx::globaltimer_ns();
#pragma unroll 1
  while (true) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (ptx::globaltimer_ns() - t0 > KVB_WAIT_NS) {
      *abort_flag = 1;
      if (status) atomicOr(status, code);
      return false;
    }
  }
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <typename T>
__host__ __device__ constexpr int ab_format() {
  return std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
}

// Packed fp32 pair helpers (sm_100 f32x2 ALU forms).
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float f2lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f2hi(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.ftz.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.ftz.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fsub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.ftz.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair on the FMA pipe, to take load off the MUFU unit (which
// would otherwise bound the softmax at one ex2 per lane per 8 cycles).
// Cody-Waite style split x = j + f with j = round-to-nearest(x) obtained by
// adding 1.5 * 2^23 (the integer lands in the low mantissa bits), f in
// [-0.5, 0.5]; 2^f from a degree-3 polynomial fitted here by a Remez
// exchange for minimax relative error on [-0.5, 0.5] (max 7.5e-5, below the
// half-ulp of bf16 and fp16 probabilities); the result's exponent field is
// then advanced by j.  Inputs are clamped to >= -126 so the result stays a
// normal float; used only for unmasked columns, where that clamp only
// replaces values below 2^-126.
__device__ __forceinline__ void ex2_poly_pair(uint64_t x, float& p0, float& p1) {
  const uint64_t magic = f2pack(12582912.f, 12582912.f);
  const uint64_t c3 = f2pack(0.0551716685295105f, 0.0551716685295105f);
  const uint64_t c2 = f2pack(0.2426111251115799f, 0.2426111251115799f);
  const uint64_t c1 = f2pack(0.6932609677314758f, 0.6932609677314758f);
  const uint64_t c0 = f2pack(0.9999280571937561f, 0.9999280571937561f);
  x = f2pack(fmaxf(f2lo(x), -126.f), fmaxf(f2hi(x), -126.f));
  const uint64_t t = fadd2(x, magic);
  const uint64_t f = fsub2(x, fsub2(t, magic));
  uint64_t p = ffma2(c3, f, c2);
  p = ffma2(p, f, c1);
  p = ffma2(p, f, c0);
  p0 = __uint_as_float(static_cast<uint32_t>(p) + (static_cast<uint32_t>(t) << 23));
  p1 = __uint_as_float(static_cast<uint32_t>(p >> 32) + (static_cast<uint32_t>(t >> 32) << 23));
}

// Convert a pair of probabilities to the MMA operand type, low half = first.
template <typename T>
__device__ __forceinline__ uint32_t cvt_pair(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t cvt_pair<__nv_bfloat16>(float lo, float hi) {
  uint32_t d;
#if KVB_PACK_INT
  // Probabilities are finite and non-negative: adding half an ulp of the
  // 16-bit result and keeping the high halves rounds to nearest (ties up).
  asm("prmt.b32 %0, %1, %2, 0x7632;"
      : "=r"(d)
      : "r"(__float_as_uint(lo) + 0x8000u), "r"(__float_as_uint(hi) + 0x8000u));
#else
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
#endif
  return d;
}
template <>
__device__ __forceinline__ uint32_t cvt_pair<__half>(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// TMEM load of CW (16 or 32) consecutive columns of this warp's 32 lanes.
template <int CW>
__device__ __forceinline__ void tmem_ld_cw(uint32_t taddr, uint32_t (&r)[CW]) {
  if constexpr (CW == 32)
    ptx::tmem_ld32(taddr, r);
  else
    ptx::tmem_ld16(taddr, r);
}

// Row maximum of the raw scores in NCH chunks of CW S columns starting at TMEM
// address tS (tile column c0).  Columns past `lim` are masked when MASK.
template <bool MASK, int NCH, int CW>
__device__ __forceinline__ float cols_row_max(uint32_t tS, int c0, int lim) {
  float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll 1
  for (int k = 0; k < NCH; ++k) {
    uint32_t r[CW];
    tmem_ld_cw<CW>(tS + k * CW, r);
    ptx::tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < CW; i += 4) {
      float x[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        x[e] = (MASK && c0 + k * CW + i + e > lim) ? -INFINITY : __uint_as_float(r[i + e]);
      m0 = fmax3(m0, x[0], x[1]);
      m1 = fmax3(m1, x[2], x[3]);
    }
  }
  return fmaxf(m0, m1);
}

// Softmax work on one chunk of CW columns already in registers (tile column
// c): P pairs packed into pk, partial sums updated.
template <typename T, bool MASK, int CW, int POLY>
__device__ __forceinline__ void chunk_exp(const uint32_t (&r)[CW], int c, int lim, uint64_t sc2,
                                          uint64_t nm2, uint64_t& acc0, uint64_t& acc1,
                                          uint32_t (&pk)[CW / 2]) {
#pragma unroll
  for (int i = 0; i < CW / 2; ++i) {
    float x0 = __uint_as_float(r[2 * i]);
    float x1 = __uint_as_float(r[2 * i + 1]);
    if (MASK) {
      if (c + 2 * i > lim) x0 = -INFINITY;
      if (c + 2 * i + 1 > lim) x1 = -INFINITY;
    }
    const uint64_t a = ffma2(f2pack(x0, x1), sc2, nm2);
    float p0, p1;
    if (!MASK && (i & 7) < POLY) {
      ex2_poly_pair(a, p0, p1);
    } else {
      p0 = ptx::ex2(f2lo(a));
      p1 = ptx::ex2(f2hi(a));
    }
    if (i & 1)
      acc1 = fadd2(acc1, f2pack(p0, p1));
    else
      acc0 = fadd2(acc0, f2pack(p0, p1));
    pk[i] = cvt_pair<T>(p0, p1);
  }
}

// P = exp2(s * sl2 - m) for NCH chunks of CW S columns starting at TMEM
// address tS (tile column c0), packed as 16-bit pairs into pk (pair i of
// columns c0+2i, c0+2i+1).  The chunks are double-buffered: the TMEM load of
// chunk k+1 is in flight while chunk k is exponentiated.  S in TMEM is left
// intact (the caller stores P only once the row sums pass the range check).
// Returns the row sum of P over these columns (fp32, before rounding).
template <typename T, bool MASK, int NCH, int CW, int POLY>
__device__ __forceinline__ float cols_exp(uint32_t tS, int c0, float sl2, float m_use, int lim,
                                          uint32_t (&pk)[NCH * CW / 2]) {
  const uint64_t sc2 = f2pack(sl2, sl2);
  const uint64_t nm2 = f2pack(-m_use, -m_use);
  uint64_t acc0 = 0, acc1 = 0;
  uint32_t ra[CW], rb[CW];
  tmem_ld_cw<CW>(tS, ra);
  ptx::tmem_wait_ld();
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    if (k + 1 < NCH) tmem_ld_cw<CW>(tS + (k + 1) * CW, (k & 1) ? ra : rb);
    chunk_exp<T, MASK, CW, POLY>((k & 1) ? rb : ra, c0 + k * CW, lim, sc2, nm2, acc0, acc1,
                           *reinterpret_cast<uint32_t(*)[CW / 2]>(&pk[k * CW / 2]));
    if (k + 1 < NCH) ptx::tmem_wait_ld();
  }
  const uint64_t t = fadd2(acc0, acc1);
  return f2lo(t) + f2hi(t);
}

// Write packed P over S columns this thread has already consumed: S columns
// [c, c+32) of its range become P columns [c/2, c/2+16) relative to the range
// start tP (its own S columns, so the other half's S is never overwritten).
template <int NW>
__device__ __forceinline__ void store_p(uint32_t tP, const uint32_t (&pk)[NW]) {
#pragma unroll
  for (int k = 0; k < NW / 32; ++k)
    ptx::tmem_st32(tP + 32 * k, *reinterpret_cast<const uint32_t(*)[32]>(&pk[32 * k]));
}

// Gather one 128-token K or V tile for the paged path into the swizzled
// shared-memory layout the MMA reads (the same layout a 128-byte-swizzle TMA
// box produces: row r, 16-byte unit u of a 64-element atom lands at
// atom*16K + r*128 + ((u ^ (r & 7)) * 16)).  Tokens below the cached prefix
// come from the int8 pool through the block table and are dequantised as
// q * scale in fp32, rounded once to the compute type; tokens of the suffix
// are copied from the fresh K/V; rows past the end (and padding columns past
// head_dim) are zero.  Block ids outside the pool, and table positions past
// max_blocks (a per-sequence prefix longer than the table), read as zeros
// and set KVB_STATUS_BAD_BLOCK.
template <typename T, int D>
__device__ __forceinline__ void gather_kv_tile(uint8_t* dst, const PagedArgs& pa, int b, int kvh,
                                               int tok0, int P, int kv_len, int kv, int ct,
                                               int nct, int* status) {
  using G = Geo<D>;
  constexpr int NCH = G::DP / 16;  // 16-element chunks per row (padding included)
  const T* fresh = reinterpret_cast<const T*>(kv ? pa.v_new : pa.k_new);
  const int64_t f_bs = kv ? pa.vn_bs : pa.kn_bs;
  const int64_t f_hs = kv ? pa.vn_hs : pa.kn_hs;
  const int64_t f_rs = kv ? pa.vn_rs : pa.kn_rs;
#pragma unroll 1
  for (int idx = ct; idx < BN * NCH; idx += nct) {
    const int row = idx / NCH;
    const int ch = idx - row * NCH;
    const int tok = tok0 + row;
    uint4 w0 = make_uint4(0, 0, 0, 0), w1 = make_uint4(0, 0, 0, 0);
    if (ch * 16 < D && tok < kv_len) {
      if (tok < P) {
        const int bi = tok >> 4;
        const int blk =
            bi < pa.max_blocks ? __ldg(pa.block_table + (int64_t)b * pa.max_blocks + bi) : -1;
        if (blk < 0 || blk >= pa.num_blocks) {
          if (status) atomicOr(status, KVB_STATUS_BAD_BLOCK);
        } else if (pa.pool16) {
          const uint4* src = reinterpret_cast<const uint4*>(
              reinterpret_cast<const T*>(pa.pool) +
              ((((int64_t)blk * 2 + kv) * pa.num_kv_heads + kvh) * 16 + (tok & 15)) * D + ch * 16);
          w0 = __ldg(src);
          w1 = __ldg(src + 1);
        } else {
          const int slot = tok & 15;
          const int64_t hb = (int64_t)blk * pa.num_kv_heads + kvh;
          const uint4 q = __ldg(reinterpret_cast<const uint4*>(
              pa.pool + (((int64_t)blk * 2 + kv) * pa.num_kv_heads + kvh) * 16 * D +
              (int64_t)slot * D + ch * 16));
          float sc[16];
          if (kv == 0) {
            const float s = __ldg(pa.k_scale + hb * 16 + slot);
#pragma unroll
            for (int e = 0; e < 16; ++e) sc[e] = s;
          } else {
            const float4* sp = reinterpret_cast<const float4*>(pa.v_scale + hb * D + ch * 16);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float4 f = __ldg(sp + e);
              sc[4 * e] = f.x; sc[4 * e + 1] = f.y; sc[4 * e + 2] = f.z; sc[4 * e + 3] = f.w;
            }
          }
          // int8 -> fp32 exactly: bias the byte to unsigned, drop it into the
          // mantissa of 2^23, subtract 2^23 + 128.
          const uint32_t qw[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u,
                                  q.w ^ 0x80808080u};
          uint32_t o[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint32_t word = qw[e >> 1];
            const int sh = (e & 1) * 2;
            const float f0 = __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7650 + sh)) -
                             8388736.f;
            const float f1 = __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7651 + sh)) -
                             8388736.f;
            o[e] = pack2<T>(f0 * sc[2 * e], f1 * sc[2 * e + 1]);
          }
          w0 = make_uint4(o[0], o[1], o[2], o[3]);
          w1 = make_uint4(o[4], o[5], o[6], o[7]);
        }
      } else {
        const uint4* src = reinterpret_cast<const uint4*>(
            fresh + (int64_t)b * f_bs + (int64_t)kvh * f_hs + (int64_t)(tok - P) * f_rs + ch * 16);
        w0 = __ldg(src);
        w1 = __ldg(src + 1);
      }
    }
    uint8_t* rowp = dst + (ch >> 2) * G::ATOM_BYTES + row * 128;
    const int u = (ch & 3) * 2;
    *reinterpret_cast<uint4*>(rowp + ((u ^ (row & 7)) << 4)) = w0;
    *reinterpret_cast<uint4*>(rowp + (((u + 1) ^ (row & 7)) << 4)) = w1;
  }
}

// Materialise the paged prefix (dequantised) and the fresh suffix of every
// sequence into a dense workspace K/V [batch, num_kv_heads, kv_pad, D] of the
// compute dtype, for the strategy used when many CTAs would otherwise each
// dequantise the same tiles (long suffixes under GQA).  One thread per 16
// elements; token rows in [kv_len_b, kv_len_b rounded up to 128) are zeroed so
// the attention kernel never reads uninitialised padding.
// Context-parallel shards read in place over NVLink: rank r's shard buffer
// (peer-mapped into this process) holds its prefix blocks, their scales and
// the suffix K/V of its zig-zag query rows:
//   [pool int8  shard_blocks x 2 x Hkv x 16 x D]
//   [k_scale f32 shard_blocks x Hkv x 16] [v_scale f32 shard_blocks x Hkv x D]
//   [suffix K  Hkv x 2c x D] [suffix V  Hkv x 2c x D]   (c = zig-zag chunk rows)
// Gathered block id blk lives on rank blk / shard_blocks; suffix row s lies in
// zig-zag chunk n = s / c, owned by rank n (n < world) or 2 world - 1 - n.
constexpr int kMaxPeers = 8;
struct PeerArgs {
  const uint8_t* base[kMaxPeers];
  int world;
  int shard_blocks;
  int zz_rows;
  int64_t kscale_off, vscale_off, suffix_off, suffix_v_off;
};

// peer.base[r] by a select chain, so the kernel parameter is read from
// parameter space rather than copied to local memory for a dynamic index.
__device__ __forceinline__ const uint8_t* peer_base(const PeerArgs& peer, int r) {
  const uint8_t* b = peer.base[0];
#pragma unroll
  for (int i = 1; i < kMaxPeers; ++i) b = (r == i) ? peer.base[i] : b;
  return b;
}

template <typename T, int D, bool PEER>
__global__ void __launch_bounds__(256)
    kvb_paged_materialize_kernel(PagedArgs pa, T* wk, T* wv, int q_len, int kv_pad, int* status,
                                 PeerArgs peer) {
  constexpr int NCH = D / 16;
  // The prefill launch that reads this workspace may start its CTAs' setup
  // now; it waits for this grid before touching memory.
  ptx::griddep_launch_dependents();
  const int b = blockIdx.z;
  const int kvh = blockIdx.y;
  const int P = pa.prefix_lens ? pa.prefix_lens[b] : pa.prefix_len;
  const int kv_len = P + q_len;
  const int kv_end = min(kv_pad, (kv_len + BN - 1) / BN * BN);
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)kv_end * NCH * 2) return;
  const int kv = (int)(idx / ((int64_t)kv_end * NCH));       // 0 = K, 1 = V
  const int rem = (int)(idx - (int64_t)kv * kv_end * NCH);
  const int tok = rem / NCH;
  const int ch = rem - tok * NCH;
  uint4 w0 = make_uint4(0, 0, 0, 0), w1 = make_uint4(0, 0, 0, 0);
  if (tok < kv_len) {
    if (tok < P) {
      const int bi = tok >> 4;
      const int blk =
          bi < pa.max_blocks ? __ldg(pa.block_table + (int64_t)b * pa.max_blocks + bi) : -1;
      if (blk < 0 || blk >= pa.num_blocks) {
        if (status) atomicOr(status, KVB_STATUS_BAD_BLOCK);
      } else if (!PEER && pa.pool16) {
        const uint4* src = reinterpret_cast<const uint4*>(
            reinterpret_cast<const T*>(pa.pool) +
            ((((int64_t)blk * 2 + kv) * pa.num_kv_heads + kvh) * 16 + (tok & 15)) * D + ch * 16);
        w0 = __ldg(src);
        w1 = __ldg(src + 1);
      } else {
        const int slot = tok & 15;
        const int8_t* pool = pa.pool;
        const float* kscale = pa.k_scale;
        const float* vscale = pa.v_scale;
        int lb = blk;
        if (PEER) {  // the owning rank's shard, read in place (plain loads over NVLink)
          const int r = blk / peer.shard_blocks;
          lb = blk - r * peer.shard_blocks;
          const uint8_t* base = peer_base(peer, r);
          pool = reinterpret_cast<const int8_t*>(base);
          kscale = reinterpret_cast<const float*>(base + peer.kscale_off);
          vscale = reinterpret_cast<const float*>(base + peer.vscale_off);
        }
        const int64_t hb = (int64_t)lb * pa.num_kv_heads + kvh;
        const uint4* qp = reinterpret_cast<const uint4*>(
            pool + (((int64_t)lb * 2 + kv) * pa.num_kv_heads + kvh) * 16 * D +
            (int64_t)slot * D + ch * 16);
        const uint4 q = PEER ? *qp : __ldg(qp);
        float sc[16];
        if (kv == 0) {
          const float sk = PEER ? kscale[hb * 16 + slot] : __ldg(kscale + hb * 16 + slot);
#pragma unroll
          for (int e = 0; e < 16; ++e) sc[e] = sk;
        } else {
          const float4* sp = reinterpret_cast<const float4*>(vscale + hb * D + ch * 16);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float4 f = PEER ? sp[e] : __ldg(sp + e);
            sc[4 * e] = f.x; sc[4 * e + 1] = f.y; sc[4 * e + 2] = f.z; sc[4 * e + 3] = f.w;
          }
        }
        const uint32_t qw[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u,
                                q.w ^ 0x80808080u};
        uint32_t o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const uint32_t word = qw[e >> 1];
          const int sh = (e & 1) * 2;
          const float f0 = __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7650 + sh)) - 8388736.f;
          const float f1 = __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7651 + sh)) - 8388736.f;
          o[e] = pack2<T>(f0 * sc[2 * e], f1 * sc[2 * e + 1]);
        }
        w0 = make_uint4(o[0], o[1], o[2], o[3]);
        w1 = make_uint4(o[4], o[5], o[6], o[7]);
      }
    } else if (PEER) {
      const int sr = tok - P;
      const int n = sr / peer.zz_rows;
      const int r = n < peer.world ? n : 2 * peer.world - 1 - n;
      const int row = (n < peer.world ? 0 : peer.zz_rows) + (sr - n * peer.zz_rows);
      const T* fresh = reinterpret_cast<const T*>(
          peer_base(peer, r) + (kv ? peer.suffix_v_off : peer.suffix_off));
      const uint4* src = reinterpret_cast<const uint4*>(
          fresh + ((int64_t)kvh * 2 * peer.zz_rows + row) * D + ch * 16);
      w0 = src[0];
      w1 = src[1];
    } else {
      const T* fresh = reinterpret_cast<const T*>(kv ? pa.v_new : pa.k_new);
      const int64_t bs = kv ? pa.vn_bs : pa.kn_bs, hs = kv ? pa.vn_hs : pa.kn_hs,
                    rs = kv ? pa.vn_rs : pa.kn_rs;
      const uint4* src = reinterpret_cast<const uint4*>(
          fresh + (int64_t)b * bs + (int64_t)kvh * hs + (int64_t)(tok - P) * rs + ch * 16);
      w0 = __ldg(src);
      w1 = __ldg(src + 1);
    }
  }
  T* dst = (kv ? wv : wk) + (((int64_t)b * pa.num_kv_heads + kvh) * kv_pad + tok) * D + ch * 16;
  reinterpret_cast<uint4*>(dst)[0] = w0;
  reinterpret_cast<uint4*>(dst)[1] = w1;
}

// Merge of split-key partials, the second launch of a split-key call.  One
// thread per (packed row, 8 features) of every group: LSE-weighted sum of the
// row's partials ([splits][batch][num_kv_heads][group rows][D], normalised,
// compute dtype; LSE fp32 [splits][batch][num_kv_heads][group rows]), online over
// batches of 16 splits whose loads are all in flight at once (a running maximum
// keeps the weights in range), written through the caller's strides; ch == 0
// threads also write the merged LSE.  Launched with programmatic dependent launch
// after the split kernel, so its CTAs are resident when that grid completes.
// (Merging in each group's last split CTA instead was slower at every measured
// shape: one CTA's loads pay a dependent L2 round trip per batch of splits.)
template <typename T, int D>
__global__ void __launch_bounds__(256)
    kvb_split_merge_kernel(const DenseArgs a, const PagedArgs pa, int splits, int64_t rows) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  constexpr int NCH = D / 8;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * NCH) return;
  const int64_t row = idx / NCH;                   // [batch][num_kv_heads][packed]
  const int ch = (int)(idx - row * NCH);
  const int packed = a.q_len;
  const int r = (int)(row % packed);
  const int64_t bg = row / packed;
  const int g = (int)(bg % pa.num_kv_heads);
  const int b = (int)(bg / pa.num_kv_heads);
  const T* o_part = reinterpret_cast<const T*>(a.o);
  constexpr int MB = 16;
  float m = -INFINITY, sum = 0.f;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
  for (int sp0 = 0; sp0 < splits; sp0 += MB) {
    float l[MB];
    uint4 v[MB];
#pragma unroll
    for (int u = 0; u < MB; ++u) {
      l[u] = -INFINITY;
      if (sp0 + u < splits) {
        l[u] = __ldcg(a.lse + (int64_t)(sp0 + u) * pa.lse_split_stride + row);
        v[u] = __ldcg(reinterpret_cast<const uint4*>(
            o_part + (int64_t)(sp0 + u) * pa.o_split_stride + row * D + ch * 8));
      }
    }
    float bm = m;
#pragma unroll
    for (int u = 0; u < MB; ++u) bm = fmaxf(bm, l[u]);
    if (bm == -INFINITY) continue;                  // no keys in any split so far
    const float c = __expf(m - bm);                 // 0 when m is still -inf
    sum *= c;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] *= c;
    m = bm;
#pragma unroll
    for (int u = 0; u < MB; ++u) {
      if (sp0 + u >= splits || l[u] == -INFINITY) continue;
      const float wt = __expf(l[u] - m);
      sum += wt;
      const uint32_t wv[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f;
        if constexpr (std::is_same<T, __half>::value)
          f = __half22float2(*reinterpret_cast<const __half2*>(&wv[e]));
        else
          f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv[e]));
        acc[2 * e] += wt * f.x;
        acc[2 * e + 1] += wt * f.y;
      }
    }
  }
  const float inv = sum > 0.f ? 1.f / sum : 0.f;
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) o[e] = pack2<T>(acc[2 * e] * inv, acc[2 * e + 1] * inv);
  const int head = g * pa.group_heads + r / pa.rows_per_head;
  const int i = r % pa.rows_per_head;
  T* dst = reinterpret_cast<T*>(pa.o_final) + (int64_t)b * pa.of_bs + (int64_t)head * pa.of_hs +
           (int64_t)i * pa.of_rs + ch * 8;
  *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
  if (pa.lse_final != nullptr && ch == 0)
    pa.lse_final[(int64_t)b * pa.lf_bs + (int64_t)head * pa.lf_hs + i] =
        sum > 0.f ? m + __logf(sum) : -INFINITY;
}

// DUALOK (dense launches only): a CTA whose second query tile has no rows (a
// varlen sequence's last odd tile, a single-tile sequence) gives slot 1 the
// same tile and the second half of the key range, so its two slots still run
// two chains in ping-pong; slot 0 merges the two halves in the epilogue.
template <typename T, int D, bool PAGED, bool SPLITKV = false, bool DUALOK = false>
__global__ void __launch_bounds__(Roles<PAGED>::kThreads)
    kvb_prefill_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const DenseArgs a,
                       const PagedArgs pa) {
  using G = Geo<D>;
  constexpr int kWarpTma = Roles<PAGED>::kWarpTma;
  constexpr int kWarpMma = Roles<PAGED>::kWarpMma;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;                                  // kSlots tiles
  uint8_t* sK = sQ + kSlots * G::TILE_BYTES;           // NS tiles
  uint8_t* sV = sK + G::NS * G::TILE_BYTES;            // NS tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + G::NS * G::TILE_BYTES);
  SharedCtl* ctl = reinterpret_cast<SharedCtl*>(bars + 32);
  float* xmax = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + G::BAR_BYTES);
  float* xsum = xmax + kSlots * 2 * 128;
  volatile int* abort_flag = &ctl->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  KVB_TRACE_SETUP();
  if (threadIdx.x == 0) KVB_TRACE_GT(4);
  auto bar = [&](int i) { return ptx::smem_u32(&bars[i]); };

  // ---- setup that touches no global memory ------------------------------
  // Runs while the preceding grid in the stream may still be finishing (the
  // launch allows programmatic dependent launch); everything from the wait
  // on sees that grid's writes.  TMEM is allocated here too: a dependent
  // launch only starts once every CTA of the preceding grid has signalled
  // (these kernels signal after their own allocation) or exited, so no CTA of
  // that grid can still be waiting to allocate on this SM.
  if (threadIdx.x == 0) {
    for (int sl = 0; sl < kSlots; ++sl) {
      ptx::mbar_init(bar(BAR_Q_FULL + sl), 1);
      ptx::mbar_init(bar(BAR_S_FULL + sl), 1);
      ptx::mbar_init(bar(BAR_P_FULL + sl), 4 * Roles<PAGED>::kHalves);  // one per softmax warp
      ptx::mbar_init(bar(BAR_O_FULL + sl), 1);
    }
    ptx::mbar_init(bar(BAR_DRAIN), 1);
    for (int st = 0; st < G::KSD; ++st) {
      ptx::mbar_init(bar(BAR_K_FULL + st), PAGED ? Roles<PAGED>::kConvWarps : 1);
      ptx::mbar_init(bar(BAR_K_EMPTY + st), 1);
    }
    for (int st = 0; st < G::NS; ++st) {
      ptx::mbar_init(bar(BAR_V_FULL + st), PAGED ? Roles<PAGED>::kConvWarps : 1);
      ptx::mbar_init(bar(BAR_V_EMPTY + st), 1);
    }
    ctl->abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kWarpTma && lane == 0) {
    ptx::prefetch_tmap(&tm_q);
    if (!PAGED) {
      ptx::prefetch_tmap(&tm_k);
      ptx::prefetch_tmap(&tm_v);
    }
  }
  if (warp == kWarpMma) {
    ptx::tmem_alloc(ptx::smem_u32(&ctl->tmem_base), G::TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  // ---- work item: two query tiles sharing one KV head ---------------------
  const int b = blockIdx.z;
  int head[kSlots], mtile[kSlots];
  const bool dual_split = SPLITKV && pa.dual;
  const int ctas = SPLITKV ? (int)gridDim.x / pa.tile_pairs : 1;  // CTAs per tile pair
  const int csplit = SPLITKV ? (int)blockIdx.x % ctas : 0;
  const int tpair = SPLITKV ? (int)blockIdx.x / ctas : 0;
  int vsplit[kSlots];                                              // key split of each slot
  vsplit[0] = dual_split ? 2 * csplit : csplit;
  vsplit[1] = dual_split ? 2 * csplit + 1 : csplit;
  if (SPLITKV) {  // two packed tiles of one KV head's group (or one tile twice), one key range each
    head[0] = head[1] = blockIdx.y;
    mtile[0] = dual_split ? 0 : 2 * tpair;
    mtile[1] = dual_split ? 0 : 2 * tpair + 1;
  } else if (a.pair_heads) {
    // grid (head pairs, query tiles, batch): blocks go out head-fastest, so every
    // head's heaviest (last) query tile is dispatched before any lighter one
    const int m = gridDim.y - 1 - blockIdx.y;
    head[0] = 2 * blockIdx.x;
    head[1] = 2 * blockIdx.x + 1;
    mtile[0] = mtile[1] = m;
  } else {
    const int x = gridDim.y - 1 - blockIdx.y;  // grid (heads, tile pairs, batch)
    head[0] = head[1] = blockIdx.x;
    mtile[0] = 2 * x;
    mtile[1] = 2 * x + 1;
  }
  const int kvh = head[0] / a.group;
  if (!PAGED && !SPLITKV && warp == kWarpTma && lane == 0 && a.cu_q == nullptr &&
      a.kv_prefix == nullptr) {
    // While the preceding grid finishes, pull this CTA's query tiles and first
    // key / value tiles into L2 (plain dense layout only: the coordinates come
    // from the kernel's parameters, no global read).  L2 is where every write
    // of that grid lands, so the loads after the wait below still see them;
    // the prefetch only moves the first HBM reads ahead.
#pragma unroll
    for (int sl = 0; sl < kSlots; ++sl)
      if (mtile[sl] * BM < a.q_len)
#pragma unroll
        for (int at = 0; at < G::NATOM; ++at)
          ptx::tma_prefetch_l2_4d(&tm_q, at * 64, mtile[sl] * BM, head[sl], b);
#pragma unroll
    for (int at = 0; at < G::NATOM; ++at) {
      ptx::tma_prefetch_l2_4d(&tm_k, at * 64, 0, kvh, b);
      ptx::tma_prefetch_l2_4d(&tm_v, at * 64, 0, kvh, b);
    }
  }
  ptx::griddep_wait();
  if (threadIdx.x == 0) KVB_TRACE_GT(5);
  int q_len = a.q_len, kv_len = a.kv_len, q_base = 0, k_base = 0, tb = b;
  int P = 0;  // paged: cached-prefix tokens of this sequence
  if (PAGED) {
    P = pa.prefix_lens ? pa.prefix_lens[b] : pa.prefix_len;
    kv_len = P + q_len;
  } else if (a.kv_prefix != nullptr) {
    kv_len = a.kv_prefix[b] + q_len;
  } else if (a.cu_q != nullptr) {
    q_base = a.cu_q[b];
    q_len = a.cu_q[b + 1] - q_base;
    k_base = a.cu_k[b];
    kv_len = a.cu_k[b + 1] - k_base;
    tb = 0;
  }
  // causal 1: bottom-right (j <= i + kv_len - q_len); 2: top-left (j <= i)
  const int off = (a.causal == 2) ? 0 : kv_len - (SPLITKV ? pa.rows_per_head : q_len);
  int q0[kSlots], q_rows[kSlots], n_t[kSlots], jbase[kSlots];   // jbase: first key tile
#pragma unroll
  for (int sl = 0; sl < kSlots; ++sl) {
    q0[sl] = mtile[sl] * BM;
    q_rows[sl] = max(0, min(BM, q_len - q0[sl]));
    int kv_end = (a.causal && !SPLITKV) ? min(kv_len, q0[sl] + q_rows[sl] + off) : kv_len;
    kv_end = max(kv_end, 0);
    n_t[sl] = q_rows[sl] > 0 ? (kv_end + BN - 1) / BN : 0;
    jbase[sl] = SPLITKV ? vsplit[sl] * pa.split_tiles : 0;
    if (SPLITKV) n_t[sl] = max(0, min(n_t[sl] - jbase[sl], pa.split_tiles));
  }
  if (q_rows[0] == 0 && q_rows[1] == 0) {        // uniform, before any barrier wait
    if (warp == kWarpMma) ptx::tmem_dealloc(tmem, G::TMEM_COLS);
    return;
  }
  bool dual_dense = false;
  if (DUALOK && !SPLITKV && !PAGED && q_rows[1] == 0 && n_t[0] >= 4) {
    // slot 1 takes slot 0's rows and the second half of its key tiles
    dual_dense = true;
    head[1] = head[0];
    q0[1] = q0[0];
    q_rows[1] = q_rows[0];
    const int half = (n_t[0] + 1) / 2;
    jbase[1] = half;
    n_t[1] = n_t[0] - half;
    n_t[0] = half;
  }
  const bool dual = dual_split || dual_dense;
  const int n_max = max(n_t[0], n_t[1]);
  // Position of slot s's key tile j in the K/V load sequence: the step j when
  // both slots read the same tile; in dual mode the loads alternate between
  // the slots while both have tiles (2j + s), then slot 0's continue in order
  // (slot 1 never has more tiles than slot 0).  Producer and consumers derive
  // ring stages and phases from it, so every stage is used in sequence.
  auto ring_pos = [&](int s, int j) -> int {
    return !dual ? j : (j < n_t[1] ? 2 * j + s : n_t[1] + j);
  };

  // Every CTA of this grid is resident or done once all have passed here: the
  // next launch may begin its own setup.
  ptx::griddep_launch_dependents();
  if (threadIdx.x == 0) KVB_TRACE_AT(0);

  if (PAGED && warp >= kWarpTma && warp < kWarpTma + Roles<PAGED>::kConvWarps) {
    // ===================================================== paged gather
    const int ct = threadIdx.x - kWarpTma * 32;
    constexpr int nct = Roles<PAGED>::kConvWarps * 32;
    if (n_max > 0) {
      if (ct == 0) {
#pragma unroll
        for (int sl = 0; sl < kSlots; ++sl) {
          if (n_t[sl] == 0) continue;
          ptx::mbar_arrive_expect_tx(bar(BAR_Q_FULL + sl), G::TILE_BYTES);
#pragma unroll
          for (int at = 0; at < G::NATOM; ++at)
            ptx::tma_load_4d(ptx::smem_u32(sQ + sl * G::TILE_BYTES + at * G::ATOM_BYTES), &tm_q,
                             at * 64, q0[sl], head[sl], b, bar(BAR_Q_FULL + sl));
        }
      }
#pragma unroll 1
      for (int j = 0; j < n_max; ++j) {
        const int st = j % G::NS;
        const uint32_t ph = (j / G::NS) & 1;
        bool ok = wait_bar(bar(BAR_K_EMPTY + st), ph ^ 1, abort_flag, a.status,
                           KVB_STATUS_LOAD_WAIT);
        if (!__all_sync(0xffffffffu, ok)) break;
        gather_kv_tile<T, D>(sK + st * G::TILE_BYTES, pa, b, kvh, j * BN, P, kv_len, 0, ct, nct,
                             a.status);
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar(BAR_K_FULL + st));
        ok = wait_bar(bar(BAR_V_EMPTY + st), ph ^ 1, abort_flag, a.status, KVB_STATUS_LOAD_WAIT);
        if (!__all_sync(0xffffffffu, ok)) break;
        gather_kv_tile<T, D>(sV + st * G::TILE_BYTES, pa, b, kvh, j * BN, P, kv_len, 1, ct, nct,
                             a.status);
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar(BAR_V_FULL + st));
      }
      if (*abort_flag && ct == 0) {
        // Drain the Q loads this thread issued before leaving.
        for (int sl = 0; sl < kSlots; ++sl)
          if (n_t[sl] > 0) wait_bar(bar(BAR_Q_FULL + sl), 0, abort_flag, nullptr, 0);
      }
    }
  } else if (!PAGED && warp == kWarpTma) {
    // ================================================================ TMA
    if (lane == 0 && n_max > 0) {
      // Q of slot 0, then K0, then (once K0 has landed) Q of slot 1
      auto load_q = [&](int sl) {
        if (n_t[sl] == 0) return;
        ptx::mbar_arrive_expect_tx(bar(BAR_Q_FULL + sl), G::TILE_BYTES);
#pragma unroll
        for (int at = 0; at < G::NATOM; ++at)
          ptx::tma_load_4d(ptx::smem_u32(sQ + sl * G::TILE_BYTES + at * G::ATOM_BYTES), &tm_q,
                           at * 64, q_base + q0[sl], head[sl], tb, bar(BAR_Q_FULL + sl));
      };
      load_q(0);
      // Ring position r = ring_pos(slot, j): stage r % depth, phase (r / depth) & 1,
      // the K ring KSD deep in dual mode (its last stage in slot 1's Q buffer).
      const int per = dual ? 2 : 1;
      const int ks = dual ? G::KSD : G::NS;
      int last_k[4], last_v[4];   // phase of each stage's last issued load
#pragma unroll
      for (int i = 0; i < 4; ++i) last_k[i] = last_v[i] = -1;
      bool go = true;
#pragma unroll 1
      for (int j = 0; go && j < n_max; ++j) {
#pragma unroll 1
        for (int t = 0; t < per; ++t) {
          if (dual && j >= n_t[t]) continue;
          const int r = ring_pos(t, j);
          const int st = r % ks;
          const uint32_t ph = (r / ks) & 1;
          const int ky = k_base + ((dual && t) ? jbase[1] : jbase[0]) * BN + j * BN;
          if (!wait_bar(bar(BAR_K_EMPTY + st), ph ^ 1, abort_flag, a.status, KVB_STATUS_LOAD_WAIT)) {
            go = false;
            break;
          }
          if (j < 16 && t == 0) KVB_TRACE_AT(16 + j);
          ptx::mbar_arrive_expect_tx(bar(BAR_K_FULL + st), G::TILE_BYTES);
          uint8_t* kdst = st < G::NS ? sK + st * G::TILE_BYTES : sQ + G::TILE_BYTES;
#pragma unroll
          for (int at = 0; at < G::NATOM; ++at)
            ptx::tma_load_4d(ptx::smem_u32(kdst + at * G::ATOM_BYTES), &tm_k,
                             at * 64, ky, kvh, tb, bar(BAR_K_FULL + st));
          last_k[st] = (int)ph;
          if (j == 0 && t == 0 && !dual) {
            // Q of slot 1, V0 and the next K tiles are needed only after slot 0's
            // first S: hold them back until K0 has landed, so that the first S
            // MMA's operands do not share DRAM bandwidth with them at launch.
            if (!wait_bar(bar(BAR_K_FULL), 0, abort_flag, a.status, KVB_STATUS_LOAD_WAIT)) {
              go = false;
              break;
            }
            for (int sl = 1; sl < kSlots; ++sl) load_q(sl);
          }
        }
#pragma unroll 1
        for (int t = 0; go && t < per; ++t) {
          if (dual && j >= n_t[t]) continue;
          const int r = ring_pos(t, j);
          const int st = r % G::NS;
          const uint32_t ph = (r / G::NS) & 1;
          const int ky = k_base + ((dual && t) ? jbase[1] : jbase[0]) * BN + j * BN;
          if (!wait_bar(bar(BAR_V_EMPTY + st), ph ^ 1, abort_flag, a.status, KVB_STATUS_LOAD_WAIT)) {
            go = false;
            break;
          }
          if (j < 16 && t == 0) KVB_TRACE_AT(32 + j);
          ptx::mbar_arrive_expect_tx(bar(BAR_V_FULL + st), G::TILE_BYTES);
#pragma unroll
          for (int at = 0; at < G::NATOM; ++at)
            ptx::tma_load_4d(ptx::smem_u32(sV + st * G::TILE_BYTES + at * G::ATOM_BYTES), &tm_v,
                             at * 64, ky, kvh, tb, bar(BAR_V_FULL + st));
          last_v[st] = (int)ph;
        }
      }
      if (*abort_flag) {
        // Drain: wait (bounded) for each stage's last issued loads to land.
        for (int st = 0; st < 4; ++st) {
          if (last_k[st] >= 0) wait_bar(bar(BAR_K_FULL + st), last_k[st], abort_flag, nullptr, 0);
          if (last_v[st] >= 0) wait_bar(bar(BAR_V_FULL + st), last_v[st], abort_flag, nullptr, 0);
        }
      }
    }
  } else if (warp == kWarpMma) {
    // ================================================================ MMA
    if (lane == 0 && n_max > 0) {
      constexpr uint32_t idesc_s = ptx::idesc_f16(BM, BN, ab_format<T>(), 0, 0);
      constexpr uint32_t idesc_o = ptx::idesc_f16(BM, G::DP, ab_format<T>(), 0, 1);
      const uint32_t sQa = ptx::smem_u32(sQ);
      const uint32_t sKa = ptx::smem_u32(sK);
      const uint32_t sVa = ptx::smem_u32(sV);

      // Descriptor words are built once; between instructions only the low
      // word advances (one add per operand), which keeps the single issuing
      // thread ahead of the tensor pipe.
      constexpr uint32_t hi = ptx::desc_hi_sw128(1024);
      const uint32_t q_lo = ptx::desc_lo(sQa, 16);
      const uint32_t k_lo = ptx::desc_lo(sKa, 16);
      const uint32_t v_lo = ptx::desc_lo(sVa, G::ATOM_BYTES);
      constexpr uint32_t TILE16 = G::TILE_BYTES >> 4;

      auto issue_s = [&](int sl, int j, int kst) {
        if (j < 16) KVB_TRACE_AT(48 + 96 * sl + j);
        const uint32_t qa = q_lo + (dual ? 0 : sl) * TILE16;
        // stage NS (dual mode only) is slot 1's Q buffer
        const uint32_t kb = kst < G::NS ? k_lo + kst * TILE16 : q_lo + TILE16;
        const uint32_t tS = tmem + G::s_col(sl);
#pragma unroll
        for (int kk = 0; kk < G::QK_STEPS; ++kk) {
          const uint32_t off16 = ((kk >> 2) * G::ATOM_BYTES + (kk & 3) * 32) >> 4;
          ptx::mma_ss_lohi(tS, qa + off16, hi, kb + off16, hi, idesc_s, kk > 0 ? 1u : 0u);
        }
        ptx::mma_commit(bar(BAR_S_FULL + sl));
        if (sl == 0 && j < 16) KVB_TRACE_AT(224 + j);
      };
      // P of S columns [c, c+16) sits at P column (c / PC) * PC + (c % PC) / 2:
      // each softmax warpgroup packs its PC columns over the start of its own range.
      constexpr int PC = BN / Roles<PAGED>::kHalves;
      auto issue_pv = [&](int sl, int j, int vst) {
        if (j < 16) KVB_TRACE_AT(96 + 96 * sl + j);
        const uint32_t vb = v_lo + vst * TILE16;
        const uint32_t tP = tmem + G::s_col(sl);
        const uint32_t tO = tmem + G::o_col(sl);
#pragma unroll
        for (int kk = 0; kk < G::PV_STEPS; ++kk)
          ptx::mma_ts_lohi(tO, tP + (16 * kk / PC) * PC + (16 * kk % PC) / 2,
                           vb + ((kk * 16 * 128) >> 4), hi, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        if (sl == 0 && j < 16) KVB_TRACE_AT(240 + j);
      };

      if (dual) {
        // Each slot streams its own key range; slot sl's tile j sits at ring
        // position ring_pos(sl, j) (K stage r % KSD, V stage r % NS).
        bool ok = true;
#pragma unroll
        for (int sl = 0; sl < kSlots && ok; ++sl) {
          if (n_t[sl] == 0) continue;
          ok = wait_bar(bar(BAR_K_FULL + sl), 0, abort_flag, a.status, KVB_STATUS_MMA_WAIT) &&
               wait_bar(bar(BAR_Q_FULL), 0, abort_flag, a.status, KVB_STATUS_MMA_WAIT);
          if (!ok) break;
          ptx::tc_fence_after();
          issue_s(sl, 0, sl);   // ring positions 0 and 1: K stages 0 and 1
          ptx::mma_commit(bar(BAR_K_EMPTY + sl));
        }
#pragma unroll 1
        for (int j = 0; ok && j < n_max; ++j) {
#pragma unroll
          for (int sl = 0; sl < kSlots; ++sl) {
            if (j >= n_t[sl]) continue;
            const int r = ring_pos(sl, j), r1 = ring_pos(sl, j + 1);
            const int st = r % G::NS, st1 = r1 % G::KSD;
            const uint32_t ph = (r / G::NS) & 1, ph1 = (r1 / G::KSD) & 1;
            if (!wait_bar(bar(BAR_P_FULL + sl), j & 1, abort_flag, a.status, KVB_STATUS_MMA_WAIT) ||
                !wait_bar(bar(BAR_V_FULL + st), ph, abort_flag, a.status, KVB_STATUS_MMA_WAIT)) {
              ok = false;
              break;
            }
            if (sl == 0 && j < 16) KVB_TRACE_AT(128 + j);
            ptx::tc_fence_after();
            issue_pv(sl, j, st);
            ptx::mma_commit(bar(BAR_V_EMPTY + st));
            if (j + 1 < n_t[sl]) {
              if (!wait_bar(bar(BAR_K_FULL + st1), ph1, abort_flag, a.status, KVB_STATUS_MMA_WAIT)) {
                ok = false;
                break;
              }
              issue_s(sl, j + 1, st1);
              ptx::mma_commit(bar(BAR_K_EMPTY + st1));
            } else {
              ptx::mma_commit(bar(BAR_O_FULL + sl));  // this slot's last PV
            }
          }
        }
      } else {
        bool ok = wait_bar(bar(BAR_K_FULL), 0, abort_flag, a.status, KVB_STATUS_MMA_WAIT);
#pragma unroll
        for (int sl = 0; sl < kSlots && ok; ++sl) {
          if (n_t[sl] == 0) continue;
          ok = wait_bar(bar(BAR_Q_FULL + sl), 0, abort_flag, a.status, KVB_STATUS_MMA_WAIT);
          if (!ok) break;
          ptx::tc_fence_after();
          issue_s(sl, 0, 0);
        }
        if (ok) ptx::mma_commit(bar(BAR_K_EMPTY));
#pragma unroll 1
        for (int j = 0; ok && j < n_max; ++j) {
          const int st = j % G::NS;
          const uint32_t ph = (j / G::NS) & 1;
          const int st1 = (j + 1) % G::NS;
          const uint32_t ph1 = ((j + 1) / G::NS) & 1;
          bool v_ready = false, k_next_ready = false;
#pragma unroll
          for (int sl = 0; sl < kSlots; ++sl) {
            if (j >= n_t[sl]) continue;
            if (!wait_bar(bar(BAR_P_FULL + sl), j & 1, abort_flag, a.status, KVB_STATUS_MMA_WAIT)) {
              ok = false;
              break;
            }
            if (sl == 0 && j < 16) KVB_TRACE_AT(112 + j);
            if (!v_ready) {
              if (!wait_bar(bar(BAR_V_FULL + st), ph, abort_flag, a.status, KVB_STATUS_MMA_WAIT)) {
                ok = false;
                break;
              }
              v_ready = true;
            }
            if (sl == 0 && j < 16) KVB_TRACE_AT(128 + j);
            ptx::tc_fence_after();
            issue_pv(sl, j, st);
            if (j + 1 < n_t[sl]) {
              if (!k_next_ready) {
                if (!wait_bar(bar(BAR_K_FULL + st1), ph1, abort_flag, a.status,
                              KVB_STATUS_MMA_WAIT)) {
                  ok = false;
                  break;
                }
                k_next_ready = true;
              }
              issue_s(sl, j + 1, st1);
            } else {
              ptx::mma_commit(bar(BAR_O_FULL + sl));  // this slot's last PV
            }
          }
          if (!ok) break;
          ptx::mma_commit(bar(BAR_V_EMPTY + st));
          if (k_next_ready) ptx::mma_commit(bar(BAR_K_EMPTY + st1));
        }
      }
      // Drain: every MMA issued above completes before TMEM can be freed.
      ptx::mma_commit(bar(BAR_DRAIN));
      wait_bar(bar(BAR_DRAIN), 0, abort_flag, nullptr, 0);
    }
  } else {
    // ============================================================ softmax
    // Each row of a slot is owned by one thread per column half (kHalves
    // warpgroups); the two threads of a row sit in the "pair" of warps
    // w and w + 4 and agree on every decision that touches the row (running
    // maximum, exact path, abort) through a 64-thread barrier reduction.
    constexpr int H = Roles<PAGED>::kHalves;
    constexpr int COLS = BN / H;                  // S columns per thread
    constexpr int CW = (H == 1) ? 32 : 16;        // TMEM load width
    constexpr int NCH = COLS / CW;
    constexpr int kPoly = poly_pairs_of_8<D>();
    constexpr int DH = D / H;                     // O columns per thread
    constexpr int OCW = (DH % 32 == 0) ? 32 : 16;
    const int grp = warp >> 2;
    const int sl = grp / H;                       // slot of this warpgroup
    const int hf = grp % H;                       // column half
    const int t = threadIdx.x & 127;              // row within the tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_base + G::s_col(sl) + hf * COLS;
    const uint32_t tO = tmem + lane_base + G::o_col(sl) + hf * DH;
    const uint32_t pair_bar = 1 + sl * 4 + (warp & 3);
    auto pair_any = [&](bool v) -> bool {
      if constexpr (H == 1)
        return __any_sync(0xffffffffu, v);
      else
        return ptx::bar_red_or(pair_bar, 64, v);
    };
    const int h = head[sl];
    const int q0s = q0[sl];
    const int n_tiles = n_t[sl];
    const int jb = (SPLITKV || DUALOK) ? jbase[sl] : 0;
    const int qi = q0s + t;
    const float sl2 = a.scale_log2;
    constexpr float kSumLimit = std::is_same<T, __half>::value ? 32768.f : 1.0995116e12f;
    constexpr bool kGuessMax = SPLITKV && std::is_same<T, __nv_bfloat16>::value;
    constexpr float kSumFloor = 5.42101086e-20f;   // 2^-64
    float m_run = -INFINITY;
    float l_run = 0.f;   // row sum over this thread's columns
    bool ok = true;

#pragma unroll 1
    for (int j = 0; j < n_tiles; ++j) {
      ok = wait_bar(bar(BAR_S_FULL + sl), j & 1, abort_flag, a.status, KVB_STATUS_SOFTMAX_WAIT);
      ptx::tc_fence_after();
      if (t == 0 && hf == 0 && j < 16) KVB_TRACE_AT(64 + 96 * sl + j);

      const int kv0 = (jb + j) * BN;
      // split decode: packed row qi is row qi % rows_per_head of its head
      const int qrow = SPLITKV ? qi % pa.rows_per_head : qi;
      const bool need_mask =
          (kv0 + BN > kv_len) || (a.causal && kv0 + BN - 1 > (SPLITKV ? 0 : q0s) + off);
      const int lim = (a.causal ? min(kv_len - 1, qrow + off) : kv_len - 1) - kv0;

      // Stale-maximum softmax.  After the first tile, each tile is
      // exponentiated against the running maximum in one pass with no max
      // tracking.  The maximum only has to be raised before a probability
      // could leave the range of the P operand (2^40 keeps bf16 P and the
      // fp32 sums far from overflow; fp16 P tops out at 65504, so 2^15
      // there).  Every probability is bounded by the sum over the thread's
      // columns, so that sum is the check.  Rows that fail it (in either
      // half), and rows without a maximum yet, take the exact path: tile
      // maximum, O rescale, redo.  The final normalisation uses the same
      // maximum as the exponentials, so the result is exact up to rounding.
      //
      // Split-key launches in bf16: a row's first tile tries the maximum 0
      // (log2 domain) before it has one; bf16 P keeps float32's exponent range,
      // so any sum in [2^-64, 2^40] over the thread's columns leaves every
      // probability that matters normal and finite, and the rounding of P is
      // the same relative to any maximum.  Rows outside that range (and fp16,
      // whose P range is narrow) take the exact path as before.  A split of a
      // few key tiles saves the first tile's maximum pass (16 new tokens over
      // 32 K keys: 60.4 -> 59.5 us); the prefill launches keep the exact first
      // tile (no gain on the reuse prefill, 2.4 % slower on long causal prefill).
      float alpha = 1.f;
      float sum = 0.f;
      uint32_t pk[COLS / 2];
      const bool first = m_run == -INFINITY;
      bool need = !ok || (!kGuessMax && first);
      if (!__any_sync(0xffffffffu, need)) {
        const float m_try = (kGuessMax && first) ? 0.f : m_run;
        sum = need_mask ? cols_exp<T, true, NCH, CW, kPoly>(tS, hf * COLS, sl2, m_try, lim, pk)
                        : cols_exp<T, false, NCH, CW, kPoly>(tS, hf * COLS, sl2, m_try, lim, pk);
        need = !(sum <= kSumLimit) ||   // also catches inf / NaN
               (kGuessMax && first && !(sum >= kSumFloor));
      }
      if (t == 0 && sl == 0 && j < 16) KVB_TRACE_AT(256 + 48 * hf + j);
      const bool redo = pair_any(need);
      if (t == 0 && sl == 0 && hf == 0 && j < 16) KVB_TRACE_AT(272 + j);
      if (kGuessMax && !redo && first) m_run = 0.f;   // both threads of the row took the guess
      if (redo) {
        if (pair_any(!ok)) {
          ok = false;
          break;
        }
        float raw_mx = need_mask ? cols_row_max<true, NCH, CW>(tS, hf * COLS, lim)
                                 : cols_row_max<false, NCH, CW>(tS, hf * COLS, lim);
        if constexpr (H == 2) {
          xmax[(sl * 2 + hf) * 128 + t] = raw_mx;
          ptx::bar_sync(pair_bar, 64);
          raw_mx = fmaxf(raw_mx, xmax[(sl * 2 + (hf ^ 1)) * 128 + t]);
        }
        const float m_tile = raw_mx * sl2;
        const bool raise = m_tile > m_run && raw_mx > -INFINITY;
        if (raise) {
          alpha = ptx::ex2(m_run - m_tile);
          m_run = m_tile;
        }
        // O rescale over this thread's columns (PV_{j-1} completed before S_j
        // was committed)
        if (j > 0 && __any_sync(0xffffffffu, raise)) {
          const float f = raise ? alpha : 1.f;
#pragma unroll 1
          for (int c = 0; c < DH; c += OCW) {
            uint32_t r[OCW];
            tmem_ld_cw<OCW>(tO + c, r);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < OCW; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * f);
            if constexpr (OCW == 32)
              ptx::tmem_st32(tO + c, r);
            else
              ptx::tmem_st16(tO + c, r);
          }
        }
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        sum = need_mask ? cols_exp<T, true, NCH, CW, kPoly>(tS, hf * COLS, sl2, m_use, lim, pk)
                        : cols_exp<T, false, NCH, CW, kPoly>(tS, hf * COLS, sl2, m_use, lim, pk);
      }
      store_p<COLS / 2>(tS, pk);
      l_run = l_run * alpha + sum;
      ptx::tmem_wait_st();
      if (t == 0 && sl == 0 && j < 16) KVB_TRACE_AT(288 + 32 * hf + j);
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar(BAR_P_FULL + sl));
      if (lane == 0 && warp == 3 && j < 16) KVB_TRACE_AT(208 + j);
      if (lane == 0 && sl == 0 && j == 4) KVB_TRACE_AT(8 + (warp & 7));   // every warp, tile 4
      if (t == 0 && hf == 0 && j < 16) KVB_TRACE_AT(80 + 96 * sl + j);
    }

    // ---- epilogue --------------------------------------------------------
    bool have_o = n_tiles > 0 && ok;
    if (have_o) {
      have_o = wait_bar(bar(BAR_O_FULL + sl), 0, abort_flag, a.status, KVB_STATUS_EPILOGUE_WAIT);
      have_o = __all_sync(0xffffffffu, have_o);
      ptx::tc_fence_after();
    }
    if (t == 0 && sl == 0 && hf == 0) KVB_TRACE_AT(2);
    float l_tot = l_run;
    if constexpr (H == 2) {  // both warps of the pair always reach this barrier once
      xsum[(sl * 2 + hf) * 128 + t] = l_run;
      ptx::bar_sync(pair_bar, 64);
      l_tot += xsum[(sl * 2 + (hf ^ 1)) * 128 + t];
    }
    const bool row_valid = t < q_rows[sl];
    const float inv_l = (l_tot > 0.f) ? 1.f / l_tot : 0.f;
    // dual split-key CTAs merge their two key splits and write one partial (index csplit)
    const bool merge2 = (DUALOK && dual_dense) || dual_split;
    const int part = dual_split ? csplit : vsplit[sl];
    T* obase = reinterpret_cast<T*>(a.o) + hf * DH + (SPLITKV ? part * pa.o_split_stride : 0) +
               (a.cu_q ? (int64_t)q_base * a.o_rs + (int64_t)h * a.o_hs
                       : (int64_t)b * a.o_bs + (int64_t)h * a.o_hs);
    constexpr int NC = DH / 8;                   // 16-byte pieces per row segment
    constexpr int ROT = 8 / (NC % 8 == 0 ? 8 : NC % 4 == 0 ? 4 : 2);
    constexpr int RPS = 32 / NC;                 // rows per store instruction
    const int wrow = (warp & 3) * 32;            // first row of this warp within the tile
    if (merge2) {
      // Two key ranges of one query tile: slot 1 hands each row's maximum and sum
      // to slot 0 (through the exact path's exchange slots, idle now), and slot 0
      // writes O = (O0 2^(m0-m) + O1 2^(m1-m)) / (l0 2^(m0-m) + l1 2^(m1-m)).
      if (sl == 1 && hf == 0) {
        xmax[256 + t] = have_o ? m_run : -INFINITY;
        xmax[384 + t] = have_o ? l_tot : 0.f;
      }
      ptx::bar_sync(9, 4 * kSlots * H * 32);     // every softmax warp, once
      if (sl == 0) {
        bool have_o1 = n_t[1] > 0 && wait_bar(bar(BAR_O_FULL + 1), 0, abort_flag, a.status,
                                              KVB_STATUS_EPILOGUE_WAIT);
        have_o1 = __all_sync(0xffffffffu, have_o1);
        ptx::tc_fence_after();
        const float m1 = xmax[256 + t], l1 = xmax[384 + t];
        const float m0 = have_o ? m_run : -INFINITY, l0 = have_o ? l_tot : 0.f;
        const float mm = fmaxf(m0, m1);
        const float a0 = (m0 == -INFINITY) ? 0.f : ptx::ex2(m0 - mm);
        const float a1 = (m1 == -INFINITY || !have_o1) ? 0.f : ptx::ex2(m1 - mm);
        const float L = l0 * a0 + l1 * a1;
        const float inv = L > 0.f ? 1.f / L : 0.f;
        const float w0 = a0 * inv, w1 = a1 * inv;
        const uint32_t tO1 = tmem + lane_base + G::o_col(1) + hf * DH;
        // every MMA has completed (both O_FULL commits): the Q tile is free
        uint4* stage = reinterpret_cast<uint4*>(sQ) + (hf * 4 + (warp & 3)) * 32 * NC;
#pragma unroll 1
        for (int c = 0; c < DH; c += OCW) {
          uint32_t r0[OCW], r1[OCW];
          tmem_ld_cw<OCW>(tO + c, r0);
          tmem_ld_cw<OCW>(tO1 + c, r1);
          ptx::tmem_wait_ld();
          uint32_t pk[OCW / 2];
#pragma unroll
          for (int i = 0; i < OCW / 2; ++i)
            pk[i] = pack2<T>(__uint_as_float(r0[2 * i]) * w0 + __uint_as_float(r1[2 * i]) * w1,
                             __uint_as_float(r0[2 * i + 1]) * w0 +
                                 __uint_as_float(r1[2 * i + 1]) * w1);
#pragma unroll
          for (int i = 0; i < OCW / 8; ++i)
            stage[lane * NC + (c / 8 + i + lane / ROT) % NC] =
                make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
        __syncwarp();
        const int pr = lane / NC, pc = lane % NC;
#pragma unroll 1
        for (int r0_ = 0; r0_ < 32; r0_ += RPS) {
          const int rr = r0_ + pr;
          if (pr < RPS && rr < 32 && wrow + rr < q_rows[0])
            *reinterpret_cast<uint4*>(obase + (int64_t)(q0s + wrow + rr) * a.o_rs + pc * 8) =
                stage[rr * NC + (pc + rr / ROT) % NC];
        }
        if (hf == 0 && row_valid && a.lse != nullptr) {
          const float lse = L > 0.f ? (mm + ptx::lg2(L)) * 0.69314718055994531f : -INFINITY;
          if (a.cu_q)
            a.lse[(int64_t)h * a.lse_hs + q_base + qi] = lse;
          else
            a.lse[(SPLITKV ? part * pa.lse_split_stride : 0) + (int64_t)b * a.lse_bs +
                  (int64_t)h * a.lse_hs + qi] = lse;
        }
      }
    } else if (have_o) {
      // The warp's 32 output row segments go through shared memory, so that the
      // global stores write whole segments (NC lanes per row) instead of one
      // 16-byte piece of 32 different rows per instruction.  The slot's Q tile
      // is free: the O_FULL commit follows every MMA that read it.  Pieces are
      // rotated by row so that neither pass has bank conflicts.
      uint4* stage = reinterpret_cast<uint4*>(sQ + sl * G::TILE_BYTES) +
                     (hf * 4 + (warp & 3)) * 32 * NC;
#pragma unroll 1
      for (int c = 0; c < DH; c += OCW) {
        uint32_t r[OCW];
        tmem_ld_cw<OCW>(tO + c, r);
        ptx::tmem_wait_ld();
        uint32_t pk[OCW / 2];
#pragma unroll
        for (int i = 0; i < OCW / 2; ++i)
          pk[i] = pack2<T>(__uint_as_float(r[2 * i]) * inv_l, __uint_as_float(r[2 * i + 1]) * inv_l);
#pragma unroll
        for (int i = 0; i < OCW / 8; ++i)
          stage[lane * NC + (c / 8 + i + lane / ROT) % NC] =
              make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      }
      __syncwarp();
      const int pr = lane / NC, pc = lane % NC;
#pragma unroll 1
      for (int r0 = 0; r0 < 32; r0 += RPS) {
        const int rr = r0 + pr;
        if (pr < RPS && rr < 32 && wrow + rr < q_rows[sl])
          *reinterpret_cast<uint4*>(obase + (int64_t)(q0s + wrow + rr) * a.o_rs + pc * 8) =
              stage[rr * NC + (pc + rr / ROT) % NC];
      }
    } else if (row_valid) {
      // no key tiles (or an aborted launch): zeros
      uint4* dst = reinterpret_cast<uint4*>(obase + (int64_t)qi * a.o_rs);
#pragma unroll
      for (int i = 0; i < DH / 8; ++i) dst[i] = make_uint4(0, 0, 0, 0);
    }
    if (!merge2 && hf == 0 && row_valid && a.lse != nullptr) {
      const float lse = (l_tot > 0.f && have_o) ? (m_run + ptx::lg2(l_tot)) * 0.69314718055994531f
                                                : -INFINITY;
      if (a.cu_q)
        a.lse[(int64_t)h * a.lse_hs + q_base + qi] = lse;
      else
        a.lse[(SPLITKV ? part * pa.lse_split_stride : 0) + (int64_t)b * a.lse_bs +
              (int64_t)h * a.lse_hs + qi] = lse;
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) KVB_TRACE_AT(3);
  if (threadIdx.x == 0) KVB_TRACE_GT(6);
  if (warp == kWarpMma) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, G::TMEM_COLS);
  }
}

// ============================================================================
// Host side
// ============================================================================

static thread_local std::string g_last_error;

static int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 4-D map over (head_dim, rows, heads, batch) with a 64 x 128 x 1 x 1 box and
// 128-byte swizzle.  Strides are in elements.
static bool make_map(CUtensorMap* m, const void* base, int dtype, int head_dim, int64_t rows,
                     int64_t heads, int64_t batch, int64_t row_stride, int64_t head_stride,
                     int64_t batch_stride, std::string* err) {
  auto enc = tensor_map_encoder();
  if (!enc) {
    *err = "cuTensorMapEncodeTiled unavailable from the CUDA driver";
    return false;
  }
  cuuint64_t dims[4] = {(cuuint64_t)head_dim, (cuuint64_t)rows, (cuuint64_t)heads,
                        (cuuint64_t)batch};
  cuuint64_t strides[3] = {(cuuint64_t)row_stride * 2, (cuuint64_t)head_stride * 2,
                           (cuuint64_t)batch_stride * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)BM, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m,
                   dtype == KVB_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r);
    return false;
  }
  return true;
}

// Launch with programmatic dependent launch allowed: the kernel's CTAs may
// start, and run their setup that touches no global memory, while the
// preceding grid in the stream finishes.  The prefill kernel orders every
// global access after griddepcontrol.wait, so results are as with plain
// stream order.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, int threads, int smem,
                              cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

template <typename T, int D>
static int launch_dense_core(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                             const DenseArgs& a, int batch, int num_q_heads, int q_len,
                             cudaStream_t stream) {
  using G = Geo<D>;
  const int q_tiles = (q_len + BM - 1) / BM;
  // Launches that can have a CTA whose second query tile is empty (varlen, or an
  // odd tile count of one head) take the DUALOK instantiation; the others keep
  // the plain kernel.
  const bool dualok = !a.pair_heads && (a.cu_q != nullptr || q_tiles % 2 == 1);
  auto kern = dualok ? kvb_prefill_kernel<T, D, false, false, true>
                     : kvb_prefill_kernel<T, D, false>;
  static thread_local int configured_device[2] = {-1, -1};
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device[dualok] != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         G::SMEM_BYTES);
    if (e != cudaSuccess)
      return fail(KVB_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    configured_device[dualok] = dev;
  }
  // head-fastest grids: each head's (pair's) heaviest query tiles go out first
  dim3 grid = a.pair_heads ? dim3(num_q_heads / 2, q_tiles, batch)
                           : dim3(num_q_heads, (q_tiles + 1) / 2, batch);
  PagedArgs none = {};
  cudaError_t e = launch_pdl(kern, grid, Roles<false>::kThreads, G::SMEM_BYTES, stream, tq, tk,
                             tv, a, none);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(KVB_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
  return KVB_OK;
}

template <typename T, int D>
static int launch_dense(const KvbPrefillParams& p, cudaStream_t stream) {
  using G = Geo<D>;
  const bool varlen = p.cu_seqlens_q != nullptr;
  CUtensorMap tq, tk, tv;
  std::string err;
  const int64_t qrows = varlen ? p.total_q : p.q_len;
  const int64_t krows = std::max<int64_t>(1, varlen ? p.total_k : p.kv_len);
  const int64_t nb = varlen ? 1 : p.batch;
  // batch stride of a 1-batch varlen map only has to be a valid multiple of 16 bytes
  const int64_t qbs = varlen ? 8 : p.q_batch_stride;
  const int64_t kbs = varlen ? 8 : p.k_batch_stride;
  const int64_t vbs = varlen ? 8 : p.v_batch_stride;
  if (!make_map(&tq, p.q, p.dtype, D, qrows, p.num_q_heads, nb, p.q_row_stride, p.q_head_stride,
                qbs, &err) ||
      !make_map(&tk, p.k, p.dtype, D, krows, p.num_kv_heads, nb, p.k_row_stride, p.k_head_stride,
                kbs, &err) ||
      !make_map(&tv, p.v, p.dtype, D, krows, p.num_kv_heads, nb, p.v_row_stride, p.v_head_stride,
                vbs, &err))
    return fail(KVB_ERR_INVALID, err);

  DenseArgs a = {};
  a.o = p.o;
  a.lse = p.lse;
  a.o_bs = p.o_batch_stride;
  a.o_hs = p.o_head_stride;
  a.o_rs = p.o_row_stride;
  a.lse_bs = p.lse_batch_stride;
  a.lse_hs = p.lse_head_stride;
  a.cu_q = p.cu_seqlens_q;
  a.cu_k = p.cu_seqlens_k;
  a.q_len = p.q_len;
  a.kv_len = p.kv_len;
  a.group = p.num_q_heads / p.num_kv_heads;
  a.pair_heads = (a.group % 2 == 0) ? 1 : 0;
  a.causal = p.causal;
  a.scale_log2 = p.softmax_scale * 1.4426950408889634f;
  a.status = p.status;

  return launch_dense_core<T, D>(tq, tk, tv, a, p.batch, p.num_q_heads, p.q_len, stream);
}

// Split-key attention: the workspace holds the partials the merge launch reads.
// Layout: [KVB_DECODE_COUNTER_BYTES reserved][partial O][partial LSE].
static int64_t decode_workspace_bytes(const KvbPrefillParams& p, int splits) {
  const int64_t rows = (int64_t)p.batch * p.num_q_heads * p.q_len;
  const int64_t o_bytes = (int64_t)splits * rows * p.head_dim * 2;
  return KVB_DECODE_COUNTER_BYTES + (o_bytes + 255) / 256 * 256 + (int64_t)splits * rows * 4;
}

static int decode_split_tiles(const KvbPrefillParams& p, int splits, int* eff) {
  const int n_t = (p.kv_len + BN - 1) / BN;
  const int st = max(1, (n_t + max(splits, 1) - 1) / max(splits, 1));
  *eff = max(1, (n_t + st - 1) / st);
  return st;
}

// Dual mode: all packed rows of a group fit one 128-row tile, so each CTA runs
// two key splits, one per slot, in ping-pong (the second slot would be idle).
static bool decode_dual(const KvbPrefillParams& p, int eff_splits) {
  return (int64_t)(p.num_q_heads / p.num_kv_heads) * p.q_len <= BM && eff_splits >= 2;
}

// Partial results per packed row: one per key split, rounded up to even in dual
// mode (a last CTA with one split left writes an empty second partial).
static int decode_partials(const KvbPrefillParams& p, int eff_splits) {
  return decode_dual(p, eff_splits) ? (eff_splits + 1) / 2 * 2 : eff_splits;
}

// Arguments of a split-key launch: partials in the workspace after its reserved
// header, merged into params.o / params.lse by kvb_split_merge_kernel.
static void decode_args(const KvbPrefillParams& p, int splits, int split_tiles, void* ws, DenseArgs* a,
                        PagedArgs* sp) {
  const int group = p.num_q_heads / p.num_kv_heads;
  const int packed = group * p.q_len;
  const int D = p.head_dim;
  const int64_t rows = (int64_t)p.batch * p.num_kv_heads * packed;
  uint8_t* o_part = reinterpret_cast<uint8_t*>(ws) + KVB_DECODE_COUNTER_BYTES;
  const int64_t o_bytes = (int64_t)splits * rows * D * 2;
  *a = DenseArgs{};
  a->o = o_part;
  a->lse = reinterpret_cast<float*>(o_part + (o_bytes + 255) / 256 * 256);
  a->o_rs = D;
  a->o_hs = (int64_t)packed * D;
  a->o_bs = (int64_t)p.num_kv_heads * packed * D;
  a->lse_hs = packed;
  a->lse_bs = (int64_t)p.num_kv_heads * packed;
  a->q_len = packed;
  a->kv_len = p.kv_len;
  a->group = 1;
  a->pair_heads = 0;
  a->causal = p.causal;
  a->scale_log2 = p.softmax_scale * 1.4426950408889634f;
  a->status = p.status;
  *sp = PagedArgs{};
  sp->rows_per_head = p.q_len;
  sp->split_tiles = split_tiles;
  sp->o_split_stride = rows * D;
  sp->lse_split_stride = rows;
  sp->num_kv_heads = p.num_kv_heads;
  sp->o_final = p.o;
  sp->lse_final = p.lse;
  sp->of_bs = p.o_batch_stride;
  sp->of_hs = p.o_head_stride;
  sp->of_rs = p.o_row_stride;
  sp->lf_bs = p.lse_batch_stride;
  sp->lf_hs = p.lse_head_stride;
  sp->group_heads = group;
  sp->tile_pairs = (packed + 2 * BM - 1) / (2 * BM);
}


template <typename T, int D>
static int launch_decode(const KvbPrefillParams& p, int splits_req, void* ws, cudaStream_t stream) {
  using G = Geo<D>;
  const int group = p.num_q_heads / p.num_kv_heads;
  const int packed = group * p.q_len;
  int splits = 1;
  const int split_tiles = decode_split_tiles(p, splits_req, &splits);
  const bool dual = decode_dual(p, splits);
  const int parts = decode_partials(p, splits);
  DenseArgs a;
  PagedArgs sp;
  decode_args(p, parts, split_tiles, ws, &a, &sp);
  sp.dual = dual ? 1 : 0;
  const int packed_rows = (p.num_q_heads / p.num_kv_heads) * p.q_len;
  const int ctas = dual ? parts / 2 : splits;   // CTAs per (sequence, KV head, tile pair)
  const int64_t q_rs = p.q_len == 1 ? p.q_head_stride : p.q_row_stride;
  CUtensorMap tq, tk, tv;
  std::string err;
  if (!make_map(&tq, p.q, p.dtype, D, packed, p.num_kv_heads, p.batch, q_rs,
                (int64_t)group * p.q_head_stride, p.batch > 1 ? p.q_batch_stride : 8, &err) ||
      !make_map(&tk, p.k, p.dtype, D, std::max(1, p.kv_len), p.num_kv_heads, p.batch,
                p.k_row_stride, p.k_head_stride, p.batch > 1 ? p.k_batch_stride : 8, &err) ||
      !make_map(&tv, p.v, p.dtype, D, std::max(1, p.kv_len), p.num_kv_heads, p.batch,
                p.v_row_stride, p.v_head_stride, p.batch > 1 ? p.v_batch_stride : 8, &err))
    return fail(KVB_ERR_INVALID, err);
  auto kern = kvb_prefill_kernel<T, D, false, true>;
  static thread_local int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         G::SMEM_BYTES);
    if (e != cudaSuccess)
      return fail(KVB_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    configured_device = dev;
  }
  cudaError_t e = launch_pdl(kern, dim3(ctas * sp.tile_pairs, p.num_kv_heads, p.batch),
                             Roles<false>::kThreads, G::SMEM_BYTES, stream, tq, tk, tv, a, sp);
  if (e == cudaSuccess) {
    const int64_t rows = (int64_t)p.batch * p.num_kv_heads * packed_rows;
    const int64_t items = rows * (D / 8);
    // dual CTAs have already merged their two key splits: one partial per CTA
    e = launch_pdl(kvb_split_merge_kernel<T, D>, dim3((unsigned)((items + 255) / 256)), 256, 0,
                   stream, a, sp, dual ? ctas : parts, rows);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return fail(KVB_ERR_CUDA, std::string("decode launch: ") + cudaGetErrorString(e));
  return KVB_OK;
}

// Workspace the paged path uses to dequantise the prefix once instead of in
// every CTA: chosen when each KV tile would be read (and dequantised) by at
// least kMaterializeMinReaders CTAs.  0 = the fused path is used.
constexpr int kMaterializeMinReaders = 4;

// Bytes of the dense K/V copy the materialise kernel writes for these params:
// K and V, [batch, num_kv_heads, kv_pad, D] each, 2-byte elements.
static int64_t paged_materialize_bytes(const KvbPagedPrefillParams& p) {
  const int64_t kv_pad = (int64_t)(p.prefix_len + p.q_len + BN - 1) / BN * BN;
  return 2 * (int64_t)p.batch * p.num_kv_heads * kv_pad * p.head_dim * 2;
}

static int64_t paged_workspace_bytes(const KvbPagedPrefillParams& p) {
  if (p.q_len <= 0 || p.num_kv_heads <= 0 || p.num_q_heads % p.num_kv_heads) return 0;
  const int group = p.num_q_heads / p.num_kv_heads;
  const int q_tiles = (p.q_len + BM - 1) / BM;
  const int64_t readers = (group % 2 == 0) ? (int64_t)q_tiles * (group / 2) : (q_tiles + 1) / 2;
  if (readers < kMaterializeMinReaders) return 0;
  return paged_materialize_bytes(p);
}

static PagedArgs paged_args(const KvbPagedPrefillParams& p) {
  PagedArgs pa;
  pa.pool = p.kv_pool;
  pa.k_scale = p.k_scale;
  pa.v_scale = p.v_scale;
  pa.block_table = p.block_tables;
  pa.prefix_lens = p.prefix_lens;
  pa.k_new = p.k_new;
  pa.v_new = p.v_new;
  pa.kn_bs = p.k_new_batch_stride;
  pa.kn_hs = p.k_new_head_stride;
  pa.kn_rs = p.k_new_row_stride;
  pa.vn_bs = p.v_new_batch_stride;
  pa.vn_hs = p.v_new_head_stride;
  pa.vn_rs = p.v_new_row_stride;
  pa.max_blocks = p.max_blocks_per_seq;
  pa.num_blocks = p.num_blocks;
  pa.num_kv_heads = p.num_kv_heads;
  pa.prefix_len = p.prefix_len;
  pa.pool16 = p.pool_format == KVB_POOL_COMPUTE ? 1 : 0;
  return pa;
}

// Dense K and V of every sequence, [batch, num_kv_heads, kv_pad, D] each, into
// the workspace: kv_pad = round_up(prefix_len + q_len, 128).
template <typename T, int D>
static int launch_materialize(const KvbPagedPrefillParams& p, cudaStream_t stream,
                              const PeerArgs* peer = nullptr) {
  const PagedArgs pa = paged_args(p);
  const int kv_pad = (p.prefix_len + p.q_len + BN - 1) / BN * BN;
  T* wk = reinterpret_cast<T*>(p.workspace);
  T* wv = wk + (int64_t)p.batch * p.num_kv_heads * kv_pad * D;
  const int64_t threads = (int64_t)kv_pad * (D / 16) * 2;
  dim3 mgrid((unsigned)((threads + 255) / 256), p.num_kv_heads, p.batch);
  if (peer)
    kvb_paged_materialize_kernel<T, D, true><<<mgrid, 256, 0, stream>>>(
        pa, wk, wv, p.q_len, kv_pad, p.status, *peer);
  else
    kvb_paged_materialize_kernel<T, D, false><<<mgrid, 256, 0, stream>>>(
        pa, wk, wv, p.q_len, kv_pad, p.status, PeerArgs{});
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(KVB_ERR_CUDA, std::string("materialize launch: ") + cudaGetErrorString(e));
  return KVB_OK;
}

// force_materialize: take the materialise strategy whatever the reader count
// (the no-allocation entry point, whose workspace is always present).
template <typename T, int D>
static int launch_paged(const KvbPagedPrefillParams& p, cudaStream_t stream,
                        bool force_materialize = false) {
  using G = Geo<D>;
  CUtensorMap tq;
  std::string err;
  if (!make_map(&tq, p.q, p.dtype, D, p.q_len, p.num_q_heads, p.batch, p.q_row_stride,
                p.q_head_stride, p.batch > 1 ? p.q_batch_stride : 8, &err))
    return fail(KVB_ERR_INVALID, err);
  DenseArgs a = {};
  a.o = p.o;
  a.lse = p.lse;
  a.o_bs = p.o_batch_stride;
  a.o_hs = p.o_head_stride;
  a.o_rs = p.o_row_stride;
  a.lse_bs = p.lse_batch_stride;
  a.lse_hs = p.lse_head_stride;
  a.q_len = p.q_len;
  a.kv_len = p.prefix_len + p.q_len;
  a.group = p.num_q_heads / p.num_kv_heads;
  a.pair_heads = (a.group % 2 == 0) ? 1 : 0;
  a.causal = p.causal;
  a.scale_log2 = p.softmax_scale * 1.4426950408889634f;
  a.status = p.status;
  const PagedArgs pa = paged_args(p);

  const int64_t need = force_materialize ? paged_materialize_bytes(p) : paged_workspace_bytes(p);
  if (need > 0 && p.workspace != nullptr && p.workspace_bytes >= need) {
    // Many CTAs read each KV tile: dequantise the prefix once into the
    // workspace, then run the dense kernel over it.
    const int kv_pad = (p.prefix_len + p.q_len + BN - 1) / BN * BN;
    T* wk = reinterpret_cast<T*>(p.workspace);
    T* wv = wk + (int64_t)p.batch * p.num_kv_heads * kv_pad * D;
    const int64_t threads = (int64_t)kv_pad * (D / 16) * 2;
    dim3 mgrid((unsigned)((threads + 255) / 256), p.num_kv_heads, p.batch);
    kvb_paged_materialize_kernel<T, D, false><<<mgrid, 256, 0, stream>>>(
        pa, wk, wv, p.q_len, kv_pad, p.status, PeerArgs{});
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
      return fail(KVB_ERR_CUDA, std::string("materialize launch: ") + cudaGetErrorString(e));
    CUtensorMap tk, tv;
    const int64_t hs = (int64_t)kv_pad * D, bs = (int64_t)p.num_kv_heads * kv_pad * D;
    if (!make_map(&tk, wk, p.dtype, D, kv_pad, p.num_kv_heads, p.batch, D, hs, bs, &err) ||
        !make_map(&tv, wv, p.dtype, D, kv_pad, p.num_kv_heads, p.batch, D, hs, bs, &err))
      return fail(KVB_ERR_INVALID, err);
    if (p.prefix_lens != nullptr) {
      a.kv_prefix = p.prefix_lens;
    }
    return launch_dense_core<T, D>(tq, tk, tv, a, p.batch, p.num_q_heads, p.q_len, stream);
  }

  auto kern = kvb_prefill_kernel<T, D, true>;
  static thread_local int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         G::SMEM_BYTES);
    if (e != cudaSuccess)
      return fail(KVB_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    configured_device = dev;
  }
  const int q_tiles = (p.q_len + BM - 1) / BM;
  dim3 grid = a.pair_heads ? dim3(p.num_q_heads / 2, q_tiles, p.batch)
                           : dim3(p.num_q_heads, (q_tiles + 1) / 2, p.batch);
  cudaError_t e = launch_pdl(kern, grid, Roles<true>::kThreads, G::SMEM_BYTES, stream, tq, tq, tq,
                             a, pa);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(KVB_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
  return KVB_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static int validate(const KvbPrefillParams& p) {
  if (p.dtype != KVB_DTYPE_BF16 && p.dtype != KVB_DTYPE_FP16)
    return fail(KVB_ERR_INVALID, "dtype must be KVB_DTYPE_BF16 or KVB_DTYPE_FP16");
  if (p.head_dim != 64 && p.head_dim != 96 && p.head_dim != 128)
    return fail(KVB_ERR_INVALID,
                "head_dim must be one of 64, 96, 128, got " + std::to_string(p.head_dim));
  if (p.batch < 1 || p.num_q_heads < 1 || p.num_kv_heads < 1)
    return fail(KVB_ERR_INVALID, "batch and head counts must be positive");
  if (p.num_q_heads % p.num_kv_heads)
    return fail(KVB_ERR_INVALID, "num_q_heads (" + std::to_string(p.num_q_heads) +
                                     ") must be divisible by num_kv_heads (" +
                                     std::to_string(p.num_kv_heads) + ")");
  if (p.batch > 65535 || p.num_q_heads > 65535)
    return fail(KVB_ERR_UNSUPPORTED, "batch and num_q_heads must be <= 65535");
  if (p.causal < 0 || p.causal > 2)
    return fail(KVB_ERR_INVALID, "causal must be 0 (none), 1 (bottom-right) or 2 (top-left)");
  if (p.q_len < 0 || p.kv_len < 0)
    return fail(KVB_ERR_INVALID, "sequence lengths must be non-negative");
  if (p.q_len > 65535 * BM)  // query tiles are the grid's y dimension
    return fail(KVB_ERR_UNSUPPORTED, "q_len must be <= " + std::to_string(65535 * BM));
  const bool varlen = p.cu_seqlens_q != nullptr;
  // An empty key side may come with null k/v (an empty tensor's data pointer).
  const bool no_keys = varlen ? p.total_k == 0 : p.kv_len == 0;
  if (!p.q || !p.o || (!no_keys && (!p.k || !p.v)))
    return fail(KVB_ERR_INVALID, "q, k, v and o must be non-null");
  if (!aligned16(p.q) || !aligned16(p.k) || !aligned16(p.v) || !aligned16(p.o))
    return fail(KVB_ERR_INVALID, "q, k, v and o must be 16-byte aligned");
  if (varlen != (p.cu_seqlens_k != nullptr))
    return fail(KVB_ERR_INVALID, "cu_seqlens_q and cu_seqlens_k must both be set or both NULL");
  if (varlen && (p.total_q < 0 || p.total_k < 0))
    return fail(KVB_ERR_INVALID, "total_q/total_k must be non-negative in varlen mode");
  const int64_t st[] = {p.q_head_stride, p.q_row_stride, p.k_head_stride, p.k_row_stride,
                        p.v_head_stride, p.v_row_stride, p.o_head_stride, p.o_row_stride};
  for (int64_t s : st)
    if (s <= 0 || (s % 8) != 0)
      return fail(KVB_ERR_INVALID, "row and head strides must be positive multiples of 8 elements");
  if (!varlen) {
    const int64_t bst[] = {p.q_batch_stride, p.k_batch_stride, p.v_batch_stride, p.o_batch_stride};
    for (int64_t s : bst)
      if ((p.batch > 1 && s <= 0) || (s % 8) != 0)
        return fail(KVB_ERR_INVALID, "batch strides must be positive multiples of 8 elements");
  }
  return KVB_OK;
}

}  // namespace kvb

// ============================================================================
// C ABI
// ============================================================================
using namespace kvb;

extern "C" int kvb_prefill_fwd(const KvbPrefillParams* params, void* stream) {
  if (!params) return fail(KVB_ERR_INVALID, "params is NULL");
  const KvbPrefillParams& p = *params;
  int rc = validate(p);
  if (rc != KVB_OK) return rc;
  if (p.q_len == 0) return KVB_OK;
  const bool varlen = p.cu_seqlens_q != nullptr;
  if (varlen && (p.total_q == 0)) return KVB_OK;
  // The TMA maps need at least one row; an empty key side is handled by the
  // kernel (no tiles) but the map must still be encodable.
  KvbPrefillParams q = p;
  if (varlen ? q.total_k == 0 : q.kv_len == 0) {
    // No keys: no tile is ever loaded, but the K/V maps must still encode.
    q.k = p.q; q.v = p.q;
    q.k_head_stride = p.q_head_stride; q.k_row_stride = p.q_row_stride;
    q.k_batch_stride = p.q_batch_stride;
    q.v_head_stride = p.q_head_stride; q.v_row_stride = p.q_row_stride;
    q.v_batch_stride = p.q_batch_stride;
    if (varlen) q.total_k = 1;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool bf = p.dtype == KVB_DTYPE_BF16;
  switch (p.head_dim) {
    case 64: return bf ? launch_dense<__nv_bfloat16, 64>(q, s) : launch_dense<__half, 64>(q, s);
    case 96: return bf ? launch_dense<__nv_bfloat16, 96>(q, s) : launch_dense<__half, 96>(q, s);
    default: return bf ? launch_dense<__nv_bfloat16, 128>(q, s) : launch_dense<__half, 128>(q, s);
  }
}

extern "C" int kvb_flash_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                                  int batch, int heads, int seqlen, int head_dim, int dtype,
                                  float softmax_scale, int causal, void* stream) {
  KvbPrefillParams p = {};
  p.dtype = dtype;
  p.head_dim = head_dim;
  p.batch = batch;
  p.num_q_heads = heads;
  p.num_kv_heads = heads;
  p.q_len = seqlen;
  p.kv_len = seqlen;
  p.causal = causal;
  p.softmax_scale = softmax_scale;
  p.q = q;
  p.k = k;
  p.v = v;
  p.o = o;
  p.lse = lse;
  const int64_t rs = head_dim, hs = (int64_t)seqlen * head_dim, bs = (int64_t)heads * hs;
  p.q_row_stride = p.k_row_stride = p.v_row_stride = p.o_row_stride = rs;
  p.q_head_stride = p.k_head_stride = p.v_head_stride = p.o_head_stride = hs > 0 ? hs : rs;
  p.q_batch_stride = p.k_batch_stride = p.v_batch_stride = p.o_batch_stride = bs > 0 ? bs : rs;
  p.lse_head_stride = seqlen;
  p.lse_batch_stride = (int64_t)heads * seqlen;
  return kvb_prefill_fwd(&p, stream);
}

static int validate_paged(const KvbPagedPrefillParams& p) {
  if (p.dtype != KVB_DTYPE_BF16 && p.dtype != KVB_DTYPE_FP16)
    return fail(KVB_ERR_INVALID, "dtype must be KVB_DTYPE_BF16 or KVB_DTYPE_FP16");
  if (p.head_dim != 64 && p.head_dim != 96 && p.head_dim != 128)
    return fail(KVB_ERR_INVALID,
                "head_dim must be one of 64, 96, 128, got " + std::to_string(p.head_dim));
  if (p.batch < 1 || p.num_q_heads < 1 || p.num_kv_heads < 1)
    return fail(KVB_ERR_INVALID, "batch and head counts must be positive");
  if (p.num_q_heads % p.num_kv_heads)
    return fail(KVB_ERR_INVALID, "num_q_heads must be divisible by num_kv_heads");
  if (p.batch > 65535 || p.num_q_heads > 65535)
    return fail(KVB_ERR_UNSUPPORTED, "batch and num_q_heads must be <= 65535");
  if (p.causal < 0 || p.causal > 2)
    return fail(KVB_ERR_INVALID, "causal must be 0 (none), 1 (bottom-right) or 2 (top-left)");
  if (p.q_len < 0 || p.prefix_len < 0)
    return fail(KVB_ERR_INVALID, "q_len and prefix_len must be non-negative");
  if (p.q_len > 65535 * BM)  // query tiles are the grid's y dimension
    return fail(KVB_ERR_UNSUPPORTED, "q_len must be <= " + std::to_string(65535 * BM));
  if (p.block_size != 16)
    return fail(KVB_ERR_UNSUPPORTED, "block_size must be 16");
  if (p.num_blocks < 1 || p.max_blocks_per_seq < 0)
    return fail(KVB_ERR_INVALID, "num_blocks must be positive");
  if ((int64_t)p.max_blocks_per_seq * 16 < p.prefix_len)
    return fail(KVB_ERR_INVALID, "block table too short for prefix_len");
  if (p.pool_format != KVB_POOL_INT8_KIVI && p.pool_format != KVB_POOL_COMPUTE)
    return fail(KVB_ERR_INVALID, "pool_format must be KVB_POOL_INT8_KIVI or KVB_POOL_COMPUTE");
  const bool scales = p.pool_format == KVB_POOL_INT8_KIVI;
  if (!p.q || !p.o || !p.kv_pool || !p.block_tables || (scales && (!p.k_scale || !p.v_scale)))
    return fail(KVB_ERR_INVALID, "q, o, kv_pool, scales and block_tables must be non-null");
  if (p.q_len > 0 && (!p.k_new || !p.v_new))
    return fail(KVB_ERR_INVALID, "k_new and v_new must be non-null when q_len > 0");
  if (!aligned16(p.q) || !aligned16(p.o) || !aligned16(p.kv_pool) ||
      (scales && !aligned16(p.v_scale)) ||
      (p.k_new && !aligned16(p.k_new)) || (p.v_new && !aligned16(p.v_new)))
    return fail(KVB_ERR_INVALID, "q, o, k_new, v_new, kv_pool and v_scale must be 16-byte aligned");
  const int64_t st[] = {p.q_head_stride, p.q_row_stride, p.o_head_stride, p.o_row_stride,
                        p.k_new_head_stride, p.k_new_row_stride, p.v_new_head_stride,
                        p.v_new_row_stride};
  for (int64_t s : st)
    if (s <= 0 || (s % 8) != 0)
      return fail(KVB_ERR_INVALID, "row and head strides must be positive multiples of 8 elements");
  return KVB_OK;
}

static int validate_decode(const KvbPrefillParams& p, int splits) {
  int rc = validate(p);
  if (rc != KVB_OK) return rc;
  if (p.cu_seqlens_q) return fail(KVB_ERR_UNSUPPORTED, "split decode takes dense batches");
  if (splits < 1 || splits > 4096) return fail(KVB_ERR_INVALID, "num_splits must be in [1, 4096]");
  if (p.q_len < 1 || p.kv_len < p.q_len)
    return fail(KVB_ERR_INVALID, "split decode needs 1 <= q_len <= kv_len");
  const int group = p.num_q_heads / p.num_kv_heads;
  const int64_t packed = (int64_t)group * p.q_len;
  if (packed > (int64_t)1 << 24)
    return fail(KVB_ERR_UNSUPPORTED, "split-key attention packs (q heads per KV head) * q_len "
                                     "<= 2^24 rows");
  if (p.q_len > 1 && p.q_head_stride != (int64_t)p.q_len * p.q_row_stride)
    return fail(KVB_ERR_INVALID, "with q_len > 1 the rows of a head must be contiguous in q "
                                 "(head stride = q_len * row stride)");
  return KVB_OK;
}

extern "C" int64_t kvb_decode_workspace_bytes(const KvbPrefillParams* params, int num_splits) {
  if (!params || validate_decode(*params, num_splits) != KVB_OK) return -1;
  int eff = 1;
  decode_split_tiles(*params, num_splits, &eff);
  return decode_workspace_bytes(*params, decode_partials(*params, eff));
}

extern "C" int kvb_decode_fwd(const KvbPrefillParams* params, int num_splits, void* workspace,
                              int64_t workspace_bytes, void* stream) {
  if (!params) return fail(KVB_ERR_INVALID, "params is NULL");
  const KvbPrefillParams& p = *params;
  int rc = validate_decode(p, num_splits);
  if (rc != KVB_OK) return rc;
  int eff = 1;
  decode_split_tiles(p, num_splits, &eff);
  const int64_t need = decode_workspace_bytes(p, decode_partials(p, eff));
  if (!workspace || !aligned16(workspace) || workspace_bytes < need)
    return fail(KVB_ERR_INVALID, "workspace must hold " + std::to_string(need) + " bytes");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool bf = p.dtype == KVB_DTYPE_BF16;
  switch (p.head_dim) {
    case 64:
      return bf ? launch_decode<__nv_bfloat16, 64>(p, num_splits, workspace, s)
                : launch_decode<__half, 64>(p, num_splits, workspace, s);
    case 96:
      return bf ? launch_decode<__nv_bfloat16, 96>(p, num_splits, workspace, s)
                : launch_decode<__half, 96>(p, num_splits, workspace, s);
    default:
      return bf ? launch_decode<__nv_bfloat16, 128>(p, num_splits, workspace, s)
                : launch_decode<__half, 128>(p, num_splits, workspace, s);
  }
}

extern "C" int64_t kvb_paged_prefill_workspace_bytes(const KvbPagedPrefillParams* params) {
  if (!params || validate_paged(*params) != KVB_OK) return 0;
  return paged_workspace_bytes(*params);
}

extern "C" int kvb_paged_prefill_fwd(const KvbPagedPrefillParams* params, void* stream) {
  if (!params) return fail(KVB_ERR_INVALID, "params is NULL");
  const KvbPagedPrefillParams& p = *params;
  int rc = validate_paged(p);
  if (rc != KVB_OK) return rc;
  if (p.q_len == 0) return KVB_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool bf = p.dtype == KVB_DTYPE_BF16;
  switch (p.head_dim) {
    case 64: return bf ? launch_paged<__nv_bfloat16, 64>(p, s) : launch_paged<__half, 64>(p, s);
    case 96: return bf ? launch_paged<__nv_bfloat16, 96>(p, s) : launch_paged<__half, 96>(p, s);
    default: return bf ? launch_paged<__nv_bfloat16, 128>(p, s) : launch_paged<__half, 128>(p, s);
  }
}

extern "C" int kvb_paged_materialize(const KvbPagedPrefillParams* params, void* stream) {
  if (!params) return fail(KVB_ERR_INVALID, "params is NULL");
  const KvbPagedPrefillParams& p = *params;
  if (p.dtype != KVB_DTYPE_BF16 && p.dtype != KVB_DTYPE_FP16)
    return fail(KVB_ERR_INVALID, "dtype must be KVB_DTYPE_BF16 or KVB_DTYPE_FP16");
  if (p.head_dim != 64 && p.head_dim != 96 && p.head_dim != 128)
    return fail(KVB_ERR_INVALID,
                "head_dim must be one of 64, 96, 128, got " + std::to_string(p.head_dim));
  if (p.batch < 1 || p.num_kv_heads < 1 || p.batch > 65535 || p.num_kv_heads > 65535)
    return fail(KVB_ERR_INVALID, "batch and num_kv_heads must be in [1, 65535]");
  if (p.q_len < 0 || p.prefix_len < 0)
    return fail(KVB_ERR_INVALID, "q_len and prefix_len must be non-negative");
  if (p.block_size != 16) return fail(KVB_ERR_UNSUPPORTED, "block_size must be 16");
  if (p.num_blocks < 1 || p.max_blocks_per_seq < 0 ||
      (int64_t)p.max_blocks_per_seq * 16 < p.prefix_len)
    return fail(KVB_ERR_INVALID, "num_blocks must be positive and the table cover prefix_len");
  if (p.pool_format != KVB_POOL_INT8_KIVI && p.pool_format != KVB_POOL_COMPUTE)
    return fail(KVB_ERR_INVALID, "pool_format must be KVB_POOL_INT8_KIVI or KVB_POOL_COMPUTE");
  const bool scales = p.pool_format == KVB_POOL_INT8_KIVI;
  if (!p.kv_pool || !p.block_tables || (scales && (!p.k_scale || !p.v_scale)))
    return fail(KVB_ERR_INVALID, "kv_pool, scales and block_tables must be non-null");
  if (p.q_len > 0 && (!p.k_new || !p.v_new))
    return fail(KVB_ERR_INVALID, "k_new and v_new must be non-null when q_len > 0");
  if (!aligned16(p.kv_pool) || (scales && !aligned16(p.v_scale)) || !aligned16(p.workspace) ||
      (p.k_new && !aligned16(p.k_new)) || (p.v_new && !aligned16(p.v_new)))
    return fail(KVB_ERR_INVALID, "kv_pool, v_scale, k_new, v_new and workspace must be 16-byte aligned");
  if (p.q_len > 0) {
    const int64_t st[] = {p.k_new_head_stride, p.k_new_row_stride, p.v_new_head_stride,
                          p.v_new_row_stride};
    for (int64_t x : st)
      if (x <= 0 || (x % 8) != 0)
        return fail(KVB_ERR_INVALID, "k_new/v_new row and head strides must be positive multiples of 8");
  }
  const int64_t need = paged_materialize_bytes(p);
  if (!p.workspace || p.workspace_bytes < need)
    return fail(KVB_ERR_INVALID, "workspace must hold " + std::to_string(need) + " bytes");
  if (p.prefix_len + p.q_len == 0) return KVB_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool bf = p.dtype == KVB_DTYPE_BF16;
  switch (p.head_dim) {
    case 64:
      return bf ? launch_materialize<__nv_bfloat16, 64>(p, s) : launch_materialize<__half, 64>(p, s);
    case 96:
      return bf ? launch_materialize<__nv_bfloat16, 96>(p, s) : launch_materialize<__half, 96>(p, s);
    default:
      return bf ? launch_materialize<__nv_bfloat16, 128>(p, s)
                : launch_materialize<__half, 128>(p, s);
  }
}

extern "C" int64_t kvb_peer_shard_layout(int num_kv_heads, int head_dim, int shard_blocks,
                                         int zigzag_rows, int64_t* offsets) {
  if (num_kv_heads < 1 || (head_dim != 64 && head_dim != 96 && head_dim != 128) ||
      shard_blocks < 1 || zigzag_rows < 0)
    return -1;
  const int64_t pool = (int64_t)shard_blocks * 2 * num_kv_heads * 16 * head_dim;
  const int64_t ks = (int64_t)shard_blocks * num_kv_heads * 16 * 4;
  const int64_t vs = (int64_t)shard_blocks * num_kv_heads * head_dim * 4;
  const int64_t sfx = (int64_t)num_kv_heads * 2 * zigzag_rows * head_dim * 2;
  if (offsets) {
    offsets[0] = 0;                     // pool
    offsets[1] = pool;                  // k_scale
    offsets[2] = pool + ks;             // v_scale
    offsets[3] = pool + ks + vs;        // suffix K
    offsets[4] = pool + ks + vs + sfx;  // suffix V
  }
  return pool + ks + vs + 2 * sfx;
}

extern "C" int kvb_paged_materialize_peers(const KvbPagedPrefillParams* params,
                                           const KvbPeerShards* shards, void* stream) {
  if (!params || !shards) return fail(KVB_ERR_INVALID, "params and shards must be non-null");
  const KvbPagedPrefillParams& p = *params;
  const KvbPeerShards& sh = *shards;
  if (p.dtype != KVB_DTYPE_BF16 && p.dtype != KVB_DTYPE_FP16)
    return fail(KVB_ERR_INVALID, "dtype must be KVB_DTYPE_BF16 or KVB_DTYPE_FP16");
  if (p.batch != 1) return fail(KVB_ERR_UNSUPPORTED, "peer shards hold one sequence (batch 1)");
  if (p.pool_format != KVB_POOL_INT8_KIVI)
    return fail(KVB_ERR_UNSUPPORTED, "peer shards hold int8 KIVI pools");
  if (sh.world < 1 || sh.world > kMaxPeers)
    return fail(KVB_ERR_UNSUPPORTED, "world must be in [1, 8]");
  if (sh.shard_blocks < 1 || p.num_blocks != sh.world * sh.shard_blocks)
    return fail(KVB_ERR_INVALID, "num_blocks must equal world * shard_blocks");
  if (p.q_len != 2 * sh.world * sh.zigzag_rows || p.q_len < 0)
    return fail(KVB_ERR_INVALID, "q_len must equal 2 * world * zigzag_rows");
  if (p.num_kv_heads < 1 || p.num_kv_heads > 65535 || p.prefix_len < 0)
    return fail(KVB_ERR_INVALID, "bad num_kv_heads or prefix_len");
  if (p.block_size != 16) return fail(KVB_ERR_UNSUPPORTED, "block_size must be 16");
  if (!p.block_tables || (int64_t)p.max_blocks_per_seq * 16 < p.prefix_len)
    return fail(KVB_ERR_INVALID, "block_tables must be set and cover prefix_len");
  int64_t off[5];
  if (kvb_peer_shard_layout(p.num_kv_heads, p.head_dim, sh.shard_blocks, sh.zigzag_rows, off) < 0)
    return fail(KVB_ERR_INVALID, "head_dim must be one of 64, 96, 128");
  PeerArgs peer = {};
  for (int r = 0; r < sh.world; ++r) {
    if (!sh.base[r] || !aligned16(sh.base[r]))
      return fail(KVB_ERR_INVALID, "every shard base must be non-null and 16-byte aligned");
    peer.base[r] = reinterpret_cast<const uint8_t*>(sh.base[r]);
  }
  peer.world = sh.world;
  peer.shard_blocks = sh.shard_blocks;
  peer.zz_rows = sh.zigzag_rows;
  peer.kscale_off = off[1];
  peer.vscale_off = off[2];
  peer.suffix_off = off[3];
  peer.suffix_v_off = off[4];
  const int64_t need = paged_materialize_bytes(p);
  if (!p.workspace || !aligned16(p.workspace) || p.workspace_bytes < need)
    return fail(KVB_ERR_INVALID, "workspace must hold " + std::to_string(need) + " bytes");
  if (p.prefix_len + p.q_len == 0) return KVB_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool bf = p.dtype == KVB_DTYPE_BF16;
  switch (p.head_dim) {
    case 64:
      return bf ? launch_materialize<__nv_bfloat16, 64>(p, s, &peer)
                : launch_materialize<__half, 64>(p, s, &peer);
    case 96:
      return bf ? launch_materialize<__nv_bfloat16, 96>(p, s, &peer)
                : launch_materialize<__half, 96>(p, s, &peer);
    default:
      return bf ? launch_materialize<__nv_bfloat16, 128>(p, s, &peer)
                : launch_materialize<__half, 128>(p, s, &peer);
  }
}

// ── hooks for the no-allocation entry point (kvb_noalloc_sm100.cu) ──────────
// Validate the params and return the workspace bytes the materialise strategy
// needs, or a negative KVB_ERR_* code (the reason is in kvb_last_error).
int64_t kvb_detail_paged_materialize_bytes(const KvbPagedPrefillParams& p) {
  const int rc = validate_paged(p);
  if (rc != KVB_OK) return -(int64_t)rc;
  return p.q_len == 0 ? 0 : paged_materialize_bytes(p);
}

// Paged prefill with the prefix always materialised into `scratch`, which the
// caller has checked holds kvb_detail_paged_materialize_bytes(p) bytes.
int kvb_detail_paged_prefill_scratch(const KvbPagedPrefillParams& params, void* scratch,
                                     int64_t scratch_bytes, cudaStream_t s) {
  if (params.q_len == 0) return KVB_OK;
  KvbPagedPrefillParams p = params;
  p.workspace = scratch;
  p.workspace_bytes = scratch_bytes;
  const bool bf = p.dtype == KVB_DTYPE_BF16;
  switch (p.head_dim) {
    case 64:
      return bf ? launch_paged<__nv_bfloat16, 64>(p, s, true) : launch_paged<__half, 64>(p, s, true);
    case 96:
      return bf ? launch_paged<__nv_bfloat16, 96>(p, s, true) : launch_paged<__half, 96>(p, s, true);
    default:
      return bf ? launch_paged<__nv_bfloat16, 128>(p, s, true)
                : launch_paged<__half, 128>(p, s, true);
  }
}

int kvb_detail_fail(int code, const std::string& msg) { return fail(code, msg); }

extern "C" const char* kvb_last_error(void) { return g_last_error.c_str(); }

extern "C" int kvb_abi_version(void) { return KVB_ABI_VERSION; }

#ifdef KVB_TRACE
extern "C" int kvb_debug_set_trace(void* dev_ptr) {
  return cudaMemcpyToSymbol(kvb::g_kvb_trace, &dev_ptr, sizeof(dev_ptr)) == cudaSuccess ? 0 : -1;
}
#endif
