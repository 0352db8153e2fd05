/*
 * kvb_attn.h -- C ABI of the kvboost_b200 prefill-attention library
 * (libkvb_attn: kvboost_b200/_kvb_attn.so), B200 / sm_100a only.
 *
 * Plain pointers, sizes and a CUDA stream handle (cudaStream_t passed as
 * void*); no framework types.  Every entry point validates its arguments on
 * the host before launching anything and returns
 *
 *     KVB_OK (0)            launched (asynchronous: nothing is synchronised)
 *     KVB_ERR_INVALID (1)   bad argument; nothing launched
 *     KVB_ERR_UNSUPPORTED(2) well-formed but outside what the kernels support
 *     KVB_ERR_CUDA (-1)     the CUDA runtime refused the launch
 *
 * with a human-readable reason available from kvb_last_error() (per host
 * thread).  Device-side waits are bounded: a kernel that gives up on a wait
 * ORs a non-zero code into the optional caller-owned `status` word
 * (KVB_STATUS_*) and exits cleanly instead of hanging.
 *
 * Attention semantics (all entry points): O = softmax(Q K^T * scale) V per
 * query head, query head h reading KV head h / (num_q_heads / num_kv_heads)
 * (GQA grouping as KVBoost's repeat_interleave, cpu_paged/paged_attn_cpu.py:87-88).
 * causal = 1 (KVB_CAUSAL_BOTTOM_RIGHT): key j is visible to query i iff
 * j <= i + (kv_len - q_len), i.e. HuggingFace's reuse-prefill mask; for
 * q_len == kv_len it equals the reference kernel's mask
 * (csrc/flash_attn_kernel.cu:148,193).  causal = 2 (KVB_CAUSAL_TOP_LEFT):
 * j <= i, torch SDPA's is_causal, which the reference's paged path applies
 * (cpu_paged/paged_attn_cpu.py:103).  causal = 0: no mask.  LSE is log(sum_j exp(scale*q.k_j))
 * in natural log (flash_attn_kernel.cu:236-245); rows with no visible key
 * get O = 0 and LSE = -inf.
 */
#ifndef KVB_ATTN_H_
#define KVB_ATTN_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVB_ABI_VERSION 2

enum {
  KVB_DTYPE_BF16 = 0,
  KVB_DTYPE_FP16 = 1
};

enum {
  KVB_CAUSAL_NONE = 0,
  KVB_CAUSAL_BOTTOM_RIGHT = 1,
  KVB_CAUSAL_TOP_LEFT = 2
};

enum {
  KVB_OK = 0,
  KVB_ERR_INVALID = 1,
  KVB_ERR_UNSUPPORTED = 2,
  KVB_ERR_CUDA = -1
};

/* Bits a kernel ORs into `status` when a bounded wait gives up. */
enum {
  KVB_STATUS_LOAD_WAIT = 1,    /* producer waited too long for a free stage   */
  KVB_STATUS_MMA_WAIT = 2,     /* MMA issuer waited too long for operands     */
  KVB_STATUS_SOFTMAX_WAIT = 4, /* softmax warps waited too long for scores    */
  KVB_STATUS_EPILOGUE_WAIT = 8,/* epilogue waited too long for the output     */
  KVB_STATUS_BAD_BLOCK = 16,    /* a block-table entry was outside the pool    */
  KVB_STATUS_BAD_LENGTH = 32,   /* a chunk's token count did not fit its blocks */
  KVB_STATUS_PEER_WAIT = 64     /* a cross-GPU barrier waited too long for a peer */
};

/*
 * kvb_flash_attn_fwd -- drop-in for the reference extension's
 * flash_attn_fwd_dispatch(Q, K, V, O, L, scale, causal)
 * (src/kvboost/csrc/flash_attn.h:5-12, flash_attn_kernel.cu:250-294) together
 * with its argument checks (flash_attn.cpp:16-54), behind the Python op
 * kvboost._flash_attn_cuda.flash_attn_fwd (flash_attn.cpp:85-102).
 *
 * q, k, v, o : contiguous [batch, heads, seqlen, head_dim], dtype KVB_DTYPE_*
 * lse        : contiguous float32 [batch, heads, seqlen] (may be NULL)
 * head_dim   : 64, 96 or 128.  Same q and kv length, same head count (as the
 *              reference requires).  Launched on `stream` (the reference used
 *              the legacy default stream).
 */
int kvb_flash_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                       int batch, int heads, int seqlen, int head_dim, int dtype,
                       float softmax_scale, int causal, void* stream);

/*
 * Extended prefill: GQA, q_len != kv_len (reuse prefill over a cached
 * prefix), arbitrary row/head/batch strides, and packed variable-length
 * batches.  Replaces the SDPA call that KVBoost's reuse prefill reaches
 * through HF's attention registry (flash_attn_ext.py:86-103 and
 * transformers integrations/sdpa_attention.py).
 *
 * Dense mode (cu_seqlens_q == NULL): q/o are [batch, q_len] rows per head,
 * k/v [batch, kv_len]; element (b, h, i, d) of q sits at
 *   q + b*q_batch_stride + h*q_head_stride + i*q_row_stride + d.
 * lse (optional) element (b, h, i) at lse + b*lse_batch_stride + h*lse_head_stride + i.
 *
 * Varlen mode (cu_seqlens_q and cu_seqlens_k set, device int32 [batch+1]):
 * q/o are packed [total_q, heads, head_dim] (batch stride ignored), k/v
 * [total_k, kv_heads, head_dim]; sequence b owns rows cu[b]..cu[b+1]-1;
 * q_len / kv_len carry the maxima over sequences; lse element (h, row) at
 * lse + h*lse_head_stride + row.
 *
 * Requirements: innermost stride 1; row/head/batch strides multiples of 8
 * elements; base pointers 16-byte aligned; batch, num_q_heads <= 65535 and
 * q_len <= 65535 * 128 (KVB_ERR_UNSUPPORTED otherwise).
 */
typedef struct KvbPrefillParams {
  int32_t dtype;
  int32_t head_dim;
  int32_t batch;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t q_len;
  int32_t kv_len;
  int32_t causal;
  float softmax_scale;
  int32_t total_q; /* varlen only: rows of q/o */
  int32_t total_k; /* varlen only: rows of k/v */
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse;
  int64_t q_batch_stride, q_head_stride, q_row_stride;
  int64_t k_batch_stride, k_head_stride, k_row_stride;
  int64_t v_batch_stride, v_head_stride, v_row_stride;
  int64_t o_batch_stride, o_head_stride, o_row_stride;
  int64_t lse_batch_stride, lse_head_stride;
  const int32_t* cu_seqlens_q;
  const int32_t* cu_seqlens_k;
  int32_t* status;
} KvbPrefillParams;

int kvb_prefill_fwd(const KvbPrefillParams* params, void* stream);

/*
 * Split-key attention for few queries per head over many keys: decode steps
 * (q_len 1), the selective-recompute seams (q_len <= 16) and short reuse
 * suffixes that reach the SDPA call of the reference's engine
 * (flash_attn_ext.py:86-103).  Same params and semantics as kvb_prefill_fwd in
 * dense mode, restricted to 1 <= q_len <= kv_len; with q_len > 1 each head's
 * rows must be contiguous in q (head stride = q_len * row stride).  The query
 * heads sharing a KV head are packed as rows ((q heads per KV head) * q_len
 * of them, two 128-row tiles per CTA), so every key tile is read once per
 * group and tile pair, and the key range is split over num_splits CTAs; a
 * second launch merges the partial outputs by their LSE.  workspace: device
 * memory of at least kvb_decode_workspace_bytes(params, num_splits) bytes (-1:
 * invalid params, reason in kvb_last_error), 16-byte aligned, holding the
 * partials after a reserved header of KVB_DECODE_COUNTER_BYTES (no
 * initialisation needed); calls that overlap on the GPU must not share one.
 * No counterpart in the reference, whose decode steps run the same SDPA call
 * as its prefill.
 */
#define KVB_DECODE_COUNTER_BYTES (64 * 1024)
int64_t kvb_decode_workspace_bytes(const KvbPrefillParams* params, int num_splits);
int kvb_decode_fwd(const KvbPrefillParams* params, int num_splits, void* workspace,
                   int64_t workspace_bytes, void* stream);

/*
 * Reuse prefill over an int8 paged prefix: the suffix's queries attend to
 * the cached prefix (KVBoost's 128-token chunks, KIVI int8, stored in
 * 16-token blocks) followed by the suffix's own fresh K/V, bottom-right
 * causal.  Replaces the host path that dequantises each cached chunk
 * (kv_quantize.py:102-109), gathers it through the block table
 * (cpu_paged/block_allocator.py:178-206, cpu_paged/chunk_to_blocks.py:57-125)
 * and concatenates it before SDPA (cache_manager.py:460-471): here the
 * gather and the dequantisation happen in the kernel's K/V load stage.
 *
 * Pool layout (one layer): kv_pool int8 [num_blocks, 2, num_kv_heads, 16,
 * head_dim] (index 0 = K, 1 = V; the reference pool's layout,
 * block_allocator.py:67-73); k_scale float32 [num_blocks, num_kv_heads, 16]
 * (the per-token K scale of each slot); v_scale float32 [num_blocks,
 * num_kv_heads, head_dim] (the per-channel V scale of the chunk the block
 * belongs to).  Scales are the reference's float16 values widened to
 * float32.  Logical token t of sequence b lives in block
 * block_tables[b * max_blocks_per_seq + t / 16], slot t % 16.  Dequantised
 * values are q * scale rounded once to the compute dtype.
 *
 * q/o: [batch, num_q_heads, q_len, head_dim] strided; k_new/v_new: the
 * suffix's K/V [batch, num_kv_heads, q_len, head_dim] strided.  Sequence b
 * has kv_len = prefix_len_b + q_len.  block_size must be 16.  Block ids
 * outside [0, num_blocks) read as zeros and set KVB_STATUS_BAD_BLOCK.
 */
enum {
  KVB_POOL_INT8_KIVI = 0,
  KVB_POOL_COMPUTE = 1
};

typedef struct KvbPagedPrefillParams {
  int32_t dtype;
  int32_t head_dim;
  int32_t batch;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t q_len;
  int32_t causal;
  float softmax_scale;
  const void* q;
  void* o;
  float* lse;
  int64_t q_batch_stride, q_head_stride, q_row_stride;
  int64_t o_batch_stride, o_head_stride, o_row_stride;
  int64_t lse_batch_stride, lse_head_stride;
  const void* k_new;
  const void* v_new;
  int64_t k_new_batch_stride, k_new_head_stride, k_new_row_stride;
  int64_t v_new_batch_stride, v_new_head_stride, v_new_row_stride;
  const int8_t* kv_pool;
  const float* k_scale;
  const float* v_scale;
  int32_t num_blocks;
  int32_t block_size;
  const int32_t* block_tables;
  int32_t max_blocks_per_seq;
  int32_t prefix_len;           /* uniform (or maximum) cached tokens        */
  const int32_t* prefix_lens;   /* device [batch] per-sequence, or NULL      */
  int32_t* status;
  void* workspace;              /* optional device scratch, see below        */
  int64_t workspace_bytes;
  /* ABI 2: the pool's element format.  KVB_POOL_INT8_KIVI (0, the default of
   * a zero-initialised struct): int8 codes with k_scale / v_scale as above.
   * KVB_POOL_COMPUTE: the pool holds K/V in the compute dtype (the
   * reference's paged engine pool, block_allocator.py:67-73, with its
   * float16/bfloat16 dtype); k_scale and v_scale are not used. */
  int32_t pool_format;
  int32_t reserved0;
} KvbPagedPrefillParams;

/*
 * When many CTAs would read (and dequantise) each KV tile -- long suffixes
 * under GQA, e.g. 2048 new tokens over 8 query heads per KV head -- the
 * library can instead dequantise the prefix once into a dense workspace and
 * run the dense kernel over it.  kvb_paged_prefill_workspace_bytes returns the
 * bytes that strategy needs for these params (0 when the fused path is the
 * right one); pass at least that much as params->workspace to enable it.
 * Without a (large enough) workspace the fused path runs; results agree to
 * rounding either way.
 */
int64_t kvb_paged_prefill_workspace_bytes(const KvbPagedPrefillParams* params);

int kvb_paged_prefill_fwd(const KvbPagedPrefillParams* params, void* stream);

/* Dequantise and gather the paged prefix of every sequence, followed by its
 * fresh suffix, into dense K and V: params->workspace receives K then V, each
 * [batch, num_kv_heads, round_up(prefix_len + q_len, 128), head_dim] in the
 * compute dtype (rows past a sequence's prefix_len_b + q_len, up to the next
 * multiple of 128, are zeros; rows past that are left as they were).
 * workspace_bytes must be at least 2 * batch * num_kv_heads * round_up(...) *
 * head_dim * 2.  q, o and lse are not used.  The device form of the host path
 * that gathers each sequence's blocks (cpu_paged/block_allocator.py:178-206),
 * dequantises them (kv_quantize.py:102-109) and concatenates the chunks
 * (cache_manager.py:460-471); used where the dense K/V feed several query
 * ranges (context-parallel query chunks over one gathered pool). */
int kvb_paged_materialize(const KvbPagedPrefillParams* params, void* stream);

/* Context-parallel shards read in place.  Each rank of a G-GPU group keeps,
 * in a buffer peer-mapped into every rank (symmetric memory over NVLink), its
 * shard of a prompt's paged prefix (the gathered block ids
 * [r * shard_blocks, (r + 1) * shard_blocks)) and the suffix K/V of its
 * zig-zag query rows (chunks r and 2G-1-r of 2G chunks of zigzag_rows rows),
 * laid out by kvb_peer_shard_layout.  base[r] is rank r's buffer as mapped in
 * the calling process. */
typedef struct KvbPeerShards {
  const void* base[8];
  int32_t world;
  int32_t shard_blocks;
  int32_t zigzag_rows;
  int32_t reserved0;
} KvbPeerShards;

/* Byte offsets of a shard buffer's five regions (pool int8 [shard_blocks, 2,
 * Hkv, 16, D]; k_scale f32 [shard_blocks, Hkv, 16]; v_scale f32
 * [shard_blocks, Hkv, D]; suffix K and suffix V [Hkv, 2 * zigzag_rows, D] in
 * the 16-bit compute dtype) into offsets[0..4]; returns the buffer's size in
 * bytes, or -1 for invalid arguments.  No counterpart in the reference. */
int64_t kvb_peer_shard_layout(int num_kv_heads, int head_dim, int shard_blocks,
                              int zigzag_rows, int64_t* offsets);

/* kvb_paged_materialize for one sequence whose prefix blocks and suffix rows
 * are spread over the ranks' shard buffers: every block and suffix row is
 * read from its owner's buffer with plain loads (peer memory over NVLink), so
 * the gather needs no separate collective.  params: batch 1, num_blocks =
 * world * shard_blocks, block_tables in gathered ids, q_len = 2 * world *
 * zigzag_rows, workspace as for kvb_paged_materialize; kv_pool, scales,
 * k_new and v_new are not used.  The caller orders the peers' writes before
 * this call (a cross-GPU barrier).  No counterpart in the reference, whose
 * pool is one host process's memory. */
int kvb_paged_materialize_peers(const KvbPagedPrefillParams* params,
                                const KvbPeerShards* shards, void* stream);

/* Signal words of a bounded cross-GPU barrier.  slot[r] is rank r's array of
 * `world` uint32 words (zero before the first barrier) as mapped in the calling
 * process (peer-mapped memory, e.g. symmetric memory over NVLink). */
typedef struct KvbPeerSignals {
  uint32_t* slot[8];
  int32_t world;
  int32_t rank;
} KvbPeerSignals;

/* Barrier of the context-parallel group before kvb_paged_materialize_peers:
 * enqueued on `stream`, it stores `epoch` into word `rank` of every rank's
 * array, then waits until every word of this rank's array has reached `epoch`
 * (epochs grow by one per barrier, starting at 1).  Every write this GPU made
 * before the launch is visible to a peer once it sees the word.  A wait still
 * unsatisfied after timeout_ns ORs KVB_STATUS_PEER_WAIT into *status and the
 * kernel returns (no trap, the context stays usable).  Plain peer stores and
 * loads only.  No counterpart in the reference, which runs on one host. */
int kvb_peer_barrier(const KvbPeerSignals* signals, uint32_t epoch, int64_t timeout_ns,
                     int* status, void* stream);

/* Size of the static device scratch of kvb_paged_prefill_fwd_noalloc: 32 MiB. */
#define KVB_NOALLOC_SCRATCH_BYTES (32ll << 20)

/* Paged reuse prefill that allocates nothing.  No counterpart in the
 * reference: it serves callers that must not allocate device memory while a
 * request runs (a serving loop whose memory is planned up front, a caching
 * allocator that must not grow between a pool reservation and its release).
 *
 * Same params, results and errors as kvb_paged_prefill_fwd, with the prefix
 * always dequantised once into a fixed static device array of
 * KVB_NOALLOC_SCRATCH_BYTES per device (params->workspace and
 * params->workspace_bytes are ignored); the dense attention kernel then reads
 * it.  Needs 2 * batch * num_kv_heads * round_up(prefix_len + q_len, 128) *
 * head_dim * 2 bytes; larger requests return KVB_ERR_UNSUPPORTED with the
 * sizes in kvb_last_error.  Nothing in the scratch needs to start at zero:
 * the materialise kernel writes every row the attention kernel reads.
 *
 * The first call on a device looks up the scratch's address (which loads the
 * library's module on that device); make it before any stream capture.  The
 * address is looked up again after a context teardown (cudaDeviceReset), so
 * the first call after one should also precede any capture.  Under lazy module
 * loading (the default since CUDA 12.2) only processes that use the library's
 * kernels on a device hold the 32 MiB there; with CUDA_MODULE_LOADING=EAGER
 * every process that loads the library holds it on each device it uses.
 * Calls share one scratch per device: two calls that overlap in time
 * (different streams or host threads) race on it.
 */
int kvb_paged_prefill_fwd_noalloc(const KvbPagedPrefillParams* params, void* stream);

/* ---- Quantise-on-store: a freshly encoded chunk into the int8 block pool ----
 *
 * Replaces, for one encoded chunk, the reference's store path: the K/V taken
 * out of the model's cache (engine.py:846-850), KIVI int8 quantisation on the
 * store (cache_manager.py:164-175 -> kv_quantize.py:73-100) and the copy into
 * 16-token blocks (cpu_paged/chunk_to_blocks.py:57-101).  One launch covers
 * every layer; the source is read once and nothing goes through the host.
 *
 * Arithmetic: the reference's, in the source dtype (torch rounds every step of
 * kv_quantize.py to the tensor's dtype): K scale per token = round(round(max(
 * amax_d|k|, 1e-8)) / 127), V scale per channel over the chunk's tokens,
 * q = clamp(rint(round(x / scale)), -128, 127), 0 where x / scale is NaN
 * (0 / 0); scales stored as float16 (kv_quantize.py:93-97) and, where the
 * float32 arrays are given, as the float32 value of that float16.  Token t
 * goes to block_ids[t / 16], slot t % 16; slots of the last block past the
 * chunk's end are zeroed (q and K scale); every block of the chunk gets the
 * chunk's V scales.  Sources must hold finite values.
 */
#define KVB_MAX_LAYERS 128
#define KVB_MAX_CHUNK_BLOCKS 128

typedef struct KvbQuantizeStoreParams {
  int32_t dtype;              /* source K/V dtype, KVB_DTYPE_*; the arithmetic runs in it */
  int32_t head_dim;           /* 64, 96 or 128 */
  int32_t num_layers;         /* 1 .. KVB_MAX_LAYERS */
  int32_t num_kv_heads;
  int32_t num_tokens;         /* chunk length S >= 1 */
  int32_t num_chunk_blocks;   /* ceil(S / 16) .. KVB_MAX_CHUNK_BLOCKS */
  int32_t block_ids[KVB_MAX_CHUNK_BLOCKS];
  int64_t num_pool_blocks;    /* every block id must lie in [0, num_pool_blocks) */
  /* Source, per layer: element (h, t, d) at src_k[l] + h * src_head_stride +
   * t * src_row_stride + d (elements).  Host arrays of device pointers. */
  const void* const* src_k;
  const void* const* src_v;
  int64_t src_head_stride;
  int64_t src_row_stride;
  /* Destination, per layer (host arrays of device pointers): the int8 pool
   * [num_pool_blocks][2][num_kv_heads][16][head_dim] (K at index 0, V at 1),
   * float16 scales K [num_pool_blocks][num_kv_heads][16] and V
   * [num_pool_blocks][num_kv_heads][head_dim], and their float32 copies.
   * Any of the four scale arrays may be NULL (not written). */
  void* const* pool;
  void* const* k_scale16;
  void* const* v_scale16;
  void* const* k_scale;
  void* const* v_scale;
} KvbQuantizeStoreParams;

int kvb_quantize_store(const KvbQuantizeStoreParams* params, void* stream);

/*
 * The same store for several chunks in one launch (a warm of many chunks):
 * every pointer below is DEVICE memory, so the tables are built once per call
 * and copied with the data's stream.  Chunk c has num_tokens[c] tokens (1 ..
 * 16 * max_chunk_blocks) in blocks block_ids[c][0 .. ceil(num_tokens[c] / 16));
 * its layer l's K and V are src[(c * num_layers + l) * 2 + 0 / 1], 16-byte
 * aligned, with the chunk's head and row strides src_strides[c][0 / 1]
 * (elements, multiples of 8).  tables[k * num_layers + l] for k = 0..4: the
 * pool, K scale fp16, V scale fp16, K scale fp32, V scale fp32 of layer l (a
 * NULL scale table entry is not written).  The chunks' blocks must not overlap.
 * Block ids outside [0, num_pool_blocks) are skipped and set
 * KVB_STATUS_BAD_BLOCK; a token count out of range, a misaligned source or a
 * stride that is not a multiple of 8 skips that chunk and sets
 * KVB_STATUS_BAD_LENGTH, in the optional *status.
 */
typedef struct KvbQuantizeStoreBatch {
  int32_t dtype;
  int32_t head_dim;
  int32_t num_layers;
  int32_t num_kv_heads;
  int32_t num_chunks;         /* num_chunks * num_layers <= 65535 */
  int32_t max_chunk_blocks;   /* row length of block_ids, <= KVB_MAX_CHUNK_BLOCKS */
  int64_t num_pool_blocks;
  const int32_t* num_tokens;  /* device [num_chunks] */
  const int32_t* block_ids;   /* device [num_chunks][max_chunk_blocks] */
  const void* const* src;     /* device [num_chunks][num_layers][2] */
  const int64_t* src_strides; /* device [num_chunks][2] */
  void* const* tables;        /* device [5][num_layers] */
  int32_t* status;
} KvbQuantizeStoreBatch;

int kvb_quantize_store_batch(const KvbQuantizeStoreBatch* params, void* stream);

/* ---- CacheBlend: deviation-guided patch of stitched chunk K/V ----
 *
 * Replaces CacheBlendRecompute._deviation_recompute after its full-context
 * forward (cacheblend.py:141-197), device-resident: for each cached position
 * t, the mean over layers of 1 - cos(cached K_t, fresh K_t), the K vectors of
 * all KV heads flattened into one (cosine as torch's: x.y / (max(|x|, 1e-8)
 * max(|y|, 1e-8)), float32 here); positions with deviation > min_deviation
 * are candidates; the min(num_select, #candidates) largest are chosen (lower
 * position first among equal deviations; torch's topk leaves that order
 * unspecified), written ascending to `selected` (-1 after the count) with
 * their count in *num_selected, and with patch = 1 the fresh K and V rows of
 * every layer and head are copied over the cached ones there.  No host
 * synchronisation: the count stays on the device.
 */
typedef struct KvbCacheBlendParams {
  int32_t dtype;              /* KVB_DTYPE_*, all four K/V operands */
  int32_t head_dim;           /* 64, 96 or 128 */
  int32_t num_layers;         /* 1 .. KVB_MAX_LAYERS */
  int32_t num_kv_heads;
  int32_t num_tokens;         /* S, cached positions compared, >= 1 */
  int32_t num_select;         /* max(1, int(S * recompute_ratio)) (cacheblend.py:163) */
  float min_deviation;
  int32_t patch;              /* 0: deviation and selection only; 1: also patch */
  /* Per layer (host arrays of device pointers): element (h, t, d) at
   * ptr[l] + h * head_stride + t * row_stride + d.  Strides in elements, multiples
   * of 8; pointers 16-byte aligned.  cached_v / fresh_v may be NULL when patch = 0. */
  void* const* cached_k;
  void* const* cached_v;
  const void* const* fresh_k;
  const void* const* fresh_v;
  int64_t cached_head_stride;
  int64_t cached_row_stride;
  int64_t fresh_head_stride;
  int64_t fresh_row_stride;
  float* deviation;           /* device [S], written */
  int32_t* selected;          /* device [num_select], written */
  int32_t* num_selected;      /* device [1], written */
} KvbCacheBlendParams;

int kvb_cacheblend_fwd(const KvbCacheBlendParams* params, void* stream);

/* Human-readable reason for the last non-zero return on this host thread. */
const char* kvb_last_error(void);

/* KVB_ABI_VERSION of the loaded library. */
int kvb_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* KVB_ATTN_H_ */
