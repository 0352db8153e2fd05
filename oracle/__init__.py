"""CPU oracle for the kvboost_b200 prefill-attention path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
directory.  It may be imported by ``tests/``, by ``__graft_entry__.smoke()``
and by ``bench.py`` (its CPU-baseline leg and ``--impl reference`` arm), and
there only as the checker or as the timed CPU restatement -- never as the
thing whose output is shipped.

What it restates (each function cites the KVBoost file:line it follows):

* ``attention``  -- softmax attention with bottom-right (offset) causal mask,
  GQA head grouping and the natural-log LSE of the reference kernel
  (``src/kvboost/csrc/flash_attn_kernel.cu:184-245``), varlen and paged
  variants (``src/kvboost/cpu_paged/paged_attn_cpu.py:33-108``).
* ``kv_quant``   -- KIVI int8 quantize / dequantize with the reference's
  float16 rounding (``src/kvboost/kv_quantize.py:73-109``), also on bfloat16
  K/V as a model hands them to the store.
* ``cacheblend`` -- CacheBlend's per-position deviation, top-k selection and
  patch (``src/kvboost/cacheblend.py:103-197``).
* ``paged``      -- the block allocator's LIFO free list, ref counts,
  copy-on-write, the chunk->block mapper and ``read_kv`` gather
  (``src/kvboost/cpu_paged/block_allocator.py``,
  ``src/kvboost/cpu_paged/chunk_to_blocks.py``).
* ``hashing``    -- prefix-chained SHA-256 chunk keys and the fixed 128-token
  split (``src/kvboost/models.py:131-148``,
  ``src/kvboost/chunk_registry.py:98-110``).

Parity pin: every module here is checked against golden vectors produced by
running the reference itself (``tests/golden/make_golden.py``; fixtures in
``tests/golden/``) by ``tests/test_oracle_golden.py``.
"""
