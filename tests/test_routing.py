"""Host: which kernel prefill_attention picks for a shape (split_key_plan)."""

from kvboost_b200.ops import decode_splits, split_key_plan


def test_dense_configs_keep_prefill_kernel():
    # prefix-reuse op (B4, 32/8 heads, 256 new over 1152), single causal op, long paged suffix
    assert not split_key_plan(4, 32, 8, 256, 1152)[0]
    assert not split_key_plan(2, 16, 16, 1024, 1024)[0]
    assert not split_key_plan(1, 64, 8, 2048, 34816)[0]
    assert not split_key_plan(1, 32, 8, 8192, 8192)[0]


def test_short_suffixes_take_split_key():
    use, splits = split_key_plan(8, 16, 2, 1, 4096)      # decode step: 9 CTAs x 2 ranges per group
    assert use and splits == 16
    assert split_key_plan(8, 16, 2, 16, 32784)[0]         # seam over a 32K prefix
    assert split_key_plan(1, 32, 32, 16, 8208)[0]         # MHA short suffix
    assert split_key_plan(1, 64, 8, 64, 32832)[0]         # short suffix, 64/8 heads


def test_not_for_queries_longer_than_keys_or_tiny_kv():
    assert not split_key_plan(1, 16, 2, 300, 200)[0]
    assert not split_key_plan(8, 16, 2, 1, 100)[0]


def test_splits_fill_one_wave():
    # one CTA per split per (sequence, KV head, 256 packed rows), at least two key tiles
    # each; two splits per CTA when a group's packed rows fit one 128-row tile
    assert decode_splits(8, 2, 4096) == 16
    assert decode_splits(8, 2, 32768, packed_rows=128) == 18
    assert decode_splits(8, 2, 32768, packed_rows=129) == 9
    assert decode_splits(1, 8, 32768, packed_rows=8 * 64) == 9
    assert decode_splits(1, 2, 300) == 1
    assert decode_splits(200, 2, 4096) == 2      # more groups than SMs: still both slots busy
    assert decode_splits(200, 2, 4096, packed_rows=129) == 1
