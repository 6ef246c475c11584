"""Hybrid KV-cache sizing and grouping (the arithmetic of plugins/vllm_lrkv/vllm_lrkv/kv_cache.py:56-134)."""

import math

from belt_b200 import kv_cache


def test_block_holds_n_latent_gdn_states():
    # 16 compressed layers of 1024-column BF16 rows (2 KB per token each), a GDN state of 1.1 MB
    pages = kv_cache.latent_page_sizes({"layers": {f"l{i}": {"row_width": 1024} for i in range(16)}})
    assert pages == [2048] * 16
    mamba = 1_114_112
    block, padded = kv_cache.hybrid_block_size(pages, mamba, 16, 16, 16)
    assert block % 16 == 0
    assert block * sum(pages) >= 16 * mamba                       # the block holds n_latent GDN states
    assert (block - 16) * sum(pages) < 16 * mamba                 # and is the smallest aligned such size
    assert padded is None or (padded >= mamba and padded == math.ceil(block * sum(pages) / 16))


def test_learned_ranks_and_alignment():
    # per-layer widths of a learned-rank export (not all equal), the backends' blocks 16 and 64 (lcm 64)
    widths = [1024, 896, 1024, 768, 1024, 960]
    pages = kv_cache.latent_page_sizes({"layers": {f"l{i}": {"row_width": w} for i, w in enumerate(widths)}})
    mamba = 600_000
    align = kv_cache.backend_alignment([16, 64])
    assert align == 64
    block, padded = kv_cache.hybrid_block_size(pages, mamba, kv_cache.KERNEL_BLOCK_UNIT, 16, align)
    assert block % 64 == 0 and block * sum(pages) >= len(pages) * mamba
    assert (block - 64) * sum(pages) < len(pages) * mamba or block == 64
    assert padded == math.ceil(block * sum(pages) / len(pages)) and padded >= mamba


def test_exact_fit_needs_no_padding():
    # one layer of 4 KB per token, a state of exactly 16 tokens' worth: block 16, no padding
    assert kv_cache.hybrid_block_size([4096], 16 * 4096, 16, 1, 16) == (16, None)


def test_nothing_to_size():
    assert kv_cache.hybrid_block_size([], 1000, 16, 32, 16) == (32, None)
    assert kv_cache.hybrid_block_size([2048], 0, 16, 32, 16) == (32, None)


def test_groups_in_model_order():
    latent = ["a0", "a1", "a2"]
    mamba = [f"m{i}" for i in range(8)]
    assert kv_cache.group_layers(latent, mamba) == [latent, ["m0", "m1", "m2"], ["m3", "m4", "m5"], ["m6", "m7"]]
    assert kv_cache.group_layers([], ["m0", "m1"]) == [["m0"], ["m1"]]
