"""KV-cache block size and layer grouping for hybrid models (GDN + compressed full-attention layers), the arithmetic of
the reference's vLLM hooks (plugins/vllm_lrkv/vllm_lrkv/kv_cache.py:56-138), written as plain functions of the sizes
they read from the vLLM config:

* ``hybrid_block_size``: the smallest backend-aligned block size B (tokens) with B * sum_i(row bytes_i) >= n_latent *
  GDN state bytes, so that one block of all compressed layers holds as many bytes as n_latent GDN states, and the GDN
  page padded to that block's bytes / n_latent (``_resize_block``, kv_cache.py:56-88);
* ``group_layers``: every compressed layer in one group and the GDN layers in groups of n_latent, in model order
  (``_packed_kv_cache_groups``, kv_cache.py:103-134), so that every group fills the same block;
* ``latent_page_sizes``: per-token cache bytes of every compressed layer of a ``kv_lowrank`` config block
  (kv_cache.py:47-53).

The hooks that patch vLLM's platform and ``kv_cache_utils`` with these decisions need vLLM 0.32's plugin API and are
not part of this package; the functions take the same inputs, so a plugin calls them from its own hooks. This
backend's kernels accept block sizes 16, 32, 64 and multiples of 128 (``KERNEL_BLOCK_UNIT`` is the smallest).
"""

from __future__ import annotations

import math

# the smallest block size the decode and decompress kernels accept (the reference's backend: MultipleOf(64))
KERNEL_BLOCK_UNIT = 16


def latent_page_sizes(kv_lowrank: dict, dtype_size: int = 2) -> list:
    """Per-token cache bytes of every compressed layer: row_width * dtype size (kv_cache.py:47-53)."""
    return [int(info["row_width"]) * int(dtype_size) for info in kv_lowrank["layers"].values()]


def hybrid_block_size(latent_page_bytes: list, mamba_page: int, kernel_block_unit: int = KERNEL_BLOCK_UNIT,
                      pre_block_size: int = 1, backend_alignment: int = 1):
    """(block_size, padded GDN page or None when no padding is needed) for a hybrid model whose compressed layers store
    ``latent_page_bytes[i]`` bytes per token and whose GDN state takes ``mamba_page`` bytes (kv_cache.py:56-88):
    B = unit * ceil(n_latent * mamba_page / (unit * sum(latent bytes))), unit = max(kernel unit, the block size set
    before, 1), rounded up to a multiple of ``backend_alignment`` (the lcm of the attention backends' smallest block
    sizes); the GDN page padded to ceil(B * sum / n_latent). Returns (pre_block_size, None) when there is nothing to
    size (no compressed layer or no GDN state)."""
    if not latent_page_bytes or mamba_page <= 0:
        return pre_block_size, None
    n_latent, per_token = len(latent_page_bytes), sum(latent_page_bytes)
    unit = max(int(kernel_block_unit), int(pre_block_size), 1)
    block = unit * math.ceil(n_latent * mamba_page / (unit * per_token))
    align = max(int(backend_alignment), 1)
    block = align * math.ceil(block / align)
    padded = math.ceil(block * per_token / n_latent)
    return block, (padded if padded != mamba_page else None)


def backend_alignment(smallest_block_sizes: list) -> int:
    """lcm of the attention backends' smallest supported block sizes (kv_cache.py:72-74)."""
    return math.lcm(*[int(s) for s in smallest_block_sizes]) if smallest_block_sizes else 1


def group_layers(latent_layers: list, mamba_layers: list) -> list:
    """KV-cache groups: the compressed layers together, then the GDN layers in model order in groups of
    len(latent_layers) (kv_cache.py:103-134). With no compressed layer the GDN layers stay one group each."""
    groups = [list(latent_layers)] if latent_layers else []
    n = len(latent_layers) or 1
    for i in range(0, len(mamba_layers), n):
        groups.append(list(mamba_layers[i:i + n]))
    return groups
