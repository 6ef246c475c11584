"""The vLLM side of this package: the plugin API names it binds to, the plugin entry point, and the hybrid KV-cache
hooks (the reference's ``plugins/vllm_lrkv/vllm_lrkv/__init__.py:28-41`` and ``kv_cache.py:56-148``).

``vllm_api()`` returns the vLLM 0.32 plugin-API names the backend classes are built on (``AttentionBackend``,
``AttentionType``, ``MultipleOf``, ``FullAttentionSpec``, ``KVCacheLayout``, ...) or None when the running vLLM does
not provide them; ``latent_backend`` then falls back to stand-ins of the same shape, so the package imports and runs
without vLLM.

``register()`` is the plugin entry point (``vllm.general_plugins``): it registers ``LatentAttentionBackend`` under the
reference's backend name ``LRKV_LATENT`` -- the swap that makes a vLLM serving a latent export run this package's
kernels -- and installs the two KV-cache hooks. Model classes are not registered here: the compressed layers' model
code stays the plugin's own (it reaches the backend through the name).

The hooks replace two decisions vLLM makes for hybrid (GDN + full attention) models, for ``latent`` models only:

* ``Platform._align_hybrid_block_size``: after vLLM's own sizing, the block size becomes the smallest backend-aligned
  B with B * (all compressed layers' bytes per token) >= n_latent * GDN state bytes, and the GDN page is padded to
  that block's bytes / n_latent (``kv_cache.hybrid_block_size``);
* ``kv_cache_utils._get_packed_kv_cache_groups``: with a block-outermost layout and pages of different sizes, one group
  of all compressed layers and the GDN layers in model order in groups of n_latent (``kv_cache.group_layers``), so
  that every group fills the same block.

Every other model goes through vLLM's functions unchanged.
"""

from __future__ import annotations

from functools import wraps
import logging
from types import SimpleNamespace

from . import kv_cache

logger = logging.getLogger(f"vllm.{__name__}")

BACKEND_NAME = "LRKV_LATENT"
BACKEND_PATH = "belt_b200.latent_backend.LatentAttentionBackend"
LATENT_FORMAT = "latent"


def vllm_api():
    """The vLLM plugin-API names this package binds to, or None when they cannot be imported. Only a vLLM that is
    already loaded is probed (this package running inside a vLLM process; importing vLLM just to look takes seconds),
    unless ``BELT_B200_BIND_VLLM=1`` asks for the import."""
    import os
    import sys
    if "vllm" not in sys.modules and os.environ.get("BELT_B200_BIND_VLLM") != "1":
        return None
    try:
        from vllm.v1.attention.backend import AttentionBackend, AttentionType, MultipleOf
        from vllm.v1.kv_cache_interface import FullAttentionSpec
        from vllm.v1.kv_cache_layout import KVCacheLayout
    except Exception:
        return None
    return SimpleNamespace(AttentionBackend=AttentionBackend, AttentionType=AttentionType, MultipleOf=MultipleOf,
                           FullAttentionSpec=FullAttentionSpec, KVCacheLayout=KVCacheLayout)


# ------------------------------------------------------------------------------------------------------ the hooks
def latent_block(vllm_config):
    """The model's ``kv_lowrank`` block when it is a ``latent`` export, else None."""
    mc = getattr(vllm_config, "model_config", None)
    block = getattr(getattr(mc, "hf_text_config", None), "kv_lowrank", None) if mc is not None else None
    return block if isinstance(block, dict) and block.get("format") == LATENT_FORMAT else None


def gdn_state_bytes(vllm_config) -> int:
    """The unpadded GDN state page of the model, from the model class's state-shape helpers (as vLLM's platform
    computes it before padding)."""
    from vllm.model_executor.models import ModelRegistry
    from vllm.v1.kv_cache_interface import MambaSpec

    mc = vllm_config.model_config
    cls, _ = ModelRegistry.resolve_model_cls(mc.architecture, model_config=mc)
    if hasattr(cls, "get_mamba_specs_from_config"):
        return max(spec.page_size_bytes for spec in cls.get_mamba_specs_from_config(vllm_config))
    return MambaSpec(shapes=cls.get_mamba_state_shape_from_config(vllm_config),
                     dtypes=cls.get_mamba_state_dtype_from_config(vllm_config), block_size=-1).page_size_bytes


def _dtype_bytes(dtype) -> int:
    import torch
    return torch.empty((), dtype=dtype).element_size()


def resize_hybrid_block(platform_cls, vllm_config, backend_cls, pre_block_size: int) -> None:
    """Set the cache config's block size and GDN page padding for a ``latent`` model (a no-op for others)."""
    block = latent_block(vllm_config)
    if block is None:
        return
    from vllm.config.vllm import set_current_vllm_config
    from vllm.v1.attention.backend import MultipleOf

    pages = kv_cache.latent_page_sizes(block, _dtype_bytes(vllm_config.model_config.dtype))
    state = gdn_state_bytes(vllm_config)
    if not pages or state <= 0:
        return

    def smallest(sizes):
        return min(s.base if isinstance(s, MultipleOf) else int(s) for s in sizes)

    with set_current_vllm_config(vllm_config):
        unit = smallest(backend_cls.get_supported_kernel_block_sizes())
        others = [smallest(sizes) for b in platform_cls._find_non_ssm_backends(vllm_config)
                  if (sizes := b.get_supported_kernel_block_sizes())]
    size, padded = kv_cache.hybrid_block_size(pages, state, unit, pre_block_size, kv_cache.backend_alignment(others))
    cc = vllm_config.cache_config
    cc.block_size = size
    if getattr(cc, "mamba_cache_mode", None) == "align":
        cc.mamba_block_size = size
    cc.mamba_page_size_padded = padded
    logger.info("belt_b200: %d compressed layers (%d cache bytes per token), block size %d tokens, GDN page %s",
                len(pages), sum(pages), size, padded if padded is not None else "unpadded")


def wrap_align_hybrid_block_size(original):
    """``Platform._align_hybrid_block_size`` followed by ``resize_hybrid_block`` for latent models."""
    @wraps(original)
    def align(cls, vllm_config, backend_cls):
        pre = vllm_config.cache_config.block_size
        original(cls, vllm_config, backend_cls)
        resize_hybrid_block(cls, vllm_config, backend_cls, pre)

    align._belt_b200 = True
    return align


def wrap_packed_kv_cache_groups(original):
    """``kv_cache_utils._get_packed_kv_cache_groups`` with the latent grouping (``kv_cache.group_layers``)."""
    @wraps(original)
    def groups_for(vllm_config, kv_cache_spec):
        from vllm.v1.core import kv_cache_utils
        from vllm.v1.kv_cache_interface import KVCacheGroupSpec, MambaSpec, UniformTypeKVCacheSpecs

        from .latent_backend import LatentKVSpec

        if latent_block(vllm_config) is None:
            return original(vllm_config, kv_cache_spec)
        layout = vllm_config.cache_config.get_resolved_kv_cache_layout()
        if not layout.is_block_outermost or len({s.page_size_bytes for s in kv_cache_spec.values()}) <= 1:
            return original(vllm_config, kv_cache_spec)
        latent = [n for n, s in kv_cache_spec.items() if isinstance(s, LatentKVSpec)]
        states = [n for n, s in kv_cache_spec.items() if isinstance(s, MambaSpec)]
        if not latent or len(latent) + len(states) != len(kv_cache_spec):
            return original(vllm_config, kv_cache_spec)
        groups = []
        for names in kv_cache.group_layers(latent, states):
            spec = UniformTypeKVCacheSpecs.from_specs({n: kv_cache_spec[n] for n in names})
            if spec is None:
                return original(vllm_config, kv_cache_spec)
            groups.append(KVCacheGroupSpec(list(names), spec))
        kv_cache_utils._annotate_eagle_groups(
            vllm_config, kv_cache_spec, groups,
            use_trailing_layer_fallback=kv_cache_utils._uses_trailing_mtp_layers(vllm_config))
        kv_cache_utils._warn_if_unannotated_eagle_mamba(vllm_config, groups)
        logger.info("belt_b200: KV cache groups: %d compressed layers, %d GDN groups", len(latent), len(groups) - 1)
        return groups

    groups_for._belt_b200 = True
    return groups_for


def install_kv_cache_hooks() -> None:
    """Wrap vLLM's two KV-cache decisions (once; installing twice changes nothing)."""
    from vllm.platforms import interface
    from vllm.v1.core import kv_cache_utils

    if not getattr(kv_cache_utils._get_packed_kv_cache_groups, "_belt_b200", False):
        kv_cache_utils._get_packed_kv_cache_groups = wrap_packed_kv_cache_groups(
            kv_cache_utils._get_packed_kv_cache_groups)
    current = interface.Platform.__dict__["_align_hybrid_block_size"].__func__
    if not getattr(current, "_belt_b200", False):
        interface.Platform._align_hybrid_block_size = classmethod(wrap_align_hybrid_block_size(current))


def register() -> bool:
    """Plugin entry point: register ``LRKV_LATENT`` -> this package's backend and install the KV-cache hooks. Returns
    False (and changes nothing) when the running vLLM lacks the plugin API."""
    if vllm_api() is None:
        return False
    from vllm.v1.attention.backends.registry import AttentionBackendEnum
    if BACKEND_NAME not in AttentionBackendEnum._member_map_:
        AttentionBackendEnum.register(BACKEND_NAME, BACKEND_PATH)
    install_kv_cache_hooks()
    logger.info("belt_b200: attention backend %s -> %s", BACKEND_NAME, BACKEND_PATH)
    return True
