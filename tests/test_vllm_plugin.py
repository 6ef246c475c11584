"""The vLLM binding and plugin hooks (``belt_b200.vllm_plugin``), driven through a fake vLLM module tree.

vLLM 0.32 (the plugin API the reference targets) is not in this image, so the names the binding and the hooks import
are provided by small stand-in modules shaped like vLLM's: the backend base class and its types, the KV-cache spec
classes, the layout enum, the backend registry, the platform's hybrid block sizing and ``kv_cache_utils``' packing.
Checked: the backend classes bind to vLLM's own types when present (``MultipleOf``, ``KVCacheLayout``,
``AttentionBackend``, ``FullAttentionSpec``); ``register`` adds ``LRKV_LATENT`` once and wraps the two KV-cache
decisions once; for a latent model the block size and GDN padding are the ones ``kv_cache.hybrid_block_size``
computes from the config's layer widths and the model's GDN state, and the groups are one of all compressed layers
plus GDN groups of n_latent in model order; other models keep vLLM's decisions.
"""

from contextlib import contextmanager
from dataclasses import dataclass
import enum
import sys
import types

import pytest
import torch

from belt_b200 import kv_cache, latent_backend, vllm_plugin

GDN_STATE = 1_114_112


def _module(name, **attrs):
    m = types.ModuleType(name)
    m.__path__ = []
    for k, v in attrs.items():
        setattr(m, k, v)
    return m


@pytest.fixture
def fake_vllm(monkeypatch):
    class AttentionBackend:
        pass

    class AttentionType:
        DECODER = "decoder"

    @dataclass(frozen=True)
    class MultipleOf:
        base: int

    @dataclass(frozen=True, kw_only=True)
    class FullAttentionSpec:
        block_size: int
        num_kv_heads: int
        head_size: int
        dtype: torch.dtype

        @property
        def page_size_bytes(self):
            return self.block_size * self.num_kv_heads * self.head_size * torch.finfo(self.dtype).bits // 8

    @dataclass(frozen=True)
    class MambaSpec:
        page_size_bytes: int = GDN_STATE

    @dataclass
    class KVCacheGroupSpec:
        layer_names: list
        kv_cache_spec: object

    class UniformTypeKVCacheSpecs:
        @classmethod
        def from_specs(cls, specs):
            kinds = {type(s) for s in specs.values()}
            return types.SimpleNamespace(specs=dict(specs)) if len(kinds) == 1 else None

    class KVCacheLayout(enum.Enum):
        NHD = "NHD"
        BLHNC = "BLHNC"
        BLNHC = "BLNHC"

        @property
        def is_block_outermost(self):
            return self.name.startswith("BL")

    class AttentionBackendEnum:
        _member_map_ = {}

        @classmethod
        def register(cls, name, path):
            cls._member_map_[name] = path

    class FlashAttention:
        @staticmethod
        def get_supported_kernel_block_sizes():
            return [MultipleOf(16)]

    class Platform:
        @classmethod
        def _align_hybrid_block_size(cls, vllm_config, backend_cls):
            vllm_config.cache_config.block_size = 64          # stand-in for vLLM's own sizing

        @classmethod
        def _find_non_ssm_backends(cls, vllm_config):
            return [FlashAttention]

    calls = {"annotate": 0}

    def original_groups(vllm_config, kv_cache_spec):
        return "vllm's grouping"

    def annotate(vllm_config, kv_cache_spec, groups, use_trailing_layer_fallback):
        calls["annotate"] += 1

    class HybridModel:
        @staticmethod
        def get_mamba_specs_from_config(vllm_config):
            return [MambaSpec(), MambaSpec(GDN_STATE // 2)]

    class ModelRegistry:
        @staticmethod
        def resolve_model_cls(arch, model_config):
            return HybridModel, arch

    @contextmanager
    def set_current_vllm_config(cfg):
        yield

    kv_utils = _module("vllm.v1.core.kv_cache_utils", _get_packed_kv_cache_groups=original_groups,
                       _annotate_eagle_groups=annotate, _uses_trailing_mtp_layers=lambda cfg: False,
                       _warn_if_unannotated_eagle_mamba=lambda cfg, groups: None)
    tree = {
        "vllm": _module("vllm"), "vllm.v1": _module("vllm.v1"), "vllm.v1.attention": _module("vllm.v1.attention"),
        "vllm.v1.attention.backend": _module("vllm.v1.attention.backend", AttentionBackend=AttentionBackend,
                                             AttentionType=AttentionType, MultipleOf=MultipleOf),
        "vllm.v1.attention.backends": _module("vllm.v1.attention.backends"),
        "vllm.v1.attention.backends.registry": _module("vllm.v1.attention.backends.registry",
                                                       AttentionBackendEnum=AttentionBackendEnum),
        "vllm.v1.kv_cache_interface": _module("vllm.v1.kv_cache_interface", FullAttentionSpec=FullAttentionSpec,
                                              MambaSpec=MambaSpec, KVCacheGroupSpec=KVCacheGroupSpec,
                                              UniformTypeKVCacheSpecs=UniformTypeKVCacheSpecs),
        "vllm.v1.kv_cache_layout": _module("vllm.v1.kv_cache_layout", KVCacheLayout=KVCacheLayout),
        "vllm.v1.core": _module("vllm.v1.core", kv_cache_utils=kv_utils), "vllm.v1.core.kv_cache_utils": kv_utils,
        "vllm.platforms": _module("vllm.platforms"),
        "vllm.platforms.interface": _module("vllm.platforms.interface", Platform=Platform),
        "vllm.config": _module("vllm.config"),
        "vllm.config.vllm": _module("vllm.config.vllm", set_current_vllm_config=set_current_vllm_config),
        "vllm.model_executor": _module("vllm.model_executor"),
        "vllm.model_executor.models": _module("vllm.model_executor.models", ModelRegistry=ModelRegistry),
    }
    tree["vllm.platforms"].interface = tree["vllm.platforms.interface"]
    for name, mod in tree.items():
        monkeypatch.setitem(sys.modules, name, mod)
    api = vllm_plugin.vllm_api()
    assert api is not None
    # the classes a vLLM process would have bound at import
    KV = latent_backend.make_kv_spec_class(api)
    monkeypatch.setattr(latent_backend, "LatentKVSpec", KV)
    monkeypatch.setattr(latent_backend, "LatentAttentionBackend", latent_backend.make_backend_class(api))
    return types.SimpleNamespace(api=api, KV=KV, MambaSpec=MambaSpec, KVCacheLayout=KVCacheLayout,
                                 KVCacheGroupSpec=KVCacheGroupSpec, Platform=Platform, registry=AttentionBackendEnum,
                                 kv_utils=kv_utils, calls=calls, MultipleOf=MultipleOf,
                                 AttentionBackend=AttentionBackend, FullAttentionSpec=FullAttentionSpec)


def _config(latent=True, widths=(1024, 896, 1024, 768), layout="BLHNC", fake=None):
    block = {"format": "latent", "layers": {str(3 + 4 * i): {"row_width": w} for i, w in enumerate(widths)}}
    hf = types.SimpleNamespace(kv_lowrank=block if latent else None)
    mc = types.SimpleNamespace(hf_text_config=hf, dtype=torch.bfloat16, architecture="HybridModel")
    cc = types.SimpleNamespace(block_size=16, mamba_cache_mode="align", mamba_block_size=None,
                               mamba_page_size_padded=None,
                               get_resolved_kv_cache_layout=lambda: fake.KVCacheLayout[layout])
    return types.SimpleNamespace(model_config=mc, cache_config=cc)


def test_backend_binds_to_vllm_types(fake_vllm):
    B = latent_backend.LatentAttentionBackend
    assert issubclass(B, fake_vllm.AttentionBackend)
    sizes = B.get_supported_kernel_block_sizes()
    assert sizes[:3] == [16, 32, 64] and isinstance(sizes[3], fake_vllm.MultipleOf) and sizes[3].base == 128
    assert B.supported_kv_cache_layouts() == (fake_vllm.KVCacheLayout.BLHNC, fake_vllm.KVCacheLayout.BLNHC)
    spec = fake_vllm.KV(block_size=16, num_kv_heads=1, head_size=1024, dtype=torch.bfloat16)
    assert isinstance(spec, fake_vllm.FullAttentionSpec) and spec.head_size_v == 0
    assert spec.page_size_bytes == 16 * 1024 * 2
    assert B.get_name() == "LRKV_LATENT" and B.get_impl_cls() is latent_backend.LatentAttentionImpl


def test_without_vllm_the_stand_ins_are_used():
    if "vllm" in sys.modules:
        pytest.skip("a vLLM is loaded in this process")
    assert vllm_plugin.vllm_api() is None
    assert latent_backend.MultipleOf is latent_backend._StandInMultipleOf
    assert vllm_plugin.register() is False


def test_register_adds_the_backend_and_wraps_once(fake_vllm):
    assert vllm_plugin.register()
    assert fake_vllm.registry._member_map_["LRKV_LATENT"] == "belt_b200.latent_backend.LatentAttentionBackend"
    wrapped_groups = fake_vllm.kv_utils._get_packed_kv_cache_groups
    wrapped_align = fake_vllm.Platform.__dict__["_align_hybrid_block_size"].__func__
    assert wrapped_groups._belt_b200 and wrapped_align._belt_b200
    assert vllm_plugin.register()
    assert fake_vllm.kv_utils._get_packed_kv_cache_groups is wrapped_groups
    assert fake_vllm.Platform.__dict__["_align_hybrid_block_size"].__func__ is wrapped_align


def test_hybrid_block_size_for_a_latent_model(fake_vllm):
    vllm_plugin.register()
    cfg = _config(fake=fake_vllm)
    fake_vllm.Platform._align_hybrid_block_size(cfg, latent_backend.LatentAttentionBackend)
    pages = [w * 2 for w in (1024, 896, 1024, 768)]
    exp, padded = kv_cache.hybrid_block_size(pages, GDN_STATE, 16, 16, 16)
    assert cfg.cache_config.block_size == exp and cfg.cache_config.mamba_block_size == exp
    assert cfg.cache_config.mamba_page_size_padded == padded
    assert exp * sum(pages) >= len(pages) * GDN_STATE
    other = _config(latent=False, fake=fake_vllm)
    fake_vllm.Platform._align_hybrid_block_size(other, latent_backend.LatentAttentionBackend)
    assert other.cache_config.block_size == 64 and other.cache_config.mamba_page_size_padded is None


def test_kv_cache_groups_for_a_latent_model(fake_vllm):
    vllm_plugin.register()
    KV, M = fake_vllm.KV, fake_vllm.MambaSpec
    spec = {}
    for i in range(10):                              # model order: layers 3 and 7 compressed, the rest GDN
        if i in (3, 7):
            spec[f"l{i}"] = KV(block_size=16, num_kv_heads=1, head_size=1024 if i == 3 else 896, dtype=torch.bfloat16)
        else:
            spec[f"l{i}"] = M()
    groups = fake_vllm.kv_utils._get_packed_kv_cache_groups(_config(fake=fake_vllm), spec)
    assert [g.layer_names for g in groups] == [["l3", "l7"], ["l0", "l1"], ["l2", "l4"], ["l5", "l6"], ["l8", "l9"]]
    assert fake_vllm.calls["annotate"] == 1
    # other models, or a layout that is not block-outermost: vLLM's grouping
    assert fake_vllm.kv_utils._get_packed_kv_cache_groups(_config(latent=False, fake=fake_vllm), spec) == \
        "vllm's grouping"
    assert fake_vllm.kv_utils._get_packed_kv_cache_groups(_config(layout="NHD", fake=fake_vllm), spec) == \
        "vllm's grouping"
