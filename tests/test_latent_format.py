"""The latent export directory: this package's writer and reader against the reference's own exporter.

``tests/golden/export.json`` holds what the reference's ``export()`` (``lrkv/runtime/export_latent.py:208-305``)
wrote for the synthetic base model and factor checkpoint of ``tests/golden/export_case.py`` (packed and
``rope_align``), and the checksums of the per-layer constants the reference's ``derive_latent_tensors``
(``qwen3_5_latent.py:161-202``) builds from it (``tests/golden/make_export_golden.py`` made both). Here the same inputs
go through ``belt_b200.latent_format``: every exported tensor must be bit-identical to the reference's, the configs and
the accounting equal, and the reader must rebuild the reference's constants bit for bit.
"""

import hashlib
import json
import os
import sys

import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

import export_case  # noqa: E402

from belt_b200 import latent_format  # noqa: E402

VARIANTS = {"packed": False, "rope_align": True}


def sha(t):
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(HERE, "golden", "export.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def exports(tmp_path_factory):
    tmp = tmp_path_factory.mktemp("latent_export")
    base = export_case.write_base_model(str(tmp / "base"))
    ckpt = export_case.write_checkpoint(str(tmp / "ckpt.pt"))
    out = {}
    for name, rope_align in VARIANTS.items():
        out[name] = str(tmp / name)
        latent_format.export_latent_model(base, ckpt, out[name], rope_align=rope_align)
    return out


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_export_matches_reference_exporter(golden, exports, variant):
    got = export_case.describe_export(exports[variant])
    exp = golden["variants"][variant]["export"]
    assert got["files"] == exp["files"]
    assert got["config"] == exp["config"]
    assert got["kv_lowrank"] == exp["kv_lowrank"]
    assert got["weight_map"] == exp["weight_map"]
    assert got["metadata"] == exp["metadata"]
    assert got["record"] == exp["record"]
    assert sorted(got["tensors"]) == sorted(exp["tensors"])
    for name, t in exp["tensors"].items():
        assert got["tensors"][name] == t, name


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_reader_rebuilds_reference_constants(golden, exports, variant):
    exp = latent_format.read_latent_export(exports[variant])
    assert sorted(exp.layers) == [1, 3]
    cos_sin = exp.cos_sin()
    assert sha(cos_sin) == golden["cos_sin_f32"]
    for i, d in golden["variants"][variant]["derive"].items():
        lat = exp.latent_layer(int(i), cos_sin=cos_sin)
        assert sha(lat.qmap) == d["qmap"], i
        assert sha(lat.u_cat) == d["u_cat"], i
        assert lat.k_segs.tolist() == d["k_segs"] == lat.k_segs_host
        assert sha(lat.rope_gain) == d["rope_gain"]
        assert [list(g) for g in lat.rope.groups] == d["groups"]
        assert sha(lat.rope.blocks) == d["blocks"]
        assert sha(lat.rope.cos_sin) == d["cos_sin"]
        assert sha(lat.rope_up) == d["rope_up"]
        assert sha(lat.v_up) == d["v_up_t"]
        assert lat.n_k == d["n_k"]
        L = exp.layers[int(i)]
        assert tuple(L.tensors["q_gate_proj.weight"].shape) == (24 * 512, export_case.HIDDEN)
        assert tuple(L.tensors["o_proj.weight"].shape) == (export_case.HIDDEN, 24 * 256)


def test_load_latent_layers_and_layer_selection(exports):
    layers = latent_format.load_latent_layers(exports["packed"], layers=[3])
    assert list(layers) == [3]
    lat = layers[3]
    assert lat.v_rank == 1024 and lat.v_offset == 128        # layer 3 keeps V at full rank (not compressed)
    with pytest.raises(KeyError):
        latent_format.read_latent_export(exports["packed"], layers=[0])


def test_reader_takes_the_multimodal_layout(exports, tmp_path):
    """Checkpoints of the multimodal model keep the text layers under model.language_model.layers.{i}."""
    from safetensors import safe_open
    from safetensors.torch import save_file
    src = exports["packed"]
    with open(os.path.join(src, "model.safetensors.index.json")) as f:
        wm = json.load(f)["weight_map"]
    tensors = {}
    for shard in set(wm.values()):
        with safe_open(os.path.join(src, shard), framework="pt") as f:
            for n in f.keys():
                tensors[n.replace("model.layers.", "model.language_model.layers.")] = f.get_tensor(n)
    save_file(tensors, str(tmp_path / "model.safetensors"))
    with open(os.path.join(src, "config.json")) as f:
        cfg = json.load(f)
    with open(tmp_path / "config.json", "w") as f:
        json.dump({"architectures": cfg["architectures"], "text_config": cfg}, f)
    exp = latent_format.read_latent_export(str(tmp_path))
    ref = latent_format.read_latent_export(src)
    for i in (1, 3):
        assert exp.layers[i].prefix == f"model.language_model.layers.{i}.self_attn."
        for k, t in ref.layers[i].tensors.items():
            assert torch.equal(exp.layers[i].tensors[k], t), (i, k)


def test_factor_checkpoint_reader(tmp_path):
    sd = export_case.factor_state_dict()
    f = latent_format.read_factor_checkpoint(sd)
    assert sorted(f) == [1, 3]
    assert f[1]["k"][2] == export_case.K_RANKS[1] and f[1]["v"] is not None
    assert f[3]["v"] is None
    path = tmp_path / "wrapped.pt"
    torch.save({"state_dict": sd}, path)
    assert sorted(latent_format.read_factor_checkpoint(str(path))) == [1, 3]
    bad = dict(sd)
    bad["model.layers.1.self_attn.k_proj.group_ranks"] = torch.tensor([2])
    with pytest.raises(ValueError, match="per-head K"):
        latent_format.read_factor_checkpoint(bad)
    with pytest.raises(ValueError, match="no low-rank factors"):
        latent_format.read_factor_checkpoint({"model.embed_tokens.weight": torch.zeros(2)})


def test_row_layout_rejects_rope_align_with_a_wide_rotary_dim():
    with pytest.raises(ValueError, match="divide 64"):
        latent_format.row_layout([128] * 4, 512, 128, rope_align=True)
