"""A small synthetic base model directory and low-rank factor checkpoint, built from fixed seeds.

Used by ``make_export_golden.py`` (which runs the reference's exporter on them) and by ``tests/test_latent_format.py``
(which runs this package's exporter and reader on the same inputs). The geometry is the compressed layers' (24 query
heads, 4 KV heads, head_dim 256, 64 rotary channels, theta 1e7) with a small hidden size, so that the files stay a
few MB:

* a text model of four layers, full attention at layers 1 and 3, in two safetensors shards (layer 3 alone in the
  second), plus stand-in tensors for the other layers and a non-weight file that the export copies;
* a checkpoint compressing K and V of layer 1 (head ranks 48 / 72 / 64 / 80, r_v 96) and only K of layer 3 (ranks
  16 / 64 / 40 / 8, V stays the base projection).
"""

from __future__ import annotations

import json
import os

import torch

HIDDEN, HEADS, KV_HEADS, HEAD_DIM = 64, 24, 4, 256
LAYERS = 4
CONFIG = {
    "architectures": ["Qwen3_5ForCausalLM"], "model_type": "qwen3_5_text", "hidden_size": HIDDEN,
    "num_attention_heads": HEADS, "num_key_value_heads": KV_HEADS, "head_dim": HEAD_DIM, "num_hidden_layers": LAYERS,
    "layer_types": ["linear_attention", "full_attention", "linear_attention", "full_attention"],
    "rms_norm_eps": 1e-6, "max_position_embeddings": 4096, "torch_dtype": "bfloat16",
    "rope_parameters": {"rope_type": "default", "rope_theta": 1e7, "partial_rotary_factor": 0.25},
}
K_RANKS = {1: [48, 72, 64, 80], 3: [16, 64, 40, 8]}
V_RANK = {1: 96}


def _bf16(g, *shape, std=1.0):
    return (torch.randn(*shape, generator=g) * std).to(torch.bfloat16)


def base_tensors(seed: int = 20) -> dict:
    """{shard name: {tensor name: tensor}} of the base model."""
    g = torch.Generator().manual_seed(seed)
    s1, s2 = {}, {}
    s1["model.embed_tokens.weight"] = _bf16(g, 128, HIDDEN)
    for i in range(LAYERS):
        dst = s2 if i == 3 else s1
        if CONFIG["layer_types"][i] == "linear_attention":
            dst[f"model.layers.{i}.linear_attn.in_proj.weight"] = _bf16(g, 96, HIDDEN, std=0.1)
        else:
            p = f"model.layers.{i}.self_attn."
            dst[p + "q_proj.weight"] = _bf16(g, HEADS * 2 * HEAD_DIM, HIDDEN, std=HIDDEN ** -0.5)
            dst[p + "k_proj.weight"] = _bf16(g, KV_HEADS * HEAD_DIM, HIDDEN, std=HIDDEN ** -0.5)
            dst[p + "v_proj.weight"] = _bf16(g, KV_HEADS * HEAD_DIM, HIDDEN, std=HIDDEN ** -0.5)
            dst[p + "o_proj.weight"] = _bf16(g, HIDDEN, HEADS * HEAD_DIM, std=(HEADS * HEAD_DIM) ** -0.5)
            dst[p + "q_norm.weight"] = _bf16(g, HEAD_DIM, std=0.1)
            dst[p + "k_norm.weight"] = _bf16(g, HEAD_DIM, std=0.1)
        dst[f"model.layers.{i}.input_layernorm.weight"] = _bf16(g, HIDDEN, std=0.1)
    s1["model.norm.weight"] = _bf16(g, HIDDEN, std=0.1)
    return {"model-00001-of-00002.safetensors": s1, "model-00002-of-00002.safetensors": s2}


def write_base_model(path: str, seed: int = 20) -> str:
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    shards = base_tensors(seed)
    weight_map = {}
    for name, tensors in shards.items():
        save_file(tensors, os.path.join(path, name), metadata={"format": "pt"})
        weight_map.update({n: name for n in tensors})
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": 0}, "weight_map": weight_map}, f, indent=2)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(CONFIG, f, indent=2)
    with open(os.path.join(path, "tokenizer_config.json"), "w") as f:
        json.dump({"model_max_length": 4096}, f)
    return path


def factor_state_dict(seed: int = 21) -> dict:
    """The low-rank checkpoint (the reference's lrkv/checkpoint.py layout), fp32 factors."""
    g = torch.Generator().manual_seed(seed)
    sd = {}
    for i, ranks in K_RANKS.items():
        p = f"model.layers.{i}.self_attn."
        total = sum(ranks)
        sd[p + "k_proj.VS.weight"] = torch.randn(total, HIDDEN, generator=g) / HIDDEN ** 0.5
        U = torch.zeros(KV_HEADS * HEAD_DIM, total)
        col = 0
        for h, r in enumerate(ranks):
            U[h * HEAD_DIM:(h + 1) * HEAD_DIM, col:col + r] = torch.randn(HEAD_DIM, r, generator=g) / r ** 0.5
            col += r
        sd[p + "k_proj.U.weight"] = U
        sd[p + "k_proj.head_ranks"] = torch.tensor(ranks, dtype=torch.int32)
    for i, r_v in V_RANK.items():
        p = f"model.layers.{i}.self_attn."
        sd[p + "v_proj.VS.weight"] = torch.randn(r_v, HIDDEN, generator=g) / HIDDEN ** 0.5
        sd[p + "v_proj.U.weight"] = torch.randn(KV_HEADS * HEAD_DIM, r_v, generator=g) / r_v ** 0.5
    return sd


def write_checkpoint(path: str, seed: int = 21) -> str:
    torch.save(factor_state_dict(seed), path)
    return path


def describe_export(out: str) -> dict:
    """What the golden records of an export directory: the config and index, every tensor's shape, dtype and
    sha256, each shard's metadata, the latent_export.json accounting, and the files present. Paths and timings are
    left out (they depend on where and when the export ran)."""
    import hashlib
    from safetensors import safe_open

    def sha(t):
        t = t.contiguous()
        if t.dtype == torch.bfloat16:
            t = t.view(torch.int16)
        return hashlib.sha256(t.numpy().tobytes()).hexdigest()

    with open(os.path.join(out, "config.json")) as f:
        config = json.load(f)
    block = dict(config["kv_lowrank"])
    block.pop("checkpoint")
    config = {k: v for k, v in config.items() if k != "kv_lowrank"}
    with open(os.path.join(out, "model.safetensors.index.json")) as f:
        index = json.load(f)
    with open(os.path.join(out, "latent_export.json")) as f:
        record = json.load(f)
    for k in ("base_model", "checkpoint", "checkpoint_sha256", "seconds"):
        record.pop(k)
    tensors, metadata = {}, {}
    for shard in sorted(set(index["weight_map"].values())):
        with safe_open(os.path.join(out, shard), framework="pt") as f:
            metadata[shard] = f.metadata()
            for n in f.keys():
                t = f.get_tensor(n)
                tensors[n] = {"shape": list(t.shape), "dtype": str(t.dtype), "sha256": sha(t)}
    return {"config": config, "kv_lowrank": block, "weight_map": index["weight_map"], "record": record,
            "tensors": tensors, "metadata": metadata, "files": sorted(os.listdir(out))}
