"""The latent export: the on-disk model directory this backend serves, its reader, and a writer.

A latent export is a Hugging Face model directory in which every compressed full-attention layer keeps one cache row
per token instead of keys and values (the reference's format, ``lrkv/runtime/export_latent.py:1-34``):

* ``config.json`` (or its ``text_config``) carries a ``kv_lowrank`` block: ``format`` "latent", ``rotary_dim``,
  ``alignment_elements``, ``rope_align`` and per compressed layer its row layout (``layers``: K ranks per KV group,
  ``v_rank``, ``lk``, ``v_offset``, ``pe_offset`` = ``row_width``, ``rope_ranks``, ``k_segments``, ``rope_offsets``);
* per compressed layer, under its attention prefix (``model.layers.{i}.self_attn.`` or
  ``model.language_model.layers.{i}.self_attn.``): ``kv_latent_proj.weight`` [row_width, hidden] (the rows of the
  cache row: every group's latent projection at its columns, zero rows at the alignment gaps, the joint V
  projection at ``v_offset``), ``k_up.weight`` [G, head_dim, r_max] (U_g), ``v_up.weight`` [G * head_dim, r_v] (U_v),
  the query + gate projection renamed ``q_gate_proj.weight``, and the stock ``o_proj`` / ``q_norm`` / ``k_norm``;
* safetensors shards listed by ``model.safetensors.index.json`` (or one ``model.safetensors``).

The factors come from a low-rank checkpoint (the reference's ``lrkv/checkpoint.py`` layout: a ``torch.save``'d
state dict holding, per compressed layer, ``k_proj.VS.weight`` [sum r_g, hidden], ``k_proj.U.weight``
[G * head_dim, sum r_g] (block diagonal), ``k_proj.head_ranks`` [G] and ``v_proj.VS.weight`` / ``v_proj.U.weight``).
Before a group's factors are written its latent basis is rotated (an orthogonal Q from a float64 QR of the rotary
rows of U_g) so that the rotary rows of U_g Q are zero past the first min(rot, r_g) coordinates: the RoPE keys are
then rebuilt from those coordinates only. The writer reproduces the reference exporter's tensors bit for bit; the
golden test of this module compares them with the reference's own output.

``read_latent_export`` / ``load_latent_layers`` read a directory (the reference's or this module's) into the
backend's per-layer constants (``LatentLayer``) and the attention block's weights.
"""

from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass, field
import hashlib
import itertools
import json
import os
import shutil
import time

import torch

FORMAT = "latent"
ALIGN = 8                                   # BF16 elements in 16 bytes: every part of a row starts 16-byte aligned
Q_GATE = "q_gate_proj"
ARCH_VLM = "Qwen3_5LowRankLatentForConditionalGeneration"
ARCH_TEXT = "Qwen3_5LowRankLatentForCausalLM"
_WEIGHT_SUFFIXES = (".safetensors", ".bin", ".pt", ".pth", ".msgpack", ".h5", ".gguf")
_ATTN_PREFIXES = ("model.language_model.layers.{}.self_attn.", "model.layers.{}.self_attn.")


# --------------------------------------------------------------------------------------------------------- row layout
def _round_up(n: int, m: int = ALIGN) -> int:
    return (n + m - 1) // m * m


def group_runs(k_ranks, rotary_dim: int, rope_align: bool = False) -> list:
    """Cache columns of every KV group's latent coordinates, as [start, length] runs in the group's latent order.

    Packed: the groups one after another. ``rope_align``: first the leading min(rot, r_g) coordinates of every
    group (the only ones its RoPE keys read) -- groups with the most of them first, ties in group order -- then the
    remaining coordinates of every group in group order."""
    ranks = [int(r) for r in k_ranks]
    if not rope_align:
        starts = itertools.accumulate([0] + ranks[:-1])
        return [[[s, r]] for s, r in zip(starts, ranks)]
    lead = [min(rotary_dim, r) for r in ranks]
    runs = [[] for _ in ranks]
    col = 0
    for g in sorted(range(len(ranks)), key=lambda g: (-lead[g], g)):
        runs[g].append([col, lead[g]])
        col += lead[g]
    for g, r in enumerate(ranks):
        if r > lead[g]:
            runs[g].append([col, r - lead[g]])
            col += r - lead[g]
    return runs


def row_layout(k_ranks, v_rank: int, rotary_dim: int, rope_align: bool = False) -> dict:
    """The row layout of one compressed layer, with the keys of the ``kv_lowrank`` layer entries: the K part from
    column 0, the V part from the next 16-byte boundary, the row padded to a 16-byte multiple."""
    if rope_align and 64 % rotary_dim:
        raise ValueError(f"a rope-aligned row keeps each group's {rotary_dim} RoPE coordinates inside one 64-column "
                         "chunk, so the rotary dim must divide 64")
    ranks = [int(r) for r in k_ranks]
    runs = group_runs(ranks, rotary_dim, rope_align)
    lk = sum(ranks)
    v_offset = _round_up(lk)
    width = _round_up(v_offset + int(v_rank))
    return {"k_head_ranks": ranks, "v_rank": int(v_rank), "lk": lk, "v_offset": v_offset, "pe_offset": width,
            "row_width": width, "rope_ranks": [min(rotary_dim, r) for r in ranks], "k_segments": runs,
            "rope_offsets": [g[0][0] for g in runs]}


# ------------------------------------------------------------------------------------------------- the layer's tensors
def _rotary_basis(U: torch.Tensor, rotary_dim: int) -> torch.Tensor | None:
    """The float64 orthogonal Q [r, r] (complete QR of the transposed rotary rows of U [head_dim, r]) that zeroes the
    rotary rows of U Q past column rot; None when r <= rot (nothing to rotate)."""
    if U.shape[1] <= rotary_dim:
        return None
    basis, _ = torch.linalg.qr(U[:rotary_dim].double().T, mode="complete")
    return basis


def latent_tensors(k_factors, v_factors, head_dim: int, rotary_dim: int, dtype: torch.dtype = torch.bfloat16,
                   rope_align: bool = False):
    """(kv_latent_proj [row_width, hidden], k_up [G, head_dim, r_max], v_up [G * head_dim, r_v], layout) of one
    compressed layer from per-group K factors ``k_factors`` [(VS_g [r_g, hidden], U_g [head_dim, r_g])] and the joint
    V factors ``v_factors`` (VS_v [r_v, hidden], U_v [G * head_dim, r_v])."""
    G = len(k_factors)
    VS_v, U_v = v_factors[0].float(), v_factors[1].float()
    if U_v.shape[0] != G * head_dim:
        raise ValueError(f"U_v has {U_v.shape[0]} rows; {G} KV groups of head dim {head_dim} need {G * head_dim}")
    ranks = [int(VS.shape[0]) for VS, _ in k_factors]
    layout = row_layout(ranks, int(VS_v.shape[0]), rotary_dim, rope_align)
    hidden = int(VS_v.shape[1])
    proj = torch.zeros(layout["row_width"], hidden)
    k_up = torch.zeros(G, head_dim, max(ranks))
    for g, (VS, U) in enumerate(k_factors):
        VS, U, r = VS.float(), U.float(), ranks[g]
        basis = _rotary_basis(U, rotary_dim)
        if basis is None:
            basis = torch.eye(r, dtype=torch.float64)
        VS = (basis.T @ VS.double()).float()
        U = (U.double() @ basis).float()
        U[:rotary_dim, min(rotary_dim, r):] = 0.0        # exactly zero (the QR leaves rounding residue)
        cols = torch.cat([torch.arange(s, s + n) for s, n in layout["k_segments"][g]])
        proj[cols] = VS
        k_up[g, :, :r] = U
    vo = layout["v_offset"]
    proj[vo:vo + layout["v_rank"]] = VS_v
    return proj.to(dtype), k_up.to(dtype), U_v.to(dtype), layout


# ----------------------------------------------------------------------------------------------- factor checkpoints
def _attn_key(i: int, name: str) -> str:
    return f"model.layers.{i}.self_attn.{name}"


def read_factor_checkpoint(source) -> dict:
    """{layer: {"k": (VS, U, head_ranks) or None, "v": (VS, U) or None}} of a low-rank checkpoint (a path to a
    ``torch.save``'d state dict, optionally under "state_dict", or the dict itself)."""
    sd = source
    if isinstance(source, (str, os.PathLike)):
        sd = torch.load(source, map_location="cpu", weights_only=False)
        if isinstance(sd, dict) and isinstance(sd.get("state_dict"), dict):
            sd = sd["state_dict"]
    layers = defaultdict(lambda: {"k": None, "v": None})
    for key in sd:
        parts = key.split(".")
        if len(parts) < 6 or parts[:2] != ["model", "layers"] or parts[3] != "self_attn" or \
                ".".join(parts[5:]) != "VS.weight" or parts[4] not in ("k_proj", "v_proj"):
            continue
        i = int(parts[2])
        proj = parts[4]
        if proj == "k_proj":
            if _attn_key(i, "k_proj.group_ranks") in sd:
                raise ValueError(f"layer {i}: a latent export needs per-head K factors, not grouped ones")
            layers[i]["k"] = (sd[key], sd[_attn_key(i, "k_proj.U.weight")],
                              [int(r) for r in sd[_attn_key(i, "k_proj.head_ranks")].tolist()])
        else:
            if _attn_key(i, "v_proj.head_ranks") in sd:
                raise ValueError(f"layer {i}: a latent export needs one joint V latent, not per-head V factors")
            layers[i]["v"] = (sd[key], sd[_attn_key(i, "v_proj.U.weight")])
    if not layers:
        raise ValueError("the checkpoint holds no low-rank factors (*.k_proj.VS.weight / *.v_proj.VS.weight)")
    return dict(sorted(layers.items()))


def _group_factors(entry, base_k: torch.Tensor | None, num_kv_heads: int, head_dim: int) -> list:
    """Per-group (VS_g, U_g): the checkpoint's block-diagonal K factors cut per group, or the base projection
    ``base_k`` [G * head_dim, hidden] as full-rank factors (VS_g = its rows, U_g = I) when K is not compressed."""
    if entry is None:
        rows = base_k.float().view(num_kv_heads, head_dim, -1)
        eye = torch.eye(head_dim)
        return [(rows[g], eye) for g in range(num_kv_heads)]
    VS, U, ranks = entry
    VS, U = VS.float(), U.float()
    out, start = [], 0
    for g, r in enumerate(ranks):
        out.append((VS[start:start + r], U[g * head_dim:(g + 1) * head_dim, start:start + r]))
        start += r
    return out


def _joint_v(entry, base_v: torch.Tensor | None):
    if entry is None:
        W = base_v.float()
        return W, torch.eye(W.shape[0])
    return entry[0].float(), entry[1].float()


# ------------------------------------------------------------------------------------------------------ config access
def text_config(config: dict) -> dict:
    return config.get("text_config", config)


def head_dim_of(tc: dict) -> int:
    return int(tc.get("head_dim") or tc["hidden_size"] // tc["num_attention_heads"])


def rope_params(tc: dict) -> dict:
    return tc.get("rope_parameters") or tc.get("rope_scaling") or {}


def rotary_dim_of(tc: dict) -> int:
    factor = rope_params(tc).get("partial_rotary_factor", tc.get("partial_rotary_factor", 1.0)) or 1.0
    return int(head_dim_of(tc) * float(factor))


def rope_theta_of(tc: dict) -> float:
    return float(rope_params(tc).get("rope_theta", tc.get("rope_theta", 10000.0)))


def cos_sin_table(max_pos: int, rotary_dim: int, theta: float) -> torch.Tensor:
    """The rotary embedding's NeoX cos/sin cache [max_pos, rot] in fp32 (cos half, then sin half), as vLLM's
    ``RotaryEmbedding`` builds it for plain positions."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, rotary_dim, 2, dtype=torch.float) / rotary_dim))
    t = torch.arange(max_pos, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


# ----------------------------------------------------------------------------------------------------- the directory
def _weight_map(model_dir: str) -> dict:
    index = os.path.join(model_dir, "model.safetensors.index.json")
    if os.path.exists(index):
        with open(index) as f:
            return dict(json.load(f)["weight_map"])
    single = os.path.join(model_dir, "model.safetensors")
    if os.path.exists(single):
        from safetensors import safe_open
        with safe_open(single, framework="pt") as f:
            return {n: "model.safetensors" for n in f.keys()}
    raise FileNotFoundError(f"{model_dir}: no model.safetensors.index.json or model.safetensors")


def _attn_prefix(weight_map: dict, i: int, probe: str) -> str:
    for fmt in _ATTN_PREFIXES:
        if fmt.format(i) + probe in weight_map:
            return fmt.format(i)
    raise KeyError(f"layer {i}: no {probe} under model.layers.{i} or model.language_model.layers.{i}")


def _sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 24), b""):
            h.update(block)
    return h.hexdigest()


def export_latent_model(model_dir: str, checkpoint: str, output: str, dtype: torch.dtype = torch.bfloat16,
                        rope_align: bool = False) -> dict:
    """Write ``output``: the base model ``model_dir`` with every layer the low-rank ``checkpoint`` compresses turned
    into a latent layer (k_proj / v_proj dropped, q_proj renamed q_gate_proj, kv_latent_proj / k_up / v_up added),
    the other shards and files copied, ``config.json`` given the ``kv_lowrank`` block and the plugin architecture,
    and ``latent_export.json`` recording the cache accounting. Returns that record."""
    from safetensors import safe_open
    from safetensors.torch import save_file

    t0 = time.time()
    with open(os.path.join(model_dir, "config.json")) as f:
        config = json.load(f)
    tc = text_config(config)
    if "quantization_config" in config or "quantization_config" in tc:
        raise ValueError(f"{model_dir}: a quantized base model cannot be exported (BF16 / FP16 weights needed)")
    head_dim, G, rot = head_dim_of(tc), int(tc["num_key_value_heads"]), rotary_dim_of(tc)
    weight_map = _weight_map(model_dir)
    factors = read_factor_checkpoint(checkpoint)
    shard_layers = defaultdict(list)
    for i in factors:
        prefix = _attn_prefix(weight_map, i, "q_proj.weight")
        shards = {s for n, s in weight_map.items() if n.startswith(prefix)}
        if len(shards) != 1:
            raise ValueError(f"layer {i}: its attention tensors lie in {len(shards)} shards; one is supported")
        shard_layers[shards.pop()].append((i, prefix))

    os.makedirs(output, exist_ok=True)
    for name in os.listdir(model_dir):                      # tokenizer, generation config, ... (not weights)
        src = os.path.join(model_dir, name)
        if os.path.isfile(src) and name != "config.json" and not name.endswith(_WEIGHT_SUFFIXES) \
                and not name.startswith("pytorch_model"):
            shutil.copy2(src, os.path.join(output, name))

    new_map, layer_entries = dict(weight_map), {}
    for shard in sorted(set(weight_map.values())):
        if shard not in shard_layers:
            shutil.copy2(os.path.join(model_dir, shard), os.path.join(output, shard))
            continue
        with safe_open(os.path.join(model_dir, shard), framework="pt") as f:
            metadata = f.metadata()
            tensors = {n: f.get_tensor(n) for n in f.keys()}
        for i, prefix in shard_layers[shard]:
            entry = factors[i]
            k_factors = _group_factors(entry["k"], tensors.get(prefix + "k_proj.weight"), G, head_dim)
            v_factors = _joint_v(entry["v"], tensors.get(prefix + "v_proj.weight"))
            proj, k_up, v_up, layout = latent_tensors(k_factors, v_factors, head_dim, rot, dtype, rope_align)
            for n in list(tensors):
                if n.startswith(prefix + "k_proj.") or n.startswith(prefix + "v_proj."):
                    del tensors[n], new_map[n]
                elif n.startswith(prefix + "q_proj."):
                    renamed = prefix + Q_GATE + n[len(prefix + "q_proj"):]
                    tensors[renamed] = tensors.pop(n)
                    new_map[renamed] = new_map.pop(n)
            for suffix, t in (("kv_latent_proj.weight", proj), ("k_up.weight", k_up), ("v_up.weight", v_up)):
                tensors[prefix + suffix] = t.contiguous()
                new_map[prefix + suffix] = shard
            layer_entries[str(i)] = dict(layout, k_compressed=entry["k"] is not None,
                                         v_compressed=entry["v"] is not None)
        save_file({n: t.contiguous() for n, t in tensors.items()}, os.path.join(output, shard), metadata=metadata)

    index_path = os.path.join(model_dir, "model.safetensors.index.json")
    index = {"metadata": {}}
    if os.path.exists(index_path):
        with open(index_path) as f:
            index = json.load(f)
    index["weight_map"] = new_map
    with open(os.path.join(output, "model.safetensors.index.json"), "w") as f:
        json.dump(index, f, indent=2)

    dname = str(dtype).replace("torch.", "")
    tc["kv_lowrank"] = {"format": FORMAT, "rotary_dim": rot, "nope_dim": head_dim - rot, "rope_slice": "rebuilt",
                        "norm_folded": True, "alignment_elements": ALIGN, "latent_dtype": dname, "cache_dtype": dname,
                        "rope_align": rope_align, "q_gate_proj": Q_GATE, "layers": layer_entries,
                        "base_architectures": config.get("architectures"),
                        "checkpoint": os.path.abspath(checkpoint)}
    config["architectures"] = [ARCH_VLM if "text_config" in config else ARCH_TEXT]
    with open(os.path.join(output, "config.json"), "w") as f:
        json.dump(config, f, indent=2)

    full = 2 * G * head_dim
    widths = {i: e["row_width"] for i, e in layer_entries.items()}
    packed = {i: e["lk"] + e["v_rank"] for i, e in layer_entries.items()}
    n = len(widths)
    record = {"base_model": os.path.abspath(model_dir), "checkpoint": os.path.abspath(checkpoint),
              "checkpoint_sha256": _sha256(checkpoint), "format": FORMAT, "dtype": str(dtype), "cache_dtype": dname,
              "compressed_layers": sorted(int(i) for i in layer_entries), "layers": layer_entries,
              "cache_elements_per_token": {"compressed_layers": widths, "total": sum(widths.values()),
                                           "packed_total": sum(packed.values()), "full_kv_total": full * n,
                                           "ratio": sum(widths.values()) / (full * n)},
              "cache_bytes_ratio": sum(widths.values()) * dtype.itemsize / (2 * full * n),
              "seconds": round(time.time() - t0, 1)}
    with open(os.path.join(output, "latent_export.json"), "w") as f:
        json.dump(record, f, indent=2)
    return record


# -------------------------------------------------------------------------------------------------------- the reader
@dataclass
class ExportedLayer:
    """One compressed layer of a latent export: its index, attention prefix, row layout and tensors (by suffix:
    ``kv_latent_proj.weight``, ``k_up.weight``, ``v_up.weight``, ``k_norm.weight`` and, when present,
    ``q_gate_proj.weight``, ``o_proj.weight``, ``q_norm.weight``)."""

    index: int
    prefix: str
    layout: dict
    tensors: dict = field(default_factory=dict)


@dataclass
class LatentExport:
    """A latent export read from disk: the text config, its ``kv_lowrank`` block and the compressed layers."""

    path: str
    config: dict
    block: dict
    layers: dict

    @property
    def head_dim(self) -> int:
        return head_dim_of(self.config)

    @property
    def rotary_dim(self) -> int:
        return int(self.block["rotary_dim"])

    @property
    def eps(self) -> float:
        return float(self.config.get("rms_norm_eps", 1e-6))

    def cos_sin(self, max_pos: int | None = None) -> torch.Tensor:
        """The model's rotary cos/sin table (fp32) for positions [0, max_pos) (default: max_position_embeddings)."""
        n = int(max_pos if max_pos is not None else self.config.get("max_position_embeddings", 32768))
        return cos_sin_table(n, self.rotary_dim, rope_theta_of(self.config))

    def latent_layer(self, i: int, device=None, max_pos: int | None = None, cos_sin: torch.Tensor | None = None):
        """The backend's ``LatentLayer`` of compressed layer ``i`` (``derive_latent_tensors`` of its tensors)."""
        from .layer import derive_latent_tensors
        L = self.layers[i]
        t = L.tensors
        if cos_sin is None:
            cos_sin = self.cos_sin(max_pos)
        return derive_latent_tensors(t["k_up.weight"], t["v_up.weight"], t["k_norm.weight"], L.layout, cos_sin,
                                     rotary_dim=self.rotary_dim, eps=self.eps, device=device)


_LAYER_SUFFIXES = ("kv_latent_proj.weight", "k_up.weight", "v_up.weight", "k_norm.weight")
_BLOCK_SUFFIXES = ("q_gate_proj.weight", "o_proj.weight", "q_norm.weight")


def read_latent_export(model_dir: str, layers=None, block_weights: bool = True) -> LatentExport:
    """Read a latent export's config and the tensors of its compressed layers (all, or the indices in ``layers``);
    ``block_weights`` also reads the attention block's q_gate_proj / o_proj / q_norm. Tensors stay in the stored
    dtype on the CPU."""
    from safetensors import safe_open

    with open(os.path.join(model_dir, "config.json")) as f:
        config = json.load(f)
    tc = text_config(config)
    block = tc.get("kv_lowrank")
    if not isinstance(block, dict) or block.get("format") != FORMAT:
        raise ValueError(f"{model_dir}: config.json has no kv_lowrank block of format {FORMAT!r}")
    weight_map = _weight_map(model_dir)
    wanted = sorted(int(i) for i in block["layers"]) if layers is None else sorted(int(i) for i in layers)
    out = {}
    by_shard = defaultdict(list)
    for i in wanted:
        layout = block["layers"].get(str(i))
        if layout is None:
            raise KeyError(f"{model_dir}: layer {i} is not a compressed layer")
        prefix = _attn_prefix(weight_map, i, "kv_latent_proj.weight")
        out[i] = ExportedLayer(i, prefix, layout)
        suffixes = _LAYER_SUFFIXES + (_BLOCK_SUFFIXES if block_weights else ())
        for s in suffixes:
            name = prefix + s
            if name in weight_map:
                by_shard[weight_map[name]].append((i, s, name))
            elif s in _LAYER_SUFFIXES:
                raise KeyError(f"{model_dir}: {name} is missing")
    for shard, items in by_shard.items():
        with safe_open(os.path.join(model_dir, shard), framework="pt") as f:
            for i, s, name in items:
                out[i].tensors[s] = f.get_tensor(name)
    for i, L in out.items():
        t, lay = L.tensors, L.layout
        G, D = t["k_up.weight"].shape[0], t["k_up.weight"].shape[1]
        if t["kv_latent_proj.weight"].shape[0] != lay["row_width"] or t["v_up.weight"].shape != (G * D, lay["v_rank"]):
            raise ValueError(f"{model_dir}: layer {i}'s tensors do not match its kv_lowrank layout")
    return LatentExport(model_dir, tc, block, out)


def load_latent_layers(model_dir: str, device=None, layers=None, max_pos: int | None = None) -> dict:
    """{layer index: ``LatentLayer``} of a latent export, ready for ``LatentAttentionImpl`` (``layer.latent``)."""
    exp = read_latent_export(model_dir, layers, block_weights=False)
    cos_sin = exp.cos_sin(max_pos)
    return {i: exp.latent_layer(i, device, cos_sin=cos_sin) for i in exp.layers}
