"""The latent export format this backend reads: cache row layout, per-group column runs, the RoPE change of basis and
the per-layer tensors of a ``latent`` model directory.

Format of one compressed layer (the reference's ``lrkv/runtime/export_latent.py``):

* cache row ``[c~_1 | ... | c~_G | 0 | c_v | 0]`` of ``row_width = pe_offset`` BF16 elements; the K part starts at
  column 0, the V part at ``v_offset = align8(lk)``, and the row ends at ``align8(v_offset + r_v)`` (``row_layout``,
  ``export_latent.py:143-166``); every part starts on a 16-byte boundary;
* ``k_segments``: every group's latent columns as [start, length] runs, packed or ``rope_align``-ed
  (``export_latent.py:116-133``);
* ``rope_basis``: per group an orthogonal Q with (U_g Q)[:rot, min(rot, r_g):] = 0, so the rotary rows of U_g read only
  the first ``rr_g = min(rot, r_g)`` latent coordinates (``export_latent.py:169-176``);
* tensors ``kv_latent_proj.weight [pe_offset, hidden]``, ``k_up.weight [G, head_dim, r_max]``,
  ``v_up.weight [G * head_dim, r_v]`` and the ``config.json`` ``kv_lowrank`` block (``export_latent.py:179-205,
  278-287``).

The layout and the tensors are the same as the reference's so that one exported directory serves both.
"""

from __future__ import annotations

import torch

ALIGN = 8            # BF16 elements per 16 bytes: TMA box starts and row strides
FORMAT = "latent"


def _align(x: int, align: int = ALIGN) -> int:
    return -(-x // align) * align


def k_segments(k_head_ranks, rotary_dim: int, rope_align: bool = False) -> list:
    """Cache columns of every KV group's latent coordinates as [start, length] runs in latent order.

    Packed: group after group. ``rope_align``: the leading min(rot, r_g) coordinates of every group first (groups with
    a full rot of them in group order, then the others largest first), then the rest of every group in group order
    (``export_latent.py:116-133``)."""
    if not rope_align:
        offsets = [sum(k_head_ranks[:g]) for g in range(len(k_head_ranks))]
        return [[[o, int(r)]] for o, r in zip(offsets, k_head_ranks)]
    rr = [min(rotary_dim, int(r)) for r in k_head_ranks]
    segments, col = [[] for _ in rr], 0
    for g in sorted(range(len(rr)), key=lambda g: -rr[g]):
        segments[g].append([col, rr[g]])
        col += rr[g]
    for g, r in enumerate(k_head_ranks):
        if r > rr[g]:
            segments[g].append([col, int(r) - rr[g]])
            col += int(r) - rr[g]
    return segments


def row_layout(k_head_ranks, v_rank: int, num_kv_heads: int, rotary_dim: int, align: int = ALIGN,
               rope_align: bool = False) -> dict:
    """Offsets of one compressed layer's cache row (``export_latent.py:143-166``)."""
    if rope_align and 64 % rotary_dim:
        raise ValueError(f"rope_align keeps every group's RoPE coordinates in one 64-column chunk: rot {rotary_dim} "
                         "must divide 64")
    if len(k_head_ranks) != num_kv_heads:
        raise ValueError(f"{len(k_head_ranks)} K ranks for {num_kv_heads} KV heads")
    lk = sum(int(r) for r in k_head_ranks)
    v_offset = _align(lk, align)
    pe_offset = _align(v_offset + v_rank, align)
    segments = k_segments(k_head_ranks, rotary_dim, rope_align)
    return {
        "k_head_ranks": [int(r) for r in k_head_ranks],
        "v_rank": int(v_rank),
        "lk": lk,
        "v_offset": v_offset,
        "pe_offset": pe_offset,
        "row_width": pe_offset,
        "rope_ranks": [min(rotary_dim, int(r)) for r in k_head_ranks],
        "k_segments": segments,
        "rope_offsets": [runs[0][0] for runs in segments],
    }


def rope_basis(U: torch.Tensor, rotary_dim: int) -> torch.Tensor:
    """Orthogonal Q [r, r] (float64) with (U Q)[:rotary_dim, min(rotary_dim, r):] = 0 for U [head_dim, r]
    (QR of the rotary rows, ``export_latent.py:169-176``)."""
    r = U.shape[1]
    if r <= rotary_dim:
        return torch.eye(r, dtype=torch.float64)
    Q, _ = torch.linalg.qr(U[:rotary_dim].double().T, mode="complete")
    return Q


def build_latent_layer(k_blocks, v_factors, num_kv_heads: int, head_dim: int, rotary_dim: int,
                       dtype: torch.dtype = torch.bfloat16, align: int = ALIGN, rope_align: bool = False):
    """(kv_latent_proj [pe_offset, hidden], k_up [G, head_dim, r_max], v_up [G * head_dim, r_v], layout) from per-group
    K factors (VS_g [r_g, hidden], U_g [head_dim, r_g]) and joint V factors (VS_v [r_v, hidden], U_v [G * head_dim,
    r_v]), after each group's change of basis (``export_latent.py:179-205``)."""
    ranks = [int(VS.shape[0]) for VS, _ in k_blocks]
    VS_v, U_v = (t.float() for t in v_factors)
    if len(ranks) != num_kv_heads or U_v.shape[0] != num_kv_heads * head_dim:
        raise ValueError(f"{len(ranks)} K blocks / U_v {tuple(U_v.shape)} for {num_kv_heads} KV heads")
    layout = row_layout(ranks, int(VS_v.shape[0]), num_kv_heads, rotary_dim, align, rope_align)
    hidden = int(VS_v.shape[1])
    proj = torch.zeros(layout["pe_offset"], hidden, dtype=torch.float32)
    k_up = torch.zeros(num_kv_heads, head_dim, max(ranks), dtype=torch.float32)
    for g, ((VS, U), r) in enumerate(zip(k_blocks, ranks)):
        Q = rope_basis(U, rotary_dim)
        VS, U = (Q.T @ VS.double()).float(), (U.double() @ Q).float()
        U[:rotary_dim, min(rotary_dim, r):] = 0.0              # exactly zero, not rounding residue
        i = 0
        for start, n in layout["k_segments"][g]:
            proj[start:start + n] = VS[i:i + n]
            i += n
        k_up[g, :, :r] = U
    proj[layout["v_offset"]:layout["v_offset"] + layout["v_rank"]] = VS_v
    return proj.to(dtype), k_up.to(dtype), U_v.to(dtype), layout


def kv_lowrank_block(layers: dict, rotary_dim: int, head_dim: int, dtype: torch.dtype = torch.bfloat16,
                     rope_align: bool = False) -> dict:
    """The ``config.json`` ``kv_lowrank`` block of a latent export (``export_latent.py:278-284``); ``layers`` maps a
    layer index (str) to its ``row_layout``."""
    name = str(dtype).replace("torch.", "")
    return {"format": FORMAT, "rotary_dim": rotary_dim, "nope_dim": head_dim - rotary_dim, "rope_slice": "rebuilt",
            "norm_folded": True, "alignment_elements": ALIGN, "latent_dtype": name, "cache_dtype": name,
            "rope_align": rope_align, "q_gate_proj": "q_gate_proj", "layers": layers}


def latent_layers(config) -> dict:
    """{layer index: layout} of a config carrying a ``kv_lowrank`` block of format ``latent``
    (``qwen3_5_latent.py:48-52``)."""
    block = config.get("kv_lowrank") if isinstance(config, dict) else getattr(config, "kv_lowrank", None)
    if not isinstance(block, dict) or block.get("format") != FORMAT:
        return {}
    return {int(i): info for i, info in block["layers"].items()}
