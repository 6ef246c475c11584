"""Per-layer constants of a compressed layer (``LatentLayer``) derived from the loaded latent-export weights.

``derive_latent_tensors`` restates the reference's load-time derivation
(plugins/vllm_lrkv/vllm_lrkv/models/qwen3_5_latent.py:161-202, k_segs :156-158, rope groups :122) so that every tensor
the decode path reads is the reference's, bit for bit: the absorbed-query map ``qmap``, ``u_cat``, ``k_segs``, the
RoPE gain, the rope blocks (``rope_blocks``), ``rope_up``, the BF16 cos/sin table and U_v transposed. The derivation
runs on the CPU (it is load-time only) and the results are moved to the device.
"""

from __future__ import annotations

from dataclasses import dataclass, field
import math

import torch

from . import latent_ops
from .decode import CHUNK, RopeRebuild, rope_blocks


@dataclass
class LatentLayer:
    """Constants of one compressed layer, attached to its attention layer after weight loading
    (latent_backend.py:66-93)."""

    num_kv_heads: int
    head_dim: int
    rotary_dim: int
    v_rank: int
    v_offset: int
    pe_offset: int
    n_k: int                    # 64-column chunks of the K part the decode kernel reads
    qmap: torch.Tensor          # [G, D, n_k * 64 + G * rot]: query -> block-diagonal decode query
    v_up: torch.Tensor          # [G, r_v, D]: U_v transposed
    u_cat: torch.Tensor         # [lk, G * D] BF16: U_g^T at the group's columns
    k_segs: torch.Tensor        # [G, 4] int32: every group's latent columns as two runs (start, length) x 2
    rope_gain: torch.Tensor     # [rot] fp32: k_norm gain of the rotary channels
    eps: float
    rotary: object = None       # the layer's rotary embedding, if any (its cos/sin cache is ``rope.cos_sin``)
    mrope_section: tuple | None = None
    rope: RopeRebuild = None    # RoPE keys rebuilt in-kernel from the K latent
    rope_up: torch.Tensor = None  # [G, rot, n_k * 64] gain * rotary rows of U_g by column
    k_segs_host: list = field(default_factory=list)   # k_segs as host ints (no device sync on the hot path)
    wk: torch.Tensor = None     # [G, D, n_k * 64]: per group rope_up then qmap's nope rows (the keys of decompress)

    @property
    def col_runs(self) -> list:
        return latent_ops.group_column_runs(self.k_segs_host, self.n_k, self.rotary_dim)

    def block_diag_query(self, q: torch.Tensor) -> torch.Tensor:
        """[T, H, head_dim] normed rotated query -> [T, H, n_k * 64 + G * rot] (latent_backend.py:87-89)."""
        return latent_ops.block_diag_query(q, self.qmap, self.col_runs)

    def up_project(self, a: torch.Tensor, out: torch.Tensor) -> None:
        """[T, H, r_v] latent-space attention output -> out [T, H, head_dim] (latent_backend.py:91-93)."""
        latent_ops.up_project(a, self.v_up, out)

    def decompress_paged(self, cache: torch.Tensor, block_table_row: torch.Tensor, seq_len: int, pos0: int,
                         count: int, k_out=None, v_out=None):
        """Keys and values [count, G, D] of positions [pos0, pos0 + count) of one request, rebuilt on the tensor cores
        from its rows in ``cache`` [blocks, page, W] (``latent_ops.decompress_paged``): ``decompress`` of the gathered
        rows in one kernel."""
        return latent_ops.decompress_paged(cache, block_table_row, seq_len, pos0, count, self.wk, self.k_segs_host,
                                           self.v_up, self.v_offset, self.rope.cos_sin, k_out, v_out)

    def decompress_varlen(self, cache: torch.Tensor, block_table: torch.Tensor, pieces, k_out=None, v_out=None):
        """Keys and values of several requests' position ranges in one launch (``latent_ops.decompress_varlen``):
        ``pieces`` = [(request row of ``block_table``, seq_len, pos0, count), ...], concatenated in that order."""
        return latent_ops.decompress_varlen(cache, block_table, pieces, self.wk, self.k_segs_host, self.v_up,
                                            self.v_offset, self.rope.cos_sin, k_out, v_out)


def k_segs_rows(layout: dict) -> list:
    """[[start, length, start, length]] per group from the layout's ``k_segments`` (qwen3_5_latent.py:156-158)."""
    segs = [[(int(a), int(n)) for a, n in runs] for runs in layout["k_segments"]]
    return [[x for run in runs + [(0, 0)] * (2 - len(runs)) for x in run] for runs in segs]


def derive_latent_tensors(k_up: torch.Tensor, v_up: torch.Tensor, k_norm_weight: torch.Tensor, layout: dict,
                          cos_sin_cache: torch.Tensor, *, rotary_dim: int = 64, eps: float = 1e-6,
                          dtype: torch.dtype = torch.bfloat16, device=None, rotary=None,
                          mrope_section=None) -> LatentLayer:
    """``LatentLayer`` of one compressed layer from its export tensors (qwen3_5_latent.py:161-202).

    k_up [G, D, r_max], v_up [G * D, r_v] (BF16, as loaded), k_norm_weight [D] (zero-centred RMSNorm weight: the
    gain is 1 + weight), ``layout`` (``latent_format.row_layout``: the kv_lowrank entry of the layer), cos_sin_cache [max_pos, rot] (the rotary
    embedding's table, any float dtype; stored BF16)."""
    device = torch.device(device) if device is not None else k_up.device
    k_up = k_up.detach().to("cpu")
    v_up = v_up.detach().to("cpu")
    gain = 1.0 + k_norm_weight.detach().to("cpu").float()
    U = k_up.float()
    rot = rotary_dim
    G, D, _ = k_up.shape
    ranks = [int(r) for r in layout["k_head_ranks"]]
    segments = [[(int(a), int(n)) for a, n in runs] for runs in layout["k_segments"]]
    lk = sum(ranks)
    v_offset, r_v = int(layout["v_offset"]), int(layout["v_rank"])
    n_k = math.ceil(v_offset / CHUNK)
    qmap = torch.zeros(G, D, n_k * CHUNK + G * rot, dtype=torch.float32)
    u_cat = torch.zeros(lk, G * D, dtype=torch.float32)
    for g, (runs, r) in enumerate(zip(segments, ranks)):
        cols = torch.cat([torch.arange(a, a + n) for a, n in runs])
        qmap[g, :rot, n_k * CHUNK + g * rot:n_k * CHUNK + (g + 1) * rot] = torch.eye(rot)
        qmap[g, rot:, cols] = gain[rot:, None] * U[g, rot:, :r]
        u_cat[cols, g * D:(g + 1) * D] = U[g, :, :r].T
    groups = tuple((runs[0][0], int(rr)) for runs, rr in zip(segments, layout["rope_ranks"]))
    if any(runs[0][1] < rr for runs, (_, rr) in zip(segments, groups)):
        raise ValueError("every group's RoPE coordinates must lead its first column run")
    u_rot = [gain[:rot, None] * U[g, :rot, :rr] for g, (off, rr) in enumerate(groups)]
    blocks = rope_blocks(u_rot, groups).to(dtype)
    rope_up = torch.zeros(G, rot, n_k * CHUNK, dtype=dtype)
    for g, ((off, rr), u) in enumerate(zip(groups, u_rot)):
        rope_up[g, :, off:off + rr] = u.to(dtype)
    rows = k_segs_rows(layout)
    wk = torch.cat([rope_up, qmap[:, rot:, :n_k * CHUNK].to(dtype)], dim=1).contiguous()
    v_up_t = v_up.view(G, D, r_v).transpose(1, 2).contiguous()
    cos_sin = cos_sin_cache.detach().to("cpu").to(torch.bfloat16).contiguous()
    to = dict(device=device)
    return LatentLayer(num_kv_heads=G, head_dim=D, rotary_dim=rot, v_rank=r_v, v_offset=v_offset,
                       pe_offset=int(layout["pe_offset"]), n_k=n_k, qmap=qmap.to(dtype).to(**to),
                       v_up=v_up_t.to(dtype).to(**to), u_cat=u_cat.to(torch.bfloat16).to(**to),
                       k_segs=torch.tensor(rows, dtype=torch.int32, **to), rope_gain=gain[:rot].clone().to(**to),
                       eps=float(eps), rotary=rotary, mrope_section=mrope_section,
                       rope=RopeRebuild(groups=groups, blocks=blocks.to(**to), cos_sin=cos_sin.to(**to)),
                       rope_up=rope_up.to(**to), k_segs_host=rows, wk=wk.to(**to))
