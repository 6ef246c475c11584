"""Split-KV latent decode on B200: the public surface of the reference's ``vllm_lrkv.cute_decode``
(plugins/vllm_lrkv/vllm_lrkv/cute_decode.py) over this package's sm_100a kernels.

Same names, arguments and buffers as the reference: ``DecodeSchedule`` / ``make_schedule`` / ``schedule`` (a device
work split computed once per step and shared by all layers, graph-safe), ``latent_decode`` (``latent_decode_cute``),
``merge_segments``, ``RopeRebuild`` / ``rope_blocks`` and the reference construction ``block_diag_query``. The tile
of the split is 128 tokens (the reference's CuTe kernel used 64), and page sizes of 16, 32, 64 or any multiple of 128
are accepted (the reference required multiples of 64).
"""

from __future__ import annotations

from dataclasses import dataclass
import math
import os

import torch

from . import _lib
from . import ops as _ops  # noqa: F401  (registers torch.ops.lrkv_b200)

H, G, ROT = 24, 4, 64
TILE_T = 128          # tokens per split-KV tile (BELT_DECODE_TILE)
CHUNK = 64            # features per TMA box
MAX_LV = 640          # r_v bound of the decode kernel (5 TMEM accumulator blocks)
MAX_LK_PAD = 768      # v_offset bound (12 K chunks + 4 RoPE chunks of query in shared memory)

_ERR_WORDS: dict = {}


def error_word(device) -> torch.Tensor:
    """The device's int32 error word: decode and schedule kernels record a nonzero code there if a bounded wait in
    the kernel gave up (a bug, never a data condition)."""
    device = torch.device(device)
    w = _ERR_WORDS.get(device)
    if w is None:
        w = _ERR_WORDS[device] = torch.zeros(1, dtype=torch.int32, device=device)
    return w


def check_device_errors(device=None) -> None:
    """Raise if a kernel on ``device`` recorded an error (synchronises the device; for tests and debugging)."""
    devs = [torch.device(device)] if device is not None else list(_ERR_WORDS)
    for d in devs:
        w = _ERR_WORDS.get(d)
        if w is not None:
            code = int(w.item())
            if code:
                w.zero_()
                raise _lib.BeltError(f"device error 0x{code:x} recorded by a belt kernel on {d}")


def _stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


@dataclass
class DecodeSchedule:
    """The split-KV work of one decode step, in device memory (interchangeable with the reference's buffers,
    cute_decode.py:545-559). It is computed once per step and read by the decode and merge of every layer.

    ``work`` has one row per segment -- a run of consecutive tiles of one request -- holding (request, first tile,
    end tile, unused); rows are sorted by request, then tile. ``seg_base[b]`` is the first row of request b (its rows
    end at ``seg_base[b + 1]``), ``cta_seg[c]`` the first row CTA c processes (up to ``cta_seg[c + 1]``)."""

    num_ctas: int
    work: torch.Tensor              # [num_reqs + num_ctas, 4] int32 (the capacity)
    cta_seg: torch.Tensor           # first segment row per CTA, plus the end: [num_ctas + 1] int32
    seg_base: torch.Tensor          # first segment row per request, plus the end: [max_reqs + 1] int32
    # 0: the reference's split (equal runs of tiles); > 0: equal runs of cost, a tile costing 8 and a request's first
    # tile this much more (belt_decode_schedule_weighted)
    start_cost: int = 0
    # balanced split (belt_decode_schedule_balanced; None: off): per CTA the decode time of the step so far (int64 ns,
    # added by the decode launches), its speed weight (fp32) and the cost it was dealt (int64)
    cta_ns: torch.Tensor | None = None
    cta_w: torch.Tensor | None = None
    cta_cap: torch.Tensor | None = None

    @property
    def capacity(self) -> int:
        return self.work.shape[0]


# Extra cost of a request's first tile in the weighted split, in eighths of a tile: a segment switch costs the decode
# kernel a query reload and a partial-output epilogue, measured at 11.9 us against 7.4 us per tile (1.6 tiles).
SCHEDULE_START_COST = 13
# Balanced split by default (BELT_B200_BALANCE=0 turns it off): the CTAs' shares follow their measured speed, so the
# split of a step depends on the times of the step before (outputs then differ between runs at the rounding level).
SCHEDULE_BALANCE = os.environ.get("BELT_B200_BALANCE", "1") != "0"


def make_schedule(max_reqs: int, device, num_ctas: int | None = None, start_cost: int = SCHEDULE_START_COST,
                  balance: bool | None = None) -> DecodeSchedule:
    """Buffers for up to ``max_reqs`` decode requests; one CTA per SM by default (cute_decode.py:562-568).
    ``start_cost`` 0 keeps the reference's split; the default weights request starts (``DecodeSchedule``).
    ``balance`` (default ``SCHEDULE_BALANCE``, only with ``start_cost`` > 0) deals the cost out by the CTAs' measured
    speed: the decode launches time every CTA, the next ``schedule`` call updates the weights."""
    device = torch.device(device)
    if num_ctas is None:
        num_ctas = torch.cuda.get_device_properties(device).multi_processor_count
    if balance is None:
        balance = SCHEDULE_BALANCE
    i32 = dict(device=device, dtype=torch.int32)
    sched = DecodeSchedule(num_ctas, torch.zeros(max_reqs + num_ctas, 4, **i32), torch.zeros(num_ctas + 1, **i32),
                           torch.zeros(max_reqs + 1, **i32), int(start_cost))
    if balance and start_cost > 0:
        sched.cta_ns = torch.zeros(num_ctas, dtype=torch.int64, device=device)
        sched.cta_w = torch.ones(num_ctas, dtype=torch.float32, device=device)
        sched.cta_cap = torch.zeros(num_ctas, dtype=torch.int64, device=device)
    return sched


def schedule(sched: DecodeSchedule, seq_lens: torch.Tensor, min_tiles: int = 1) -> None:
    """Fill ``sched`` for the decode requests ``seq_lens`` [B] (int32, on the device): runs of
    max(ceil(tiles / num_ctas), ``min_tiles``) tiles per CTA (cute_decode.py:601-607), or with
    ``sched.start_cost`` > 0 runs of equal cost; a request of length 0 gets no segment."""
    B = seq_lens.shape[0]
    if B + 1 > sched.seg_base.shape[0]:
        raise ValueError(f"schedule: {B} requests exceed the schedule's capacity {sched.seg_base.shape[0] - 1}")
    if seq_lens.dtype != torch.int32 or not seq_lens.is_contiguous():
        raise ValueError("schedule: seq_lens must be contiguous int32")
    if sched.cta_w is not None:
        torch.ops.lrkv_b200.decode_schedule_balanced(seq_lens, sched.work, sched.cta_seg, sched.seg_base, sched.cta_ns,
                                                     sched.cta_w, sched.cta_cap, sched.num_ctas, int(min_tiles),
                                                     int(sched.start_cost))
    else:
        torch.ops.lrkv_b200.decode_schedule(seq_lens, sched.work, sched.cta_seg, sched.seg_base, sched.num_ctas,
                                            int(min_tiles), int(sched.start_cost))


def block_diag_query(q_lat: torch.Tensor, q_rot: torch.Tensor, k_off: list, k_ranks: list, lk_pad: int,
                     dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """[B, H, n_k * 64 + G * rot] query of the score GEMM: q_lat(h) at its group's K columns, the rotated query at its
    group's RoPE chunk, zeros elsewhere (the reference construction, cute_decode.py:610-623; the backend computes it
    with ``latent_ops.block_diag_query``)."""
    B = q_lat.shape[0]
    n_k = math.ceil(lk_pad / CHUNK)
    q = torch.zeros(B, H, n_k * CHUNK + G * ROT, device=q_lat.device, dtype=dtype)
    hpg = H // G
    for g in range(G):
        hs = slice(g * hpg, (g + 1) * hpg)
        q[:, hs, k_off[g]:k_off[g] + k_ranks[g]] = q_lat[:, hs, :k_ranks[g]]
        q[:, hs, n_k * CHUNK + g * ROT:n_k * CHUNK + (g + 1) * ROT] = q_rot[:, hs]
    return q


@dataclass
class RopeRebuild:
    """RoPE-key inputs of the decode kernel: RoPE keys rebuilt in-kernel from the K latent (cute_decode.py:626-632)."""

    groups: tuple                   # ((k_off_g, rr_g) per group): latent columns the group's keys depend on
    blocks: torch.Tensor            # [1, rot, n_blocks * 64] BF16: resident blocks of gain * B_g (``rope_blocks``)
    cos_sin: torch.Tensor           # [max_pos, rot] BF16: the model's cos_sin_cache (cos half | sin half)


def rope_blocks(u_rot: list, groups) -> torch.Tensor:
    """[1, rot, n_blocks * 64] blocks in the dtype of u_rot: u_rot[g] [rot, >= rr_g] are the rotary rows of U_g times
    the k_norm gain, reading latent columns k_off_g .. k_off_g + rr_g; block (g, c) holds them at the columns of the
    64-column cache chunk c, groups then chunks (cute_decode.py:635-646)."""
    blocks = []
    for U, (off, rr) in zip(u_rot, groups):
        for c in range(off // CHUNK, (off + rr - 1) // CHUNK + 1):
            blk = torch.zeros(ROT, CHUNK, dtype=U.dtype, device=U.device)
            lo, hi = max(off, c * CHUNK), min(off + rr, (c + 1) * CHUNK)
            blk[:, lo - c * CHUNK:hi - c * CHUNK] = U[:, lo - off:hi - off]
            blocks.append(blk)
    return torch.cat(blocks, dim=1).unsqueeze(0).contiguous()


def _check_cache(cache: torch.Tensor):
    if cache.dtype != torch.bfloat16 or cache.dim() != 3 or cache.stride(-1) != 1:
        raise ValueError("cache must be a [blocks, page, W] BF16 view with contiguous rows")
    if cache.stride(1) % 8 or cache.stride(0) % 8:
        raise ValueError("cache rows must start 16-byte aligned")


def latent_decode(q_bd: torch.Tensor, cache: torch.Tensor, block_table: torch.Tensor, seq_lens: torch.Tensor,
                  sched: DecodeSchedule, part: torch.Tensor, sm_scale: float, lk_pad: int, lv: int, *,
                  rope: RopeRebuild) -> None:
    """Partial attention of one compressed layer over the segments of ``sched`` (``schedule`` of these seq_lens) into
    ``part`` [>= B + num_ctas - 1, H, lv + 1] fp32: per segment the normalised latent V-space output and its LSE
    (cute_decode.py:649-678).

    q_bd [B, H, n_k * 64 + G * rot] BF16 (``block_diag_query``); cache [num_blocks, page, W] BF16: the layer's
    (possibly strided) view with 16-byte aligned rows; block_table [B, max_pages] int32; ``rope``: ``RopeRebuild``.
    """
    B = q_bd.shape[0]
    _check_cache(cache)
    if q_bd.dtype != torch.bfloat16 or not q_bd.is_contiguous():
        raise ValueError("q_bd must be contiguous BF16")
    if part.dtype != torch.float32 or part.stride(-1) != 1 or part.shape[-1] != lv + 1:
        raise ValueError("part must be fp32 [segments, H, lv + 1] with a contiguous last dim")
    if part.shape[0] < B + sched.num_ctas - 1:
        raise ValueError(f"part holds {part.shape[0]} segments, need >= B + num_ctas - 1 = {B + sched.num_ctas - 1}")
    if block_table.dtype != torch.int32 or block_table.stride(-1) != 1:
        raise ValueError("block_table must be int32 with contiguous rows")
    if seq_lens.dtype != torch.int32 or not seq_lens.is_contiguous():
        raise ValueError("seq_lens must be contiguous int32")
    blocks, cos_sin = rope.blocks, rope.cos_sin
    if blocks.dtype != torch.bfloat16 or not blocks.is_contiguous() or blocks.shape[1] != ROT:
        raise ValueError("rope blocks must be contiguous BF16 [1, 64, n * 64]")
    if cos_sin.dtype != torch.bfloat16 or not cos_sin.is_contiguous() or cos_sin.shape[1] != ROT:
        raise ValueError("cos_sin must be contiguous BF16 [max_pos, 64]")
    groups = [int(x) for gr in rope.groups for x in gr]
    if sched.cta_ns is not None:   # balanced split: time every CTA for the next step's weights
        torch.ops.lrkv_b200.latent_decode_timed(q_bd, cache, block_table, seq_lens, sched.work, sched.cta_seg, part,
                                                sched.num_ctas, float(sm_scale), int(lk_pad), int(lv), groups, blocks,
                                                cos_sin, sched.cta_ns)
    else:
        torch.ops.lrkv_b200.latent_decode(q_bd, cache, block_table, seq_lens, sched.work, sched.cta_seg, part,
                                          sched.num_ctas, float(sm_scale), int(lk_pad), int(lv), groups, blocks,
                                          cos_sin)


latent_decode_cute = latent_decode   # the reference's name for the same entry


def merge_segments(part: torch.Tensor, sched: DecodeSchedule, out: torch.Tensor, lse: torch.Tensor) -> None:
    """Segment partials ``part`` [segments, H, lv + 1] -> out [B, H, lv] (BF16), lse [B, H] (fp32)
    (cute_decode.py:715-722)."""
    B, nh, lv = out.shape
    if out.stride(-1) != 1 or part.shape[-1] != lv + 1 or out.dtype != torch.bfloat16:
        raise ValueError("merge_segments: out must be BF16 [B, H, lv] with a contiguous last dim")
    if lse.dtype != torch.float32 or lse.stride(-1) != 1:
        raise ValueError("merge_segments: lse must be fp32 [B, H]")
    torch.ops.lrkv_b200.merge_segments(part, sched.seg_base, out, lse)


def partial_buffer(rows: int, r_v: int, device) -> torch.Tensor:
    """Partial outputs for ``latent_decode`` / ``merge_segments`` / ``merge_up_project``: fp32 [rows, H, r_v + 1]
    (the r_v normalised features and the natural-log LSE of every segment and head), allocated with the head stride
    rounded up to a multiple of 4 floats so that every row starts on 16 bytes (the fused merge then reads the rows as
    float4). A view of that allocation; any other [rows, H, r_v + 1] layout with a contiguous last dim works as well."""
    width = (r_v + 1 + 3) // 4 * 4
    return torch.empty(rows, H, width, dtype=torch.float32, device=device)[:, :, :r_v + 1]


def merge_up_project(part: torch.Tensor, sched: DecodeSchedule, v_up_t: torch.Tensor, out: torch.Tensor,
                     lse: torch.Tensor) -> None:
    """``merge_segments`` and the V up-projection in one kernel: part [segments, H, lv + 1] -> out [B, H, 256] (BF16,
    written in place, e.g. the first rows of the attention output) = U_v,g(h) bf16(merged a), and lse [B, H] (fp32).
    The merged output never leaves the chip; the roundings are those of ``merge_segments`` + ``up_project``."""
    B, nh, D = out.shape
    lv = v_up_t.shape[1]
    if part.dtype != torch.float32 or part.stride(-1) != 1 or part.shape[-1] != lv + 1:
        raise ValueError("merge_up_project: part must be fp32 [segments, H, lv + 1] with a contiguous last dim")
    if out.dtype != torch.bfloat16 or out.stride(-1) != 1 or nh != H or D != 256:
        raise ValueError("merge_up_project: out must be BF16 [B, 24, 256] with contiguous channels")
    if v_up_t.dtype != torch.bfloat16 or not v_up_t.is_contiguous() or v_up_t.shape[0] != G or v_up_t.shape[2] != 256:
        raise ValueError("merge_up_project: v_up_t must be a contiguous BF16 [4, lv, 256]")
    if lse.dtype != torch.float32 or lse.stride(-1) != 1 or lse.shape[0] < B:
        raise ValueError("merge_up_project: lse must be fp32 [B, H]")
    torch.ops.lrkv_b200.merge_up_project(part, sched.seg_base, v_up_t, out, lse)
