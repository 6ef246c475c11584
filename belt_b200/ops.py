"""The C ABI as torch custom operators: ``torch.ops.lrkv_b200.*``.

Every kernel entry point of ``libbelt_b200.so`` is registered with ``torch.library.custom_op`` so that torch sees one
opaque operator per kernel launch, with its mutated arguments declared: ``torch.compile`` traces through the backend
and keeps each launch as one node (its fake implementation gives the output metadata without running anything), and
vLLM's piecewise graph splitting can name the ops. The real implementations pass device pointers, strides and the
current CUDA stream to the C ABI (``_lib``) and raise ``ValueError`` / ``BeltError`` on a bad status; there is no CPU
implementation (``device_types="cuda"``), so a call on CPU tensors fails instead of falling back.

The reference invokes its operators as plain Python functions inside vLLM's attention op
(``plugins/vllm_lrkv/vllm_lrkv/latent_backend.py:251-295``); the Python surface of this package
(``decode.latent_decode``, ``latent_ops.block_diag_query``, ...) keeps those names and dispatches here. Every kernel
records a timed-out wait in the device's error word (``decode.error_word``), which the implementations fetch
themselves: it is not an argument torch tracks.

Operators (mutated arguments marked !):
  cache_write(c, slot_mapping, cache!, u_cat, k_segs, eps)
  proj_cache_write(x, w_down, slot_mapping, cache!, u_cat, k_segs, eps)
  decode_schedule(seq_lens, work!, cta_seg!, seg_base!, num_ctas, min_tiles, start_cost)
  decode_schedule_balanced(seq_lens, work!, cta_seg!, seg_base!, cta_ns!, cta_w!, cta_cap!, num_ctas, min_tiles,
                           start_cost)
  latent_decode(q_bd, cache, block_table, seq_lens, work, cta_seg, part!, num_ctas, sm_scale, lk_pad, lv,
                rope_groups, rope_blocks, cos_sin)
  latent_decode_timed(..., as latent_decode, cta_ns!)
  merge_segments(part, seg_base, out!, lse!)
  merge_up_project(part, seg_base, v_up_t, out!, lse!)
  block_diag_query(q, qmap, col_runs) -> q_bd
  up_project(a, v_up_t, out!)
  decompress(cache, block_table_row, seq_len, pos0, wk, k_segs, v_up_t, v_offset, cos_sin, k_out!, v_out!)
  prefill_attention(q, k, v, q_pos0, k_pos0, scale, causal, out!, lse!)
  decompress_varlen(cache, block_table, pieces, wk, k_segs, v_up_t, v_offset, cos_sin, k_out!, v_out!)
  prefill_attention_varlen(q, k, v, pieces, scale, causal, out!, lse!, out2!, lse2!)
  attn_fold(out!, lse!, part, part_lse, pieces)
  linear(x, weight) -> x weight^T  (the model's linear layers, BF16)
"""

from __future__ import annotations

import torch
from torch.library import custom_op

from . import _lib

NS = "lrkv_b200"


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _err(t: torch.Tensor) -> int:
    from .decode import error_word
    return error_word(t.device).data_ptr()


def _aligned(*ts) -> None:
    for t in ts:
        if t.data_ptr() % 16:
            raise ValueError("tensors passed to the kernels must start 16-byte aligned")


# ------------------------------------------------------------------------------------------------------- cache write
@custom_op(f"{NS}::cache_write", mutates_args=("cache",), device_types="cuda")
def cache_write(c: torch.Tensor, slot_mapping: torch.Tensor, cache: torch.Tensor, u_cat: torch.Tensor,
                k_segs: list[int], eps: float) -> None:
    T = slot_mapping.shape[0]
    _lib.call("belt_latent_rows_to_cache", c.data_ptr(), T, c.stride(0), slot_mapping.data_ptr(),
              int(slot_mapping.dtype == torch.int64), cache.data_ptr(), cache.shape[0], cache.shape[1], cache.shape[2],
              cache.stride(0), cache.stride(1), u_cat.data_ptr(), u_cat.shape[0], _lib.int_array(k_segs), float(eps),
              _stream(c))


@cache_write.register_fake
def _(c, slot_mapping, cache, u_cat, k_segs, eps):
    return None


@custom_op(f"{NS}::proj_cache_write", mutates_args=("cache",), device_types="cuda")
def proj_cache_write(x: torch.Tensor, w_down: torch.Tensor, slot_mapping: torch.Tensor, cache: torch.Tensor,
                     u_cat: torch.Tensor, k_segs: list[int], eps: float) -> None:
    T = slot_mapping.shape[0]
    _lib.call("belt_latent_proj_rows_to_cache", x.data_ptr(), T, x.stride(0), x.shape[1], w_down.data_ptr(),
              w_down.stride(0), slot_mapping.data_ptr(), int(slot_mapping.dtype == torch.int64), cache.data_ptr(),
              cache.shape[0], cache.shape[1], cache.shape[2], cache.stride(0), cache.stride(1), u_cat.data_ptr(),
              u_cat.shape[0], _lib.int_array(k_segs), float(eps), _err(x), _stream(x))


@proj_cache_write.register_fake
def _(x, w_down, slot_mapping, cache, u_cat, k_segs, eps):
    return None


# ----------------------------------------------------------------------------------------------------------- decode
@custom_op(f"{NS}::decode_schedule", mutates_args=("work", "cta_seg", "seg_base"), device_types="cuda")
def decode_schedule(seq_lens: torch.Tensor, work: torch.Tensor, cta_seg: torch.Tensor, seg_base: torch.Tensor,
                    num_ctas: int, min_tiles: int, start_cost: int) -> None:
    B = seq_lens.shape[0]
    if start_cost > 0:
        _lib.call("belt_decode_schedule_weighted", seq_lens.data_ptr(), B, num_ctas, min_tiles, start_cost,
                  work.data_ptr(), work.shape[0], cta_seg.data_ptr(), seg_base.data_ptr(), _err(seq_lens),
                  _stream(seq_lens))
    else:
        _lib.call("belt_decode_schedule", seq_lens.data_ptr(), B, num_ctas, min_tiles, work.data_ptr(),
                  work.shape[0], cta_seg.data_ptr(), seg_base.data_ptr(), _err(seq_lens), _stream(seq_lens))


@decode_schedule.register_fake
def _(seq_lens, work, cta_seg, seg_base, num_ctas, min_tiles, start_cost):
    return None


@custom_op(f"{NS}::decode_schedule_balanced", mutates_args=("work", "cta_seg", "seg_base", "cta_ns", "cta_w", "cta_cap"),
           device_types="cuda")
def decode_schedule_balanced(seq_lens: torch.Tensor, work: torch.Tensor, cta_seg: torch.Tensor, seg_base: torch.Tensor,
                             cta_ns: torch.Tensor, cta_w: torch.Tensor, cta_cap: torch.Tensor, num_ctas: int,
                             min_tiles: int, start_cost: int) -> None:
    _lib.call("belt_decode_schedule_balanced", seq_lens.data_ptr(), seq_lens.shape[0], num_ctas, min_tiles, start_cost,
              cta_ns.data_ptr(), cta_w.data_ptr(), cta_cap.data_ptr(), work.data_ptr(), work.shape[0],
              cta_seg.data_ptr(), seg_base.data_ptr(), _err(seq_lens), _stream(seq_lens))


@decode_schedule_balanced.register_fake
def _(seq_lens, work, cta_seg, seg_base, cta_ns, cta_w, cta_cap, num_ctas, min_tiles, start_cost):
    return None


@custom_op(f"{NS}::latent_decode", mutates_args=("part",), device_types="cuda")
def latent_decode(q_bd: torch.Tensor, cache: torch.Tensor, block_table: torch.Tensor, seq_lens: torch.Tensor,
                  work: torch.Tensor, cta_seg: torch.Tensor, part: torch.Tensor, num_ctas: int, sm_scale: float,
                  lk_pad: int, lv: int, rope_groups: list[int], rope_blocks: torch.Tensor,
                  cos_sin: torch.Tensor) -> None:
    _aligned(cache)
    _lib.call("belt_latent_decode", q_bd.data_ptr(), q_bd.shape[0], q_bd.shape[2], cache.data_ptr(), cache.shape[0],
              cache.shape[1], cache.shape[2], cache.stride(0), cache.stride(1), block_table.data_ptr(),
              block_table.stride(0), seq_lens.data_ptr(), work.data_ptr(), cta_seg.data_ptr(), num_ctas,
              part.data_ptr(), part.stride(0), part.stride(1), float(sm_scale), int(lk_pad), int(lv),
              _lib.int_array(rope_groups), rope_blocks.data_ptr(), rope_blocks.shape[-1] // 64, cos_sin.data_ptr(),
              cos_sin.shape[0], _err(q_bd), _stream(q_bd))


@latent_decode.register_fake
def _(q_bd, cache, block_table, seq_lens, work, cta_seg, part, num_ctas, sm_scale, lk_pad, lv, rope_groups,
      rope_blocks, cos_sin):
    return None


@custom_op(f"{NS}::latent_decode_timed", mutates_args=("part", "cta_ns"), device_types="cuda")
def latent_decode_timed(q_bd: torch.Tensor, cache: torch.Tensor, block_table: torch.Tensor, seq_lens: torch.Tensor,
                        work: torch.Tensor, cta_seg: torch.Tensor, part: torch.Tensor, num_ctas: int, sm_scale: float,
                        lk_pad: int, lv: int, rope_groups: list[int], rope_blocks: torch.Tensor,
                        cos_sin: torch.Tensor, cta_ns: torch.Tensor) -> None:
    _aligned(cache)
    _lib.call("belt_latent_decode_timed", q_bd.data_ptr(), q_bd.shape[0], q_bd.shape[2], cache.data_ptr(),
              cache.shape[0], cache.shape[1], cache.shape[2], cache.stride(0), cache.stride(1), block_table.data_ptr(),
              block_table.stride(0), seq_lens.data_ptr(), work.data_ptr(), cta_seg.data_ptr(), num_ctas,
              part.data_ptr(), part.stride(0), part.stride(1), float(sm_scale), int(lk_pad), int(lv),
              _lib.int_array(rope_groups), rope_blocks.data_ptr(), rope_blocks.shape[-1] // 64, cos_sin.data_ptr(),
              cos_sin.shape[0], _err(q_bd), cta_ns.data_ptr(), _stream(q_bd))


@latent_decode_timed.register_fake
def _(q_bd, cache, block_table, seq_lens, work, cta_seg, part, num_ctas, sm_scale, lk_pad, lv, rope_groups,
      rope_blocks, cos_sin, cta_ns):
    return None


@custom_op(f"{NS}::merge_segments", mutates_args=("out", "lse"), device_types="cuda")
def merge_segments(part: torch.Tensor, seg_base: torch.Tensor, out: torch.Tensor, lse: torch.Tensor) -> None:
    B, nh, lv = out.shape
    _lib.call("belt_merge_segments", part.data_ptr(), part.stride(0), part.stride(1), seg_base.data_ptr(), B, nh, lv,
              out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(), lse.stride(0), _stream(out))


@merge_segments.register_fake
def _(part, seg_base, out, lse):
    return None


@custom_op(f"{NS}::merge_up_project", mutates_args=("out", "lse"), device_types="cuda")
def merge_up_project(part: torch.Tensor, seg_base: torch.Tensor, v_up_t: torch.Tensor, out: torch.Tensor,
                     lse: torch.Tensor) -> None:
    B = out.shape[0]
    lv = v_up_t.shape[1]
    _lib.call("belt_merge_up_project", part.data_ptr(), part.stride(0), part.stride(1), seg_base.data_ptr(), B, lv,
              v_up_t.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(), lse.stride(0),
              _err(part), _stream(out))


@merge_up_project.register_fake
def _(part, seg_base, v_up_t, out, lse):
    return None


# ------------------------------------------------------------------------------------------ per-head projections
@custom_op(f"{NS}::block_diag_query", mutates_args=(), device_types="cuda")
def block_diag_query(q: torch.Tensor, qmap: torch.Tensor, col_runs: list[int]) -> torch.Tensor:
    T, H, _ = q.shape
    KQ = qmap.shape[-1]
    out = torch.empty(T, H, KQ, device=q.device, dtype=q.dtype)
    _lib.call("belt_block_diag_query", q.data_ptr(), T, q.stride(0), q.stride(1), qmap.data_ptr(), KQ,
              _lib.int_array(col_runs), out.data_ptr(), _err(q), _stream(q))
    return out


@block_diag_query.register_fake
def _(q, qmap, col_runs):
    return q.new_empty(q.shape[0], q.shape[1], qmap.shape[-1])


@custom_op(f"{NS}::up_project", mutates_args=("out",), device_types="cuda")
def up_project(a: torch.Tensor, v_up_t: torch.Tensor, out: torch.Tensor) -> None:
    _lib.call("belt_up_project", a.data_ptr(), a.shape[0], a.stride(0), a.stride(1), v_up_t.shape[1],
              v_up_t.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1), _err(a), _stream(a))


@up_project.register_fake
def _(a, v_up_t, out):
    return None


# ---------------------------------------------------------------------------------------------------------- prefill
@custom_op(f"{NS}::decompress", mutates_args=("k_out", "v_out"), device_types="cuda")
def decompress(cache: torch.Tensor, block_table_row: torch.Tensor, seq_len: int, pos0: int, wk: torch.Tensor,
               k_segs: list[int], v_up_t: torch.Tensor, v_offset: int, cos_sin: torch.Tensor, k_out: torch.Tensor,
               v_out: torch.Tensor) -> None:
    count = k_out.shape[0]
    _lib.call("belt_latent_decompress", cache.data_ptr(), cache.shape[0], cache.shape[1], cache.shape[2],
              cache.stride(0), cache.stride(1), block_table_row.data_ptr(), int(seq_len), int(pos0), int(count),
              wk.data_ptr(), wk.shape[2], _lib.int_array(k_segs), v_up_t.data_ptr(), int(v_offset), v_up_t.shape[1],
              cos_sin.data_ptr(), cos_sin.shape[0], k_out.data_ptr(), v_out.data_ptr(), k_out.stride(0),
              k_out.stride(1), _err(cache), _stream(cache))


@decompress.register_fake
def _(cache, block_table_row, seq_len, pos0, wk, k_segs, v_up_t, v_offset, cos_sin, k_out, v_out):
    return None


@custom_op(f"{NS}::prefill_attention", mutates_args=("out", "lse"), device_types="cuda")
def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_pos0: int, k_pos0: int, scale: float,
                      causal: bool, out: torch.Tensor, lse: torch.Tensor) -> None:
    _lib.call("belt_prefill_attention", q.data_ptr(), q.shape[0], q.stride(0), q.stride(1), k.data_ptr(), v.data_ptr(),
              k.shape[0], k.stride(0), k.stride(1), int(q_pos0), int(k_pos0), int(bool(causal)), float(scale),
              out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(), lse.stride(0), _err(q), _stream(q))


@prefill_attention.register_fake
def _(q, k, v, q_pos0, k_pos0, scale, causal, out, lse):
    return None


@custom_op(f"{NS}::decompress_varlen", mutates_args=("k_out", "v_out"), device_types="cuda")
def decompress_varlen(cache: torch.Tensor, block_table: torch.Tensor, pieces: list[int], wk: torch.Tensor,
                      k_segs: list[int], v_up_t: torch.Tensor, v_offset: int, cos_sin: torch.Tensor,
                      k_out: torch.Tensor, v_out: torch.Tensor) -> None:
    _lib.call("belt_latent_decompress_varlen", cache.data_ptr(), cache.shape[0], cache.shape[1], cache.shape[2],
              cache.stride(0), cache.stride(1), block_table.data_ptr(), block_table.stride(0), len(pieces) // 4,
              _lib.int_array(pieces), wk.data_ptr(), wk.shape[2], _lib.int_array(k_segs), v_up_t.data_ptr(),
              int(v_offset), v_up_t.shape[1], cos_sin.data_ptr(), cos_sin.shape[0], k_out.data_ptr(), v_out.data_ptr(),
              k_out.stride(0), k_out.stride(1), _err(cache), _stream(cache))


@decompress_varlen.register_fake
def _(cache, block_table, pieces, wk, k_segs, v_up_t, v_offset, cos_sin, k_out, v_out):
    return None


@custom_op(f"{NS}::prefill_attention_varlen", mutates_args=("out", "lse", "out2", "lse2"), device_types="cuda")
def prefill_attention_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pieces: list[int], scale: float,
                             causal: bool, out: torch.Tensor, lse: torch.Tensor, out2: torch.Tensor,
                             lse2: torch.Tensor) -> None:
    _lib.call("belt_prefill_attention_varlen", q.data_ptr(), q.shape[0], q.stride(0), q.stride(1), k.data_ptr(),
              v.data_ptr(), k.shape[0], k.stride(0), k.stride(1), len(pieces) // 8, _lib.int_array(pieces),
              int(bool(causal)), float(scale), out.data_ptr(), out2.data_ptr(), out.stride(0), out.stride(1),
              lse.data_ptr(), lse2.data_ptr(), lse.stride(0), _err(q), _stream(q))


@prefill_attention_varlen.register_fake
def _(q, k, v, pieces, scale, causal, out, lse, out2, lse2):
    return None


@custom_op(f"{NS}::attn_fold", mutates_args=("out", "lse"), device_types="cuda")
def attn_fold(out: torch.Tensor, lse: torch.Tensor, part: torch.Tensor, part_lse: torch.Tensor,
              pieces: list[int]) -> None:
    _lib.call("belt_attn_fold", out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(), lse.stride(0),
              part.data_ptr(), part.stride(0), part.stride(1), part_lse.data_ptr(), part_lse.stride(0),
              len(pieces) // 3, _lib.int_array(pieces), _stream(out))


@attn_fold.register_fake
def _(out, lse, part, part_lse, pieces):
    return None


# ---------------------------------------------------------------------------------------------------------- linear
@custom_op(f"{NS}::linear", mutates_args=(), device_types="cuda")
def linear(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    M, K = x.shape
    N = weight.shape[0]
    out = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
    _lib.call("belt_gemm_bf16", x.data_ptr(), M, K, x.stride(0), weight.data_ptr(), N, weight.stride(0),
              out.data_ptr(), out.stride(0), _err(x), _stream(x))
    return out


@linear.register_fake
def _(x, weight):
    return x.new_empty(x.shape[0], weight.shape[0])


OPS = ("cache_write", "proj_cache_write", "decode_schedule", "decode_schedule_balanced", "latent_decode",
       "latent_decode_timed", "merge_segments", "merge_up_project",
       "block_diag_query",
       "up_project", "decompress", "prefill_attention", "decompress_varlen", "prefill_attention_varlen", "attn_fold",
       "linear")
