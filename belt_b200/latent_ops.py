"""The operators around the latent decode, the public surface of the reference's ``vllm_lrkv.latent_ops``
(plugins/vllm_lrkv/vllm_lrkv/latent_ops.py), on this package's sm_100a kernels:

* ``block_diag_query``: the normed, rotated query [T, H, D] times each KV group's map [D, n_k * 64 + G * rot] ->
  the block-diagonal decode query [T, H, n_k * 64 + G * rot] (latent_ops.py:67-73);
* ``up_project``: the merged latent output [T, H, r_v] times U_v of each head's group (stored transposed as
  [G, r_v, D]) -> the attention output [T, H, D], in place (latent_ops.py:76-81);
* ``latent_rows_to_cache``: the per-token cache rows ``[c_K / rho | 0 | c_v | 0]`` into the paged KV cache
  (latent_ops.py:138-158);
* ``project_rows_to_cache``: the same rows computed from the layer inputs, the model's ``kv_latent_proj`` linear
  (models/qwen3_5_latent.py:139-140, 213) fused into the write on the tensor cores;
* ``decompress_paged``: keys and values of a request's cached positions rebuilt from its latent rows (the prefill
  path's ``LatentLayer.decompress``, latent_backend.py:95-108) on the tensor cores;
* ``prefill_attention``: a request's new tokens over those keys and values (causal, with the LSE), the attention of
  the reference's prefill path (latent_backend.py:285-320).
"""

from __future__ import annotations

import torch

from . import ops as _ops  # noqa: F401  (registers torch.ops.lrkv_b200)

HEAD_DIM = 256


def host_k_segs(k_segs) -> list:
    """k_segs as a flat host list of 16 ints. A device tensor is copied to the host (a synchronisation): hot paths pass
    the host rows (``LatentLayer.k_segs_host``)."""
    if not isinstance(k_segs, torch.Tensor):
        return [int(x) for row in k_segs for x in (row if isinstance(row, (list, tuple)) else [row])]
    return [int(x) for x in k_segs.flatten().tolist()]


def _runs_dense(kq: int, groups: int = 4):
    return [[(0, kq), (0, 0), (0, 0)] for _ in range(groups)]


def group_column_runs(k_segs, n_k: int, rot: int = 64) -> list:
    """Per group the query columns its map can make non-zero: its latent column runs (``k_segs`` rows
    (start, length, start, length)) and its RoPE chunk n_k * 64 + g * rot."""
    flat = host_k_segs(k_segs)
    rows = [flat[4 * g:4 * g + 4] for g in range(len(flat) // 4)]
    runs = []
    for g, (a, n, b, m) in enumerate(rows):
        rope = n_k * 64 + g * rot
        runs.append([(a, a + n), (b, b + m), (rope, rope + rot)])
    return runs


def block_diag_query(q: torch.Tensor, qmap: torch.Tensor, col_runs=None) -> torch.Tensor:
    """q [T, H, D] (normed, rotated) and qmap [G, D, KQ] -> the decode kernel's block-diagonal query [T, H, KQ] (BF16,
    FP32 accumulation). ``col_runs`` (``group_column_runs``) limits the work to the columns a group's map can make
    non-zero; without it the full product is computed."""
    T, Hq, D = q.shape
    KQ = qmap.shape[-1]
    if q.dtype != torch.bfloat16 or qmap.dtype != torch.bfloat16 or q.stride(-1) != 1 or not qmap.is_contiguous():
        raise ValueError("block_diag_query: BF16 q with a contiguous last dim and a contiguous BF16 qmap")
    if Hq != 24 or D != HEAD_DIM or qmap.shape[0] != 4 or qmap.shape[1] != D:
        raise ValueError(f"block_diag_query: q {tuple(q.shape)} / qmap {tuple(qmap.shape)} (24 heads, 4 groups, 256)")
    runs = col_runs if col_runs is not None else _runs_dense(KQ)
    flat = [int(x) for g in runs for r in g for x in r]
    return torch.ops.lrkv_b200.block_diag_query(q, qmap, flat)


def up_project(a: torch.Tensor, v_up_t: torch.Tensor, out: torch.Tensor) -> None:
    """a [T, H, r_v] (merged latent output) and v_up_t [G, r_v, D] (U_v transposed) -> out [T, H, D] =
    U_v,g(h) a(h), in place."""
    R, D = v_up_t.shape[1], v_up_t.shape[2]
    if a.shape[-1] != R or v_up_t.stride(2) != 1 or not v_up_t.is_contiguous():
        raise ValueError("up_project: a [T, H, r_v] and a contiguous v_up_t [G, r_v, D]")
    if a.stride(-1) != 1 or out.stride(-1) != 1 or out.shape[:2] != a.shape[:2] or D != HEAD_DIM:
        raise ValueError("up_project: shapes / strides")
    if a.dtype != torch.bfloat16 or out.dtype != torch.bfloat16 or v_up_t.dtype != torch.bfloat16:
        raise ValueError("up_project: BF16 tensors")
    torch.ops.lrkv_b200.up_project(a, v_up_t, out)


def latent_rows_to_cache(c: torch.Tensor, slot_mapping: torch.Tensor, cache: torch.Tensor, u_cat: torch.Tensor,
                         k_segs: torch.Tensor, eps: float) -> None:
    """Write the cache rows of new tokens: c [T, >= pe_offset] (the latent projection; its first pe_offset columns are
    [c_K | 0 | c_v | 0]) -> cache[slot] = [c_K / rho | 0 | c_v | 0] per group.

    u_cat [lk, G * D] (BF16): U_g^T at the rows of the group's columns; k_segs [G, 4] int32: every group's columns as
    two runs (start, length, start, length); cache [blocks, page, W]. Slots < 0 are padding."""
    T = slot_mapping.shape[0]
    if T == 0:
        return
    lk, ngd = u_cat.shape
    segs = host_k_segs(k_segs)
    ng = len(segs) // 4
    if len(segs) != 16 or ngd != ng * HEAD_DIM:
        raise ValueError("latent_rows_to_cache: head dim 256, 4 groups, k_segs [4, 4]")
    W = cache.shape[-1]
    if c.stride(-1) != 1 or cache.stride(-1) != 1 or not u_cat.is_contiguous():
        raise ValueError("latent_rows_to_cache: contiguous rows")
    if c.dtype != torch.bfloat16 or cache.dtype != torch.bfloat16 or u_cat.dtype != torch.bfloat16:
        raise ValueError("latent_rows_to_cache: BF16 c, cache and u_cat")
    if c.shape[1] < W:
        raise ValueError(f"latent_rows_to_cache: c has {c.shape[1]} columns, the row width is {W}")
    if slot_mapping.dtype not in (torch.int32, torch.int64) or not slot_mapping.is_contiguous():
        raise ValueError("latent_rows_to_cache: contiguous int32 / int64 slot_mapping")
    torch.ops.lrkv_b200.cache_write(c, slot_mapping, cache, u_cat, segs, float(eps))


def _check_kv_out(t: torch.Tensor, rows: int, name: str) -> None:
    if t.dtype != torch.bfloat16 or tuple(t.shape) != (rows, 4, HEAD_DIM) or t.stride(2) != 1:
        raise ValueError(f"{name} must be BF16 [{rows}, 4, 256] with contiguous channels")


def decompress_varlen(cache: torch.Tensor, block_table: torch.Tensor, pieces, wk: torch.Tensor, k_segs,
                      v_up_t: torch.Tensor, v_offset: int, cos_sin: torch.Tensor, k_out: torch.Tensor | None = None,
                      v_out: torch.Tensor | None = None):
    """Keys and values of several requests' position ranges in one launch: ``pieces`` = [(request row of
    ``block_table``, its seq_len, pos0, count), ...]; piece i fills rows [sum of the earlier counts, + count) of
    k_out / v_out [sum counts, 4, 256] (allocated when not given). Per piece the same result as
    ``decompress_paged``."""
    flat = [int(x) for pc in pieces for x in pc]
    rows = sum(int(pc[3]) for pc in pieces)
    dev = cache.device
    if k_out is None:
        k_out = torch.empty(rows, 4, HEAD_DIM, dtype=torch.bfloat16, device=dev)
    if v_out is None:
        v_out = torch.empty(rows, 4, HEAD_DIM, dtype=torch.bfloat16, device=dev)
    if rows == 0:
        return k_out, v_out
    if cache.dtype != torch.bfloat16 or cache.stride(-1) != 1 or block_table.dtype != torch.int32 or \
            block_table.stride(-1) != 1:
        raise ValueError("decompress_varlen: BF16 cache with contiguous rows, int32 block table with contiguous rows")
    _check_kv_out(k_out, rows, "k_out")
    _check_kv_out(v_out, rows, "v_out")
    if k_out.stride() != v_out.stride():
        raise ValueError("decompress_varlen: k_out and v_out with the same strides")
    torch.ops.lrkv_b200.decompress_varlen(cache, block_table, flat, wk, host_k_segs(k_segs), v_up_t, int(v_offset),
                                          cos_sin, k_out, v_out)
    return k_out, v_out


def prefill_attention_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pieces, scale: float, out: torch.Tensor,
                             lse: torch.Tensor, out2: torch.Tensor | None = None, lse2: torch.Tensor | None = None,
                             causal: bool = True) -> None:
    """Several pieces of prefill attention in one launch. q [Tq, 24, 256], k / v [Tk, 4, 256] BF16; ``pieces`` =
    [(q_row, ql, k_row, S, q_pos0, k_pos0, o_row, to2), ...]: queries [q_row, q_row + ql) at positions q_pos0.. over
    keys [k_row, k_row + S) at positions k_pos0.. (causal by position), written from row o_row of out / lse, or of
    out2 / lse2 when to2 (same shapes and strides)."""
    flat = [int(x) for pc in pieces for x in pc]
    if not flat:
        return
    for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
        if t.dtype != torch.bfloat16 or t.dim() != 3 or t.shape[2] != HEAD_DIM or t.stride(2) != 1:
            raise ValueError(f"prefill_attention_varlen: {name} [n, heads, 256] BF16 with contiguous channels")
    if lse.dtype != torch.float32 or lse.stride(1) != 1:
        raise ValueError("prefill_attention_varlen: lse [rows, 24] fp32 with contiguous heads")
    if out2 is None:
        out2, lse2 = out, lse
    if out2.stride() != out.stride() or lse2.stride() != lse.stride():
        raise ValueError("prefill_attention_varlen: out2 / lse2 with the strides of out / lse")
    if out2 is out:
        # one destination: the op's second pair may not alias the first, so give it an empty pair (no piece uses it)
        if any(int(pc[7]) for pc in pieces):
            raise ValueError("prefill_attention_varlen: a piece writes to out2, which was not given")
        out2 = out.new_empty(0, out.shape[1], HEAD_DIM).as_strided((0, out.shape[1], HEAD_DIM), out.stride())
        lse2 = lse.new_empty(0, lse.shape[1]).as_strided((0, lse.shape[1]), lse.stride())
    torch.ops.lrkv_b200.prefill_attention_varlen(q, k, v, flat, float(scale), bool(causal), out, lse, out2, lse2)


def attn_fold(out: torch.Tensor, lse: torch.Tensor, part: torch.Tensor, part_lse: torch.Tensor, pieces) -> None:
    """Fold a chunk's attention result into the running one, in place, by log-sum-exp: ``pieces`` = [(destination row
    of out / lse, source row of part / part_lse, rows), ...]."""
    flat = [int(x) for pc in pieces for x in pc]
    if not flat:
        return
    for name, t in (("out", out), ("part", part)):
        if t.dtype != torch.bfloat16 or t.dim() != 3 or t.shape[2] != HEAD_DIM or t.stride(2) != 1:
            raise ValueError(f"attn_fold: {name} [rows, 24, 256] BF16 with contiguous channels")
    torch.ops.lrkv_b200.attn_fold(out, lse, part, part_lse, flat)


def linear(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """x [M, K] @ weight[N, K]^T on the tensor cores (``belt_gemm_bf16``): BF16 operands with contiguous rows (any row
    strides that are multiples of 8), FP32 accumulation, BF16 out [M, N]. The model's linear layers (q_gate_proj,
    o_proj, kv_latent_proj at prefill sizes)."""
    if x.dim() != 2 or weight.dim() != 2 or x.shape[1] != weight.shape[1]:
        raise ValueError(f"linear: x {tuple(x.shape)} and weight {tuple(weight.shape)} ([M, K] and [N, K])")
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or x.stride(1) != 1 or weight.stride(1) != 1:
        raise ValueError("linear: BF16 x and weight with contiguous rows")
    return torch.ops.lrkv_b200.linear(x, weight)


# From this many tokens on (prefill chunks) the projection runs as a GEMM (``linear``) followed by the cache write: the
# fused kernel re-streams W_down for every 128 tokens, which costs more than the round trip of c (8192 tokens); below
# it the fused kernel is as fast and needs no buffer for c.
FUSED_WRITE_MAX_TOKENS = 2048


def project_rows_to_cache(x: torch.Tensor, w_down: torch.Tensor, slot_mapping: torch.Tensor, cache: torch.Tensor,
                          u_cat: torch.Tensor, k_segs, eps: float, fused: bool | None = None) -> None:
    """``latent_rows_to_cache(bf16(x @ w_down^T), ...)``: x [T, hidden] BF16 (the layer inputs of the new tokens),
    w_down [>= W, hidden] BF16 (``kv_latent_proj.weight``, zero rows at the gaps), the other arguments as
    ``latent_rows_to_cache``. ``fused`` (default: fewer than FUSED_WRITE_MAX_TOKENS tokens) runs it as one kernel that
    never materialises the projection; otherwise the projection is this package's GEMM (``linear``) into a [T, W]
    buffer, then the cache write."""
    T = slot_mapping.shape[0]
    if T == 0:
        return
    lk, ngd = u_cat.shape
    segs = host_k_segs(k_segs)
    if len(segs) != 16 or ngd != 4 * HEAD_DIM:
        raise ValueError("project_rows_to_cache: head dim 256, 4 groups, k_segs [4, 4]")
    W = cache.shape[-1]
    for name, t in (("x", x), ("w_down", w_down), ("cache", cache), ("u_cat", u_cat)):
        if t.dtype != torch.bfloat16 or t.stride(-1) != 1:
            raise ValueError(f"project_rows_to_cache: {name} must be BF16 with contiguous rows")
    if x.shape[0] < T or w_down.shape[0] < W or w_down.shape[1] != x.shape[1] or not u_cat.is_contiguous():
        raise ValueError("project_rows_to_cache: x [T, hidden], w_down [>= W, hidden], contiguous u_cat")
    if slot_mapping.dtype not in (torch.int32, torch.int64) or not slot_mapping.is_contiguous():
        raise ValueError("project_rows_to_cache: contiguous int32 / int64 slot_mapping")
    if fused is None:
        fused = T < FUSED_WRITE_MAX_TOKENS
    if not fused:
        latent_rows_to_cache(linear(x[:T], w_down[:W]), slot_mapping, cache, u_cat, k_segs, eps)
        return
    torch.ops.lrkv_b200.proj_cache_write(x, w_down, slot_mapping, cache, u_cat, segs, float(eps))


def decompress_paged(cache: torch.Tensor, block_table_row: torch.Tensor, seq_len: int, pos0: int, count: int,
                     wk: torch.Tensor, k_segs, v_up_t: torch.Tensor, v_offset: int, cos_sin: torch.Tensor,
                     k_out: torch.Tensor | None = None, v_out: torch.Tensor | None = None):
    """Keys and values [count, G, D] BF16 of positions [pos0, pos0 + count) of one request, rebuilt from its latent rows
    in ``cache`` [blocks, page, W] (rows gathered through ``block_table_row``) on the tensor cores: the reference's
    ``LatentLayer.decompress`` (latent_backend.py:95-108) of the gathered rows (latent_backend.py:214-225). ``wk``
    [G, D, n_k * 64]: per group the rope rows of U_g times the gain, then the nope rows of qmap (``LatentLayer.wk``)."""
    G, D, kc = wk.shape
    r_v = v_up_t.shape[1]
    dev = cache.device
    if k_out is None:
        k_out = torch.empty(count, G, D, dtype=torch.bfloat16, device=dev)
    if v_out is None:
        v_out = torch.empty(count, G, D, dtype=torch.bfloat16, device=dev)
    if count == 0:
        return k_out, v_out
    if cache.dtype != torch.bfloat16 or cache.stride(-1) != 1 or block_table_row.dtype != torch.int32:
        raise ValueError("decompress_paged: BF16 cache with contiguous rows, int32 block table")
    if G != 4 or D != HEAD_DIM or not wk.is_contiguous() or not v_up_t.is_contiguous() or v_up_t.shape[0] != G:
        raise ValueError("decompress_paged: wk [4, 256, kc] and v_up [4, r_v, 256] contiguous")
    for name, t in (("k_out", k_out), ("v_out", v_out)):
        if t.dtype != torch.bfloat16 or tuple(t.shape) != (count, G, D) or t.stride(2) != 1:
            raise ValueError(f"decompress_paged: {name} [count, 4, 256] BF16 with contiguous channels")
    if k_out.stride() != v_out.stride():
        raise ValueError("decompress_paged: k_out and v_out with the same strides")
    torch.ops.lrkv_b200.decompress(cache, block_table_row, int(seq_len), int(pos0), wk, host_k_segs(k_segs), v_up_t,
                                   int(v_offset), cos_sin, k_out, v_out)
    return k_out, v_out


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_pos0: int, k_pos0: int, scale: float,
                      causal: bool = True, out: torch.Tensor | None = None, lse: torch.Tensor | None = None):
    """softmax(scale q k^T) v on the tensor cores for one request's new tokens: q [ql, 24, 256] BF16 at positions
    q_pos0.., k / v [S, 4, 256] BF16 at positions k_pos0.. (head h reads group h // 6), causal by position. Returns
    (out [ql, 24, 256] BF16, lse [ql, 24] fp32, natural log; -inf where a query sees no key). The operation of the
    reference's flash_attn_varlen_func call in its prefill path (latent_backend.py:285-320)."""
    ql, H, D = q.shape
    S = k.shape[0]
    dev = q.device
    if out is None:
        out = torch.empty(ql, H, D, dtype=torch.bfloat16, device=dev)
    if lse is None:
        lse = torch.empty(ql, H, dtype=torch.float32, device=dev)
    if ql == 0:
        return out, lse
    for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
        if t.dtype != torch.bfloat16 or t.dim() != 3 or t.shape[2] != HEAD_DIM or t.stride(2) != 1:
            raise ValueError(f"prefill_attention: {name} [n, heads, 256] BF16 with contiguous channels")
    if H != 24 or k.shape[1] != 4 or k.shape != v.shape or k.stride() != v.stride() or tuple(out.shape) != (ql, H, D):
        raise ValueError("prefill_attention: q [ql, 24, 256], k / v [S, 4, 256] with equal strides, out like q")
    if lse.dtype != torch.float32 or tuple(lse.shape) != (ql, H) or lse.stride(1) != 1:
        raise ValueError("prefill_attention: lse [ql, 24] fp32 with contiguous heads")
    torch.ops.lrkv_b200.prefill_attention(q, k, v, int(q_pos0), int(k_pos0), float(scale), bool(causal), out, lse)
    return out, lse
