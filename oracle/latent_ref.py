"""CPU restatement of BELT's latent-KV decode path — the parity oracle (test infrastructure, never shipped).

Every function restates one piece of the reference (``liuyaoyang04/BELT``), cited by file:line within that project:

* export format: ``lrkv/runtime/export_latent.py`` (``row_layout``, ``k_segments``, ``rope_basis``,
  ``build_latent_layer``);
* load-time constants: ``plugins/vllm_lrkv/vllm_lrkv/models/qwen3_5_latent.py:161-202`` (``derive_latent_tensors``)
  and ``cute_decode.py:635-646`` (``rope_blocks``);
* the cache write: ``latent_ops.py:85-135`` (``_latent_rows``);
* the absorbed query and V up-projection: ``latent_ops.py:23-81`` (``_group_gemm``);
* the reference's own torch attention path: ``latent_backend.py:95-108`` (``LatentLayer.decompress``) followed by
  causal softmax attention in fp32 (the CPU stand-in for ``flash_attn_varlen_func`` at ``latent_backend.py:290``);
* the split-KV schedule and merge: ``cute_decode.py:571-607`` and ``:681-722``.

Torch on the CPU (fp32 arithmetic, BF16 only where the reference stores BF16); numpy for the integer schedule.
"""

from __future__ import annotations

import math

import numpy as np
import torch

H, G, D, ROT, CHUNK = 24, 4, 256, 64, 64
HPG = H // G
ALIGN = 8

__all__ = [
    "H", "G", "D", "ROT", "CHUNK", "HPG", "ALIGN", "align", "k_segments", "row_layout", "rope_basis",
    "build_latent_layer", "rope_cos_sin", "derive", "rope_blocks", "latent_rows", "project_rows", "block_diag_query",
    "block_diag_query_construct", "up_project", "decompress", "attend", "gather_rows", "decode_reference",
    "decode_fp32", "q_norm_rope", "gate_mul", "schedule", "schedule_weighted", "decode_partials", "merge_segments", "decode_kernel_path",
]


def align(x: int, a: int = ALIGN) -> int:
    """``export_latent.py:112-113`` (``_align``)."""
    return -(-x // a) * a


def k_segments(k_head_ranks, rotary_dim, rope_align=False):
    """Cache columns of every group's latent coordinates as [start, length] runs (``export_latent.py:116-133``)."""
    if not rope_align:
        offsets = [sum(k_head_ranks[:g]) for g in range(len(k_head_ranks))]
        return [[[o, int(r)]] for o, r in zip(offsets, k_head_ranks)]
    rr = [min(rotary_dim, int(r)) for r in k_head_ranks]
    segs, col = [[] for _ in rr], 0
    for g in sorted(range(len(rr)), key=lambda g: -rr[g]):
        segs[g].append([col, rr[g]])
        col += rr[g]
    for g, r in enumerate(k_head_ranks):
        if r > rr[g]:
            segs[g].append([col, int(r) - rr[g]])
            col += int(r) - rr[g]
    return segs


def row_layout(k_head_ranks, v_rank, rotary_dim, rope_align=False):
    """Offsets of one compressed layer's cache row (``export_latent.py:143-166``)."""
    lk = sum(k_head_ranks)
    v_offset = align(lk)
    pe_offset = align(v_offset + v_rank)
    segs = k_segments(k_head_ranks, rotary_dim, rope_align)
    return {"k_head_ranks": list(k_head_ranks), "v_rank": int(v_rank), "lk": lk, "v_offset": v_offset,
            "pe_offset": pe_offset, "row_width": pe_offset,
            "rope_ranks": [min(rotary_dim, int(r)) for r in k_head_ranks], "k_segments": segs,
            "rope_offsets": [runs[0][0] for runs in segs]}


def rope_basis(U, rotary_dim):
    """Orthogonal Q with (U Q)[:rot, min(rot, r):] = 0 (``export_latent.py:169-176``)."""
    r = U.shape[1]
    if r <= rotary_dim:
        return torch.eye(r, dtype=torch.float64)
    Q, _ = torch.linalg.qr(U[:rotary_dim].double().T, mode="complete")
    return Q


def build_latent_layer(k_blocks, v_factors, num_kv_heads, head_dim, rotary_dim, dtype=torch.bfloat16,
                       rope_align=False):
    """(kv_latent_proj, k_up, v_up, layout) from per-group (VS_g, U_g) and joint (VS_v, U_v)
    (``export_latent.py:179-205``)."""
    ranks = [int(VS.shape[0]) for VS, _ in k_blocks]
    VS_v, U_v = (t.float() for t in v_factors)
    layout = row_layout(ranks, int(VS_v.shape[0]), rotary_dim, rope_align)
    hidden = int(VS_v.shape[1])
    proj = torch.zeros(layout["pe_offset"], hidden)
    k_up = torch.zeros(num_kv_heads, head_dim, max(ranks))
    for g, ((VS, U), r) in enumerate(zip(k_blocks, ranks)):
        Q = rope_basis(U, rotary_dim)
        VS, U = (Q.T @ VS.double()).float(), (U.double() @ Q).float()
        U[:rotary_dim, min(rotary_dim, r):] = 0.0
        i = 0
        for start, n in layout["k_segments"][g]:
            proj[start:start + n] = VS[i:i + n]
            i += n
        k_up[g, :, :r] = U
    proj[layout["v_offset"]:layout["v_offset"] + layout["v_rank"]] = VS_v
    return proj.to(dtype), k_up.to(dtype), U_v.to(dtype), layout


def rope_cos_sin(max_pos, rotary_dim, theta):
    """The NeoX ``cos_sin_cache`` [max_pos, rot] fp32 (cos half | sin half) the reference reads from the model's rotary
    embedding (``qwen3_5_latent.py:186``; vLLM ``RotaryEmbedding._compute_cos_sin_cache``)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, rotary_dim, 2, dtype=torch.float) / rotary_dim))
    t = torch.arange(max_pos, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


def rope_blocks(u_rot, groups):
    """[1, rot, n_blocks * 64] resident blocks of gain * B_g by 64-column chunk (``cute_decode.py:635-646``)."""
    blocks = []
    for U, (off, rr) in zip(u_rot, groups):
        for c in range(off // CHUNK, (off + rr - 1) // CHUNK + 1):
            blk = torch.zeros(ROT, CHUNK, dtype=U.dtype)
            lo, hi = max(off, c * CHUNK), min(off + rr, (c + 1) * CHUNK)
            blk[:, lo - c * CHUNK:hi - c * CHUNK] = U[:, lo - off:hi - off]
            blocks.append(blk)
    return torch.cat(blocks, dim=1).unsqueeze(0).contiguous()


def derive(k_up, v_up, k_norm_weight, layout, cos_sin, rotary_dim=ROT, eps=1e-6, dtype=torch.bfloat16):
    """Load-time constants of one compressed layer (``qwen3_5_latent.py:161-202``, k_segs ``:156-158``,
    rope groups ``:122``). ``cos_sin``: the fp32 table; it is stored in BF16 as the reference does (``:186``)."""
    G_, D_, _ = k_up.shape
    rot = rotary_dim
    gain = 1.0 + k_norm_weight.float()
    U = k_up.float()
    v_offset, r_v = layout["v_offset"], layout["v_rank"]
    segs = [[(int(a), int(n)) for a, n in runs] for runs in layout["k_segments"]]
    ranks = layout["k_head_ranks"]
    lk = sum(ranks)
    n_k = math.ceil(v_offset / CHUNK)
    qmap = torch.zeros(G_, D_, n_k * CHUNK + G_ * rot)
    u_cat = torch.zeros(lk, G_ * D_)
    for g, (runs, r) in enumerate(zip(segs, ranks)):
        cols = torch.cat([torch.arange(a, a + n) for a, n in runs])
        qmap[g, :rot, n_k * CHUNK + g * rot:n_k * CHUNK + (g + 1) * rot] = torch.eye(rot)
        qmap[g, rot:, cols] = gain[rot:, None] * U[g, rot:, :r]
        u_cat[cols, g * D_:(g + 1) * D_] = U[g, :, :r].T
    groups = tuple((runs[0][0], int(rr)) for runs, rr in zip(segs, layout["rope_ranks"]))
    u_rot = [gain[:rot, None] * U[g, :rot, :rr] for g, (off, rr) in enumerate(groups)]
    blocks = rope_blocks(u_rot, groups).to(dtype)
    rope_up = torch.zeros(G_, rot, n_k * CHUNK, dtype=dtype)
    for g, ((off, rr), u) in enumerate(zip(groups, u_rot)):
        rope_up[g, :, off:off + rr] = u.to(dtype)
    k_segs = torch.tensor([[x for run in runs + [(0, 0)] * (2 - len(runs)) for x in run] for runs in segs],
                          dtype=torch.int32)
    v_up_t = v_up.view(G_, D_, r_v).transpose(1, 2).contiguous()
    return {"num_kv_heads": G_, "head_dim": D_, "rotary_dim": rot, "v_rank": r_v, "v_offset": v_offset,
            "pe_offset": layout["pe_offset"], "n_k": n_k, "qmap": qmap.to(dtype), "v_up": v_up_t,
            "u_cat": u_cat.to(torch.bfloat16), "k_segs": k_segs, "rope_gain": gain[:rot].clone(), "eps": eps,
            "groups": groups, "blocks": blocks, "cos_sin": cos_sin.to(torch.bfloat16).contiguous(),
            "rope_up": rope_up, "k_up": k_up, "gain": gain}


# ---------------------------------------------------------------------------------------------------------------
# kernels of the path, restated
# ---------------------------------------------------------------------------------------------------------------

def latent_rows(c, slot_mapping, cache, u_cat, k_segs, eps):
    """In place on ``cache`` [blocks, page, W] (BF16): the rows [c_K / rho | c[lk:W]] of the new tokens at their
    slots; slot < 0 is padding (``latent_ops.py:85-135``; rho_g = rms over the 256 channels of U_g c_g, BF16
    operands with FP32 accumulation)."""
    T = slot_mapping.shape[0]
    lk, ngd = u_cat.shape
    ng = k_segs.shape[0]
    Dh = ngd // ng
    page, W = cache.shape[1], cache.shape[2]
    cf = c[:, :W].float()
    u = u_cat.float()
    for t in range(T):
        slot = int(slot_mapping[t])
        if slot < 0:
            continue
        blk, off = slot // page, slot % page
        row = cache[blk, off]
        row[lk:W] = c[t, lk:W].to(cache.dtype)
        for g in range(ng):
            a_lo, a_n, b_lo, b_n = (int(x) for x in k_segs[g])
            cols = torch.cat([torch.arange(a_lo, a_lo + a_n), torch.arange(b_lo, b_lo + b_n)])
            k_pre = cf[t, cols] @ u[cols, g * Dh:(g + 1) * Dh]
            inv = torch.rsqrt((k_pre * k_pre).sum() / Dh + eps)
            row[cols] = (cf[t, cols] * inv).to(cache.dtype)
    return cache


def project_rows(x, w_down, slot_mapping, cache, u_cat, k_segs, eps):
    """The model's down-projection followed by the cache write: c = bf16(x @ w_down^T) (``kv_latent_proj``,
    ``qwen3_5_latent.py:139-140, 213``: a BF16 linear with FP32 accumulation), then ``latent_rows``
    (``latent_ops.py:85-158``)."""
    W = cache.shape[2]
    c = (x.float() @ w_down[:W].float().t()).to(torch.bfloat16)
    return latent_rows(c, slot_mapping, cache, u_cat, k_segs, eps)


def block_diag_query(q, qmap):
    """q [T, H, D] x qmap[g] [D, KQ] per group -> [T, H, KQ] BF16 (FP32 accumulation; ``latent_ops.py:23-44,
    67-73``)."""
    T, H_, D_ = q.shape
    G_ = qmap.shape[0]
    hpg = H_ // G_
    out = torch.einsum("tgjd,gdk->tgjk", q.float().view(T, G_, hpg, D_), qmap.float())
    return out.reshape(T, H_, -1).to(q.dtype)


def block_diag_query_construct(q_lat, q_rot, k_off, k_ranks, lk_pad):
    """The reference construction of the block-diagonal query (``cute_decode.py:610-623``)."""
    B = q_lat.shape[0]
    n_k = math.ceil(lk_pad / CHUNK)
    q = torch.zeros(B, H, n_k * CHUNK + G * ROT, dtype=q_lat.dtype)
    for g in range(G):
        hs = slice(g * HPG, (g + 1) * HPG)
        q[:, hs, k_off[g]:k_off[g] + k_ranks[g]] = q_lat[:, hs, :k_ranks[g]]
        q[:, hs, n_k * CHUNK + g * ROT:n_k * CHUNK + (g + 1) * ROT] = q_rot[:, hs]
    return q


def up_project(a, v_up_t):
    """a [T, H, r_v] x v_up_t[g] [r_v, D] per head's group -> [T, H, D] BF16 (``latent_ops.py:76-81``)."""
    T, H_, R = a.shape
    G_ = v_up_t.shape[0]
    out = torch.einsum("tgjr,grd->tgjd", a.float().view(T, G_, H_ // G_, R), v_up_t.float())
    return out.reshape(T, H_, -1).to(torch.bfloat16)


def decompress(layer, rows, positions):
    """Rows [S, W] at positions [S] -> (k [S, G, D], v [S, G, D]) BF16 with RoPE channels first
    (``latent_backend.py:95-108``): gain * B_g c~ rounded to BF16, NeoX rotation in fp32, rounded again."""
    rot, n_k = layer["rotary_dim"], layer["n_k"]
    rows = rows.to(torch.bfloat16)
    kc = min(n_k * CHUNK, rows.shape[1])
    rf = rows[:, :kc].float()
    x = torch.einsum("sk,gdk->sgd", rf, layer["rope_up"][:, :, :kc].float()).to(torch.bfloat16).float()
    cos, sin = layer["cos_sin"][positions].float().unsqueeze(1).chunk(2, dim=-1)
    x1, x2 = x.chunk(2, dim=-1)
    k_pe = torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(torch.bfloat16)
    k_nope = torch.einsum("sk,gdk->sgd", rf, layer["qmap"][:, rot:, :kc].float()).to(torch.bfloat16)
    vo, vr = layer["v_offset"], layer["v_rank"]
    v = torch.einsum("sr,grd->sgd", rows[:, vo:vo + vr].float(), layer["v_up"].float()).to(torch.bfloat16)
    return torch.cat((k_pe, k_nope), dim=-1), v


def attend(q, k, v, scale):
    """One decode query per request over its whole context, fp32: q [H, D], k/v [S, G, D] (head h reads group
    h // HPG)."""
    H_ = q.shape[0]
    G_ = k.shape[1]
    kh = k.float().repeat_interleave(H_ // G_, dim=1)       # [S, H, D]
    vh = v.float().repeat_interleave(H_ // G_, dim=1)
    s = torch.einsum("hd,shd->hs", q.float(), kh) * scale
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hs,shd->hd", p, vh)


def gather_rows(cache, block_table, b, n):
    """The first n rows of request b through its block table, with their positions (``latent_backend.py:214-225``:
    position pos sits in block ``block_table[b, pos // page]`` at offset ``pos % page``)."""
    page = cache.shape[1]
    pos = torch.arange(n)
    blk = block_table[b, pos // page].long()
    return cache[blk, pos % page], pos


def decode_reference(q, cache, block_table, seq_lens, layer, scale):
    """Oracle A: the reference's torch latent path — ``decompress`` of every context row, then fp32 attention.
    q [B, H, D] (normed, rotated) -> [B, H, D] fp32; a request of length 0 gives zeros."""
    B = q.shape[0]
    out = torch.zeros(B, q.shape[1], layer["head_dim"])
    for b in range(B):
        n = int(seq_lens[b])
        if n == 0:
            continue
        rows, pos = gather_rows(cache, block_table, b, n)
        k, v = decompress(layer, rows, pos)
        out[b] = attend(q[b], k, v, scale)
    return out


def decode_fp32(q, cache, block_table, seq_lens, layer, scale):
    """Oracle B: the same attention with no rounding besides the stored inputs (cache rows, factors, cos/sin table):
    k_g(j) = gain * U_g c~_g(j) over all 256 channels, RoPE on the first rot, v_g(j) = U_v,g c_v(j)."""
    rot = layer["rotary_dim"]
    B = q.shape[0]
    gain = layer["gain"]
    U = layer["k_up"].float()
    Uv = layer["v_up"].float()                      # [G, r_v, D]
    segs = layer["k_segs"]
    vo, vr = layer["v_offset"], layer["v_rank"]
    out = torch.zeros(B, q.shape[1], layer["head_dim"])
    for b in range(B):
        n = int(seq_lens[b])
        if n == 0:
            continue
        rows, pos = gather_rows(cache, block_table, b, n)
        rows = rows.float()
        ks = []
        for g in range(layer["num_kv_heads"]):
            a_lo, a_n, b_lo, b_n = (int(x) for x in segs[g])
            cols = torch.cat([torch.arange(a_lo, a_lo + a_n), torch.arange(b_lo, b_lo + b_n)])
            r = len(cols)
            kg = (rows[:, cols] @ U[g, :, :r].T) * gain           # [S, D]
            cos, sin = layer["cos_sin"][pos].float().chunk(2, dim=-1)
            x1, x2 = kg[:, :rot // 2], kg[:, rot // 2:rot]
            kg = torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin, kg[:, rot:]), dim=-1)
            ks.append(kg)
        k = torch.stack(ks, dim=1)
        v = torch.einsum("sr,grd->sgd", rows[:, vo:vo + vr], Uv)
        out[b] = attend(q[b].float(), k, v, scale)
    return out


def q_norm_rope(qg, norm_weight, eps, cos_sin, positions):
    """The query side of the model's fused q-norm / RoPE (``models/qwen3_5_latent.py:209-212``): qg [T, H, >= D] ->
    [T, H, D] BF16 = NeoX rotation of the first rot channels (cos_sin [max_pos, rot] BF16, cos then sin) of
    x * rsqrt(mean(x^2) + eps) * (1 + w) (the Qwen3.5 zero-centred RMSNorm), fp32 throughout, one BF16 rounding."""
    D_ = norm_weight.shape[0]
    x = qg[..., :D_].float()
    x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * (1.0 + norm_weight.float())
    rot = cos_sin.shape[1]
    cs = cos_sin[positions.long()].float()                    # [T, rot]
    cos, sin = cs[:, None, :rot // 2], cs[:, None, rot // 2:]
    x1, x2 = x[..., :rot // 2], x[..., rot // 2:rot]
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin, x[..., rot:]), dim=-1).to(torch.bfloat16)


def gate_mul(attn, gate):
    """attn * sigmoid(gate) (``models/qwen3_5_latent.py:215``), fp32, BF16 out."""
    return (attn.float() * torch.sigmoid(gate.float())).to(torch.bfloat16)


def schedule(seq_lens, num_ctas, tile, min_tiles=1, capacity=None):
    """Split of every request's ``tile``-token tiles into equal runs per CTA (``cute_decode.py:571-607``).

    Returns (work [capacity, 4] = (request, first tile, end tile, 0), cta_seg [num_ctas + 1], seg_base [B + 1]),
    int32; entries past the live segments are zero."""
    seq = np.asarray(seq_lens, dtype=np.int64).reshape(-1)
    B = seq.shape[0]
    capacity = capacity or (B + num_ctas)
    tiles = (seq + tile - 1) // tile
    first = np.cumsum(tiles) - tiles
    total_tiles = int(tiles.sum())
    per = max(max(-(-total_tiles // num_ctas), min_tiles), 1)
    cta0 = first // per
    nseg = np.where(tiles > 0, (first + tiles - 1) // per - cta0 + 1, 0)
    base = np.cumsum(nseg) - nseg
    total = int(nseg.sum())
    work = np.zeros((capacity, 4), dtype=np.int32)
    cta_seg = np.zeros(num_ctas + 1, dtype=np.int32)
    seg_base = np.zeros(B + 1, dtype=np.int32)
    seg_base[:B] = base
    seg_base[B] = total
    for b in range(B):
        for j in range(int(nseg[b])):
            cta = int(cta0[b]) + j
            g0 = max(int(first[b]), cta * per)
            g1 = min(int(first[b] + tiles[b]), (cta + 1) * per)
            k = int(base[b]) + j
            work[k] = (b, g0 - first[b], g1 - first[b], 0)
            if g0 == cta * per:
                cta_seg[cta] = k
    for c in range(num_ctas + 1):
        if c * per >= total_tiles:
            cta_seg[c] = total
    return work, cta_seg, seg_base


def schedule_weighted(seq_lens, num_ctas, tile, start_cost, min_tiles=1, capacity=None):
    """The cost-weighted split of the decode kernel's schedule (this package's own refinement of
    ``cute_decode.py:571-607``): tiles in request order cost 8 units each and every request's first tile
    ``start_cost`` more; CTA c takes the tiles whose cost starts in [c * per, (c + 1) * per), per = max(ceil(total
    cost / num_ctas), 8 * min_tiles, 8); a CTA's tiles of one request form one segment. Same outputs as ``schedule``
    (which this equals for start_cost 0 only up to the unit: use ``schedule`` for the reference's split). Written
    tile by tile, independently of the kernel's closed forms."""
    seq = np.asarray(seq_lens, dtype=np.int64).reshape(-1)
    B = seq.shape[0]
    capacity = capacity or (B + num_ctas)
    tiles = (seq + tile - 1) // tile
    total_cost = int(sum(start_cost + 8 * t for t in tiles if t > 0))
    per = max(-(-total_cost // num_ctas), 8 * min_tiles, 8)
    segs = []                                   # (request, cta, first tile, end tile)
    cost = 0
    for b in range(B):
        t = int(tiles[b])
        if t == 0:
            continue
        cost += start_cost
        for k in range(t):
            cta = cost // per
            if segs and segs[-1][0] == b and segs[-1][1] == cta:
                segs[-1][3] = k + 1
            else:
                segs.append([b, cta, k, k + 1])
            cost += 8
    work = np.zeros((capacity, 4), dtype=np.int32)
    cta_seg = np.zeros(num_ctas + 1, dtype=np.int32)
    seg_base = np.zeros(B + 1, dtype=np.int32)
    for k, (b, cta, k0, k1) in enumerate(segs):
        work[k] = (b, k0, k1, 0)
    for b in range(B + 1):
        seg_base[b] = sum(1 for sg in segs if sg[0] < b)
    for c in range(num_ctas + 1):
        cta_seg[c] = sum(1 for sg in segs if sg[1] < c)
    return work, cta_seg, seg_base


def decode_partials(q_bd, cache, block_table, seq_lens, layer, work, num_segments, scale, tile):
    """The per-segment partial outputs the split-KV kernel writes (``cute_decode.py:310-455``), rounded as that
    kernel rounds: the rebuilt RoPE key to BF16 before and after the rotation (``:473-484``), P to BF16 before P.V
    (``:408``); fp32 scores, sums and accumulators.

    q_bd [B, H, KQ] (BF16) -> part [num_segments, H, r_v + 1] fp32: the normalised latent V-space output and the
    natural-log LSE of the scaled scores."""
    rot, n_k = layer["rotary_dim"], layer["n_k"]
    vo, vr = layer["v_offset"], layer["v_rank"]
    groups = layer["groups"]
    U = layer["k_up"].float() * layer["gain"][None, :, None]
    part = torch.zeros(num_segments, H, vr + 1)
    for s in range(num_segments):
        b, t0, t1 = (int(x) for x in work[s, :3])
        end = min(t1 * tile, int(seq_lens[b]))
        n0 = t0 * tile
        if end <= n0:
            continue
        rows, pos = gather_rows(cache, block_table, b, end)
        rows, pos = rows[n0:end].float(), pos[n0:end]
        qb = q_bd[b].float()                                           # [H, KQ]
        sc = rows[:, :n_k * CHUNK] @ qb[:, :n_k * CHUNK].T              # [S, H]
        cos, sin = layer["cos_sin"][pos].float().chunk(2, dim=-1)
        for g, (off, rr) in enumerate(groups):
            kr = (rows[:, off:off + rr] @ U[g, :rot, :rr].to(torch.bfloat16).float().T)
            kr = kr.to(torch.bfloat16).float()
            x1, x2 = kr[:, :rot // 2], kr[:, rot // 2:]
            kp = torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(torch.bfloat16).float()
            hs = slice(g * HPG, (g + 1) * HPG)
            sc[:, hs] += kp @ qb[hs, n_k * CHUNK + g * ROT:n_k * CHUNK + (g + 1) * ROT].T
        z = sc * scale
        m = z.max(dim=0).values                                         # [H]
        p = torch.exp(z - m)
        den = p.sum(dim=0)
        acc = p.to(torch.bfloat16).float().T @ rows[:, vo:vo + vr]      # [H, r_v]
        part[s, :, :vr] = acc / den[:, None]
        part[s, :, vr] = m + torch.log(den)
    return part


def merge_segments(part, seg_base, B, lv):
    """LSE merge of every request's segments -> (a [B, H, lv] fp32, lse [B, H]); a request without segments gives
    zeros and -inf (``cute_decode.py:681-712``)."""
    a = torch.zeros(B, part.shape[1], lv)
    lse = torch.full((B, part.shape[1]), float("-inf"))
    for b in range(B):
        s0, s1 = int(seg_base[b]), int(seg_base[b + 1])
        if s1 <= s0:
            continue
        l = part[s0:s1, :, lv]                                          # [n, H]
        m = l.max(dim=0).values
        w = torch.exp(l - m)
        den = w.sum(dim=0)
        a[b] = (w[:, :, None] * part[s0:s1, :, :lv]).sum(dim=0) / den[:, None]
        lse[b] = m + torch.log(den)
    return a, lse


def decode_kernel_path(q, cache, block_table, seq_lens, layer, scale, tile, num_ctas):
    """The whole decode chain the backend runs (``latent_backend.py:274-284``), restated on the CPU with the
    kernels' rounding points: block-diagonal query -> split-KV partials -> merge -> BF16 a -> U_v.
    Returns (out [B, H, D] BF16, a [B, H, r_v] BF16, lse [B, H] fp32, q_bd)."""
    B = q.shape[0]
    q_bd = block_diag_query(q, layer["qmap"])
    work, cta_seg, seg_base = schedule(seq_lens, num_ctas, tile)
    nseg = int(seg_base[B])
    part = decode_partials(q_bd, cache, block_table, seq_lens, layer, work, nseg, scale, tile)
    a, lse = merge_segments(part, seg_base, B, layer["v_rank"])
    a = a.to(torch.bfloat16)
    out = up_project(a, layer["v_up"])
    return out, a, lse, q_bd
