"""GPU parity of the sm_100a kernels against the CPU oracle and the reference's golden outputs.

Tolerances: the schedule and the cache-row placement are compared bit for bit; cache-row values within 1 BF16 ulp
(the reference's rsqrt and dot order are not bit-defined); the attention output within max-abs 2e-2 and mean-abs 2e-3
of the fp32 oracle (the north-star bound for BF16).
"""

import math

import pytest
import torch

import oracle
from belt_b200 import decode as dec
from belt_b200 import _lib, latent_ops, synth
from belt_b200.latent_backend import (CommonAttentionMetadata, LatentAttentionImpl, LatentAttentionMetadataBuilder,
                                      LatentKVSpec, latent_attention_step)
from belt_b200.layer import derive_latent_tensors

from conftest import CASES, bf16_ulp_close, golden_case

pytestmark = pytest.mark.gpu
SCALE = 256 ** -0.5
MAX_ABS, MEAN_ABS = 2e-2, 2e-3
DEV = "cuda"


def layer_pair(w, max_pos=4096, device=DEV):
    cos_sin = synth.cos_sin_table(max_pos)
    lat = derive_latent_tensors(w.k_up, w.v_up, w.k_norm_weight, w.layout, cos_sin, device=device)
    ref = oracle.derive(w.k_up, w.v_up, w.k_norm_weight, w.layout, cos_sin)
    return lat, ref


def run_decode(lat, q, cache, block_table, seq_lens, num_ctas=None):
    """The backend's decode chain on the device; returns (out, a, lse, part, sched)."""
    B = q.shape[0]
    sched = dec.make_schedule(B, q.device, num_ctas=num_ctas)
    dec.schedule(sched, seq_lens)
    q_bd = lat.block_diag_query(q)
    part = torch.full((B + sched.num_ctas, 24, lat.v_rank + 1), float("nan"), device=q.device)
    dec.latent_decode(q_bd, cache, block_table, seq_lens, sched, part, SCALE, lat.v_offset, lat.v_rank, rope=lat.rope)
    a = torch.empty(B, 24, lat.v_rank, dtype=torch.bfloat16, device=q.device)
    lse = torch.empty(B, 24, device=q.device)
    dec.merge_segments(part, sched, a, lse)
    out = torch.empty(B, 24, 256, dtype=torch.bfloat16, device=q.device)
    lat.up_project(a, out)
    torch.cuda.synchronize()
    dec.check_device_errors(q.device)
    return out, a, lse, part, sched, q_bd


def assert_close_out(out, ref, what=""):
    err = (out.float().cpu() - ref.float().cpu()).abs()
    assert torch.isfinite(out.float()).all(), f"{what}: non-finite output"
    assert float(err.max()) < MAX_ABS and float(err.mean()) < MEAN_ABS, (what, float(err.max()), float(err.mean()))


# ------------------------------------------------------------------------------------------------- schedule
@pytest.mark.parametrize("seqs,nct", [
    ([129, 513, 1025, 2001], 148), ([1, 17, 129, 300], 8), ([0, 64, 0, 65, 4096, 1], 16), ([8192] * 64, 148),
    ([5], 148), ([0, 0], 4), ([3000, 1, 1, 1, 7000, 64, 63, 65], 148), ([200] * 300, 148), ([128, 256, 127], 1),
    (list(range(0, 3000, 7)), 148),
])
def test_schedule_bit_exact(seqs, nct):
    """The reference's split (start_cost 0)."""
    B = len(seqs)
    sched = dec.make_schedule(B, DEV, num_ctas=nct, start_cost=0)
    sched.work.fill_(-7)
    dec.schedule(sched, torch.tensor(seqs, dtype=torch.int32, device=DEV))
    work, cta_seg, seg_base = oracle.schedule(seqs, nct, dec.TILE_T)
    total = int(seg_base[-1])
    torch.cuda.synchronize()
    assert torch.equal(sched.seg_base.cpu(), torch.from_numpy(seg_base))
    assert torch.equal(sched.cta_seg.cpu(), torch.from_numpy(cta_seg))
    assert torch.equal(sched.work[:total].cpu(), torch.from_numpy(work[:total]))


@pytest.mark.parametrize("start_cost", [1, dec.SCHEDULE_START_COST, 16, 1024])
@pytest.mark.parametrize("seqs,nct", [
    ([129, 513, 1025, 2001], 148), ([1, 17, 129, 300], 8), ([0, 64, 0, 65, 4096, 1], 16), ([8192] * 64, 148),
    ([5], 148), ([0, 0], 4), ([3000, 1, 1, 1, 7000, 64, 63, 65], 148), ([200] * 300, 148), ([128, 256, 127], 1),
    (list(range(0, 3000, 7)), 148),
])
def test_schedule_weighted_bit_exact(seqs, nct, start_cost):
    """The cost-weighted split against the oracle's tile-by-tile restatement."""
    B = len(seqs)
    sched = dec.make_schedule(B, DEV, num_ctas=nct, start_cost=start_cost)
    sched.work.fill_(-7)
    dec.schedule(sched, torch.tensor(seqs, dtype=torch.int32, device=DEV))
    work, cta_seg, seg_base = oracle.schedule_weighted(seqs, nct, dec.TILE_T, start_cost)
    total = int(seg_base[-1])
    torch.cuda.synchronize()
    assert torch.equal(sched.seg_base.cpu(), torch.from_numpy(seg_base))
    assert torch.equal(sched.cta_seg.cpu(), torch.from_numpy(cta_seg))
    assert torch.equal(sched.work[:total].cpu(), torch.from_numpy(work[:total]))


def balanced_split(seqs, nct, start_cost, w, tile=128, unit=8):
    """The balanced split restated tile by tile: CTA c takes the tiles whose cost position x_b + s0 + 8 k falls in
    [B_c, B_(c+1)), B_c = per * nct * W_c // W with W_c the prefix sums of the fixed-point weights."""
    import numpy as np
    tiles = [(L + tile - 1) // tile for L in seqs]
    cost = [start_cost + unit * t if t > 0 else 0 for t in tiles]
    total = sum(cost)
    per = max(-(-total // nct), unit, unit)
    wq = [int(np.float32(np.float32(x) * np.float32(1048576.0) + np.float32(0.5))) for x in w]
    pre = [0]
    for q in wq:
        pre.append(pre[-1] + q)
    bounds = [per * nct * p // pre[-1] for p in pre]
    owner = lambda pos: max(c for c in range(nct) if bounds[c] <= pos)
    work, seg_base, seg_cta = [], [], []
    x = 0
    for b, t in enumerate(tiles):
        seg_base.append(len(work))
        prev = None
        for k in range(t):
            c = owner(x + start_cost + unit * k)
            if c != prev:
                work.append([b, k, k + 1, 0])
                seg_cta.append(c)
                prev = c
            else:
                work[-1][2] = k + 1
        x += cost[b]
    seg_base.append(len(work))
    cta_seg = [next((i for i, c in enumerate(seg_cta) if c >= cc), len(work)) for cc in range(nct + 1)]
    return work, cta_seg, seg_base, bounds, wq


@pytest.mark.parametrize("seqs,nct", [([8192] * 64, 148), ([3000, 1, 1, 1, 7000, 64, 63, 65] * 20, 148),
                                      ([200] * 300, 148), (list(range(1000, 60000, 997)), 100)])
def test_schedule_balanced(seqs, nct):
    """The balanced split: a fresh schedule is the weighted split; after a step whose CTAs ran at different speeds the
    weights follow cap / ns (as belt_decode_schedule_balanced documents, in the same fp32 / fixed-point arithmetic),
    the work follows the weights tile by tile, and the times are zeroed for the next step."""
    import numpy as np
    B, sc = len(seqs), dec.SCHEDULE_START_COST
    sched = dec.make_schedule(B, DEV, num_ctas=nct, start_cost=sc, balance=True)
    sl = torch.tensor(seqs, dtype=torch.int32, device=DEV)
    dec.schedule(sched, sl)
    work, cta_seg, seg_base = oracle.schedule_weighted(seqs, nct, dec.TILE_T, sc)
    assert torch.equal(sched.cta_seg.cpu(), torch.from_numpy(cta_seg))
    assert torch.equal(sched.work[:int(seg_base[-1])].cpu(), torch.from_numpy(work[:int(seg_base[-1])]))
    for step in range(3):
        cap = sched.cta_cap.cpu().double()
        speed = 1.0 + 0.2 * torch.sin(torch.arange(nct, dtype=torch.float64) * (1.7 + step))
        ns = (cap / speed * 1000.0).round().long()
        sched.cta_ns.copy_(ns.to(DEV))
        w_prev = sched.cta_w.cpu().numpy()
        dec.schedule(sched, sl)
        torch.cuda.synchronize()
        tiles = [(L + dec.TILE_T - 1) // dec.TILE_T for L in seqs]
        per = max(-(-sum(sc + 8 * t for t in tiles if t > 0) // nct), 8)
        if per < 64:   # under 8 tiles a CTA the weights are not used: the weighted split, weights unchanged
            assert torch.equal(sched.cta_seg.cpu(), torch.from_numpy(cta_seg)), step
            assert np.array_equal(sched.cta_w.cpu().numpy(), w_prev) and not sched.cta_ns.cpu().any()
            assert sched.cta_cap.cpu().tolist() == [per] * nct
            continue
        rq = [int(float(c) / float(n) * 1e9) for c, n in zip(cap.tolist(), ns.tolist())]
        mean = sum(rq) / nct
        f32 = np.float32
        w = [min(max(f32(f32(0.5) * f32(wp) + f32(0.5) * f32(q / mean)), f32(0.8)), f32(1.25))
             for wp, q in zip(w_prev, rq)]
        ework, ecta, ebase, bounds, wq = balanced_split(seqs, nct, sc, w)
        assert sched.seg_base[:B + 1].cpu().tolist() == ebase, step
        assert sched.cta_seg.cpu().tolist() == ecta, step
        assert sched.work[:ebase[-1]].cpu().tolist() == ework, step
        assert sched.cta_cap.cpu().tolist() == [bounds[c + 1] - bounds[c] for c in range(nct)]
        assert not sched.cta_ns.cpu().any()
        got_w = sched.cta_w.cpu().numpy()
        assert np.allclose(got_w, np.array(wq, dtype=np.float64) * nct / sum(wq), rtol=1e-6)
        assert abs(got_w.mean() - 1.0) < 1e-5 and got_w.min() > 0.7 and got_w.max() < 1.4
        # slower CTAs (higher ns per cost) get less: weights move with the speeds
        if step == 0:
            assert np.corrcoef(got_w, speed.numpy())[0, 1] > 0.9


# ------------------------------------------------------------------------------------------------- cache write
@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("slot_dtype", [torch.int64, torch.int32])
def test_cache_write(name, slot_dtype):
    fx, spec, w, batch, q = golden_case(name)
    lat, ref = layer_pair(w)
    W = w.layout["row_width"]
    page = fx["page"]
    gcw = torch.Generator().manual_seed(9)
    c = (torch.randn(24, W, generator=gcw) * synth.latent_columns(w.layout)).to(torch.bfloat16)
    slots = fx["cw_slots"]
    nb = fx["cw_nb"]
    init = torch.full((nb, page, W), float("nan")).to(torch.bfloat16)
    init.view(-1, W)[::3] = 1.5                           # some untouched rows with finite content
    exp = oracle.latent_rows(c, slots, init.clone(), ref["u_cat"], ref["k_segs"], 1e-6)
    cache = init.clone().to(DEV)
    latent_ops.latent_rows_to_cache(c.to(DEV), slots.to(slot_dtype).to(DEV), cache, lat.u_cat, lat.k_segs, 1e-6)
    torch.cuda.synchronize()
    got = cache.cpu()
    live = slots >= 0
    written = slots[live].long()
    untouched = torch.ones(nb * page, dtype=torch.bool)
    untouched[written] = False
    # placement: every untouched row is bit-identical, every written row lands in its slot
    assert torch.equal(got.view(-1, W)[untouched].view(torch.int16), init.view(-1, W)[untouched].view(torch.int16))
    assert bf16_ulp_close(got.view(-1, W)[written], exp.view(-1, W)[written], ulps=1)
    assert bf16_ulp_close(got.view(-1, W)[written], fx["cw_rows"], ulps=1)


def test_cache_write_strided_view_and_padding():
    spec = synth.c50()
    w = synth.make_layer(spec)
    lat, ref = layer_pair(w)
    W = w.layout["row_width"]
    page, nb, layers = 16, 40, 3
    buf = torch.zeros(nb, layers * page * W, dtype=torch.bfloat16, device=DEV)
    view = buf.view(nb, layers, page, W)[:, 1]                    # the middle layer's pages, block stride 3 pages
    T = 300
    g = torch.Generator().manual_seed(4)
    c = (torch.randn(T, W + 64, generator=g) * torch.cat([synth.latent_columns(w.layout), torch.ones(64)])).to(
        torch.bfloat16)
    slots = torch.randperm(nb * page, generator=g)[:T]
    slots[::7] = -1
    latent_ops.latent_rows_to_cache(c.to(DEV), slots.to(DEV), view, lat.u_cat, lat.k_segs, 1e-6)
    exp = oracle.latent_rows(c[:, :W], slots, torch.zeros(nb, page, W, dtype=torch.bfloat16), ref["u_cat"],
                             ref["k_segs"], 1e-6)
    torch.cuda.synchronize()
    full = buf.view(nb, layers, page, W).cpu()
    assert bf16_ulp_close(full[:, 1], exp, ulps=1)
    assert not full[:, 0].any() and not full[:, 2].any()          # neighbouring layers untouched


def test_cache_write_prefill_chunk_and_unaligned_inputs():
    """The cache write at prefill size (an 8192-token chunk, sampled against the oracle; the tensor-core fold), with c
    rows that are not 16-byte aligned (element loads), and with a u_cat that is not 16-byte aligned (the SIMT
    kernel). Values within 1 BF16 ulp, rows never written left zero."""
    spec = synth.c50()
    w = synth.make_layer(spec)
    lat, ref = layer_pair(w)
    W = w.layout["row_width"]
    page = 16
    g = torch.Generator().manual_seed(31)
    cols = torch.cat([synth.latent_columns(w.layout), torch.ones(8)])
    u_off = torch.empty(lat.u_cat.numel() + 1, dtype=torch.bfloat16, device=DEV)[1:].view_as(lat.u_cat)
    u_off.copy_(lat.u_cat)
    for T, c_off, u_cat in ((8192, 0, lat.u_cat), (300, 1, lat.u_cat), (300, 0, u_off)):
        nb = T // page + 8
        c_full = (torch.randn(T, W + 8, generator=g) * cols).to(torch.bfloat16)
        c = c_full[:, c_off:c_off + W]
        slots = torch.randperm(nb * page, generator=g)[:T]
        slots[::11] = -1
        cache = torch.zeros(nb, page, W, dtype=torch.bfloat16, device=DEV)
        c_dev = c_full.to(DEV)[:, c_off:c_off + W]
        before = _lib.path_counts()["simt_cache_write"]
        latent_ops.latent_rows_to_cache(c_dev, slots.to(DEV), cache, u_cat, lat.k_segs, 1e-6)
        torch.cuda.synchronize()
        assert _lib.path_counts()["simt_cache_write"] == before + (u_cat is u_off)     # only the misaligned u_cat
        live = torch.nonzero(slots >= 0).flatten()
        sample = live[torch.randperm(live.numel(), generator=g)[:256]]
        exp = oracle.latent_rows(c[sample], slots[sample], torch.zeros(nb, page, W, dtype=torch.bfloat16),
                                 ref["u_cat"], ref["k_segs"], 1e-6)
        got = cache.cpu().view(-1, W)
        assert bf16_ulp_close(got[slots[sample]], exp.view(-1, W)[slots[sample]], ulps=1), (T, c_off)
        written = torch.zeros(nb * page, dtype=torch.bool)
        written[slots[slots >= 0]] = True
        assert not got[~written].any(), (T, c_off)


# ------------------------------------------------------------------------------------------------- fused down-projection
# The kernel rounds c = x W_down^T to BF16 after an FP32 sum over `hidden` terms in another order than the oracle's
# (the reference's own cuBLAS linear has the same freedom). An element of c can then sit one BF16 ulp away, and the
# folded value c * inv at most 2 ulps; near zero the sum's own error, ~sqrt(hidden) * 2^-24 * sum|x w| (~1e-5 for
# hidden = 1024 and unit-scale rows), dominates the ulp, hence the absolute floor PROJ_ATOL. Placement stays bit-exact.
PROJ_ATOL = 2e-5


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("slot_dtype", [torch.int64, torch.int32])
def test_proj_write(name, slot_dtype):
    fx, spec, w, batch, q = golden_case(name)
    lat, ref = layer_pair(w)
    W = w.layout["row_width"]
    page, nb = fx["page"], fx["cw_nb"]
    slots = fx["cw_slots"]
    T = slots.shape[0]
    x = torch.randn(T, spec.hidden, generator=torch.Generator().manual_seed(11)).to(torch.bfloat16)
    init = torch.full((nb, page, W), float("nan")).to(torch.bfloat16)
    init.view(-1, W)[::3] = 1.5
    exp = oracle.project_rows(x, w.kv_latent_proj, slots, init.clone(), ref["u_cat"], ref["k_segs"], 1e-6)
    cache = init.clone().to(DEV)
    latent_ops.project_rows_to_cache(x.to(DEV), w.kv_latent_proj.to(DEV), slots.to(slot_dtype).to(DEV), cache,
                                     lat.u_cat, lat.k_segs, 1e-6)
    torch.cuda.synchronize()
    dec.check_device_errors(DEV)
    got = cache.cpu()
    written = slots[slots >= 0].long()
    untouched = torch.ones(nb * page, dtype=torch.bool)
    untouched[written] = False
    assert torch.equal(got.view(-1, W)[untouched].view(torch.int16), init.view(-1, W)[untouched].view(torch.int16))
    assert bf16_ulp_close(got.view(-1, W)[written], exp.view(-1, W)[written], ulps=2, atol=PROJ_ATOL)


def test_proj_write_strided_view_multi_tile():
    """300 tokens (three 128-token tiles, the last one ragged), padding slots, the middle layer of a block-outermost
    buffer: neighbouring layers stay zero."""
    spec = synth.spec_from_ranks(448, 576)
    w = synth.make_layer(spec)
    lat, ref = layer_pair(w)
    W = w.layout["row_width"]
    page, nb, layers = 16, 40, 3
    buf = torch.zeros(nb, layers, page, W, dtype=torch.bfloat16, device=DEV)
    view = buf[:, 1]
    T = 300
    g = torch.Generator().manual_seed(4)
    x = torch.randn(T, spec.hidden, generator=g).to(torch.bfloat16)
    slots = torch.randperm(nb * page, generator=g)[:T]
    slots[::7] = -1
    latent_ops.project_rows_to_cache(x.to(DEV), w.kv_latent_proj.to(DEV), slots.to(DEV), view, lat.u_cat,
                                     lat.k_segs, 1e-6)
    exp = oracle.project_rows(x, w.kv_latent_proj, slots, torch.zeros(nb, page, W, dtype=torch.bfloat16),
                              ref["u_cat"], ref["k_segs"], 1e-6)
    torch.cuda.synchronize()
    dec.check_device_errors(DEV)
    full = buf.cpu()
    assert bf16_ulp_close(full[:, 1], exp, ulps=2, atol=PROJ_ATOL)
    assert not full[:, 0].any() and not full[:, 2].any()


@pytest.mark.parametrize("fused", [True, False])
def test_proj_write_prefill_chunk(fused):
    """An 8192-token chunk (the chunked-prefill write), checked on a sample of 256 tokens against the oracle: through the
    fused kernel, and as a library GEMM + the cache write (the default at this size)."""
    spec = synth.c50()
    w = synth.make_layer(spec)
    lat, ref = layer_pair(w)
    W = w.layout["row_width"]
    T, page = 8192, 16
    nb = T // page + 8
    g = torch.Generator().manual_seed(12)
    x = torch.randn(T, spec.hidden, generator=g).to(torch.bfloat16)
    slots = torch.randperm(nb * page, generator=g)[:T]
    cache = torch.zeros(nb, page, W, dtype=torch.bfloat16, device=DEV)
    latent_ops.project_rows_to_cache(x.to(DEV), w.kv_latent_proj.to(DEV), slots.to(DEV), cache, lat.u_cat,
                                     lat.k_segs, 1e-6, fused=fused)
    torch.cuda.synchronize()
    dec.check_device_errors(DEV)
    sample = torch.randperm(T, generator=g)[:256]
    exp = oracle.project_rows(x[sample], w.kv_latent_proj, slots[sample], torch.zeros(nb, page, W,
                              dtype=torch.bfloat16), ref["u_cat"], ref["k_segs"], 1e-6)
    got = cache.cpu().view(-1, W)[slots[sample]]
    assert bf16_ulp_close(got, exp.view(-1, W)[slots[sample]], ulps=2, atol=PROJ_ATOL)
    written = torch.zeros(nb * page, dtype=torch.bool)
    written[slots] = True
    assert not cache.cpu().view(-1, W)[~written].any()


# ------------------------------------------------------------------------------------------------- query / up-projection
@pytest.mark.parametrize("name", CASES)
def test_block_diag_query(name):
    fx, spec, w, batch, q = golden_case(name)
    lat, ref = layer_pair(w)
    exp = oracle.block_diag_query(q, ref["qmap"])
    got = lat.block_diag_query(q.to(DEV)).cpu()
    assert bf16_ulp_close(got, exp, ulps=1)
    assert bf16_ulp_close(got, fx["q_bd"], ulps=1)
    dense = latent_ops.block_diag_query(q.to(DEV), lat.qmap).cpu()  # the full product gives the same query
    assert bf16_ulp_close(dense, exp, ulps=1)


def test_block_diag_query_fallback_is_counted():
    """A query whose token stride is not a multiple of 16 bytes cannot be described by TMA: the product runs on the
    CUDA-core kernel, gives the same values, and the library's path count says so."""
    fx, spec, w, batch, q = golden_case(CASES[0])
    lat, ref = layer_pair(w)
    T = q.shape[0]
    buf = torch.zeros(T, 24 * 256 + 1, dtype=torch.bfloat16, device=DEV)
    q_odd = buf.as_strided((T, 24, 256), (24 * 256 + 1, 256, 1))
    q_odd.copy_(q)
    before = _lib.path_counts()
    got = lat.block_diag_query(q_odd).cpu()
    after = _lib.path_counts()
    assert after["simt_group_gemm"] == before["simt_group_gemm"] + 1
    assert after["simt_cache_write"] == before["simt_cache_write"]
    assert bf16_ulp_close(got, oracle.block_diag_query(q, ref["qmap"]), ulps=1)
    before = after
    lat.block_diag_query(q.to(DEV))
    assert _lib.path_counts() == before                       # the aligned query stays on the tensor cores


@pytest.mark.parametrize("name", CASES)
def test_up_project(name):
    fx, spec, w, batch, q = golden_case(name)
    lat, ref = layer_pair(w)
    B = q.shape[0]
    a = torch.randn(B, 24, spec.v_rank, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    out = torch.zeros(B + 3, 24, 256, dtype=torch.bfloat16, device=DEV)
    lat.up_project(a.to(DEV), out[:B])
    got = out.cpu()
    assert bf16_ulp_close(got[:B], fx["up_out"], ulps=1)
    assert not got[B:].any()


def test_merge_segments():
    g = torch.Generator().manual_seed(2)
    for seqs, nct, lv in [([129, 513, 1025, 2001], 16, 512), ([0, 300, 64, 0], 8, 96), ([40] * 12, 8, 640),
                          ([9000] * 3, 148, 512), ([300 * 128], 300, 64)]:
        B = len(seqs)
        sched = dec.make_schedule(B, DEV, num_ctas=nct)
        dec.schedule(sched, torch.tensor(seqs, dtype=torch.int32, device=DEV))
        nseg = int(sched.seg_base[B])
        part = torch.randn(nseg + 1, 24, lv + 1, generator=g)
        part[:, :, lv] *= 4
        a = torch.empty(B, 24, lv, dtype=torch.bfloat16, device=DEV)
        lse = torch.empty(B, 24, device=DEV)
        dec.merge_segments(part.to(DEV), sched, a, lse)
        ea, el = oracle.merge_segments(part, sched.seg_base.cpu(), B, lv)
        torch.cuda.synchronize()
        assert bf16_ulp_close(a.cpu(), ea.to(torch.bfloat16), ulps=1)
        live = torch.isfinite(el)
        assert torch.equal(torch.isfinite(lse.cpu()), live)
        assert torch.allclose(lse.cpu()[live], el[live], atol=1e-4)


def test_merge_up_project():
    """The fused merge + U_v projection against the two-kernel path (within 1 BF16 ulp: the same roundings, another
    FP32 summation order in the projection) and against the oracle's merge followed by its projection (2 ulp + 2e-3:
    the merged output may differ from the oracle's by one BF16 ulp in some features, which moves outputs that nearly
    cancel by more than their own ulp)."""
    g = torch.Generator().manual_seed(3)
    long = [int(x) for x in torch.randint(1, 3000, (70,), generator=g)]
    for seqs, nct, lv in [([129, 513, 1025, 2001], 16, 512), ([0, 300, 64, 0], 8, 96), ([40] * 40, 8, 640),
                          ([9000] * 3, 148, 384), ([300 * 128], 300, 64), (long, 148, 576), ([17, 5, 900], 4, 300)]:
        B = len(seqs)
        sched = dec.make_schedule(B, DEV, num_ctas=nct)
        dec.schedule(sched, torch.tensor(seqs, dtype=torch.int32, device=DEV))
        nseg = int(sched.seg_base[B])
        part = torch.randn(nseg + 1, 24, lv + 1, generator=g)
        part[:, :, lv] *= 4
        v_up_t = (torch.randn(4, lv, 256, generator=g) / lv ** 0.5).to(torch.bfloat16)
        part_d, v_d = part.to(DEV), v_up_t.to(DEV)
        out = torch.full((B, 24, 256), float("nan"), dtype=torch.bfloat16, device=DEV)
        lse = torch.full((B, 24), float("nan"), device=DEV)
        dec.merge_up_project(part_d, sched, v_d, out, lse)
        # the same partials with 16-byte aligned rows (the backend's layout: float4 loads of the rows where lv % 4 == 0),
        # into an output whose head stride is not a multiple of 8 (element stores instead of the staged 16-byte ones)
        part_p = dec.partial_buffer(nseg + 1, lv, DEV)
        part_p.copy_(part_d)
        out_p = torch.full((B, 24, 260), float("nan"), dtype=torch.bfloat16, device=DEV)[:, :, :256]
        lse_p = torch.full((B, 24), float("nan"), device=DEV)
        dec.merge_up_project(part_p, sched, v_d, out_p, lse_p)
        a2 = torch.empty(B, 24, lv, dtype=torch.bfloat16, device=DEV)
        lse2 = torch.empty(B, 24, device=DEV)
        dec.merge_segments(part_d, sched, a2, lse2)
        out2 = torch.empty(B, 24, 256, dtype=torch.bfloat16, device=DEV)
        latent_ops.up_project(a2, v_d, out2)
        torch.cuda.synchronize()
        dec.check_device_errors(DEV)
        what = f"{B} requests, {nct} CTAs, lv {lv}"
        assert bf16_ulp_close(out.cpu(), out2.cpu(), ulps=1, atol=1e-5), what
        assert torch.equal(out_p.cpu(), out.cpu()) and torch.equal(lse_p.cpu(), lse.cpu()), what + " (aligned rows)"
        assert torch.equal(torch.isinf(lse.cpu()), torch.isinf(lse2.cpu())), what
        live = torch.isfinite(lse2.cpu())
        assert torch.allclose(lse.cpu()[live], lse2.cpu()[live], atol=1e-6, rtol=0), what
        ea, el = oracle.merge_segments(part, sched.seg_base.cpu(), B, lv)
        eo = oracle.up_project(ea.to(torch.bfloat16), v_up_t)
        assert bf16_ulp_close(out.cpu(), eo, ulps=2, atol=2e-3), what


# ------------------------------------------------------------------------------------------------- decode
@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("num_ctas", [148, 7, 1])
def test_decode_partials(name, num_ctas):
    """The kernel's per-segment partials against the oracle's split with the kernel's rounding points."""
    fx, spec, w, batch, q = golden_case(name)
    lat, ref = layer_pair(w)
    out, a, lse, part, sched, q_bd = run_decode(lat, q.to(DEV), batch.cache.to(DEV), batch.block_table.to(DEV),
                                               batch.seq_lens.to(DEV), num_ctas)
    B = q.shape[0]
    nseg = int(sched.seg_base[B])
    exp = oracle.decode_partials(q_bd.cpu(), batch.cache, batch.block_table, batch.seq_lens, ref,
                                 sched.work.cpu(), nseg, SCALE, dec.TILE_T)
    got = part[:nseg].cpu()
    assert torch.isfinite(got).all()
    assert torch.allclose(got[:, :, -1], exp[:, :, -1], atol=2e-3, rtol=1e-4), \
        float((got[:, :, -1] - exp[:, :, -1]).abs().max())
    err = (got[:, :, :-1] - exp[:, :, :-1]).abs()
    assert float(err.max()) < 2e-2 and float(err.mean()) < 2e-3, (float(err.max()), float(err.mean()))


@pytest.mark.parametrize("name", CASES)
def test_decode_matches_reference_output(name):
    """Whole decode chain vs the reference's own torch path (golden) and the fp32 oracle."""
    fx, spec, w, batch, q = golden_case(name)
    lat, ref = layer_pair(w)
    out, *_ = run_decode(lat, q.to(DEV), batch.cache.to(DEV), batch.block_table.to(DEV), batch.seq_lens.to(DEV))
    assert_close_out(out, fx["out_reference"], f"{name} vs reference")
    exp_b = oracle.decode_fp32(q, batch.cache, batch.block_table, batch.seq_lens, ref, SCALE)
    assert_close_out(out, exp_b, f"{name} vs fp32")


@pytest.mark.parametrize("page", [16, 32, 64, 128, 256])
def test_decode_page_sizes_and_strided_views(page):
    spec = synth.c50()
    w = synth.make_layer(spec)
    lat, ref = layer_pair(w, max_pos=5000)
    seqs = [1, 127, 128, 129, 700, 4097, 0, 255]
    layout = w.layout
    bt, nb, owned = synth.block_tables(seqs, page, extra_blocks=3)
    W = layout["row_width"]
    layers = 2
    buf = torch.empty(nb, layers, page, W, dtype=torch.bfloat16)
    cache = buf[:, 1]                                        # strided per-layer view
    synth.fill_cache(cache, layout, bt, seqs, seed=5)
    buf[:, 0] = float("nan")
    q = synth.make_queries(len(seqs), seed=6)
    gbuf = buf.to(DEV)
    out, *_ = run_decode(lat, q.to(DEV), gbuf[:, 1], bt.to(DEV), torch.tensor(seqs, dtype=torch.int32, device=DEV))
    exp = oracle.decode_fp32(q, cache, bt, torch.tensor(seqs), ref, SCALE)
    assert_close_out(out, exp, f"page {page}")
    assert not out[6].float().abs().any()                     # a padded request (length 0) gives zeros


@pytest.mark.parametrize("r_k", [384, 448, 512, 576, 640])
@pytest.mark.parametrize("page", [16, 64])
def test_decode_learned_ranks(r_k, page):
    """Every per-layer rank split of the 16-layer config (r_v = 1024 - r_k): key and value parts whose chunk counts
    leave partial stages (n_k = 6, 7, 9, 10; 6..10 value chunks), against the fp32 oracle."""
    spec = synth.spec_from_ranks(r_k, 1024 - r_k)
    w = synth.make_layer(spec)
    lat, ref = layer_pair(w, max_pos=3000)
    seqs = [2049, 1, 700, 129, 1500]
    batch = synth.make_batch(w.layout, seqs, page=page, seed=21)
    q = synth.make_queries(len(seqs), seed=22)
    out, *_ = run_decode(lat, q.to(DEV), batch.cache.to(DEV), batch.block_table.to(DEV), batch.seq_lens.to(DEV))
    exp = oracle.decode_fp32(q, batch.cache, batch.block_table, batch.seq_lens, ref, SCALE)
    assert_close_out(out, exp, f"r_k {r_k}, page {page}")


@pytest.mark.parametrize("k_ranks,r_v,rope_align", [
    ((16, 16, 16, 16), 64, False),      # one chunk holds four groups' RoPE runs: the per-step rebuild words
    ((24, 8, 40, 16), 96, False),       # runs of two groups meeting inside a 16-column step
    ((96, 112, 144, 160), 512, True),   # rope-aligned: whole-chunk runs, then chunks without RoPE coordinates
])
def test_decode_rebuild_issue_paths(k_ranks, r_v, rope_align):
    """The decode issuer's three ways of issuing the RoPE-key rebuild (the host encodes each key chunk's rebuild steps
    as runs when they form at most two, a whole-chunk run issued straight; otherwise per step), against the fp32
    oracle."""
    spec = synth.LayerSpec(tuple(k_ranks), r_v, 1024, rope_align=rope_align)
    w = synth.make_layer(spec)
    lat, ref = layer_pair(w, max_pos=3000)
    seqs = [1500, 129, 2049, 7]
    batch = synth.make_batch(w.layout, seqs, page=16, seed=31)
    q = synth.make_queries(len(seqs), seed=32)
    out, *_ = run_decode(lat, q.to(DEV), batch.cache.to(DEV), batch.block_table.to(DEV), batch.seq_lens.to(DEV))
    exp = oracle.decode_fp32(q, batch.cache, batch.block_table, batch.seq_lens, ref, SCALE)
    assert_close_out(out, exp, f"ranks {k_ranks}, r_v {r_v}, rope_align {rope_align}")


def test_decode_invariances():
    """Bit-identical under a permutation of physical blocks; within tolerance across different CTA counts."""
    spec = synth.spec_from_ranks(448, 576)
    w = synth.make_layer(spec)
    lat, ref = layer_pair(w, max_pos=9000)
    seqs = [3000, 17, 8193, 640]
    batch = synth.make_batch(w.layout, seqs, page=16, seed=8)
    q = synth.make_queries(len(seqs), seed=9).to(DEV)
    o1, *_ = run_decode(lat, q, batch.cache.to(DEV), batch.block_table.to(DEV), batch.seq_lens.to(DEV), 148)
    # move every block to a new physical position
    nb = batch.cache.shape[0]
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(1))
    cache2 = torch.empty_like(batch.cache)
    cache2[perm] = batch.cache
    bt2 = perm[batch.block_table.long()].to(torch.int32)
    o2, *_ = run_decode(lat, q, cache2.to(DEV), bt2.to(DEV), batch.seq_lens.to(DEV), 148)
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))
    o3, *_ = run_decode(lat, q, batch.cache.to(DEV), batch.block_table.to(DEV), batch.seq_lens.to(DEV), 5)
    err = (o1.float() - o3.float()).abs()
    assert float(err.max()) < MAX_ABS and float(err.mean()) < MEAN_ABS
    exp = oracle.decode_fp32(q.cpu(), batch.cache, batch.block_table, batch.seq_lens, ref, SCALE)
    assert_close_out(o1, exp, "ragged 448/576")


def test_backend_forward_decode_step():
    """The backend surface end to end: builder -> impl.forward (cache write of this step's token, then decode)."""
    spec = synth.c50()
    w = synth.make_layer(spec)
    lat, ref = layer_pair(w)
    seqs = [40, 300, 1, 2050, 129] * 8                    # 40 decodes: the cache write runs on the side stream
    page = 16
    bt, nb, _ = synth.block_tables(seqs, page, extra_blocks=2)
    W = w.layout["row_width"]
    kv = torch.zeros(nb, 1, page, W, dtype=torch.bfloat16)
    synth.fill_cache(kv[:, 0], w.layout, bt, seqs, seed=3, poison=False)
    B = len(seqs)
    g = torch.Generator().manual_seed(12)
    x = torch.randn(B, w.kv_latent_proj.shape[1], generator=g).to(torch.bfloat16)
    c = (x.float() @ w.kv_latent_proj.float().T).to(torch.bfloat16)          # the latent projection of the new token
    pos = torch.tensor(seqs) - 1
    slots = bt[torch.arange(B), pos // page].long() * page + pos % page
    q = synth.make_queries(B, seed=13)
    # expected: write the new rows on the CPU, then the fp32 oracle
    exp_cache = oracle.latent_rows(c, slots, kv[:, 0].clone(), ref["u_cat"], ref["k_segs"], 1e-6)
    exp = oracle.decode_fp32(q, exp_cache, bt, torch.tensor(seqs), ref, SCALE)

    spec_kv = LatentKVSpec(block_size=page, num_kv_heads=1, head_size=W)
    builder = LatentAttentionMetadataBuilder(spec_kv, ["l0"], device=DEV, max_num_batched_tokens=256)
    cm = CommonAttentionMetadata(query_start_loc=torch.arange(B + 1, dtype=torch.int32, device=DEV),
                                 query_start_loc_cpu=torch.arange(B + 1, dtype=torch.int32),
                                 seq_lens=torch.tensor(seqs, dtype=torch.int32, device=DEV),
                                 block_table_tensor=bt.to(DEV), slot_mapping=slots.to(DEV), num_reqs=B,
                                 num_actual_tokens=B, max_query_len=1)
    md = builder.build(0, cm)
    impl = LatentAttentionImpl(24, 256, SCALE, 4)

    class Layer:
        latent = lat
    kv_d = kv.to(DEV)
    output = torch.empty(B, 24, 256, dtype=torch.bfloat16, device=DEV)
    impl.forward(Layer, q.to(DEV), c.to(DEV), pos.to(DEV), kv_d, md, output)
    torch.cuda.synchronize()
    assert bf16_ulp_close(kv_d[:, 0].cpu().view(-1, W)[slots], exp_cache.view(-1, W)[slots], ulps=1)
    assert_close_out(output, exp, "backend forward")
    assert impl.forward(Layer, q.to(DEV), c.to(DEV), pos.to(DEV), kv_d, None, output.clone()).abs().sum() == 0

    # the model-side step with the down-projection fused into the write gives the same rows and output
    kv_f = kv.to(DEV)
    out_f = torch.empty_like(output)
    latent_attention_step(impl, Layer, q.to(DEV), x.to(DEV), w.kv_latent_proj.to(DEV), kv_f, md, out_f)
    torch.cuda.synchronize()
    dec.check_device_errors(DEV)
    assert bf16_ulp_close(kv_f[:, 0].cpu().view(-1, W)[slots], exp_cache.view(-1, W)[slots], ulps=2, atol=PROJ_ATOL)
    assert_close_out(out_f, exp, "fused step")


def test_backend_decode_cuda_graph():
    """UNIFORM_SINGLE_TOKEN_DECODE graphs: the decode forward (side-stream cache write, absorbed query, split-KV
    decode, merge, U_v projection) captured once and replayed for two more steps whose inputs and metadata were
    refilled in place (contexts one token longer each step, new queries and new rows; the builder recomputes the
    schedule into its persistent buffers outside the graph). Every replay equals the eager forward of the same step,
    bit for bit, and so do the caches."""
    spec = synth.c50()
    w = synth.make_layer(spec)
    lat, ref = layer_pair(w)
    seqs0 = [40, 300, 1, 2050, 129] * 8
    B, page, steps = len(seqs0), 16, 3
    bt, nb, _ = synth.block_tables([s + steps for s in seqs0], page, extra_blocks=2)
    W = w.layout["row_width"]
    kv0 = torch.zeros(nb, 1, page, W, dtype=torch.bfloat16)
    synth.fill_cache(kv0[:, 0], w.layout, bt, [s + steps for s in seqs0], seed=23, poison=False)
    g = torch.Generator().manual_seed(24)
    inputs = []
    for k in range(steps):
        seqs = torch.tensor([s + k for s in seqs0], dtype=torch.int32)
        pos = seqs.long() - 1
        slots = bt[torch.arange(B), pos // page].long() * page + pos % page
        x = torch.randn(B, w.kv_latent_proj.shape[1], generator=g).to(torch.bfloat16)
        c = (x.float() @ w.kv_latent_proj.float().T).to(torch.bfloat16)
        q = torch.randn(B, 24, 256, generator=g).to(torch.bfloat16)
        inputs.append((seqs, pos, slots, c, q))
    spec_kv = LatentKVSpec(block_size=page, num_kv_heads=1, head_size=W)
    builder = LatentAttentionMetadataBuilder(spec_kv, ["l0"], device=DEV, max_num_batched_tokens=256)
    impl = LatentAttentionImpl(24, 256, SCALE, 4)

    class Layer:
        latent = lat
    # persistent device buffers, refilled in place before every step
    seq_d = torch.empty(B, dtype=torch.int32, device=DEV)
    pos_d = torch.empty(B, dtype=torch.int64, device=DEV)
    slot_d = torch.empty(B, dtype=torch.int64, device=DEV)
    c_d = torch.empty(B, W, dtype=torch.bfloat16, device=DEV)[:, :c.shape[1]]
    q_d = torch.empty(B, 24, 256, dtype=torch.bfloat16, device=DEV)
    out_d = torch.empty(B, 24, 256, dtype=torch.bfloat16, device=DEV)
    bt_d = bt.to(DEV)
    qsl = torch.arange(B + 1, dtype=torch.int32)

    def refill(k):
        seqs, pos, slots, c, q = inputs[k]
        seq_d.copy_(seqs)
        pos_d.copy_(pos)
        slot_d.copy_(slots)
        c_d.copy_(c)
        q_d.copy_(q)
        cm = CommonAttentionMetadata(query_start_loc=qsl.to(DEV), query_start_loc_cpu=qsl, seq_lens=seq_d,
                                     block_table_tensor=bt_d, slot_mapping=slot_d, num_reqs=B, num_actual_tokens=B,
                                     max_query_len=1)
        return builder.build(0, cm)

    # eager reference: all steps in order
    kv_e = kv0.to(DEV)
    eager = []
    for k in range(steps):
        md = refill(k)
        impl.forward(Layer, q_d, c_d, pos_d, kv_e, md, out_d)
        eager.append(out_d.clone())
    torch.cuda.synchronize()
    # graph: step 0 eagerly on a side stream (warm-up), capture, then replay steps 1 and 2
    kv_g = kv0.to(DEV)
    md = refill(0)
    s = torch.cuda.Stream(DEV)
    s.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(s):
        impl.forward(Layer, q_d, c_d, pos_d, kv_g, md, out_d)
    torch.cuda.current_stream(DEV).wait_stream(s)
    assert torch.equal(out_d, eager[0])
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        impl.forward(Layer, q_d, c_d, pos_d, kv_g, md, out_d)
    for k in range(1, steps):
        refill(k)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out_d, eager[k]), k
    dec.check_device_errors(DEV)
    assert torch.equal(kv_g, kv_e)


def test_decode_long_context_properties():
    """Config-2 size (B = 64, L = 8192, c50): finite, matches the oracle on a sample of requests, and a request's
    output does not depend on the others in the batch."""
    spec = synth.c50()
    w = synth.make_layer(spec)
    lat, ref = layer_pair(w, max_pos=8193)
    seqs = [8193] * 64
    bt, nb, _ = synth.block_tables(seqs, 16)
    cache = torch.empty(nb, 16, w.layout["row_width"], dtype=torch.bfloat16, device=DEV)
    synth.fill_cache(cache, w.layout, bt.to(DEV), seqs, seed=21)
    q = synth.make_queries(64, seed=22).to(DEV)
    sl = torch.tensor(seqs, dtype=torch.int32, device=DEV)
    out, *_ = run_decode(lat, q, cache, bt.to(DEV), sl)
    assert torch.isfinite(out.float()).all()
    sample = [0, 37, 63]
    cpu_cache = cache.cpu()
    exp = oracle.decode_fp32(q[sample].cpu(), cpu_cache, bt[sample], torch.tensor([8193] * 3), ref, SCALE)
    assert_close_out(out[sample], exp, "config-2 sample")
    alone, *_ = run_decode(lat, q[37:38], cache, bt[37:38].to(DEV), sl[37:38])
    err = (alone.float() - out[37:38].float()).abs()
    assert float(err.max()) < MAX_ABS


@pytest.mark.parametrize("spec_name", ["c50", "c25"])
def test_decode_config4_long_context(spec_name):
    """Config 4 shapes at full size (32 requests x 65,537 tokens, page 16; c50 rows of 1,024 columns and the c25
    variant of 512): 512 tiles per request spread over every CTA. Finite, two requests against the fp32 oracle,
    the same outputs from a 7-CTA split (other segments, other merges), and a request decoded alone."""
    spec = getattr(synth, spec_name)()
    w = synth.make_layer(spec)
    L = 65537
    lat, ref = layer_pair(w, max_pos=L)
    seqs = [L] * 32
    bt, nb, _ = synth.block_tables(seqs, 16)
    cache = torch.empty(nb, 16, w.layout["row_width"], dtype=torch.bfloat16, device=DEV)
    synth.fill_cache(cache, w.layout, bt.to(DEV), seqs, seed=41, poison=False)
    q = synth.make_queries(32, seed=42).to(DEV)
    sl = torch.tensor(seqs, dtype=torch.int32, device=DEV)
    out, *_ = run_decode(lat, q, cache, bt.to(DEV), sl)
    assert torch.isfinite(out.float()).all()
    sample = [3, 30]
    cpu_cache = cache.cpu()
    exp = oracle.decode_fp32(q[sample].cpu(), cpu_cache, bt[sample], torch.tensor([L] * 2), ref, SCALE)
    assert_close_out(out[sample], exp, f"{spec_name} long-context sample")
    out7, *_ = run_decode(lat, q, cache, bt.to(DEV), sl, num_ctas=7)
    err = (out7.float() - out.float()).abs()
    assert float(err.max()) < MAX_ABS and float(err.mean()) < MEAN_ABS
    alone, *_ = run_decode(lat, q[30:31], cache, bt[30:31].to(DEV), sl[30:31])
    assert float((alone.float() - out[30:31].float()).abs().max()) < MAX_ABS


# ------------------------------------------------------------------------------------------------- decompress (prefill)
def assert_decompress_close(k, v, ek, ev, what):
    """Values and the keys' non-rotary channels within 1 BF16 ulp. The rotary channels are x1 cos - x2 sin (and
    x2 cos + x1 sin) of x = bf16(gain B_g c~): a sum order that moves x by one BF16 ulp moves the rotated value by up
    to one ulp of |x| (2^-8 |x|), so they are held to 2^-7 (1 + |expected|) absolute, and almost all within 1 ulp."""
    assert bf16_ulp_close(v, ev, ulps=1, atol=1e-6), (what, "v")
    assert bf16_ulp_close(k[..., 64:], ek[..., 64:], ulps=1, atol=1e-6), (what, "k nope")
    kp, ep = k[..., :64].float(), ek[..., :64].float()
    assert ((kp - ep).abs() <= 2 ** -7 * (1 + ep.abs())).all(), (what, "k rope", float((kp - ep).abs().max()))
    mag = torch.maximum(kp.abs(), ep.abs()).clamp_min(1e-38)
    far = (kp - ep).abs() > 2.0 ** (torch.floor(torch.log2(mag)) - 7) + 1e-6
    assert float(far.float().mean()) < 1e-4, (what, "k rope beyond 1 ulp", float(far.float().mean()))


@pytest.mark.parametrize("r_k", [384, 448, 512, 640])
@pytest.mark.parametrize("page", [16, 64, 128])
def test_decompress_paged(r_k, page):
    """Keys and values of position ranges rebuilt from the paged rows on the tensor cores, against the oracle's
    ``decompress`` of the gathered rows: whole requests, ranges that start and end inside a 128-position tile and a
    page, and a single position. Every channel within 1 BF16 ulp (the rotation's and the sums' rounding order)."""
    spec = synth.spec_from_ranks(r_k, 1024 - r_k)
    w = synth.make_layer(spec)
    lat, ref = layer_pair(w, max_pos=3000)
    seqs = [2049, 1, 700, 129]
    batch = synth.make_batch(w.layout, seqs, page=page, seed=31)
    cache, bt = batch.cache.to(DEV), batch.block_table.to(DEV)
    for b, (pos0, count) in [(0, (0, 2049)), (1, (0, 1)), (2, (37, 600)), (3, (128, 1)), (2, (699, 1)),
                             (0, (1000, 777))]:
        L = seqs[b]
        k, v = lat.decompress_paged(cache, bt[b], L, pos0, count)
        torch.cuda.synchronize()
        dec.check_device_errors(DEV)
        rows, pos = oracle.gather_rows(batch.cache, batch.block_table, b, L)
        ek, ev = oracle.decompress(ref, rows[pos0:pos0 + count], pos[pos0:pos0 + count])
        assert_decompress_close(k.cpu(), v.cpu(), ek, ev, (r_k, page, b, pos0, count))


def test_decompress_into_strided_views():
    """Outputs written into views of a larger buffer ([count, 4, 256] slices with a token stride of 2 * 1024): the
    neighbouring halves stay untouched."""
    spec = synth.c50()
    w = synth.make_layer(spec)
    lat, ref = layer_pair(w, max_pos=1200)
    seqs = [1100]
    batch = synth.make_batch(w.layout, seqs, page=16, seed=32)
    buf = torch.zeros(300, 2, 4, 256, dtype=torch.bfloat16, device=DEV)
    k_out, v_out = buf[:, 0], buf[:, 1]
    lat.decompress_paged(batch.cache.to(DEV), batch.block_table.to(DEV)[0], 1100, 500, 300, k_out, v_out)
    torch.cuda.synchronize()
    rows, pos = oracle.gather_rows(batch.cache, batch.block_table, 0, 1100)
    ek, ev = oracle.decompress(ref, rows[500:800], pos[500:800])
    assert_decompress_close(buf[:, 0].cpu(), buf[:, 1].cpu(), ek, ev, "strided views")


def test_backend_forward_mixed_prefill(monkeypatch):
    """Decodes and prefills in one step through the backend: every new token's row written, the decodes through the
    split-KV kernel, the prefills' queries (several per request, the last positions of their contexts; one request
    entirely new) attending causally over keys and values rebuilt on the tensor cores, against the fp32 oracle
    (decompress + attention). The four prefills take one decompress launch and one attention launch."""
    import belt_b200.latent_backend as lb
    calls = {"decompress": 0, "attention": 0}
    real_d, real_a = latent_ops.decompress_varlen, latent_ops.prefill_attention_varlen

    def count_d(*a, **k):
        calls["decompress"] += 1
        return real_d(*a, **k)

    def count_a(*a, **k):
        calls["attention"] += 1
        return real_a(*a, **k)
    monkeypatch.setattr(latent_ops, "decompress_varlen", count_d)
    monkeypatch.setattr(lb.latent_ops, "prefill_attention_varlen", count_a)
    spec = synth.spec_from_ranks(448, 576)
    w = synth.make_layer(spec)
    lat, ref = layer_pair(w, max_pos=2100)
    seqs = [300, 1, 129, 700, 2050, 520, 64]  # the last four are prefills of 37, 300, 20 and 64 new tokens
    qlens = [1, 1, 1, 37, 300, 20, 64]
    page = 16
    bt, nb, _ = synth.block_tables(seqs, page, extra_blocks=2)
    W = w.layout["row_width"]
    kv = torch.zeros(nb, 1, page, W, dtype=torch.bfloat16)
    synth.fill_cache(kv[:, 0], w.layout, bt, seqs, seed=4, poison=False)
    B, T = len(seqs), sum(qlens)
    g = torch.Generator().manual_seed(14)
    c = torch.randn(T, W, generator=g).to(torch.bfloat16)                     # the new tokens' latent projections
    pos = torch.cat([torch.arange(L - ql, L) for L, ql in zip(seqs, qlens)])
    req = torch.cat([torch.full((ql,), b) for b, ql in enumerate(qlens)])
    slots = bt[req, pos // page].long() * page + pos % page
    q = torch.randn(T, 24, 256, generator=g).to(torch.bfloat16)
    exp_cache = oracle.latent_rows(c, slots, kv[:, 0].clone(), ref["u_cat"], ref["k_segs"], 1e-6)
    exp = torch.zeros(T, 24, 256)
    for t in range(T):
        b, p = int(req[t]), int(pos[t])
        rows, rpos = oracle.gather_rows(exp_cache, bt, b, p + 1)
        k, v = oracle.decompress(ref, rows, rpos)
        exp[t] = oracle.attend(q[t], k, v, SCALE)

    spec_kv = LatentKVSpec(block_size=page, num_kv_heads=1, head_size=W)
    builder = LatentAttentionMetadataBuilder(spec_kv, ["l0"], device=DEV, max_num_batched_tokens=512)
    qsl = torch.tensor([0] + list(torch.cumsum(torch.tensor(qlens), 0)), dtype=torch.int32)
    cm = CommonAttentionMetadata(query_start_loc=qsl.to(DEV), query_start_loc_cpu=qsl,
                                 seq_lens=torch.tensor(seqs, dtype=torch.int32, device=DEV),
                                 block_table_tensor=bt.to(DEV), slot_mapping=slots.to(DEV), num_reqs=B,
                                 num_actual_tokens=T, max_query_len=max(qlens))
    md = builder.build(0, cm)
    assert md.num_decodes == 3 and md.num_prefills == 4
    impl = LatentAttentionImpl(24, 256, SCALE, 4)

    class Layer:
        latent = lat
    kv_d = kv.to(DEV)
    output = torch.empty(T, 24, 256, dtype=torch.bfloat16, device=DEV)
    impl.forward(Layer, q.to(DEV), c.to(DEV), pos.to(DEV), kv_d, md, output)
    torch.cuda.synchronize()
    dec.check_device_errors(DEV)
    assert bf16_ulp_close(kv_d[:, 0].cpu().view(-1, W)[slots], exp_cache.view(-1, W)[slots], ulps=1)
    assert_close_out(output, exp, "mixed prefill")
    assert calls == {"decompress": 1, "attention": 1}, calls


# ------------------------------------------------------------------------------------------------- prefill attention
def _attention_fp32(q, k, v, q_pos0, k_pos0, scale, causal=True):
    """fp32 reference: q [ql, 24, D], k / v [S, 4, D]; returns (out [ql, 24, D], lse [ql, 24])."""
    ql, S = q.shape[0], k.shape[0]
    kh = k.float().repeat_interleave(6, dim=1)
    vh = v.float().repeat_interleave(6, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kh) * scale
    if causal:
        qp = torch.arange(ql) + q_pos0
        kp = torch.arange(S) + k_pos0
        s = s.masked_fill(kp[None, None, :] > qp[None, :, None], float("-inf"))
    lse = torch.logsumexp(s, dim=-1)                                    # [24, ql]
    p = torch.softmax(s, dim=-1).nan_to_num(0.0)
    return torch.einsum("hqk,khd->qhd", p, vh), lse.transpose(0, 1)


@pytest.mark.parametrize("ql,S,q_pos0,k_pos0,causal", [
    (1, 1, 0, 0, True), (37, 700, 663, 0, True), (300, 2050, 1750, 0, True), (129, 129, 0, 0, True),
    (200, 500, 1000, 300, True),        # a context chunk: the queries see a prefix of the chunk's keys
    (64, 300, 5000, 0, True),           # every key precedes every query (no mask)
    (50, 256, 0, 100, True),            # keys after the first queries: some rows see no key (-inf, zeros)
    (130, 777, 0, 0, False),
])
def test_prefill_attention(ql, S, q_pos0, k_pos0, causal):
    g = torch.Generator().manual_seed(ql + S)
    q = torch.randn(ql, 24, 256, generator=g).to(torch.bfloat16)
    k = torch.randn(S, 4, 256, generator=g).to(torch.bfloat16)
    v = torch.randn(S, 4, 256, generator=g).to(torch.bfloat16)
    out, lse = latent_ops.prefill_attention(q.to(DEV), k.to(DEV), v.to(DEV), q_pos0, k_pos0, SCALE, causal)
    torch.cuda.synchronize()
    dec.check_device_errors(DEV)
    eo, el = _attention_fp32(q, k, v, q_pos0, k_pos0, SCALE, causal)
    err = (out.float().cpu() - eo).abs()
    assert torch.isfinite(out.float()).all()
    assert float(err.max()) < MAX_ABS and float(err.mean()) < MEAN_ABS, (float(err.max()), float(err.mean()))
    lc = lse.cpu()
    assert torch.equal(torch.isinf(lc), torch.isinf(el))
    live = torch.isfinite(el)
    assert torch.allclose(lc[live], el[live], atol=1e-3, rtol=0)


def test_prefill_attention_strided_output():
    """Output and queries as views of the backend's [T, 24, 256] buffers (rows after the decode tokens)."""
    g = torch.Generator().manual_seed(5)
    qall = torch.randn(400, 24, 256, generator=g).to(torch.bfloat16).to(DEV)
    k = torch.randn(900, 4, 256, generator=g).to(torch.bfloat16)
    v = torch.randn(900, 4, 256, generator=g).to(torch.bfloat16)
    outall = torch.zeros(400, 24, 256, dtype=torch.bfloat16, device=DEV)
    latent_ops.prefill_attention(qall[100:350], k.to(DEV), v.to(DEV), 650, 0, SCALE, out=outall[100:350])
    torch.cuda.synchronize()
    eo, _ = _attention_fp32(qall[100:350].cpu(), k, v, 650, 0, SCALE)
    err = (outall[100:350].float().cpu() - eo).abs()
    assert float(err.max()) < MAX_ABS and float(err.mean()) < MEAN_ABS
    assert not outall[:100].any() and not outall[350:].any()


def test_backend_prefill_chunked_merge(monkeypatch):
    """A prefill whose context spans several PREFILL_CHUNK rounds: the per-round attentions folded by log-sum-exp give
    the whole-context result (the fp32 oracle)."""
    import belt_b200.latent_backend as lb
    monkeypatch.setattr(lb, "PREFILL_CHUNK", 384)
    spec = synth.c50()
    w = synth.make_layer(spec)
    lat, ref = layer_pair(w, max_pos=1100)
    L, ql, page = 1000, 70, 16
    bt, nb, _ = synth.block_tables([L], page, extra_blocks=1)
    W = w.layout["row_width"]
    kv = torch.zeros(nb, 1, page, W, dtype=torch.bfloat16)
    synth.fill_cache(kv[:, 0], w.layout, bt, [L], seed=6, poison=False)
    g = torch.Generator().manual_seed(15)
    q = torch.randn(ql, 24, 256, generator=g).to(torch.bfloat16)
    rows, rpos = oracle.gather_rows(kv[:, 0], bt, 0, L)
    k, v = oracle.decompress(ref, rows, rpos)
    exp, _ = _attention_fp32(q, k, v, L - ql, 0, SCALE)
    m = lb.LatentAttentionMetadata(num_actual_tokens=ql, num_decodes=0, num_decode_tokens=0, num_prefills=1,
                                   num_prefill_tokens=ql, block_table=bt.to(DEV),
                                   seq_lens=torch.tensor([L], dtype=torch.int32, device=DEV), sched=None)
    m.prefill_q_len, m.prefill_seq_len = [ql], [L]
    impl = LatentAttentionImpl(24, 256, SCALE, 4)
    out = torch.zeros(ql, 24, 256, dtype=torch.bfloat16, device=DEV)
    impl._prefill(lat, q.to(DEV), out, kv.to(DEV)[:, 0], m)
    torch.cuda.synchronize()
    dec.check_device_errors(DEV)
    err = (out.float().cpu() - exp).abs()
    assert float(err.max()) < MAX_ABS and float(err.mean()) < MEAN_ABS, (float(err.max()), float(err.mean()))


def test_backend_prefill_rounds_over_several_requests(monkeypatch):
    """Three prefills whose contexts (1000, 70 and 450 tokens) are cut into rounds of 384 keys across requests: the
    rounds' attentions folded by log-sum-exp give every request's whole-context result (the fp32 oracle)."""
    import belt_b200.latent_backend as lb
    monkeypatch.setattr(lb, "PREFILL_CHUNK", 384)
    spec = synth.spec_from_ranks(512, 512)
    w = synth.make_layer(spec)
    lat, ref = layer_pair(w, max_pos=1100)
    lens, qls, page = [1000, 70, 450], [70, 70, 33], 16
    rounds = lb.plan_prefill_rounds(lens, 384)
    assert len(rounds) == 4 and sum(k1 - k0 for r in rounds for _, k0, k1 in r) == sum(lens)
    bt, nb, _ = synth.block_tables(lens, page, extra_blocks=1)
    W = w.layout["row_width"]
    kv = torch.zeros(nb, 1, page, W, dtype=torch.bfloat16)
    synth.fill_cache(kv[:, 0], w.layout, bt, lens, seed=8, poison=False)
    g = torch.Generator().manual_seed(16)
    q = torch.randn(sum(qls), 24, 256, generator=g).to(torch.bfloat16)
    exp = []
    for b, (L, ql) in enumerate(zip(lens, qls)):
        rows, rpos = oracle.gather_rows(kv[:, 0], bt, b, L)
        k, v = oracle.decompress(ref, rows, rpos)
        r0 = sum(qls[:b])
        exp.append(_attention_fp32(q[r0:r0 + ql], k, v, L - ql, 0, SCALE)[0])
    exp = torch.cat(exp)
    m = lb.LatentAttentionMetadata(num_actual_tokens=sum(qls), num_decodes=0, num_decode_tokens=0, num_prefills=3,
                                   num_prefill_tokens=sum(qls), block_table=bt.to(DEV),
                                   seq_lens=torch.tensor(lens, dtype=torch.int32, device=DEV), sched=None)
    m.prefill_q_len, m.prefill_seq_len = qls, lens
    impl = LatentAttentionImpl(24, 256, SCALE, 4)
    out = torch.zeros(sum(qls), 24, 256, dtype=torch.bfloat16, device=DEV)
    impl._prefill(lat, q.to(DEV), out, kv.to(DEV)[:, 0], m)
    torch.cuda.synchronize()
    dec.check_device_errors(DEV)
    err = (out.float().cpu() - exp).abs()
    assert float(err.max()) < MAX_ABS and float(err.mean()) < MEAN_ABS, (float(err.max()), float(err.mean()))


def test_decompress_varlen_equals_per_request_launches():
    """One varlen launch over pieces of three requests (whole contexts, a range inside a tile and a single position)
    gives bit for bit the per-request launches' keys and values, concatenated."""
    spec = synth.spec_from_ranks(448, 576)
    w = synth.make_layer(spec)
    lat, _ = layer_pair(w, max_pos=3000)
    seqs = [2049, 1, 700]
    batch = synth.make_batch(w.layout, seqs, page=16, seed=33)
    cache, bt = batch.cache.to(DEV), batch.block_table.to(DEV)
    pieces = [(0, 2049, 0, 2049), (1, 1, 0, 1), (2, 700, 37, 600), (0, 2049, 1000, 1), (2, 700, 699, 1)]
    k, v = lat.decompress_varlen(cache, bt, pieces)
    ks, vs = [], []
    for b, L, pos0, count in pieces:
        kb, vb = lat.decompress_paged(cache, bt[b], L, pos0, count)
        ks.append(kb)
        vs.append(vb)
    torch.cuda.synchronize()
    dec.check_device_errors(DEV)
    assert torch.equal(k.view(torch.int16), torch.cat(ks).view(torch.int16))
    assert torch.equal(v.view(torch.int16), torch.cat(vs).view(torch.int16))


def test_prefill_attention_varlen_equals_per_piece_launches():
    """One varlen attention launch over four pieces (causal prefixes, a chunk that sees a prefix of its keys, a piece
    written to the second output) gives bit for bit the per-piece launches."""
    g = torch.Generator().manual_seed(17)
    qls, Ss = [37, 200, 1, 130], [700, 500, 1, 256]
    qp0, kp0 = [663, 1000, 0, 0], [0, 300, 0, 100]
    q = torch.randn(sum(qls), 24, 256, generator=g).to(torch.bfloat16).to(DEV)
    k = torch.randn(sum(Ss), 4, 256, generator=g).to(torch.bfloat16).to(DEV)
    v = torch.randn(sum(Ss), 4, 256, generator=g).to(torch.bfloat16).to(DEV)
    out = torch.zeros(sum(qls), 24, 256, dtype=torch.bfloat16, device=DEV)
    lse = torch.zeros(sum(qls), 24, device=DEV)
    out2, lse2 = torch.zeros_like(out), torch.zeros_like(lse)
    pieces, qr, kr = [], 0, 0
    for i in range(4):
        pieces.append((qr, qls[i], kr, Ss[i], qp0[i], kp0[i], qr, int(i == 1)))
        qr += qls[i]
        kr += Ss[i]
    latent_ops.prefill_attention_varlen(q, k, v, pieces, SCALE, out, lse, out2, lse2)
    torch.cuda.synchronize()
    dec.check_device_errors(DEV)
    for i, (q_row, ql, k_row, S, q_pos0, k_pos0, o_row, to2) in enumerate(pieces):
        o1, l1 = latent_ops.prefill_attention(q[q_row:q_row + ql], k[k_row:k_row + S], v[k_row:k_row + S], q_pos0,
                                              k_pos0, SCALE, causal=True)
        dst, dl = (out2, lse2) if to2 else (out, lse)
        assert torch.equal(dst[o_row:o_row + ql].view(torch.int16), o1.view(torch.int16)), i
        assert torch.equal(dl[o_row:o_row + ql], l1), i


def test_attn_fold():
    """The log-sum-exp fold against its fp32 restatement, with rows where the part saw no key (-inf: unchanged) and
    rows whose running result is empty (-inf: replaced)."""
    g = torch.Generator().manual_seed(18)
    R = 50
    out = torch.randn(R, 24, 256, generator=g).to(torch.bfloat16)
    part = torch.randn(R + 10, 24, 256, generator=g).to(torch.bfloat16)
    lse = torch.randn(R, 24, generator=g) * 3
    plse = torch.randn(R + 10, 24, generator=g) * 3
    lse[3, 5] = float("-inf")
    plse[10 + 7, 2] = float("-inf")
    pieces = [(0, 10, 20), (20, 30, 30)]
    o_d, l_d = out.to(DEV), lse.to(DEV)
    latent_ops.attn_fold(o_d, l_d, part.to(DEV), plse.to(DEV), pieces)
    torch.cuda.synchronize()
    exp_o, exp_l = out.float().clone(), lse.clone()
    for dst, src, n in pieces:
        for i in range(n):
            lo, lc = lse[dst + i], plse[src + i]
            m = torch.maximum(lo, lc)
            wo, wc = torch.exp(lo - m).nan_to_num(0.0), torch.exp(lc - m).nan_to_num(0.0)
            merged = (out[dst + i].float() * wo[:, None] + part[src + i].float() * wc[:, None]) / (wo + wc)[:, None]
            keep = torch.isinf(lc)
            take = torch.isinf(lo) & ~keep
            exp_o[dst + i] = torch.where(keep[:, None], out[dst + i].float(),
                                         torch.where(take[:, None], part[src + i].float(), merged))
            exp_l[dst + i] = torch.where(keep, lo, torch.where(take, lc, m + torch.log(wo + wc)))
    assert bf16_ulp_close(o_d.cpu(), exp_o.to(torch.bfloat16), ulps=1, atol=1e-6)
    assert torch.allclose(l_d.cpu(), exp_l, atol=1e-5, rtol=0)


# ------------------------------------------------------------------------------------------------- model-side block
def test_q_norm_rope_and_gate_mul():
    """The query-side norm / RoPE and the output gate against their fp32 restatements: q within 1 BF16 ulp, the gate
    within 2 (the kernel's exp approximation)."""
    from belt_b200 import model
    g = torch.Generator().manual_seed(41)
    T = 300
    qg = (torch.randn(T, 24, 512, generator=g) * 3).to(torch.bfloat16)
    w = torch.randn(256, generator=g) * 0.1
    cos_sin = synth.cos_sin_table(4096).to(torch.bfloat16)   # the layer's BF16 table
    pos = torch.randint(0, 4096, (T,), generator=g)
    for dtype in (torch.int64, torch.int32):
        q = model.q_norm_rope(qg.to(DEV)[:, :, :256], w, 1e-6, cos_sin.to(DEV), pos.to(dtype).to(DEV))
        torch.cuda.synchronize()
        assert bf16_ulp_close(q.cpu(), oracle.q_norm_rope(qg, w, 1e-6, cos_sin, pos), ulps=1, atol=1e-6)
    attn = torch.randn(T, 24, 256, generator=g).to(torch.bfloat16)
    out = model.gate_mul(attn.to(DEV), qg.to(DEV)[:, :, 256:])
    torch.cuda.synchronize()
    assert bf16_ulp_close(out.cpu(), oracle.gate_mul(attn, qg[:, :, 256:]), ulps=2, atol=1e-6)


def test_latent_self_attention_block():
    """The whole attention block of a compressed layer (q_gate GEMM, q-norm / RoPE, fused write, decode, gate, o_proj)
    for one decode step, against the fp32 oracle chain."""
    from belt_b200 import model
    spec = synth.spec_from_ranks(512, 512)
    w = synth.make_layer(spec)
    hidden_size = w.kv_latent_proj.shape[1]
    g = torch.Generator().manual_seed(42)
    q_gate = (torch.randn(24 * 512, hidden_size, generator=g) / hidden_size ** 0.5).to(torch.bfloat16)
    o_proj = (torch.randn(hidden_size, 24 * 256, generator=g) / (24 * 256) ** 0.5).to(torch.bfloat16)
    q_norm = torch.randn(256, generator=g) * 0.1
    cos_sin = synth.cos_sin_table(3000)
    blk = model.LatentSelfAttention(q_gate, o_proj, q_norm, w.k_norm_weight, w.kv_latent_proj, w.k_up, w.v_up,
                                    w.layout, cos_sin, device=DEV)
    ref = oracle.derive(w.k_up, w.v_up, w.k_norm_weight, w.layout, cos_sin)
    seqs = [300, 1, 2049, 129, 700]
    page = 16
    bt, nb, _ = synth.block_tables(seqs, page, extra_blocks=2)
    W = w.layout["row_width"]
    kv = torch.zeros(nb, 1, page, W, dtype=torch.bfloat16)
    synth.fill_cache(kv[:, 0], w.layout, bt, seqs, seed=7, poison=False)
    B = len(seqs)
    hidden = torch.randn(B, hidden_size, generator=g).to(torch.bfloat16)
    pos = torch.tensor(seqs) - 1
    slots = bt[torch.arange(B), pos // page].long() * page + pos % page
    # expected: the fp32 chain with the reference's roundings
    qg = (hidden.float() @ q_gate.float().T).to(torch.bfloat16).view(B, 24, 512)
    q = oracle.q_norm_rope(qg, q_norm, 1e-6, cos_sin.to(torch.bfloat16), pos)
    exp_cache = oracle.project_rows(hidden, w.kv_latent_proj, slots, kv[:, 0].clone(), ref["u_cat"], ref["k_segs"],
                                    1e-6)
    att = oracle.decode_fp32(q, exp_cache, bt, torch.tensor(seqs), ref, 1 / 16).to(torch.bfloat16)
    gated = oracle.gate_mul(att, qg[:, :, 256:])
    exp = gated.float().view(B, -1) @ o_proj.float().T

    spec_kv = LatentKVSpec(block_size=page, num_kv_heads=1, head_size=W)
    builder = LatentAttentionMetadataBuilder(spec_kv, ["l0"], device=DEV, max_num_batched_tokens=256)
    cm = CommonAttentionMetadata(query_start_loc=torch.arange(B + 1, dtype=torch.int32, device=DEV),
                                 query_start_loc_cpu=torch.arange(B + 1, dtype=torch.int32),
                                 seq_lens=torch.tensor(seqs, dtype=torch.int32, device=DEV),
                                 block_table_tensor=bt.to(DEV), slot_mapping=slots.to(DEV), num_reqs=B,
                                 num_actual_tokens=B, max_query_len=1)
    md = builder.build(0, cm)
    out = blk.forward(pos.to(DEV), hidden.to(DEV), kv.to(DEV), md)
    torch.cuda.synchronize()
    dec.check_device_errors(DEV)
    err = (out.float().cpu() - exp).abs()
    scale = float(exp.abs().max())
    assert float(err.max()) < 2e-2 * max(1.0, scale) and float(err.mean()) < 2e-3 * max(1.0, scale), \
        (float(err.max()), float(err.mean()), scale)
