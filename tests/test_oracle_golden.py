"""Pin the CPU oracle (and the product's export restatement) to golden vectors made by the reference's own code."""

import math

import pytest
import torch

import oracle
from belt_b200 import latent_format, synth

from conftest import CASES, bf16_ulp_close, golden_case, sha

SCALE = 256 ** -0.5


@pytest.fixture(scope="module", params=CASES)
def case(request):
    fx, spec, w, batch, q = golden_case(request.param)
    cos_sin = oracle.rope_cos_sin(4096, 64, synth.THETA)
    layer = oracle.derive(w.k_up, w.v_up, w.k_norm_weight, w.layout, cos_sin)
    return request.param, fx, spec, w, batch, q, layer


def test_inputs_regenerate(case):
    name, fx, spec, w, batch, q, layer = case
    assert sha(torch.nan_to_num(batch.cache.float(), nan=7.0)) == fx["inputs_sha"]["cache"]
    assert sha(batch.block_table) == fx["inputs_sha"]["block_table"]
    assert sha(q) == fx["inputs_sha"]["q"]


def test_export_matches_reference(case):
    """The product's ``latent_tensors`` and the oracle's ``build_latent_layer`` give the reference's tensors bit for
    bit."""
    name, fx, spec, w, batch, q, layer = case
    assert w.layout == fx["layout"]
    assert sha(w.kv_latent_proj) == fx["factors_sha"]["kv_latent_proj"]
    assert sha(w.k_up) == fx["factors_sha"]["k_up"]
    assert sha(w.v_up) == fx["factors_sha"]["v_up"]
    kb, vf, kn = synth.make_factors(spec, synth.SEED_FACTORS)
    proj, k_up, v_up, layout = oracle.build_latent_layer(kb, vf, 4, 256, 64, rope_align=spec.rope_align)
    assert layout == fx["layout"] and sha(k_up) == fx["factors_sha"]["k_up"] and sha(proj) == \
        fx["factors_sha"]["kv_latent_proj"]
    for r_k, r_v in [(512, 512), (448, 576), (640, 384)]:
        ranks = [r_k // 4] * 4
        assert latent_format.row_layout(ranks, r_v, 64) == oracle.row_layout(ranks, r_v, 64)
        assert latent_format.row_layout(ranks, r_v, 64, rope_align=True) == \
            oracle.row_layout(ranks, r_v, 64, rope_align=True)
    for ranks in ([96, 112, 144, 160], [48, 40, 64, 56], [64, 16, 64, 8]):
        assert latent_format.row_layout(ranks, 300, 64, rope_align=True) == \
            oracle.row_layout(ranks, 300, 64, rope_align=True)


def test_derive_matches_reference(case):
    name, fx, spec, w, batch, q, layer = case
    d = fx["derive"]
    assert sha(layer["qmap"]) == d["qmap"]
    assert sha(layer["u_cat"]) == d["u_cat"]
    assert torch.equal(layer["k_segs"], d["k_segs"])
    assert torch.equal(layer["rope_gain"], d["rope_gain"])
    assert [tuple(g) for g in d["groups"]] == list(layer["groups"])
    assert torch.equal(layer["blocks"], d["blocks"])
    assert sha(layer["cos_sin"]) == d["cos_sin"]
    assert sha(layer["rope_up"]) == d["rope_up"]
    assert sha(layer["v_up"]) == d["v_up_t"]
    assert layer["n_k"] == d["n_k"]


def test_cos_sin_matches_vllm(common_golden):
    t = oracle.rope_cos_sin(common_golden["max_pos"], 64, common_golden["theta"])
    assert sha(t) == common_golden["cos_sin_sha_f32"]
    assert sha(synth.cos_sin_table(common_golden["max_pos"])) == common_golden["cos_sin_sha_f32"]


def test_block_diag_query(case):
    name, fx, spec, w, batch, q, layer = case
    q_bd = oracle.block_diag_query(q, layer["qmap"])
    assert bf16_ulp_close(q_bd, fx["q_bd"], ulps=1)
    if "q_bd_construct_sha" in fx:
        # the reference construction of the same query from q_lat / q_rot (``cute_decode.py:610-623``)
        rot = 64
        k_off = [runs[0][0] for runs in w.layout["k_segments"]]
        B = q.shape[0]
        qlat = torch.zeros(B, 24, max(spec.k_ranks))
        for g, r in enumerate(spec.k_ranks):
            cols = torch.arange(k_off[g], k_off[g] + r)
            qlat[:, 6 * g:6 * g + 6, :r] = torch.einsum("bhd,dk->bhk", q[:, 6 * g:6 * g + 6, rot:].float(),
                                                        layer["qmap"][g, rot:][:, cols].float())
        assert sha(qlat.to(torch.bfloat16)) == fx["q_lat_sha"]
        qc = oracle.block_diag_query_construct(qlat.to(torch.bfloat16), q[..., :rot], k_off, list(spec.k_ranks),
                                               w.layout["v_offset"])
        assert sha(qc) == fx["q_bd_construct_sha"]
        assert bf16_ulp_close(qc, q_bd, ulps=1)


def test_decompress(case):
    name, fx, spec, w, batch, q, layer = case
    smp = fx["decompress"]
    b = smp["b"]
    rows, pos = oracle.gather_rows(batch.cache, batch.block_table, b, int(batch.seq_lens[b]))
    k, v = oracle.decompress(layer, rows[smp["idx"]], pos[smp["idx"]])
    assert bf16_ulp_close(k, smp["k"], ulps=2)
    assert bf16_ulp_close(v, smp["v"], ulps=2)


def test_decode_reference(case):
    """Oracle A (the reference's torch path) reproduces the reference's output; Oracle B (fp32) is within the BF16
    tolerance of it."""
    name, fx, spec, w, batch, q, layer = case
    out_a = oracle.decode_reference(q, batch.cache, batch.block_table, batch.seq_lens, layer, SCALE)
    ref = fx["out_reference"]
    assert torch.allclose(out_a, ref, atol=5e-4, rtol=0), float((out_a - ref).abs().max())
    out_b = oracle.decode_fp32(q, batch.cache, batch.block_table, batch.seq_lens, layer, SCALE)
    err = (out_b - ref).abs()
    assert float(err.max()) < 2e-2 and float(err.mean()) < 2e-3, (float(err.max()), float(err.mean()))


@pytest.mark.parametrize("tile,num_ctas", [(128, 148), (128, 16), (64, 148), (64, 7)])
def test_kernel_path_restatement(case, tile, num_ctas):
    """The split-KV restatement with the kernel's rounding points stays within tolerance of the fp32 oracle, for
    any tile size and CTA count."""
    name, fx, spec, w, batch, q, layer = case
    out, a, lse, q_bd = oracle.decode_kernel_path(q, batch.cache, batch.block_table, batch.seq_lens, layer, SCALE,
                                                  tile, num_ctas)
    out_b = oracle.decode_fp32(q, batch.cache, batch.block_table, batch.seq_lens, layer, SCALE)
    err = (out.float() - out_b).abs()
    assert float(err.max()) < 2e-2 and float(err.mean()) < 2e-3, (float(err.max()), float(err.mean()))


def test_up_project(case):
    name, fx, spec, w, batch, q, layer = case
    B = q.shape[0]
    a = torch.randn(B, 24, spec.v_rank, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    assert sha(a) == fx["up_a_sha"]
    assert bf16_ulp_close(oracle.up_project(a, layer["v_up"]), fx["up_out"], ulps=1)


def test_latent_rows(case):
    name, fx, spec, w, batch, q, layer = case
    W = w.layout["row_width"]
    page = fx["page"]
    gcw = torch.Generator().manual_seed(9)
    c = (torch.randn(24, W, generator=gcw) * synth.latent_columns(w.layout)).to(torch.bfloat16)
    assert sha(c) == fx["cw_c_sha"]
    nb = fx["cw_nb"]
    slots = fx["cw_slots"]
    cache = torch.full((nb, page, W), float("nan")).to(torch.bfloat16)
    oracle.latent_rows(c, slots, cache, layer["u_cat"], layer["k_segs"], 1e-6)
    live = slots >= 0
    assert bf16_ulp_close(cache.view(-1, W)[slots[live].long()], fx["cw_rows"], ulps=1)
    assert int(torch.isnan(cache.float()).sum()) == fx["cw_untouched_nan"]


def test_schedule(common_golden):
    for s in common_golden["schedule"]:
        work, cta_seg, seg_base = oracle.schedule(s["seq_lens"], s["num_ctas"], s["tile"])
        total = int(seg_base[-1])
        assert torch.equal(torch.from_numpy(work[:total]), s["work"]), s["seq_lens"]
        assert torch.equal(torch.from_numpy(cta_seg), s["cta_seg"])
        assert torch.equal(torch.from_numpy(seg_base), s["seg_base"])


def test_merge(common_golden):
    for m in common_golden["merge"]:
        g = torch.Generator().manual_seed(11)
        part = torch.randn(*m["part_shape"], generator=g)
        lv = m["part_shape"][-1] - 1
        part[:, :, lv] *= 4
        assert sha(part) == m["part_sha"]
        B = len(m["seq_lens"])
        a, lse = oracle.merge_segments(part, m["seg_base"], B, lv)
        assert torch.allclose(a, m["a"], atol=1e-5, rtol=1e-5)
        assert torch.allclose(lse, m["lse"], atol=1e-5, rtol=0) or torch.equal(torch.isinf(lse), torch.isinf(m["lse"]))
        live = torch.isfinite(m["lse"])
        assert torch.allclose(lse[live], m["lse"][live], atol=1e-5)
        assert torch.equal(torch.isinf(lse), torch.isinf(m["lse"]))


def test_schedule_invariants():
    """Every tile of every request is covered once, in order, and each CTA's run is contiguous."""
    g = torch.Generator().manual_seed(3)
    for trial in range(20):
        B = int(torch.randint(1, 300, (1,), generator=g))
        seqs = torch.randint(0, 5000, (B,), generator=g).tolist()
        nct = int(torch.randint(1, 200, (1,), generator=g))
        for tile in (64, 128):
            work, cta_seg, seg_base = oracle.schedule(seqs, nct, tile)
            total = int(seg_base[B])
            for b in range(B):
                segs = work[seg_base[b]:seg_base[b + 1]]
                tiles = math.ceil(seqs[b] / tile)
                if tiles == 0:
                    assert len(segs) == 0
                    continue
                assert segs[0][1] == 0 and segs[-1][2] == tiles and (segs[:, 0] == b).all()
                assert (segs[1:, 1] == segs[:-1, 2]).all()
            assert cta_seg[0] == 0 and cta_seg[nct] == total and (cta_seg[1:] >= cta_seg[:-1]).all()


def test_schedule_weighted_invariants():
    """The cost-weighted split: every tile covered once and in order, contiguous CTA runs, at most B + num_ctas
    segments, start cost 0 splitting like the reference split of 8-unit tiles, and a CTA holding request starts never
    getting more tiles than the cost bound allows."""
    g = torch.Generator().manual_seed(5)
    for trial in range(20):
        B = int(torch.randint(1, 200, (1,), generator=g))
        seqs = torch.randint(0, 5000, (B,), generator=g).tolist()
        nct = int(torch.randint(1, 160, (1,), generator=g))
        for start_cost in (0, 3, 10, 40):
            work, cta_seg, seg_base = oracle.schedule_weighted(seqs, nct, 128, start_cost)
            total = int(seg_base[B])
            assert total <= B + nct
            for b in range(B):
                segs = work[seg_base[b]:seg_base[b + 1]]
                tiles = math.ceil(seqs[b] / 128)
                if tiles == 0:
                    assert len(segs) == 0
                    continue
                assert segs[0][1] == 0 and segs[-1][2] == tiles and (segs[:, 0] == b).all()
                assert (segs[1:, 1] == segs[:-1, 2]).all() and (segs[:, 2] > segs[:, 1]).all()
            assert cta_seg[0] == 0 and cta_seg[nct] == total and (cta_seg[1:] >= cta_seg[:-1]).all()
            # cost per CTA (8 per tile + start_cost per request start it holds) stays within per + one tile
            cost_total = sum(start_cost + 8 * math.ceil(L / 128) for L in seqs if L > 0)
            per = max(-(-cost_total // nct), 8)
            for c in range(nct):
                segs = work[cta_seg[c]:cta_seg[c + 1]]
                cost = sum(8 * int(s[2] - s[1]) + (start_cost if s[1] == 0 else 0) for s in segs)
                assert cost <= per + 8 + start_cost, (c, cost, per)
