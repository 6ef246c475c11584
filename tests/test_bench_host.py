"""Host-side logic of ``bench.py`` that needs no GPU: the config-5 wave plan and tables, the parity sample and its
check against the fp32 oracle, and the reference arm on the CPU-runnable configuration."""

import json

import pytest
import torch

import bench
import oracle
from belt_b200 import synth


def test_plan_waves_fits_every_request_once():
    lens = synth.log_uniform_lengths(200, 1024, 65536, seed=5)
    steps, page, block = 256, 16, 16 * 16 * 1024 * 2
    need = [-(-(n + steps) // page) for n in lens]
    waves, cap, nbuf = bench.plan_waves(lens, steps, page, block, free_bytes=40 << 30)
    assert nbuf == 2 and len(waves) > 1
    assert sorted(i for w in waves for i in w) == list(range(len(lens)))
    assert all(sum(need[i] for i in w) <= cap for w in waves)
    assert max(len(w) for w in waves) >= 1
    # longest first: the first wave holds the longest request
    assert max(lens) == lens[waves[0][0]]
    waves1, cap1, nbuf1 = bench.plan_waves(lens, steps, page, block, free_bytes=sum(need) * block)
    assert nbuf1 == 1 and len(waves1) == 1 and cap1 == sum(need)
    with pytest.raises(RuntimeError, match="does not fit"):
        bench.plan_waves([70000], steps, page, block, free_bytes=2 * 1000 * block)


def test_wave_tables_slots():
    base, steps, page = [40, 1, 300], 5, 16
    npages = [-(-(n + steps) // page) for n in base]
    cap = sum(npages) + 3
    t = bench.wave_tables(base, npages, cap, steps, page, seed=1)
    bt = t["block_table"]
    owned = torch.cat([bt[j, :n] for j, n in enumerate(npages)])
    assert len(set(owned.tolist())) == len(owned) and int(owned.max()) < cap
    for s in range(steps):
        assert t["seq_lens"][s].tolist() == [n + s + 1 for n in base]
        for j, n in enumerate(base):
            p = n + s
            assert int(t["slots"][s, j]) == int(bt[j, p // page]) * page + p % page
    pf = t["prefill_slots"]
    assert t["prefill_tokens"] == sum(base) == len(pf)
    allslots = torch.cat([pf, t["slots"].flatten()])
    assert len(set(allslots.tolist())) == len(allslots)          # every written position has its own slot


def test_parity_picks():
    r_k = [448, 576, 512, 512, 384, 384, 640, 640]
    layers, reqs = bench.parity_picks([5, 900, 30, 70000, 2], r_k)
    assert layers == [4, 2, 6]
    assert reqs == [0, 1, 3, 4]                                   # shortest, two between, longest


def test_check_parity_flags_an_output_off_the_oracle():
    spec = synth.c50(hidden=256)
    w = synth.make_layer(spec)
    lens = [40, 130]
    batch = synth.make_batch(w.layout, lens, page=16, poison=False)
    q = synth.make_queries(len(lens))
    ref = oracle.derive(w.k_up, w.v_up, w.k_norm_weight, w.layout, synth.cos_sin_table(200))
    exp = oracle.decode_fp32(q, batch.cache, batch.block_table, batch.seq_lens, ref, bench.SCALE)
    buf = batch.cache.unsqueeze(1)                                # [blocks, 1 layer, page, W]
    items = bench.gather_parity(buf, batch.block_table, lens, 16, q[None], exp[None], [0], [0, 1])
    good = bench.check_parity([w], items)
    assert good["ok"] and good["max_abs"] < 1e-5
    items[1]["out"] = items[1]["out"] + 0.05                        # an output that drifted from the oracle
    bad = bench.check_parity([w], items)
    assert not bad["ok"] and bad["max_abs"] >= 0.05


def test_reference_arm_on_the_cpu_runnable_config(capsys):
    class Args:
        config, batch, rows, warmup, steps, gpus = 1, None, "c50", 0, 1, 1
        cpu_seconds, cpu_full = 5.0, True
    bench.run_reference_arm(Args, 0, 1)
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["extrapolated"] is False
    assert line["samples"]["timed_context_tokens_per_pass"] == 129 + 513 + 1025 + 2001
    assert line["value"] > 0 and line["e2e"]["h2d_bytes_per_step"] == 0


def test_prefill_rounds_cover_every_context_once():
    from belt_b200.latent_backend import plan_prefill_rounds
    lens = [1000, 70, 450, 0, 384]
    for chunk in (384, 100, 1, 5000, 0):
        rounds = plan_prefill_rounds(lens, chunk)
        for i, L in enumerate(lens):
            ranges = [(k0, k1) for r in rounds for j, k0, k1 in r if j == i]
            assert [k for rng in ranges for k in range(*rng)] == list(range(L)), (chunk, i)
        for r in rounds:
            assert len({j for j, _, _ in r}) == len(r)                       # a request at most once per round
            if chunk > 0:
                assert sum(k1 - k0 for _, k0, k1 in r) <= chunk
