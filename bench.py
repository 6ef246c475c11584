"""Benchmark of the latent-KV decode step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 3|2] [--impl ours|reference]

Workload (the headline configuration the north star names, per GPU): 16 compressed full-attention layers with learned
per-layer ranks (r_k from {384, 448, 512, 576, 640}, r_v = 1024 - r_k, row width 1024), batch 128, context lengths
log-uniform in [1k, 64k], block size 16, BF16, random-permuted block tables, one block holding all 16 layers' pages
(block-outermost, strided per-layer views). ``--config 2`` runs the single-layer c50 case (batch 64 x 8192).

A step is one decode step of the path over the batch: the split-KV schedule once, then per layer the cache write of
the new token's row, the absorbed block-diagonal query, the decode kernel, the segment merge and the U_v
up-projection. ``value`` is whole-job decode tokens/s (sequences x GPUs / step time, device-timed with CUDA events,
max over ranks); the cache (tens of GB) is far larger than L2, so every step streams it from HBM. ``e2e`` runs the same
step through the backend's public API (``LatentAttentionImpl.forward``) from pinned host buffers: this step's queries
and latent rows are copied in and the attention outputs copied out inside the timed region.

Multi-GPU: one process per GPU (torchrun), each with its own 128 sequences (weak scaling, data parallel, no
collective on the data path; a gloo barrier and a max over ranks only bracket the timing).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from belt_b200 import decode as dec  # noqa: E402
from belt_b200 import dp, latent_ops, synth  # noqa: E402

METRIC = "decode tokens/s/GPU and % of latent-attn roofline at 1/2/4/8 B200 (DP)"
H, D = 24, 256
SCALE = D ** -0.5


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=3, choices=[2, 3, 4])
    ap.add_argument("--rows", default="c50", choices=["c50", "c25"],
                    help="config 4 row format: c50 (r_k = r_v = 512, 1024-column rows) or c25 (256 + 256, 512 columns)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU work budget of one baseline sample")
    ap.add_argument("--prefill", action="store_true",
                    help="measure the prefill path instead (one GPU): keys / values rebuilt from the paged rows and "
                         "causal attention of 8192 new tokens over an 8192-token context, one c50 layer")
    return ap.parse_args()


# ------------------------------------------------------------------------------------------------------------ workload
def workload_spec(config: int, batch: int | None, rank: int, world: int, rows: str = "c50"):
    """(layer specs, this rank's seq_lens, page, description, partition imbalance). The box holds batch x world
    requests; ranks take LPT shares by context tokens (equal counts), so every rank decodes ~batch requests."""
    if config == 2:
        B = batch or 64
        return [synth.c50()], [8192 + 1] * B, 16, {"workload": "config2: 1 layer c50, batch 64 x 8192, page 16"}, 1.0
    if config == 4:
        # long context: every request 65,536 cached tokens + this step's, 512 tiles each over the CTAs
        B = batch or 32
        spec = synth.c25() if rows == "c25" else synth.c50()
        return [spec] * 16, [65536 + 1] * B, 16, {
            "workload": f"config4: 16 layers {rows} (rows of {spec.row_width} columns), batch 32 x 65536, page 16"}, 1.0
    B = batch or 128
    ranks = synth.learned_ranks(16)
    pool = synth.log_uniform_lengths(B * world, 1024, 65536, seed=synth.SEED_LENGTHS)
    parts = dp.partition_lpt(pool, world)
    lens = [pool[i] for i in parts[rank]]
    specs = [synth.spec_from_ranks(rk, rv) for rk, rv in ranks]
    return specs, [L + 1 for L in lens], 16, {
        "workload": "config3: 16 layers, learned ranks (r_k in {384..640}, r_v = 1024 - r_k), batch 128/GPU, "
                    "context log-uniform [1k, 64k], page 16"}, dp.imbalance(pool, parts)


class Workload:
    def __init__(self, specs, seq_lens, page, device, rank):
        from belt_b200.layer import derive_latent_tensors
        self.device = device
        self.L = len(specs)
        self.B = len(seq_lens)
        self.page = page
        self.seq_lens_list = seq_lens
        max_pos = max(seq_lens) + 1
        cos_sin = synth.cos_sin_table(max_pos)
        self.weights = [synth.make_layer(s, seed=synth.SEED_FACTORS + i) for i, s in enumerate(specs)]
        self.layers = [derive_latent_tensors(w.k_up, w.v_up, w.k_norm_weight, w.layout, cos_sin, device=device)
                       for w in self.weights]
        Ws = [w.layout["row_width"] for w in self.weights]
        assert len(set(Ws)) == 1, "one row width per benchmark"
        self.W = W = Ws[0]
        bt, nb, _ = synth.block_tables(seq_lens, page, extra_blocks=4, seed=synth.SEED_CACHE + rank)
        self.num_blocks = nb
        self.block_table = bt.to(device)
        self.seq_lens = torch.tensor(seq_lens, dtype=torch.int32, device=device)
        # one block holds every layer's page side by side (block-outermost)
        self.buf = torch.empty(nb, self.L, page, W, dtype=torch.bfloat16, device=device)
        for l, w in enumerate(self.weights):
            synth.fill_cache(self.buf[:, l], w.layout, self.block_table, seq_lens, seed=synth.SEED_CACHE + 101 * l + rank,
                             poison=False)
        self.caches = [self.buf[:, l] for l in range(self.L)]
        gq = torch.Generator(device=device).manual_seed(synth.SEED_QUERY + rank)
        self.q = torch.randn(self.L, self.B, H, D, generator=gq, device=device, dtype=torch.bfloat16)
        hiddens = {s.hidden for s in specs}
        assert len(hiddens) == 1, "one hidden size per benchmark"
        self.hidden = hiddens.pop()
        # this step's layer inputs of the new tokens, down-projected into the cache rows by the fused write
        self.x = torch.randn(self.L, self.B, self.hidden, generator=gq, device=device, dtype=torch.bfloat16)
        self.w_down = [w.kv_latent_proj.to(device) for w in self.weights]
        pos = torch.tensor(seq_lens) - 1
        self.slots = (bt[torch.arange(self.B), pos // page].long() * page + pos % page).to(device)
        self.sched = dec.make_schedule(self.B, device)
        self.side = torch.cuda.Stream(device)
        self.part = torch.empty(self.B + self.sched.num_ctas, H, 641, dtype=torch.float32, device=device)
        self.a = torch.empty(self.B, H, 640, dtype=torch.bfloat16, device=device)
        self.lse = torch.empty(self.B, H, dtype=torch.float32, device=device)
        self.out = torch.empty(self.L, self.B, H, D, dtype=torch.bfloat16, device=device)

    # -------------------------------------------------------------------------------------------------------- step
    def step(self, dec_events=None):
        """One decode step over all layers through the operator API; ``dec_events`` [(start, end)] brackets every
        decode-kernel launch."""
        dec.schedule(self.sched, self.seq_lens)
        main = torch.cuda.current_stream(self.device)
        for l, lat in enumerate(self.layers):
            # the new rows on the side stream, overlapping the absorbed query (the backend's side-stream write)
            self.side.wait_stream(main)
            with torch.cuda.stream(self.side):
                latent_ops.project_rows_to_cache(self.x[l], self.w_down[l], self.slots, self.caches[l], lat.u_cat,
                                                 lat.k_segs_host, lat.eps)
            q_bd = lat.block_diag_query(self.q[l])
            main.wait_stream(self.side)
            part = self.part[:, :, :lat.v_rank + 1]
            if dec_events is not None:
                dec_events[l][0].record()
            dec.latent_decode(q_bd, self.caches[l], self.block_table, self.seq_lens, self.sched, part, SCALE,
                              lat.v_offset, lat.v_rank, rope=lat.rope)
            if dec_events is not None:
                dec_events[l][1].record()
            a = self.a[:, :, :lat.v_rank]
            dec.merge_segments(part, self.sched, a, self.lse)
            lat.up_project(a, self.out[l])

    launches_per_step = property(lambda self: 1 + 5 * self.L)

    # ------------------------------------------------------------------------------------------------ algorithmic units
    def decode_kernel_bytes(self, l: int) -> int:
        """Algorithmic bytes of one decode-kernel launch: every context row read once, the block-diagonal query."""
        lat = self.layers[l]
        rows = sum(self.seq_lens_list) * self.W * 2
        kq = lat.n_k * 64 + 4 * 64
        return rows + self.B * H * kq * 2

    def step_bytes(self) -> int:
        """Algorithmic bytes of one step, summed over layers: context rows read once, the factors (U_k, U_v and the
        down-projection W_down), q in and out, the new tokens' inputs and their rows written."""
        tot = 0
        for l, lat in enumerate(self.layers):
            lay = self.weights[l].layout
            rows = sum(self.seq_lens_list) * self.W * 2
            factors = 2 * (sum(256 * r for r in lay["k_head_ranks"]) + 4 * 256 * lay["v_rank"] + self.W * self.hidden)
            qo = 2 * self.B * H * D * 2
            tot += rows + factors + qo + 2 * self.B * (self.hidden + self.W)
        return tot


# ------------------------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock, power and clock-event reasons of this rank's GPU, sampled every 10 ms by a thread reading NVML while
    the timed region runs (``nvidia-smi -lms 200`` as the fallback when NVML is unavailable)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device: torch.device):
        self.device = device
        self.samples = []            # (sm MHz, max sm MHz, power W, {reason names})
        self.thread = self.proc = self.path = None
        self.stop_flag = False
        self.source = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.device).uuid)
        for cand in (uuid, "GPU-" + uuid):
            try:
                return pynvml, pynvml.nvmlDeviceGetHandleByUUID(cand)
            except pynvml.NVMLError:
                pass
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.device.index or 0)

    def _poll(self, nv, h):
        bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
        smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while not self.stop_flag:
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((float(sm), float(smax), pw, {n for n, b in bits.items() if r & b}))
            except nv.NVMLError:
                pass
            time.sleep(0.01)

    def start(self):
        # the timed loop is Python issuing launches: a 1 ms interpreter switch interval lets the sampling thread run
        self.switch = sys.getswitchinterval()
        sys.setswitchinterval(0.001)
        try:
            import threading
            nv, h = self._nvml_handle()
            self.thread = threading.Thread(target=self._poll, args=(nv, h), daemon=True)
            self.thread.start()
            self.source = "nvml 10 ms"
            return
        except Exception:  # NVML missing or refused: fall back to nvidia-smi
            self.thread = None
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device.index or 0), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            self.source = "nvidia-smi 200 ms"
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read_smi(self):
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                self.samples.append((float(f[1]), float(f[2]), float(f[3]),
                                     {n for n, v in zip(self.REASONS, f[5:9]) if v.lower() == "active"}))
            except ValueError:
                continue
        os.unlink(self.path)

    def stop(self) -> dict:
        sys.setswitchinterval(getattr(self, "switch", 0.005))
        if self.thread is not None:
            self.stop_flag = True
            self.thread.join(timeout=5)
        elif self.proc is not None:
            self._read_smi()
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock source"]}
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        power = [s[2] for s in self.samples]
        loaded = [s for s in self.samples if s[2] > 0.3 * max(power)] or self.samples
        reasons = sorted(set().union(*(s[3] for s in self.samples)))
        return {"sm_mhz": statistics.median(s[0] for s in loaded), "sm_max_mhz": max(s[1] for s in self.samples),
                "reasons": reasons, "samples": len(self.samples), "power_w_max": max(power), "source": self.source}


# ------------------------------------------------------------------------------------------------------------ CPU arm
def cpu_reference_rate(specs, seq_lens, page, budget_s: float, rank: int = 0):
    """Decode tokens/s of the reference's torch path (the oracle port of ``LatentLayer.decompress`` + fp32 attention)
    on this host's cores, extrapolated to the whole workload from a bounded sample of requests of the first layer.
    Returns (tokens/s, cores, sample description, seconds)."""
    import oracle
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    w = synth.make_layer(specs[0], seed=synth.SEED_FACTORS)
    total_ctx = sum(seq_lens)
    # calibrate on a short request, then size the sample to the budget
    order = sorted(range(len(seq_lens)), key=lambda i: seq_lens[i])
    probe = [seq_lens[order[len(order) // 2]]]
    t_probe = _cpu_time(w, probe, page)
    per_tok = t_probe / sum(probe)
    want = max(1, int(budget_s / per_tok))
    sample, acc = [], 0
    for i in order[len(order) // 4:] + order[:len(order) // 4]:
        if acc + seq_lens[i] > want and sample:
            break
        sample.append(seq_lens[i])
        acc += seq_lens[i]
    t = _cpu_time(w, sample, page)
    per_tok = t / sum(sample)
    step_s = per_tok * total_ctx * len(specs)                 # every layer of every sequence
    rate = len(seq_lens) / step_s
    desc = (f"oracle port of the reference torch path (decompress + fp32 attention), layer 0, {len(sample)} requests "
            f"/ {sum(sample)} context tokens timed ({t:.1f} s), extrapolated per context token to {len(specs)} layers "
            f"x {total_ctx} tokens")
    return rate, cores, desc, t


def _cpu_time(w, lens, page):
    import oracle
    cos_sin = synth.cos_sin_table(max(lens) + 1)
    ref = oracle.derive(w.k_up, w.v_up, w.k_norm_weight, w.layout, cos_sin)
    batch = synth.make_batch(w.layout, lens, page=page, seed=synth.SEED_CACHE, poison=False)
    q = synth.make_queries(len(lens))
    t0 = time.perf_counter()
    oracle.decode_reference(q, batch.cache, batch.block_table, batch.seq_lens, ref, SCALE)
    return time.perf_counter() - t0


def run_reference_arm(args, rank, world):
    """The reference's CPU path on the whole box's requests (every rank's share), rank 0 only."""
    if rank != 0:
        return
    per_gpu = args.batch or {2: 64, 3: 128, 4: 32}[args.config]
    specs, seq_lens, page, cfg, _ = workload_spec(args.config, per_gpu * world, 0, 1, args.rows)
    rates, tsum = [], 0.0
    for i in range(args.warmup + args.steps):
        budget = min(args.cpu_seconds, 240.0 / max(1, args.warmup + args.steps))
        rate, cores, desc, t = cpu_reference_rate(specs, seq_lens, page, budget)
        if i >= args.warmup:
            rates.append(rate)
            tsum += t
    value = statistics.median(rates)
    ms = 1000.0 * len(seq_lens) / value
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference",
            "config": {**cfg, "global_batch": len(seq_lens), "parallelism": "dp (rank 0 only: CPU)"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": desc},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------------------ e2e
def e2e_rate(wl: Workload, steps: int, warmup: int):
    """Decode tokens/s through the backend's public surface (``latent_attention_step``: the fused down-projection
    cache write, then ``LatentAttentionImpl.forward``), with this step's inputs (queries, layer inputs of the new
    tokens, positions) copied from pinned host memory and the attention outputs copied back inside the timed region,
    on a copy stream that overlaps them with the layers' compute."""
    from belt_b200.latent_backend import (CommonAttentionMetadata, LatentAttentionImpl,
                                          LatentAttentionMetadataBuilder, LatentKVSpec, latent_attention_step)
    dev = wl.device
    B, L = wl.B, wl.L
    q_host = wl.q.cpu().pin_memory()
    x_host = wl.x.cpu().pin_memory()
    pos_host = (torch.tensor(wl.seq_lens_list) - 1).pin_memory()
    out_host = torch.empty(L, B, H, D, dtype=torch.bfloat16).pin_memory()
    q_dev, x_dev = torch.empty_like(wl.q), torch.empty_like(wl.x)
    pos_dev = torch.empty(B, dtype=torch.int64, device=dev)
    out_dev = torch.empty(L, B, H, D, dtype=torch.bfloat16, device=dev)
    spec = LatentKVSpec(block_size=wl.page, num_kv_heads=1, head_size=wl.W)
    builder = LatentAttentionMetadataBuilder(spec, [f"layers.{l}" for l in range(L)], device=dev,
                                             max_num_batched_tokens=max(256, B))
    impl = LatentAttentionImpl(H, D, SCALE, 4)

    class _Layer:
        def __init__(self, lat):
            self.latent = lat
    layer_objs = [_Layer(lat) for lat in wl.layers]
    kv = wl.buf.view(wl.num_blocks, L, 1, wl.page, wl.W)
    qsl = torch.arange(B + 1, dtype=torch.int32)
    qsl_dev = qsl.to(dev)

    # the copies run on their own stream: every layer's inputs go up at the start of the step, layer l waits only for
    # its own, and its output goes down as soon as it is written, while the next layers compute; the step ends when
    # the last output has landed in host memory
    copy = torch.cuda.Stream(dev)
    in_ready = [torch.cuda.Event() for _ in range(L)]
    out_done = [torch.cuda.Event() for _ in range(L)]

    def one():
        main = torch.cuda.current_stream(dev)
        copy.wait_stream(main)
        with torch.cuda.stream(copy):
            pos_dev.copy_(pos_host, non_blocking=True)
            for l in range(L):
                q_dev[l].copy_(q_host[l], non_blocking=True)
                x_dev[l].copy_(x_host[l], non_blocking=True)
                in_ready[l].record(copy)
        cm = CommonAttentionMetadata(query_start_loc=qsl_dev, query_start_loc_cpu=qsl, seq_lens=wl.seq_lens,
                                     block_table_tensor=wl.block_table, slot_mapping=wl.slots, num_reqs=B,
                                     num_actual_tokens=B, max_query_len=1)
        md = builder.build(0, cm)
        for l in range(L):
            main.wait_event(in_ready[l])
            latent_attention_step(impl, layer_objs[l], q_dev[l], x_dev[l], wl.w_down[l], kv[:, l], md, out_dev[l])
            out_done[l].record(main)
            copy.wait_event(out_done[l])
            with torch.cuda.stream(copy):
                out_host[l].copy_(out_dev[l], non_blocking=True)
        main.wait_stream(copy)

    for _ in range(warmup):
        one()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        one()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    h2d = q_host.numel() * 2 + x_host.numel() * 2 + pos_host.numel() * 8
    d2h = out_host.numel() * 2
    return B / (ms / 1000.0), ms, h2d, d2h


def read_traffic():
    """Per-launch DRAM bytes of the decode kernel from the committed ncu summary (None until captured)."""
    path = os.path.join(ROOT, "profiles", "decode_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


def run_prefill(args):
    """One c50 layer's prefill of an 8192-token request through the backend's kernels: decompress of the context
    (keys and values from the paged rows) and the causal attention, timed on the device (inputs resident, L2 flushed
    between steps); torch's scaled_dot_product_attention on the same keys and values timed beside it."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    from belt_b200 import build as _build
    from belt_b200 import latent_ops
    from belt_b200.layer import derive_latent_tensors
    _build.build()
    L, page = 8192, 16
    w = synth.make_layer(synth.c50(), seed=synth.SEED_FACTORS)
    lat = derive_latent_tensors(w.k_up, w.v_up, w.k_norm_weight, w.layout, synth.cos_sin_table(L + 1), device=dev)
    bt, nb, _ = synth.block_tables([L], page, extra_blocks=1, seed=synth.SEED_CACHE)
    W = w.layout["row_width"]
    cache = torch.empty(nb, page, W, dtype=torch.bfloat16, device=dev)
    synth.fill_cache(cache, w.layout, bt.to(dev), [L], seed=synth.SEED_CACHE, poison=False)
    btd = bt.to(dev)
    q = synth.make_queries(L).to(dev)
    k = torch.empty(L, 4, 256, dtype=torch.bfloat16, device=dev)
    v = torch.empty_like(k)
    out = torch.empty(L, 24, 256, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(L, 24, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def step():
        lat.decompress_paged(cache, btd[0], L, 0, L, k, v)
        latent_ops.prefill_attention(q, k, v, 0, 0, SCALE, True, out, lse)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    dec.check_device_errors(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for s, e in ev:
        flush.add_(1)
        s.record()
        step()
        e.record()
    torch.cuda.synchronize()
    ms = statistics.mean(s.elapsed_time(e) for s, e in ev)
    qh = q.transpose(0, 1).unsqueeze(0)
    kh = k.transpose(0, 1).repeat_interleave(6, 0).unsqueeze(0)
    vh = v.transpose(0, 1).repeat_interleave(6, 0).unsqueeze(0)
    lib_ms = None
    try:
        for _ in range(2):
            torch.nn.functional.scaled_dot_product_attention(qh, kh, vh, is_causal=True, scale=SCALE)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(3):
            torch.nn.functional.scaled_dot_product_attention(qh, kh, vh, is_causal=True, scale=SCALE)
        e.record()
        torch.cuda.synchronize()
        lib_ms = s.elapsed_time(e) / 3
    except RuntimeError:
        pass
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        pass
    peak_tf = peaks.get("bf16_tflops") or 1590.0
    flops = 24 * (L * (L + 1) / 2) * 256 * 2 * 2 + L * 2 * 256 * 4 * (320 + 512)   # attention + decompress
    line = {"metric": "prefill tokens/s (decompress + causal attention, one c50 layer)", "value": L / (ms / 1e3),
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "prefill: 8192 new tokens over an 8192-token context, c50 layer, page 16",
                       "l2": "flushed (256 MB write) before every step"},
            "roofline": {"bound": "tensor", "achieved": flops / (ms / 1e3) / 1e12, "peak": peak_tf,
                         "unit": "TFLOP/s", "frac": flops / (ms / 1e3) / 1e12 / peak_tf,
                         "peak_source": "measured" if "bf16_tflops" in peaks else "fallback"},
            "library_sdpa_attention_ms": lib_ms, "gpu_launches": 2 * args.steps}
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.prefill:
        if rank == 0:
            run_prefill(args)
        return
    group = dp.HostGroup()
    local = group.local_rank
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from belt_b200 import build as _build
    _build.build()
    specs, seq_lens, page, cfg, imb = workload_spec(args.config, args.batch, rank, world, args.rows)
    wl = Workload(specs, seq_lens, page, dev, rank)
    torch.cuda.synchronize()

    for _ in range(max(args.warmup, 3)):
        wl.step()
    torch.cuda.synchronize()
    dec.check_device_errors(dev)

    dec_events = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(wl.L)] for _ in range(args.steps)]
    clocks = ClockSampler(dev)
    group.barrier()
    clocks.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    group.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for k in range(args.steps):
        wl.step(dec_events[k])
    end.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    group.barrier()
    ms_local = start.elapsed_time(end) / args.steps
    ms = group.max(ms_local)
    dec.check_device_errors(dev)
    total_reqs = group.sum(wl.B)
    value = total_reqs / (ms / 1000.0)

    # the decode kernel's launches, per layer
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        pass
    peak_gbs = peaks.get("hbm_gbs") or 6650.0
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    kern_ms = [statistics.mean(dec_events[k][l][0].elapsed_time(dec_events[k][l][1]) for k in range(args.steps))
               for l in range(wl.L)]
    kern_bytes = [wl.decode_kernel_bytes(l) for l in range(wl.L)]
    achieved = sum(kern_bytes) / (sum(kern_ms) / 1000.0) / 1e9
    step_gb = wl.step_bytes() / 1e9
    step_frac = step_gb / (ms_local / 1000.0) / peak_gbs
    traffic = read_traffic()
    traffic_per_launch = None
    if traffic and traffic.get("bytes_per_context_token"):
        traffic_per_launch = traffic["bytes_per_context_token"] * sum(wl.seq_lens_list)

    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {**cfg, "global_batch": int(total_reqs), "per_gpu_batch": wl.B, "layers": wl.L,
                       "context_tokens_per_gpu": sum(wl.seq_lens_list), "parallelism": f"dp{world}",
                       "partition": "LPT by context tokens, equal request counts", "partition_imbalance": imb,
                       "l2": "inputs larger than L2 (cache %.1f GB per GPU)" % (wl.buf.numel() * 2 / 1e9),
                       "tokens_per_s_per_gpu": value / world,
                       "step_roofline_frac": step_frac, "step_algorithmic_gb": step_gb},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak_gbs, "unit": "GB/s",
                         "frac": achieved / peak_gbs, "peak_source": peak_src,
                         "kernel": "latent_decode_kernel", "kernel_ms_per_launch": sum(kern_ms) / wl.L,
                         "traffic": traffic_per_launch, "traffic_source": traffic and traffic.get("source")},
            "clocks": clk,
            "gpu_launches": wl.launches_per_step * args.steps}
    if not args.no_e2e:
        _, e_ms_local, h2d, d2h = e2e_rate(wl, max(2, args.steps // 2), 2)
        e_ms = group.max(e_ms_local)
        line["e2e"] = {"value": total_reqs / (e_ms / 1000.0), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                       "d2h_bytes_per_step": d2h, "ms_per_step": e_ms}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, cores, desc, t = cpu_reference_rate(specs, seq_lens, page, args.cpu_seconds)
        line["cpu_baseline"] = {"value": rate, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": desc}
    if rank == 0:
        print(json.dumps(line), flush=True)
    group.close()


if __name__ == "__main__":
    main()
