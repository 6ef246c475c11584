"""Benchmark of the latent-KV decode step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 3|1|2|4|5] [--impl ours|reference]

Workload (the headline configuration, per GPU): 16 compressed full-attention layers with learned per-layer ranks (r_k
from {384, 448, 512, 576, 640}, r_v = 1024 - r_k, row width 1024), batch 128, context lengths log-uniform in
[1k, 64k], block size 16, BF16, random-permuted block tables, one block holding all 16 layers' pages
(block-outermost, strided per-layer views). ``--config 2`` runs the single-layer c50 case (batch 64 x 8192),
``--config 4`` the long-context case (batch 32 x 65,536, ``--rows c25`` for the narrow rows), ``--config 1`` the
CPU-runnable case (4 requests, one layer; for the reference arm).

A step is one decode step of the path over the batch: the split-KV schedule once, then per layer the cache write of
the new token's row, the absorbed block-diagonal query, the decode kernel, and the segment merge with the U_v
up-projection (one kernel). ``value`` is whole-job decode tokens/s (sequences x GPUs / step time, device-timed with CUDA events,
max over ranks); the cache (tens of GB) is far larger than L2, so every step streams it from HBM. ``e2e`` runs the same
step through the backend's public API (``LatentAttentionImpl.forward``) from pinned host buffers: this step's queries
and latent rows are copied in and the attention outputs copied out inside the timed region.

After the timed steps the CPU leg runs the CPU restatement of the reference's path (``oracle``): as the checker of a
sample of the step just timed (``parity``: the outputs of 4 requests spanning the length range in 3 layers of
different ranks, against the fp32 oracle at max-abs 2e-2 / mean-abs 2e-3), and, at N = 1, timed on a bounded sample
as ``cpu_baseline``.

Multi-GPU: one process per GPU (torchrun), each with its own 128 sequences of the same lengths as the one-GPU run
(weak scaling with fixed work per GPU, data parallel, no collective on the data path; a gloo barrier and a max over
ranks only bracket the timing).

``--config 5`` is the box-level serving run: 1,024 sequences (config-3 ranks and lengths) partitioned across the N
ranks by LPT, each rank serving its share in waves that fit its HBM (two wave buffers: one decoding, the next one
being prefilled); every wave is prefilled by chunked latent cache writes of 8,192 tokens per layer (down-projection
+ paged scatter), then decoded for 256 steps with this step's cache write, the next wave's prefill chunks interleaved
between the decode steps. ``value`` = 1,024 x 256 decode tokens / max rank time (strong scaling: the total work is
fixed).
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
    ap.add_argument("--config", type=int, default=3, choices=[1, 2, 3, 4, 5])
    ap.add_argument("--rows", default="c50", choices=["c50", "c25"],
                    help="config 4 row format: c50 (r_k = r_v = 512, 1024-column rows) or c25 (256 + 256, 512 columns)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU work budget of one baseline sample")
    ap.add_argument("--cpu-full", action="store_true",
                    help="reference arm: time the whole workload (every request of every layer), no extrapolation")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check of the timed step's outputs")
    ap.add_argument("--decode-steps", type=int, default=256, help="config 5: decode steps per wave")
    ap.add_argument("--prefill-chunk", type=int, default=8192, help="config 5: tokens per chunked-prefill write")
    ap.add_argument("--num-seqs", type=int, default=1024, help="config 5: sequences on the box")
    ap.add_argument("--gemm", action="store_true",
                    help="measure the tensor-core GEMM on the model's linear-layer shapes instead (one GPU)")
    ap.add_argument("--prefill", action="store_true",
                    help="measure the prefill path instead (one GPU): keys / values rebuilt from the paged rows and "
                         "causal attention of 8192 new tokens over an 8192-token context, one c50 layer")
    return ap.parse_args()


# ------------------------------------------------------------------------------------------------------------ workload
def workload_spec(config: int, batch: int | None, rank: int, world: int, rows: str = "c50"):
    """(layer specs, this rank's seq_lens, page, description). Config 3 gives every rank the same request lengths
    (the one-GPU pool of ``batch`` requests), so the work per GPU is the same at every N."""
    if config == 1:
        return [synth.c50()], [129, 513, 1025, 2001], 16, {
            "workload": "config1: 1 layer c50, 4 requests with contexts {128, 512, 1024, 2000} + this step's, page 16"}
    if config == 2:
        B = batch or 64
        return [synth.c50()], [8192 + 1] * B, 16, {"workload": f"config2: 1 layer c50, batch {B} x 8192, page 16"}
    if config == 4:
        # long context: every request 65,536 cached tokens + this step's, 512 tiles each over the CTAs
        B = batch or 32
        spec = synth.c25() if rows == "c25" else synth.c50()
        return [spec] * 16, [65536 + 1] * B, 16, {
            "workload": f"config4: 16 layers {rows} (rows of {spec.row_width} columns), batch {B} x 65536, page 16"}
    ranks = synth.learned_ranks(16)
    specs = [synth.spec_from_ranks(rk, rv) for rk, rv in ranks]
    if config == 5:
        n = batch or 1024
        return specs, serving_pool(n), 16, {
            "workload": f"config5: {n} sequences on the box, 16 layers with config-3 ranks, context log-uniform "
                        "[1k, 64k], page 16"}
    B = batch or 128
    lens = synth.log_uniform_lengths(B, 1024, 65536, seed=synth.SEED_LENGTHS)
    return specs, [L + 1 for L in lens], 16, {
        "workload": f"config3: 16 layers, learned ranks (r_k in {{384..640}}, r_v = 1024 - r_k), batch {B}/GPU, "
                    "context log-uniform [1k, 64k], page 16"}


def serving_pool(n: int) -> list:
    """Prompt lengths of config 5's ``n`` sequences (the config-3 distribution, seeded apart from config 3's pool)."""
    return synth.log_uniform_lengths(n, 1024, 65536, seed=synth.SEED_LENGTHS + 50)


def load_peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


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
        # head stride 644: every partial row starts on 16 bytes (float4 loads in the fused merge)
        self.part = torch.empty(self.B + self.sched.num_ctas, H, 644, dtype=torch.float32, device=device)
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
            dec.merge_up_project(part, self.sched, lat.v_up, self.out[l], self.lse)

    launches_per_step = property(lambda self: 1 + 4 * self.L)

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


# ------------------------------------------------------------------------------------------------------------ CPU leg
# The CPU restatement of the reference's path (``oracle``) runs only here: as the checker of the outputs of the step the
# GPU just timed (``parity``) and as the CPU baseline / reference arm (timed on a bounded sample). Nothing in a timed
# GPU region touches it.
PARITY_MAX_ABS, PARITY_MEAN_ABS = 2e-2, 2e-3       # the north-star tolerance for BF16 attention outputs


def parity_picks(lens, r_k, n_reqs: int = 4):
    """(layers, requests) checked after the timed region: the layers whose K rank is nearest to 384, 512 and 640 (one
    per distinct rank), and ``n_reqs`` requests at even steps through the length order (shortest to longest)."""
    layers = []
    for target in (384, 512, 640):
        best = min(range(len(r_k)), key=lambda l: (abs(r_k[l] - target), l))
        if best not in layers:
            layers.append(best)
    order = sorted(range(len(lens)), key=lambda b: (lens[b], b))
    n = min(n_reqs, len(order))
    reqs = sorted({order[round(i * (len(order) - 1) / max(1, n - 1))] for i in range(n)})
    return layers, reqs


def gather_parity(buf, block_table, lens, page, q, out, layers, reqs):
    """Host copies, made after the timed region, of what the check needs: per (layer, request) the GPU output, the
    query and the request's cache pages of that layer (``buf`` [blocks, layers, page, W])."""
    bt = block_table.cpu()
    items = []
    for l in layers:
        for b in reqs:
            n = int(lens[b])
            blocks = bt[b, :-(-n // page)].long()
            items.append({"layer": l, "req": b, "seq_len": n, "out": out[l][b].float().cpu(), "q": q[l][b].cpu(),
                          "pages": buf[blocks.to(buf.device), l].cpu()})
    return items


def check_parity(weights, items) -> dict:
    """The gathered GPU outputs against the fp32 oracle (``oracle.decode_fp32``) on the same cache rows."""
    import oracle
    cos_sin = synth.cos_sin_table(max(it["seq_len"] for it in items) + 1)
    refs = {}
    worst, total, count = 0.0, 0.0, 0
    t0 = time.perf_counter()
    for it in items:
        l = it["layer"]
        if l not in refs:
            w = weights[l]
            refs[l] = oracle.derive(w.k_up, w.v_up, w.k_norm_weight, w.layout, cos_sin)
        pages = it["pages"]
        bt = torch.arange(pages.shape[0], dtype=torch.int32)[None]
        exp = oracle.decode_fp32(it["q"][None], pages, bt, torch.tensor([it["seq_len"]]), refs[l], SCALE)[0]
        d = (it["out"] - exp).abs()
        worst = max(worst, float(d.max()))
        total += float(d.sum())
        count += d.numel()
    mean = total / max(1, count)
    return {"max_abs": worst, "mean_abs": mean, "ok": bool(worst < PARITY_MAX_ABS and mean < PARITY_MEAN_ABS),
            "tolerance": {"max_abs": PARITY_MAX_ABS, "mean_abs": PARITY_MEAN_ABS}, "oracle": "decode_fp32",
            "layers": sorted({it["layer"] for it in items}), "requests": sorted({it["req"] for it in items}),
            "context_tokens": sorted({it["seq_len"] for it in items}), "cpu_seconds": time.perf_counter() - t0}


class CpuArm:
    """The reference's torch path restated on the CPU (``oracle.decode_reference``: ``LatentLayer.decompress`` of every
    context row, then fp32 attention) on all host cores. A bounded sample of layer 0's requests is timed and the time
    per context token extrapolated to the workload (every layer of every request), unless ``full``: then every
    request of every layer is timed and nothing is extrapolated."""

    def __init__(self, specs, seq_lens, page, budget_s: float, full: bool = False):
        import oracle
        self.cores = os.cpu_count() or 1
        torch.set_num_threads(self.cores)
        self.specs, self.seq_lens, self.page, self.full = specs, list(seq_lens), page, full
        self.layers = list(range(len(specs))) if full else [0]
        self.total_ctx = sum(self.seq_lens)
        if full:
            self.sample = list(self.seq_lens)
        else:
            # calibrate on the median request, then take requests from the 25th percentile up to the budget
            order = sorted(range(len(self.seq_lens)), key=lambda i: self.seq_lens[i])
            probe = [self.seq_lens[order[len(order) // 2]]]
            per_tok = self._time_layer(0, probe) / sum(probe)
            want = max(1, int(budget_s / per_tok))
            self.sample, acc = [], 0
            for i in order[len(order) // 4:] + order[:len(order) // 4]:
                if acc + self.seq_lens[i] > want and self.sample:
                    break
                self.sample.append(self.seq_lens[i])
                acc += self.seq_lens[i]
        self._prepared = {l: self._prepare(l, self.sample) for l in self.layers}
        self._oracle = oracle

    def _prepare(self, l, lens):
        import oracle
        w = synth.make_layer(self.specs[l], seed=synth.SEED_FACTORS + l)
        ref = oracle.derive(w.k_up, w.v_up, w.k_norm_weight, w.layout, synth.cos_sin_table(max(lens) + 1))
        batch = synth.make_batch(w.layout, lens, page=self.page, seed=synth.SEED_CACHE + 101 * l, poison=False)
        return ref, batch, synth.make_queries(len(lens))

    def _time_layer(self, l, lens, prepared=None):
        import oracle
        ref, batch, q = prepared or self._prepare(l, lens)
        t0 = time.perf_counter()
        oracle.decode_reference(q, batch.cache, batch.block_table, batch.seq_lens, ref, SCALE)
        return time.perf_counter() - t0

    def run_once(self) -> float:
        """Seconds for one pass over the sample (every sampled layer)."""
        return sum(self._time_layer(l, self.sample, self._prepared[l]) for l in self.layers)

    def rate(self, seconds: float) -> float:
        """Decode tokens/s of the whole workload implied by one pass that took ``seconds``."""
        if self.full:
            return len(self.seq_lens) / seconds
        per_tok = seconds / sum(self.sample)
        return len(self.seq_lens) / (per_tok * self.total_ctx * len(self.specs))

    def describe(self, seconds: float) -> str:
        if self.full:
            return (f"oracle port of the reference torch path (decompress + fp32 attention): the whole workload timed, "
                    f"{len(self.layers)} layers x {len(self.sample)} requests / {sum(self.sample)} context tokens "
                    f"({seconds:.1f} s), not extrapolated")
        return (f"oracle port of the reference torch path (decompress + fp32 attention), layer 0, {len(self.sample)} "
                f"requests / {sum(self.sample)} context tokens timed ({seconds:.1f} s), extrapolated per context token "
                f"to {len(self.specs)} layers x {self.total_ctx} tokens")


def run_reference_arm(args, rank, world):
    """The reference's CPU path on the box's requests (every rank's share), rank 0 only."""
    if rank != 0:
        return
    specs, seq_lens, page, cfg = workload_spec(args.config, args.batch, 0, 1, args.rows)
    seq_lens = list(seq_lens) * (world if args.config == 3 else 1)      # every rank holds the same lengths
    n = args.warmup + args.steps
    budget = min(args.cpu_seconds, 150.0 / max(1, n))
    arm = CpuArm(specs, seq_lens, page, budget, full=args.cpu_full)
    rates, secs = [], []
    for i in range(n):
        t = arm.run_once()
        if i >= args.warmup:
            rates.append(arm.rate(t))
            secs.append(t)
    value = statistics.median(rates)
    ms = 1000.0 * len(seq_lens) / value
    timed_tokens = sum(arm.sample) * len(arm.layers)
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak" if args.config == 3 else "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "impl": "reference", "extrapolated": not arm.full,
            "samples": {"timed_passes": len(secs), "seconds_per_pass": statistics.median(secs),
                        "timed_context_tokens_per_pass": timed_tokens, "timed_layers": len(arm.layers),
                        "timed_requests": len(arm.sample), "workload_layers": len(specs),
                        "workload_context_tokens": sum(seq_lens)},
            "config": {**cfg, "global_batch": len(seq_lens), "parallelism": "dp (rank 0 only: CPU)"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": arm.cores, "kind": "port",
                             "sample": arm.describe(statistics.median(secs))},
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


GEMM_SHAPES = [
    # (name, M, N, K): the model's linear layers at hidden 1024, and one large product for the peak comparison
    ("kv_latent_proj, 8192-token prefill chunk", 8192, 1024, 1024),
    ("q_gate_proj, 8192-token prefill chunk", 8192, 12288, 1024),
    ("o_proj, 8192-token prefill chunk", 8192, 1024, 6144),
    ("q_gate_proj, 128-token decode step", 128, 12288, 1024),
    ("square 8192", 8192, 8192, 8192),
]


def run_gemm(args):
    """TFLOP/s of ``latent_ops.linear`` (the tcgen05 GEMM) on the model's shapes, CUDA events around each launch with
    L2 flushed before it, torch's matmul (cuBLAS) on the same operands beside; one JSON line (the first shape's figures
    at the top level, every shape under ``shapes``)."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    from belt_b200 import build as _build
    _build.build()
    peaks = load_peaks()
    peak_tf = peaks.get("bf16_tflops") or 1590.0
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    rows = []
    clocks = ClockSampler(dev)
    clocks.start()
    for name, M, N, K in GEMM_SHAPES:
        g = torch.Generator(device=dev).manual_seed(M + N + K)
        x = torch.randn(M, K, generator=g, device=dev, dtype=torch.bfloat16)
        w = torch.randn(N, K, generator=g, device=dev, dtype=torch.bfloat16) / K ** 0.5

        def timed(fn):
            for _ in range(max(args.warmup, 3)):
                fn()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(args.steps)]
            for s_, e_ in ev:
                flush.add_(1)
                s_.record()
                fn()
                e_.record()
            torch.cuda.synchronize()
            return statistics.median(s_.elapsed_time(e_) for s_, e_ in ev)

        ms = timed(lambda: latent_ops.linear(x, w))
        lib_ms = timed(lambda: x @ w.T)
        err = float((latent_ops.linear(x, w).float() - (x @ w.T).float()).abs().max())
        tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
        rows.append({"shape": name, "M": M, "N": N, "K": K, "ms": ms, "tflops": tf, "frac": tf / peak_tf,
                     "library_ms": lib_ms, "library_tflops": 2.0 * M * N * K / (lib_ms / 1e3) / 1e12,
                     "max_abs_diff_vs_library": err})
    clk = clocks.stop()
    dec.check_device_errors(dev)
    top = rows[0]
    line = {"metric": "tensor-core GEMM TFLOP/s (model linear layers)", "value": top["tflops"], "unit": "TFLOP/s",
            "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": top["ms"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": top["shape"], "l2": "flushed (256 MB write) before every timed launch"},
            "roofline": {"bound": "tensor", "achieved": top["tflops"], "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": top["frac"], "peak_source": "measured" if "bf16_tflops" in peaks else "fallback"},
            "shapes": rows, "clocks": clk, "gpu_launches": len(rows) * (args.steps + max(args.warmup, 3) + 1)}
    print(json.dumps(line), flush=True)


def run_prefill(args):
    """The prefill path of one c50 layer through the backend's varlen kernels, two workloads:

    * ``single``: one request of 8192 new tokens over an 8192-token context (keys / values rebuilt from the paged rows,
      causal attention): the line's headline;
    * ``batched``: one step of four prefill requests of 2048, 4096, 8192 and 16384 new tokens each (whole prompts),
      through ``LatentAttentionImpl._prefill``: one decompress launch and one attention launch for all four.

    Timed on the device (inputs resident, L2 flushed before each step, NVML clocks sampled); torch's
    scaled_dot_product_attention on the single request's keys and values beside it."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    from belt_b200 import build as _build
    from belt_b200.latent_backend import LatentAttentionImpl, LatentAttentionMetadata
    from belt_b200.layer import derive_latent_tensors
    _build.build()
    page = 16
    w = synth.make_layer(synth.c50(), seed=synth.SEED_FACTORS)
    lens_b = [2048, 4096, 8192, 16384]
    max_len = max(lens_b)
    lat = derive_latent_tensors(w.k_up, w.v_up, w.k_norm_weight, w.layout, synth.cos_sin_table(max_len + 1),
                                device=dev)
    impl = LatentAttentionImpl(H, D, SCALE, 4)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def workload(lens, qls):
        bt, nb, _ = synth.block_tables(lens, page, extra_blocks=1, seed=synth.SEED_CACHE)
        cache = torch.empty(nb, page, w.layout["row_width"], dtype=torch.bfloat16, device=dev)
        synth.fill_cache(cache, w.layout, bt.to(dev), lens, seed=synth.SEED_CACHE, poison=False)
        m = LatentAttentionMetadata(num_actual_tokens=sum(qls), num_decodes=0, num_decode_tokens=0,
                                    num_prefills=len(lens), num_prefill_tokens=sum(qls), block_table=bt.to(dev),
                                    seq_lens=torch.tensor(lens, dtype=torch.int32, device=dev), sched=None)
        m.prefill_q_len, m.prefill_seq_len = list(qls), list(lens)
        q = torch.randn(sum(qls), H, D, device=dev, dtype=torch.bfloat16)
        out = torch.empty(sum(qls), H, D, dtype=torch.bfloat16, device=dev)
        return lambda: impl._prefill(lat, q, out, cache, m)

    def timed(step):
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for s_, e_ in ev:
            flush.add_(1)
            s_.record()
            step()
            e_.record()
        torch.cuda.synchronize()
        return statistics.mean(s_.elapsed_time(e_) for s_, e_ in ev)

    def flops(lens, qls):   # causal attention + the decompress of every context row
        att = sum(24 * (ql * (L - ql) + ql * (ql + 1) / 2) * 256 * 4 for L, ql in zip(lens, qls))
        return att + sum(lens) * 2 * 256 * 4 * (320 + 512)

    clocks = ClockSampler(dev)
    clocks.start()
    L = 8192
    ms = timed(workload([L], [L]))
    ms_b = timed(workload(lens_b, lens_b))
    clk = clocks.stop()
    dec.check_device_errors(dev)
    # torch's attention on the same shapes (one request), for comparison
    q = torch.randn(L, H, D, device=dev, dtype=torch.bfloat16)
    k = torch.randn(L, 4, D, device=dev, dtype=torch.bfloat16)
    qh = q.transpose(0, 1).unsqueeze(0)
    kh = k.transpose(0, 1).repeat_interleave(6, 0).unsqueeze(0)
    lib_ms = None
    try:
        lib_ms = timed(lambda: torch.nn.functional.scaled_dot_product_attention(qh, kh, kh, is_causal=True,
                                                                                 scale=SCALE))
    except RuntimeError:
        pass
    peaks = load_peaks()
    peak_tf = peaks.get("bf16_tflops") or 1590.0
    tf = flops([L], [L]) / (ms / 1e3) / 1e12
    tf_b = flops(lens_b, lens_b) / (ms_b / 1e3) / 1e12
    line = {"metric": "prefill tokens/s (decompress + causal attention, one c50 layer)", "value": L / (ms / 1e3),
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "prefill: 8192 new tokens over an 8192-token context, c50 layer, page 16",
                       "l2": "flushed (256 MB write) before every step"},
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak_tf, "unit": "TFLOP/s", "frac": tf / peak_tf,
                         "peak_source": "measured" if "bf16_tflops" in peaks else "fallback"},
            "batched": {"workload": "one step of 4 prefills of 2048, 4096, 8192, 16384 new tokens (whole prompts)",
                        "ms_per_step": ms_b, "tokens_per_s": sum(lens_b) / (ms_b / 1e3), "tflops": tf_b,
                        "frac": tf_b / peak_tf, "launches_per_step": 2},
            "library_sdpa_attention_ms": lib_ms, "clocks": clk, "gpu_launches": 4 * (args.steps + max(args.warmup, 3))}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------------ config 5
def plan_waves(lens, steps: int, page: int, block_bytes: int, free_bytes: int):
    """(waves, blocks per wave buffer, buffers): requests longest first, each wave as many as fit one buffer. One
    buffer when everything fits at once, else two (one wave decoding while the next is prefilled)."""
    need = [-(-(n + steps) // page) for n in lens]
    if sum(need) * block_bytes <= free_bytes:
        nbuf, cap = 1, sum(need)
    else:
        nbuf, cap = 2, free_bytes // 2 // block_bytes
    waves, cur, used = [], [], 0
    for i in sorted(range(len(lens)), key=lambda i: (-lens[i], i)):
        if need[i] > cap:
            raise RuntimeError(f"a sequence of {lens[i]} tokens does not fit a wave buffer of {cap} blocks")
        if used + need[i] > cap:
            waves.append(cur)
            cur, used = [], 0
        cur.append(i)
        used += need[i]
    if cur:
        waves.append(cur)
    return waves, cap, nbuf


def wave_tables(base, npages, cap: int, steps: int, page: int, seed: int) -> dict:
    """Host tables of one wave: a block table dealing ``npages[j]`` blocks of a seeded permutation of the buffer's
    ``cap`` to request j; per decode step s the context lengths (base + s + 1) and the slot of that step's token
    (position base + s); and the slots of every prompt position in request order (the prefill's token stream)."""
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(cap, generator=g)
    base = torch.tensor(list(base), dtype=torch.int64)
    bt = torch.zeros(len(base), max(npages), dtype=torch.int64)
    off = 0
    for j, n in enumerate(npages):
        bt[j, :n] = perm[off:off + n]
        off += n
    pos = base[None, :] + torch.arange(steps)[:, None]                        # [steps, B]: this step's token
    rows = torch.arange(len(base))[None, :].expand(steps, -1)
    toks = torch.cat([torch.arange(int(n)) for n in base])
    owner = torch.repeat_interleave(torch.arange(len(base)), base)
    return {"block_table": bt, "seq_lens": (pos + 1).to(torch.int32), "slots": bt[rows, pos // page] * page + pos % page,
            "prefill_slots": bt[owner, toks // page] * page + toks % page, "prefill_tokens": int(base.sum())}


class ServingRun:
    """Config 5 on one rank: its share of the box's sequences, served in waves that fit its HBM.

    Every wave's cache lives in one of (at most) two wave buffers [blocks, layers, page, W]. A wave is first prefilled:
    its prompts' latent rows are written by chunked cache writes of ``chunk`` tokens per layer (the down-projection of
    the tokens' layer inputs + the paged scatter, ``latent_ops.project_rows_to_cache``), the chunks cut from the
    wave's tokens in request order (a chunk can span requests, as a serving engine packs them). Then it is decoded for
    ``steps`` steps: each step the schedule, and per layer the cache write of this step's token, the absorbed query,
    the decode kernel, the merge and the U_v projection, with every request one token longer than the step before.
    While wave k decodes, wave k + 1's prefill chunks run between its decode steps, into the other buffer."""

    def __init__(self, specs, lens, page, device, rank, steps, chunk, reserve_bytes=10 << 30):
        from belt_b200.layer import derive_latent_tensors
        self.device, self.page, self.steps, self.chunk = device, page, steps, chunk
        self.L = len(specs)
        self.lens = list(lens)
        cos_sin = synth.cos_sin_table(max(lens) + steps + 1)
        self.weights = [synth.make_layer(sp, seed=synth.SEED_FACTORS + i) for i, sp in enumerate(specs)]
        self.layers = [derive_latent_tensors(w.k_up, w.v_up, w.k_norm_weight, w.layout, cos_sin, device=device)
                       for w in self.weights]
        self.W = self.weights[0].layout["row_width"]
        self.hidden = specs[0].hidden
        self.w_down = [w.kv_latent_proj.to(device) for w in self.weights]
        block_bytes = self.L * page * self.W * 2
        free = torch.cuda.mem_get_info(device)[0] - reserve_bytes
        self.waves, cap, nbuf = plan_waves(lens, steps, page, block_bytes, free)
        need = [-(-(n + steps) // page) for n in lens]
        self.cap, self.nbuf = cap, nbuf
        Bmax = max(len(w) for w in self.waves)
        gq = torch.Generator(device=device).manual_seed(synth.SEED_QUERY + 7 * rank)
        # inputs of one decode step and of the prefill chunks: the work is what is timed, so a few buffers are reused
        self.q = torch.randn(self.L, Bmax, H, D, generator=gq, device=device, dtype=torch.bfloat16)
        self.x = torch.randn(self.L, Bmax, self.hidden, generator=gq, device=device, dtype=torch.bfloat16)
        self.xp = torch.randn(4, chunk, self.hidden, generator=gq, device=device, dtype=torch.bfloat16)
        self.sched = dec.make_schedule(Bmax, device)
        self.part = torch.empty(Bmax + self.sched.num_ctas, H, 644, dtype=torch.float32, device=device)
        self.lse = torch.empty(Bmax, H, dtype=torch.float32, device=device)
        self.out = torch.empty(self.L, Bmax, H, D, dtype=torch.bfloat16, device=device)
        self.side = torch.cuda.Stream(device)
        self.meta = [self._wave_meta(k, w, need, rank) for k, w in enumerate(self.waves)]
        self.bufs = [torch.zeros(cap, self.L, page, self.W, dtype=torch.bfloat16, device=device)
                     for _ in range(nbuf)]

    def _wave_meta(self, k, reqs, need, rank):
        """Block table, per-step seq_lens and slots, and the prefill slots of wave k, on the device."""
        m = wave_tables([self.lens[i] for i in reqs], [need[i] for i in reqs], self.cap, self.steps, self.page,
                        seed=synth.SEED_CACHE + 1000 * rank + k)
        dev = self.device
        return {"B": len(reqs), "block_table": m["block_table"].to(torch.int32).to(dev),
                "seq_lens": m["seq_lens"].to(dev).contiguous(), "slots": m["slots"].to(dev).contiguous(),
                "prefill_slots": m["prefill_slots"].to(dev), "prefill_tokens": m["prefill_tokens"],
                "chunks": -(-m["prefill_tokens"] // self.chunk)}

    def buffer(self, k):
        return self.bufs[k % self.nbuf]

    def decode_step(self, k, s):
        m = self.meta[k]
        B = m["B"]
        buf = self.buffer(k)
        seq_lens, slots = m["seq_lens"][s], m["slots"][s]
        dec.schedule(self.sched, seq_lens)
        main = torch.cuda.current_stream(self.device)
        for l, lat in enumerate(self.layers):
            cache = buf[:, l]
            self.side.wait_stream(main)
            with torch.cuda.stream(self.side):
                latent_ops.project_rows_to_cache(self.x[l, :B], self.w_down[l], slots, cache, lat.u_cat,
                                                 lat.k_segs_host, lat.eps)
            q_bd = lat.block_diag_query(self.q[l, :B])
            main.wait_stream(self.side)
            part = self.part[:B + self.sched.num_ctas, :, :lat.v_rank + 1]
            dec.latent_decode(q_bd, cache, m["block_table"], seq_lens, self.sched, part, SCALE, lat.v_offset,
                              lat.v_rank, rope=lat.rope)
            dec.merge_up_project(part, self.sched, lat.v_up, self.out[l, :B], self.lse[:B])

    def prefill_chunk(self, k, c):
        m = self.meta[k]
        t0 = c * self.chunk
        n = min(self.chunk, m["prefill_tokens"] - t0)
        slots = m["prefill_slots"][t0:t0 + n]
        x = self.xp[c % self.xp.shape[0], :n]
        buf = self.buffer(k)
        for l, lat in enumerate(self.layers):
            latent_ops.project_rows_to_cache(x, self.w_down[l], slots, buf[:, l], lat.u_cat, lat.k_segs_host, lat.eps)

    def run(self, events=None):
        """The whole serving run: wave 0's prefill, then every wave's decode steps with the next wave's prefill
        chunks in between. ``events`` (start, end) pairs bracket the decode and the prefill work for the split."""
        for c in range(self.meta[0]["chunks"]):
            self.prefill_chunk(0, c)
        for k in range(len(self.waves)):
            nxt = k + 1 if k + 1 < len(self.waves) else None
            n_next = self.meta[nxt]["chunks"] if nxt is not None else 0
            per_step = -(-n_next // self.steps)
            c = 0
            for s in range(self.steps):
                self.decode_step(k, s)
                for _ in range(per_step):
                    if c < n_next:
                        self.prefill_chunk(nxt, c)
                        c += 1

    def launches(self) -> int:
        """This repository's kernel launches in ``run``: per decode step the schedule and four per layer, per prefill
        chunk and layer the projection GEMM (``belt_gemm_bf16``) and the cache write."""
        dec_steps = len(self.waves) * self.steps
        return dec_steps * (1 + 4 * self.L) + 2 * sum(m["chunks"] for m in self.meta) * self.L


def run_serving(args, group, dev):
    rank, world = group.rank, group.world
    specs, pool, page, cfg = workload_spec(5, args.num_seqs, rank, world)
    parts = dp.partition_lpt(pool, world)
    mine = [pool[i] for i in parts[rank]]
    run = ServingRun(specs, mine, page, dev, rank, args.decode_steps, args.prefill_chunk)
    # warm-up: a few decode steps of wave 0 and one prefill chunk (the timed run starts over from an empty cache)
    for s in range(max(args.warmup, 3)):
        run.decode_step(0, s)
    run.prefill_chunk(0, 0)
    torch.cuda.synchronize()
    dec.check_device_errors(dev)
    clocks = ClockSampler(dev)
    group.barrier()
    clocks.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    group.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    run.run()
    end.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    group.barrier()
    dec.check_device_errors(dev)
    ms_local = start.elapsed_time(end)
    ms = group.max(ms_local)
    decode_tokens = len(pool) * args.decode_steps
    value = decode_tokens / (ms / 1000.0)
    per_rank_ms = group.gather_float(ms_local)
    ctx = sum(mine)
    # algorithmic HBM bytes of this rank's run: every decode step reads each request's context rows once per layer;
    # every prefill chunk writes its rows (the down-projection's operands are counted in neither)
    steps = args.decode_steps
    dec_bytes = sum(sum(run.lens[i] + s + 1 for i in w for s in range(steps)) for w in run.waves) * run.L * run.W * 2
    pf_bytes = ctx * run.L * run.W * 2
    parity = None
    if rank == 0 and not args.no_parity:
        k = len(run.waves) - 1
        m = run.meta[k]
        lens_last = [run.lens[i] + steps for i in run.waves[k]]      # the last step's contexts
        layers, reqs = parity_picks(lens_last, [w.layout["lk"] for w in run.weights], n_reqs=2)
        items = gather_parity(run.buffer(k), m["block_table"], lens_last, page, run.q, run.out, layers[:2], reqs)
        parity = check_parity(run.weights, items)
    peaks = load_peaks()
    peak_gbs = peaks.get("hbm_gbs") or 6650.0
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms / (len(run.waves) * steps), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {**cfg, "parallelism": f"dp{world}", "global_batch": len(pool),
                       "partition": "LPT by context tokens, equal request counts",
                       "partition_imbalance": dp.imbalance(pool, parts), "decode_steps_per_wave": steps,
                       "prefill_chunk_tokens": args.prefill_chunk, "waves_rank0": len(run.waves),
                       "wave_buffers_rank0": run.nbuf, "wave_buffer_gb_rank0": run.cap * run.L * page * run.W * 2 / 1e9,
                       "context_tokens_rank0": ctx, "tokens_per_s_per_gpu": value / world,
                       "ms_per_rank": per_rank_ms, "timed_ms": ms,
                       "hbm_gb_per_s_rank0": (dec_bytes + pf_bytes) / (ms_local / 1000.0) / 1e9,
                       "hbm_frac_rank0": (dec_bytes + pf_bytes) / (ms_local / 1000.0) / 1e9 / peak_gbs,
                       "l2": "inputs larger than L2 (wave buffers of tens of GB)"},
            "roofline": None, "clocks": clk, "gpu_launches": run.launches()}
    if parity is not None:
        line["parity"] = parity
    if rank == 0:
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
    if args.gemm:
        if rank == 0:
            run_gemm(args)
        return
    group = dp.HostGroup()
    local = group.local_rank
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from belt_b200 import build as _build
    _build.build()
    if args.config == 5:
        run_serving(args, group, dev)
        group.close()
        return
    specs, seq_lens, page, cfg = workload_spec(args.config, args.batch, rank, world, args.rows)
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
        wl.step()
    end.record()
    torch.cuda.synchronize()
    # the decode kernel's own duration: the same steps again with CUDA events around every decode launch (an event
    # between two launches also stops the next one from starting early, so these launches run without overlap)
    for k in range(args.steps):
        wl.step(dec_events[k])
    torch.cuda.synchronize()
    clk = clocks.stop()
    group.barrier()
    ms_local = start.elapsed_time(end) / args.steps
    ms = group.max(ms_local)
    dec.check_device_errors(dev)
    total_reqs = group.sum(wl.B)
    value = total_reqs / (ms / 1000.0)
    # the outputs of the last timed step, for the oracle check (before anything else writes the cache)
    parity_items = None
    if rank == 0 and not args.no_parity:
        layers, reqs = parity_picks(wl.seq_lens_list, [w.layout["lk"] for w in wl.weights])
        parity_items = gather_parity(wl.buf, wl.block_table, wl.seq_lens_list, wl.page, wl.q, wl.out, layers, reqs)

    # the decode kernel's launches, per layer
    peaks = load_peaks()
    peak_gbs = peaks.get("hbm_gbs") or 6650.0
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    kern_ms = [statistics.mean(dec_events[k][l][0].elapsed_time(dec_events[k][l][1]) for k in range(args.steps))
               for l in range(wl.L)]
    kern_bytes = [wl.decode_kernel_bytes(l) for l in range(wl.L)]
    achieved = sum(kern_bytes) / (sum(kern_ms) / 1000.0) / 1e9
    rank_gbs = [group.gather_float(achieved)] if world > 1 else None
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
                       "partition": "every rank decodes the same request lengths (its own cache contents)",
                       "l2": "inputs larger than L2 (cache %.1f GB per GPU)" % (wl.buf.numel() * 2 / 1e9),
                       "tokens_per_s_per_gpu": value / world,
                       "step_roofline_frac": step_frac, "step_algorithmic_gb": step_gb},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak_gbs, "unit": "GB/s",
                         "frac": achieved / peak_gbs, "peak_source": peak_src,
                         "kernel": "latent_decode_kernel", "kernel_ms_per_launch": sum(kern_ms) / wl.L,
                         "kernel_timing": "CUDA events around each decode launch, a second pass of the timed steps",
                         "traffic": traffic_per_launch, "traffic_source": traffic and traffic.get("source")},
            "clocks": clk,
            "gpu_launches": wl.launches_per_step * args.steps}
    # the decode kernel's fraction per K rank (layers of one rank share a row layout and a stage plan)
    by_rank = {}
    for l in range(wl.L):
        r = by_rank.setdefault(str(wl.weights[l].layout["lk"]), [0.0, 0.0, 0])
        r[0] += kern_bytes[l]
        r[1] += kern_ms[l]
        r[2] += 1
    line["roofline"]["frac_by_k_rank"] = {
        k: {"layers": n, "us_per_launch": 1000.0 * t / n, "frac": b / (t / 1000.0) / 1e9 / peak_gbs}
        for k, (b, t, n) in sorted(by_rank.items(), key=lambda kv: int(kv[0]))}
    if rank_gbs is not None:
        line["roofline"]["achieved_per_rank"] = rank_gbs[0]
    if not args.no_e2e:
        _, e_ms_local, h2d, d2h = e2e_rate(wl, max(2, args.steps // 2), 2)
        e_ms = group.max(e_ms_local)
        line["e2e"] = {"value": total_reqs / (e_ms / 1000.0), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                       "d2h_bytes_per_step": d2h, "ms_per_step": e_ms}
    if parity_items is not None:
        line["parity"] = check_parity(wl.weights, parity_items)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        arm = CpuArm(specs, seq_lens, page, args.cpu_seconds)
        t = arm.run_once()
        line["cpu_baseline"] = {"value": arm.rate(t), "unit": "tokens/s", "cores": arm.cores, "kind": "port",
                                "sample": arm.describe(t)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    group.close()

if __name__ == "__main__":
    main()
