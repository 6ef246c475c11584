"""``belt_latent_decode_noalloc``: the decode step whose scratch is a fixed array inside the library.

Some callers cannot allocate device memory: a host binding the C ABI that holds only the engine's KV pool, query and
output buffers, or an engine that reserved nearly all of HBM for its KV pool. This entry point serves them by keeping
the split-KV scratch in a fixed array inside the library.

The GPU tests call it through the C ABI twice in a row, on different layers and batches, and check each result
against the regular entry points (schedule -> decode -> merge with caller-provided scratch) within the decode's
tolerance: latent output max-abs 2e-2 / mean-abs 2e-3, LSE within 2e-3. The second call runs on a smaller problem
than the first, so partials or segment records left over from the first call would show up in its result. A third
case fills the array up to its limit (258 requests at r_v 640 on 148 CTAs: the last partial rows sit at its top) and
checks the result against the fp32 oracle as well. The CPU tests check that sizes beyond the fixed array are refused
before anything touches the GPU, and the rules of the per-context address record.

This file is collected last, so the GPU test also runs after every other GPU test in the same process.
"""

import os
import shutil
import subprocess

import pytest
import torch

from belt_b200 import _lib, build
from belt_b200 import decode as dec
from belt_b200 import synth
from belt_b200.layer import derive_latent_tensors

SCALE = 256 ** -0.5
MAX_ABS, MEAN_ABS, LSE_ATOL = 2e-2, 2e-3, 2e-3
PART_BYTES = (24 << 20) - (128 << 10)


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_lib.lib_path()):
        try:
            build.build()
        except RuntimeError as e:
            pytest.skip(f"cannot build the CUDA library here: {e}")
    return _lib.load()


def _noalloc_args(q_bd, cache, block_table, seq_lens, num_ctas, lat, out, lse, min_tiles=1, stream=0, err=0,
                  num_reqs=None, lv=None):
    """Argument list of belt_latent_decode_noalloc (tensors as device pointers, ints elsewhere)."""
    groups = [x for gr in lat.rope.groups for x in gr]
    blocks, cos_sin = lat.rope.blocks, lat.rope.cos_sin
    ptr = lambda t: t.data_ptr() if hasattr(t, "data_ptr") else t
    nr = q_bd.shape[0] if num_reqs is None else num_reqs
    return [ptr(q_bd), nr, q_bd.shape[2], ptr(cache), cache.shape[0], cache.shape[1], cache.shape[2], cache.stride(0),
            cache.stride(1), ptr(block_table), block_table.stride(0), ptr(seq_lens), num_ctas, min_tiles,
            float(SCALE), int(lat.v_offset), int(lat.v_rank if lv is None else lv), _lib.int_array(groups),
            ptr(blocks), blocks.shape[2] // dec.CHUNK, ptr(cos_sin), cos_sin.shape[0], ptr(out), out.stride(0),
            out.stride(1), ptr(lse), lse.stride(0), err, stream]


class _Shape:
    """A stand-in with the shape/stride/data_ptr a size check reads (no memory behind it)."""

    def __init__(self, shape, strides):
        self.shape, self._strides = shape, strides

    def stride(self, i):
        return self._strides[i]

    def data_ptr(self):
        return 4096


def _fake_layer(lv):
    from types import SimpleNamespace
    rope = SimpleNamespace(groups=((0, 64), (128, 64), (256, 64), (384, 64)),
                           blocks=_Shape((1, 64, 256), (16384, 256, 1)), cos_sin=_Shape((4096, 64), (64, 1)))
    return SimpleNamespace(v_offset=512, v_rank=lv, rope=rope)


@pytest.mark.parametrize("num_reqs,num_ctas,lv,msg", [
    (300, 148, 640, "exceed the fixed scratch"),
    (259, 148, 640, "exceed the fixed scratch"),
    (5000, 148, 64, "num_reqs"),
    (4, 2000, 64, "num_ctas"),
])
def test_noalloc_rejects_sizes_beyond_the_fixed_array(lib, num_reqs, num_ctas, lv, msg):
    """Refused with BELT_ERR_INVALID and a message naming the limit; no CUDA call is made (this runs without a GPU)."""
    lat = _fake_layer(lv)
    q_bd = _Shape((num_reqs, 24, 768), (24 * 768, 768, 1))
    cache = _Shape((64, 16, 1152), (16 * 1152, 1152, 1))
    bt = _Shape((num_reqs, 8), (8, 1))
    out = _Shape((num_reqs, 24, lv), (24 * lv, lv, 1))
    lse = _Shape((num_reqs, 24), (24, 1))
    with pytest.raises(ValueError, match=msg):
        _lib.call("belt_latent_decode_noalloc", *_noalloc_args(q_bd, cache, bt, 4096, num_ctas, lat, out, lse,
                                                               num_reqs=num_reqs))
    assert (num_reqs + num_ctas) * 24 * (lv + 1) * 4 > PART_BYTES or num_reqs > 4096 or num_ctas > 1024


def _case(r_k, r_v, seqs, seed):
    spec = synth.spec_from_ranks(r_k, r_v)
    w = synth.make_layer(spec)
    lat = derive_latent_tensors(w.k_up, w.v_up, w.k_norm_weight, w.layout, synth.cos_sin_table(max(seqs) + 8),
                                device="cuda")
    batch = synth.make_batch(w.layout, seqs, page=16, seed=seed)
    q = synth.make_queries(len(seqs), seed=seed + 1).cuda()
    return lat, batch.cache.cuda(), batch.block_table.cuda(), batch.seq_lens.cuda(), lat.block_diag_query(q)


def _regular(lat, q_bd, cache, bt, seq_lens, num_ctas):
    """The same step through the entry points that take their scratch from the caller."""
    B = q_bd.shape[0]
    sched = dec.make_schedule(B, q_bd.device, num_ctas=num_ctas)   # the backend's weighted split, as the entry uses
    dec.schedule(sched, seq_lens)
    part = torch.full((B + num_ctas, 24, lat.v_rank + 1), float("nan"), device=q_bd.device)
    dec.latent_decode(q_bd, cache, bt, seq_lens, sched, part, SCALE, lat.v_offset, lat.v_rank, rope=lat.rope)
    a = torch.empty(B, 24, lat.v_rank, dtype=torch.bfloat16, device=q_bd.device)
    lse = torch.empty(B, 24, device=q_bd.device)
    dec.merge_segments(part, sched, a, lse)
    return a, lse


def _noalloc(lat, q_bd, cache, bt, seq_lens, num_ctas):
    B = q_bd.shape[0]
    a = torch.full((B, 24, lat.v_rank), float("nan"), dtype=torch.bfloat16, device=q_bd.device)
    lse = torch.full((B, 24), float("nan"), device=q_bd.device)
    err = dec.error_word(q_bd.device)
    _lib.call("belt_latent_decode_noalloc",
              *_noalloc_args(q_bd, cache, bt, seq_lens, num_ctas, lat, a, lse, err=err.data_ptr(),
                             stream=torch.cuda.current_stream().cuda_stream))
    return a, lse


@pytest.mark.gpu
def test_noalloc_matches_regular_entry_points_twice():
    cases = [
        # (r_k, r_v, seqs, seed, num_ctas): the first call is the larger one (more segments, wider partials)
        (448, 576, [3000, 17, 8193, 640, 0, 129, 4097, 1], 20, 148),
        (512, 384, [700, 5, 1300], 30, 7),
    ]
    for r_k, r_v, seqs, seed, nct in cases:
        lat, cache, bt, seq_lens, q_bd = _case(r_k, r_v, seqs, seed)
        a_ref, lse_ref = _regular(lat, q_bd, cache, bt, seq_lens, nct)
        a, lse = _noalloc(lat, q_bd, cache, bt, seq_lens, nct)
        torch.cuda.synchronize()
        dec.check_device_errors(q_bd.device)
        what = f"r_v {r_v}, {len(seqs)} requests, {nct} CTAs"
        assert torch.isfinite(a.float()).all() and torch.isfinite(lse[seq_lens > 0]).all(), what
        err = (a.float() - a_ref.float()).abs()
        assert float(err.max()) < MAX_ABS and float(err.mean()) < MEAN_ABS, (what, float(err.max()), float(err.mean()))
        live = seq_lens > 0
        assert torch.allclose(lse[live], lse_ref[live], atol=LSE_ATOL, rtol=0), what
        assert torch.equal(torch.isinf(lse), torch.isinf(lse_ref)), what


CACHE_TEST = r"""
#include <cstdio>
#include "scratch_cache.h"
int main() {
  belt::ScratchAddressCache<2> c;
  int ctx_a, ctx_b, ctx_c;
  char x, y, z, w;
  if (c.find(&ctx_a)) return 1;                              // nothing recorded yet: a capture-time call is refused
  c.refresh(&ctx_a, &x);
  if (c.find(&ctx_a) != &x || c.find(&ctx_b)) return 2;      // a record belongs to its context only
  c.refresh(&ctx_a, &y);                                     // a new lookup in the same context (after a reset)
  if (c.find(&ctx_a) != &y || c.size() != 1) return 3;       // replaces the old address
  c.refresh(&ctx_b, &z);
  c.refresh(&ctx_c, &w);                                     // a third context: the oldest record is dropped
  if (c.find(&ctx_a) || c.find(&ctx_b) != &z || c.find(&ctx_c) != &w) return 4;
  c.forget(&ctx_b);
  if (c.find(&ctx_b) || c.find(&ctx_c) != &w || c.size() != 1) return 5;
  std::puts("ok");
  return 0;
}
"""


def test_scratch_address_record_is_per_context(tmp_path):
    """The device address of the array is recorded per CUDA context: a new lookup in a context replaces its record
    (a device reset loads the library's device code again, maybe elsewhere), another context never sees it, and a
    context with no record has none to use during stream capture. Host-only: the record is plain C++."""
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not found")
    src = tmp_path / "cache_test.cpp"
    src.write_text(CACHE_TEST)
    exe = tmp_path / "cache_test"
    csrc = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "belt_b200", "csrc")
    subprocess.run([gxx, "-std=c++17", "-O1", "-I", csrc, str(src), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0 and r.stdout.strip() == "ok", (r.returncode, r.stdout)


@pytest.mark.gpu
def test_noalloc_at_the_array_limit_against_the_oracle():
    """258 short requests at r_v 640 on 148 CTAs: up to (258 + 148) partial rows, the last of them at the top of the
    array. The result matches the regular entry points and, after the U_v projection, the fp32 oracle for the
    requests whose partials come last."""
    import oracle
    num_ctas, B = 148, 258
    assert (B + num_ctas) * 24 * 641 * 4 <= PART_BYTES < (B + 1 + num_ctas) * 24 * 641 * 4
    g = torch.Generator().manual_seed(41)
    seqs = [int(x) for x in torch.randint(1, 300, (B,), generator=g)]
    r_k, r_v = 384, 640
    lat, cache, bt, seq_lens, q_bd = _case(r_k, r_v, seqs, 50)
    a_ref, lse_ref = _regular(lat, q_bd, cache, bt, seq_lens, num_ctas)
    a, lse = _noalloc(lat, q_bd, cache, bt, seq_lens, num_ctas)
    torch.cuda.synchronize()
    dec.check_device_errors(q_bd.device)
    err = (a.float() - a_ref.float()).abs()
    assert float(err.max()) < MAX_ABS and float(err.mean()) < MEAN_ABS, (float(err.max()), float(err.mean()))
    assert torch.allclose(lse, lse_ref, atol=LSE_ATOL, rtol=0)
    # the oracle on the last requests (their partial rows are the last ones written)
    spec = synth.spec_from_ranks(r_k, r_v)
    w = synth.make_layer(spec)
    ref = oracle.derive(w.k_up, w.v_up, w.k_norm_weight, w.layout, synth.cos_sin_table(max(seqs) + 8))
    tail = list(range(B - 4, B))
    q = synth.make_queries(B, seed=51)
    exp = oracle.decode_fp32(q[tail], cache.cpu(), bt.cpu()[tail], seq_lens.cpu()[tail], ref, SCALE)
    got = oracle.up_project(a[tail].cpu(), ref["v_up"])
    d = (got.float() - exp).abs()
    assert float(d.max()) < MAX_ABS and float(d.mean()) < MEAN_ABS, (float(d.max()), float(d.mean()))
