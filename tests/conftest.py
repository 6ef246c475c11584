import hashlib
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

CASES = ("c50", "ragged", "ragged_ra", "c25", "small_rank")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


def sha(t: torch.Tensor) -> str:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def load_golden(name):
    return torch.load(os.path.join(GOLDEN, f"{name}.pt"), weights_only=False)


def golden_case(name):
    """(fixture, LayerSpec, LayerWeights, PagedBatch, q) with the inputs regenerated from the fixture's seeds."""
    from belt_b200 import synth
    fx = load_golden(name)
    sp = fx["spec"]
    spec = synth.LayerSpec(tuple(sp["k_ranks"]), sp["v_rank"], sp["hidden"], rope_align=sp["rope_align"],
                           gain_std=sp["gain_std"])
    w = synth.make_layer(spec, synth.SEED_FACTORS)
    batch = synth.make_batch(w.layout, fx["seq_lens"], page=fx["page"], seed=synth.SEED_CACHE)
    q = synth.make_queries(len(fx["seq_lens"]), synth.SEED_QUERY)
    return fx, spec, w, batch, q


class UlpCheck:
    """Result of ``bf16_ulp_close``: truthy when every element is within the bound; ``repr`` says where it is not."""

    def __init__(self, ok, msg=""):
        self.ok, self.msg = ok, msg

    def __bool__(self):
        return self.ok

    def __repr__(self):
        return f"UlpCheck({self.ok}: {self.msg})"


def bf16_ulp_close(a, b, ulps=1, atol=0.0):
    """|a - b| <= ulps BF16 ulps of max(|a|, |b|) + atol elementwise (NaN positions must agree)."""
    a, b = a.float(), b.float()
    na, nb = torch.isnan(a), torch.isnan(b)
    if not torch.equal(na, nb):
        idx = (na != nb).nonzero()[:5].tolist()
        return UlpCheck(False, f"NaN positions differ ({int((na != nb).sum())}), first {idx}")
    m = ~na
    a, b = a[m], b[m]
    mag = torch.maximum(a.abs(), b.abs())
    ulp = torch.where(mag > 0, 2.0 ** (torch.floor(torch.log2(mag.clamp_min(1e-38))) - 7), torch.zeros_like(mag))
    bad = (a - b).abs() > ulps * ulp + atol + 1e-30
    if bad.any():
        r = ((a - b).abs() / ulp.clamp_min(1e-38))[bad]
        i = bad.nonzero()[:3].flatten().tolist()
        return UlpCheck(False, f"{int(bad.sum())} elements beyond {ulps} ulp (max {float(r.max()):.1f} ulp), first at "
                               f"flat {i}: {a[i].tolist()} vs {b[i].tolist()}")
    return UlpCheck(True)


@pytest.fixture(scope="session")
def common_golden():
    return load_golden("common")
