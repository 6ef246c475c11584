"""Generate the golden vectors that pin the CPU oracle to the reference's own code.

Run in the build container, where the reference checkout is mounted (it does not travel to the GPU box):

    python tests/golden/make_golden.py --reference <path to the BELT checkout>

What runs is the reference's code, unmodified:

* ``lrkv.runtime.export_latent.build_latent_layer`` (format, change of basis);
* ``LatentAttentionLayer.derive_latent_tensors`` (``qwen3_5_latent.py:161-202``), called on a stand-in module that
  carries the loaded weights, so the reference's own derivation builds the ``LatentLayer``;
* ``LatentLayer.decompress`` (``latent_backend.py:95-108``), then fp32 softmax attention (the CPU stand-in for
  flash-attention) -> the reference decode output ("Oracle A");
* ``cute_decode.block_diag_query`` (reference construction) and ``rope_blocks``;
* the Triton kernels ``_latent_rows``, ``_group_gemm`` (block-diagonal query, V up-projection), ``_schedule`` and
  ``_merge_segments`` under ``TRITON_INTERPRET=1``. The interpreter mishandles BF16 arrays, so they run on fp32
  tensors holding BF16 values and their stores are rounded to BF16 afterwards (the kernels' ``.to(bf16)``).
* vLLM's ``RotaryEmbedding`` cos/sin cache construction.

Modules the reference imports but this container lacks (CuTe DSL 4.8 submodules, quack, vLLM 0.32 symbols) are
replaced by inert stubs: none of them is on the CPU paths above.

Inputs come from ``belt_b200.synth`` with fixed seeds; the fixtures store the factors, the outputs and checksums.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib
import os
import re
import sys
import types
from unittest import mock

os.environ["TRITON_INTERPRET"] = "1"

import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from belt_b200 import synth  # noqa: E402

CASES = {
    # name: (LayerSpec, seq_lens, page)
    "c50": (synth.LayerSpec((128,) * 4, 512, 256, gain_std=0.1), [129, 513, 1025, 2001], 16),
    "ragged": (synth.LayerSpec((96, 112, 144, 160), 512, 256, gain_std=0.1), [1, 17, 129, 300], 16),
    "ragged_ra": (synth.LayerSpec((96, 112, 144, 160), 512, 256, rope_align=True, gain_std=0.1), [2, 64, 130], 16),
    "c25": (synth.LayerSpec((64,) * 4, 256, 256), [5, 64, 200], 32),
    "small_rank": (synth.LayerSpec((48, 40, 64, 56), 300, 256, gain_std=0.05), [3, 70], 16),
}
MAX_POS = 4096
MERGE_SETS = [([129, 513, 1025, 2001], 16), ([0, 300, 64, 0], 8), ([40] * 12, 8)]
SCHEDULE_SETS = [
    ([129, 513, 1025, 2001], 148), ([1, 17, 129, 300], 8), ([0, 64, 0, 65, 4096, 1], 16), ([8192] * 64, 148),
    ([5], 148), ([0, 0], 4), ([3000, 1, 1, 1, 7000, 64, 63, 65], 148), ([200] * 300, 148),
]


class _Stub:
    def __init__(self, *a, **k):
        pass

    def __class_getitem__(cls, item):
        return cls


def _stub_module(name):
    m = types.ModuleType(name)
    m.__path__ = []

    def __getattr__(attr, _n=name):
        if attr.startswith("__"):
            raise AttributeError(attr)
        return type(attr, (_Stub,), {}) if attr[:1].isupper() else mock.MagicMock(name=f"{_n}.{attr}")

    m.__getattr__ = __getattr__
    sys.modules[name] = m


def import_with_stubs(modname, tries=64):
    for _ in range(tries):
        try:
            return importlib.import_module(modname)
        except ModuleNotFoundError as e:
            _stub_module(e.name)
        except ImportError as e:
            m = re.search(r"cannot import name '(\w+)' from '([\w\.]+)'", str(e))
            if not m:
                raise
            attr, mod = m.groups()
            target = sys.modules.get(mod) or importlib.import_module(mod)
            setattr(target, attr, type(attr, (_Stub,), {}) if attr[:1].isupper() else mock.MagicMock(name=attr))
    raise RuntimeError(f"cannot import {modname}")


def sha(t: torch.Tensor) -> str:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def bf16_round(t):
    return t.to(torch.bfloat16)


def reference_layer(mods, w, layout, cos_sin_f32, eps=1e-6):
    """Run the reference's ``derive_latent_tensors`` on a stand-in module holding the loaded weights."""
    qm, lb = mods["model"], mods["backend"]
    G, D, _ = w["k_up"].shape
    rot = 64
    ranks = layout["k_head_ranks"]
    k_segments = [[(int(a), int(n)) for a, n in runs] for runs in layout["k_segments"]]
    self = types.SimpleNamespace()
    self.k_up = types.SimpleNamespace(weight=w["k_up"].clone())
    self.v_up = types.SimpleNamespace(weight=types.SimpleNamespace())
    self.v_up.weight = torch.nn.Parameter(w["v_up"].clone(), requires_grad=False)
    self.k_norm = types.SimpleNamespace(weight=w["k_norm"].clone())
    self.rotary_dim, self.head_dim, self.num_kv_heads = rot, D, G
    self.v_offset, self.v_rank, self.pe_offset = layout["v_offset"], layout["v_rank"], layout["pe_offset"]
    self.k_segments, self.k_head_ranks, self.lk = k_segments, ranks, sum(ranks)
    self.u_cat = torch.zeros(self.lk, G * D, dtype=torch.bfloat16)
    self.k_segs = torch.tensor([[x for run in runs + [(0, 0)] * (2 - len(runs)) for x in run] for runs in k_segments],
                               dtype=torch.int32)
    self.rope_gain = torch.zeros(rot, dtype=torch.float32)
    self.rope_groups = tuple((runs[0][0], int(rr)) for runs, rr in zip(k_segments, layout["rope_ranks"]))
    self.rotary_emb = types.SimpleNamespace(cos_sin_cache=cos_sin_f32)
    self.mrope_section = None
    self.eps = eps
    self.attn = types.SimpleNamespace(latent=None)
    qm.LatentAttentionLayer.derive_latent_tensors(self)
    lat = self.attn.latent
    assert isinstance(lat, lb.LatentLayer)
    return lat


def attention_fp32(q, k, v, scale):
    H = q.shape[0]
    G = k.shape[1]
    kh = k.float().repeat_interleave(H // G, dim=1)
    vh = v.float().repeat_interleave(H // G, dim=1)
    s = torch.einsum("hd,shd->hs", q.float(), kh) * scale
    return torch.einsum("hs,shd->hd", torch.softmax(s, dim=-1), vh)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("BELT_REFERENCE", ""), required=False)
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    ref = args.reference
    if not ref or not os.path.isdir(ref):
        raise SystemExit("pass --reference <BELT checkout>")
    sys.path.insert(0, ref)
    sys.path.insert(0, os.path.join(ref, "plugins", "vllm_lrkv"))
    el = importlib.import_module("lrkv.runtime.export_latent")
    mods = {"cute": import_with_stubs("vllm_lrkv.cute_decode"), "backend": import_with_stubs("vllm_lrkv.latent_backend"),
            "model": import_with_stubs("vllm_lrkv.models.qwen3_5_latent"), "ops": import_with_stubs("vllm_lrkv.latent_ops")}
    cd, lb, ops = mods["cute"], mods["backend"], mods["ops"]
    from vllm.model_executor.layers.rotary_embedding.base import RotaryEmbedding
    # vLLM's own cos/sin construction, run on a stand-in (a CustomOp cannot be built without a vLLM config)
    rope = types.SimpleNamespace(rotary_dim=64, base=synth.THETA, max_position_embeddings=MAX_POS)
    rope._compute_inv_freq = types.MethodType(RotaryEmbedding._compute_inv_freq, rope)
    cos_sin_f32 = RotaryEmbedding._compute_cos_sin_cache(rope).float()
    scale = 256 ** -0.5

    common = {"cos_sin_sha_f32": sha(cos_sin_f32), "cos_sin_sha_bf16": sha(cos_sin_f32.to(torch.bfloat16)),
              "max_pos": MAX_POS, "theta": synth.THETA, "cos_sin_rows": cos_sin_f32[[0, 1, 2, 100, 4095]].clone()}

    # ---- schedule (integer, TILE_T = 64 of the reference) ----
    sched = []
    for seqs, nct in SCHEDULE_SETS:
        B = len(seqs)
        s = cd.make_schedule(B, "cpu", num_ctas=nct)
        cd.schedule(s, torch.tensor(seqs, dtype=torch.int32))
        total = int(s.seg_base[B])
        sched.append({"seq_lens": seqs, "num_ctas": nct, "tile": cd.TILE_T, "work": s.work[:total].clone(),
                      "cta_seg": s.cta_seg.clone(), "seg_base": s.seg_base.clone()})
    common["schedule"] = sched

    # ---- merge (fp32) ----
    merges = []
    for seqs, nct in MERGE_SETS:
        g = torch.Generator().manual_seed(11)
        B = len(seqs)
        s = cd.make_schedule(B, "cpu", num_ctas=nct)
        cd.schedule(s, torch.tensor(seqs, dtype=torch.int32))
        nseg = int(s.seg_base[B])
        lv = 96
        part = torch.randn(nseg + 1, 24, lv + 1, generator=g)
        part[:, :, lv] *= 4
        out = torch.zeros(B, 24, lv)
        lse = torch.zeros(B, 24)
        cd.merge_segments(part, s, out, lse)
        merges.append({"seq_lens": seqs, "num_ctas": nct, "part_sha": sha(part), "part_shape": list(part.shape),
                       "seg_base": s.seg_base.clone(), "a": out, "lse": lse})
    common["merge"] = merges
    torch.save(common, os.path.join(args.out, "common.pt"))
    print("common:", len(sched), "schedules,", len(merges), "merges")

    for name, (spec, seq_lens, page) in CASES.items():
        k_blocks, v_factors, k_norm = synth.make_factors(spec, synth.SEED_FACTORS)
        proj, k_up, v_up, layout = el.build_latent_layer(k_blocks, v_factors, 4, 256, 64, torch.bfloat16,
                                                         el.ALIGN, spec.rope_align)
        w = {"k_up": k_up, "v_up": v_up, "k_norm": k_norm}
        lat = reference_layer(mods, w, layout, cos_sin_f32)
        fx = {"spec": {"k_ranks": list(spec.k_ranks), "v_rank": spec.v_rank, "hidden": spec.hidden,
                       "rope_align": spec.rope_align, "gain_std": spec.gain_std},
              "seq_lens": seq_lens, "page": page, "layout": layout,
              "factors_sha": {"kv_latent_proj": sha(proj), "k_up": sha(k_up), "v_up": sha(v_up),
                              "k_norm": sha(k_norm)},
              "derive": {"qmap": sha(lat.qmap), "u_cat": sha(lat.u_cat), "k_segs": lat.k_segs.clone(),
                         "rope_gain": lat.rope_gain.clone(), "groups": list(lat.rope.groups),
                         "blocks": lat.rope.blocks.clone(), "cos_sin": sha(lat.rope.cos_sin),
                         "rope_up": sha(lat.rope_up), "v_up_t": sha(lat.v_up), "n_k": lat.n_k}}
        # decode inputs
        batch = synth.make_batch(layout, seq_lens, page=page, seed=synth.SEED_CACHE)
        q = synth.make_queries(len(seq_lens), synth.SEED_QUERY)
        fx["inputs_sha"] = {"cache": sha(torch.nan_to_num(batch.cache.float(), nan=7.0)),
                            "block_table": sha(batch.block_table), "q": sha(q)}
        B = len(seq_lens)
        out = torch.zeros(B, 24, 256)
        sample = None
        for b in range(B):
            n = seq_lens[b]
            pos = torch.arange(n)
            blk = batch.block_table[b, pos // page].long()
            rows = batch.cache[blk, pos % page]
            k, v = lat.decompress(rows, pos)
            if sample is None:
                idx = torch.arange(0, n, max(1, n // 8))[:8]
                sample = {"b": b, "idx": idx, "k": k[idx].clone(), "v": v[idx].clone()}
            out[b] = attention_fp32(q[b], k, v, scale)
        fx["decompress"] = sample
        fx["out_reference"] = out
        # block-diagonal query (Triton _group_gemm, fp32 io) and the reference construction
        q_bd = ops.block_diag_query(q.float(), lat.qmap.float())
        fx["q_bd"] = bf16_round(q_bd)
        rot = 64
        k_off = [runs[0][0] for runs in layout["k_segments"]]
        if not spec.rope_align:
            qlat = torch.zeros(B, 24, max(spec.k_ranks))
            for g, r in enumerate(spec.k_ranks):
                cols = torch.arange(k_off[g], k_off[g] + r)
                qlat[:, 6 * g:6 * g + 6, :r] = torch.einsum(
                    "bhd,dk->bhk", q[:, 6 * g:6 * g + 6, rot:].float(), lat.qmap[g, rot:][:, cols].float())
            fx["q_bd_construct_sha"] = sha(cd.block_diag_query(qlat.to(torch.bfloat16), q[..., :rot], k_off,
                                                               list(spec.k_ranks), layout["v_offset"]))
            fx["q_lat_sha"] = sha(qlat.to(torch.bfloat16))
        # V up-projection (Triton _group_gemm, fp32 io)
        a = torch.randn(B, 24, spec.v_rank, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
        up = torch.zeros(B, 24, 256)
        ops.up_project(a.float(), lat.v_up.float(), up)
        fx["up_a_sha"], fx["up_out"] = sha(a), bf16_round(up)
        # cache write (Triton _latent_rows, fp32 io)
        T = 24
        gcw = torch.Generator().manual_seed(9)
        W = layout["row_width"]
        c = (torch.randn(T, W, generator=gcw) * synth.latent_columns(layout)).to(torch.bfloat16)
        nb = 6
        slots = torch.randperm(nb * page, generator=gcw)[:T].to(torch.int32)
        slots[[1, 7, 20]] = -1
        cache_f = torch.full((nb, page, W), float("nan"))
        ops.latent_rows_to_cache(c.float(), slots, cache_f, lat.u_cat.float(), lat.k_segs, 1e-6)
        fx["cw_c_sha"], fx["cw_slots"], fx["cw_nb"] = sha(c), slots, nb
        live = slots >= 0
        fx["cw_rows"] = bf16_round(cache_f.view(-1, W)[slots[live].long()])
        fx["cw_untouched_nan"] = int(torch.isnan(cache_f).sum())
        torch.save(fx, os.path.join(args.out, f"{name}.pt"))
        print(name, "W", W, "groups", list(lat.rope.groups), "out", float(out.abs().mean()))


if __name__ == "__main__":
    main()
