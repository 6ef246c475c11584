"""Golden record of the reference's latent exporter, for the export reader / writer of ``belt_b200.latent_format``.

Run in the build container, where the reference checkout is mounted (it does not travel to the GPU box):

    python tests/golden/make_export_golden.py --reference <path to the BELT checkout>

What runs is the reference's code, unmodified:

* ``lrkv.runtime.export_latent.export`` on the synthetic base model and factor checkpoint of ``export_case.py``,
  once packed and once with ``rope_align``;
* ``LatentAttentionLayer.derive_latent_tensors`` (``qwen3_5_latent.py:161-202``, through ``make_golden``'s stand-in
  module) on every compressed layer's exported tensors, with vLLM's cos/sin construction for the config's theta.

``export.json`` keeps, per variant, what ``export_case.describe_export`` reads of the output directory (tensor
checksums, config, index, accounting) and the checksums of the derived per-layer constants.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib
import json
import os
import sys
import tempfile
import types

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import torch  # noqa: E402

import export_case  # noqa: E402
import make_golden  # noqa: E402


def sha(t):
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def derive_record(mods, out_dir, cos_sin_f32):
    """The reference's derive on every compressed layer of an export directory: checksums by layer."""
    from safetensors import safe_open
    with open(os.path.join(out_dir, "config.json")) as f:
        config = json.load(f)
    with open(os.path.join(out_dir, "model.safetensors.index.json")) as f:
        wm = json.load(f)["weight_map"]
    rec = {}
    for i, layout in config["kv_lowrank"]["layers"].items():
        p = f"model.layers.{i}.self_attn."
        w = {}
        for key, name in (("k_up", "k_up.weight"), ("v_up", "v_up.weight"), ("k_norm", "k_norm.weight")):
            with safe_open(os.path.join(out_dir, wm[p + name]), framework="pt") as f:
                w[key] = f.get_tensor(p + name)
        lat = make_golden.reference_layer(mods, w, layout, cos_sin_f32, eps=config["rms_norm_eps"])
        rec[i] = {"qmap": sha(lat.qmap), "u_cat": sha(lat.u_cat), "k_segs": lat.k_segs.tolist(),
                  "rope_gain": sha(lat.rope_gain), "groups": [list(g) for g in lat.rope.groups],
                  "blocks": sha(lat.rope.blocks), "cos_sin": sha(lat.rope.cos_sin), "rope_up": sha(lat.rope_up),
                  "v_up_t": sha(lat.v_up), "n_k": lat.n_k}
    return rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("BELT_REFERENCE", ""))
    ap.add_argument("--out", default=os.path.join(HERE, "export.json"))
    args = ap.parse_args()
    ref = args.reference
    if not ref or not os.path.isdir(ref):
        raise SystemExit("pass --reference <BELT checkout>")
    sys.path.insert(0, ref)
    sys.path.insert(0, os.path.join(ref, "plugins", "vllm_lrkv"))
    el = importlib.import_module("lrkv.runtime.export_latent")
    mods = {"backend": make_golden.import_with_stubs("vllm_lrkv.latent_backend"),
            "model": make_golden.import_with_stubs("vllm_lrkv.models.qwen3_5_latent")}
    from vllm.model_executor.layers.rotary_embedding.base import RotaryEmbedding
    cfg = export_case.CONFIG
    rope = types.SimpleNamespace(rotary_dim=64, base=cfg["rope_parameters"]["rope_theta"],
                                 max_position_embeddings=cfg["max_position_embeddings"])
    rope._compute_inv_freq = types.MethodType(RotaryEmbedding._compute_inv_freq, rope)
    cos_sin_f32 = RotaryEmbedding._compute_cos_sin_cache(rope).float()

    golden = {"cos_sin_f32": sha(cos_sin_f32), "variants": {}}
    with tempfile.TemporaryDirectory() as tmp:
        base = export_case.write_base_model(os.path.join(tmp, "base"))
        ckpt = export_case.write_checkpoint(os.path.join(tmp, "ckpt.pt"))
        for name, rope_align in (("packed", False), ("rope_align", True)):
            out = os.path.join(tmp, name)
            el.export(base, ckpt, out, dtype=torch.bfloat16, rope_align=rope_align)
            golden["variants"][name] = {"export": export_case.describe_export(out),
                                        "derive": derive_record(mods, out, cos_sin_f32)}
            print(name, sorted(golden["variants"][name]["export"]["kv_lowrank"]["layers"]))
    with open(args.out, "w") as f:
        json.dump(golden, f, indent=1, sort_keys=True)
    print("wrote", args.out)


if __name__ == "__main__":
    main()
