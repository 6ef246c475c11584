"""Seeded synthetic workloads of the benchmark configurations.

No model weights, factor checkpoints or datasets are available offline, so every test and benchmark input is drawn
here from fixed seeds with the shapes and distributions the benchmark configurations name:

* geometry of one compressed full-attention layer: 24 query heads in 4 KV groups, head_dim 256, partial NeoX RoPE on
  the first 64 channels, theta 1e7;
* factors per group U_g [256, r_g] ~ N(0, 1/r_g), U_v [4 * 256, r_v] ~ N(0, 1/r_v), down-projections
  VS [r, hidden] ~ N(0, 1/hidden), passed through the export's change of basis (``latent_format.latent_tensors``);
* cache rows ~ N(0, 1) in every latent column, zero in the alignment gaps; physical blocks dealt to requests by a
  seeded random permutation; blocks no request owns are NaN-poisoned so a stray read shows up;
* queries ~ N(0, 1) BF16; token t of a request sits at position t.

Seeds: 0 factors, 1 cache, 2 queries, 3 lengths (and per-layer ranks).
"""

from __future__ import annotations

from dataclasses import dataclass, field
import math

import torch

from . import latent_format

H, G, D, ROT = 24, 4, 256, 64
THETA = 1e7
SEED_FACTORS, SEED_CACHE, SEED_QUERY, SEED_LENGTHS = 0, 1, 2, 3


@dataclass
class LayerSpec:
    """Ranks of one compressed layer."""

    k_ranks: tuple
    v_rank: int
    hidden: int = 1024
    rope_align: bool = False
    gain_std: float = 0.0

    @property
    def row_width(self) -> int:
        return latent_format.row_layout(self.k_ranks, self.v_rank, ROT, rope_align=self.rope_align)["row_width"]


def c50(hidden: int = 1024, **kw) -> LayerSpec:
    """r_k = 512 (4 x 128), r_v = 512: row width 1024."""
    return LayerSpec((128,) * 4, 512, hidden, **kw)


def c25(hidden: int = 1024, **kw) -> LayerSpec:
    """r_k + r_v = 512: r_k = 256 (4 x 64), r_v = 256: row width 512."""
    return LayerSpec((64,) * 4, 256, hidden, **kw)


def learned_ranks(num_layers: int = 16, budget: int = 1024, seed: int = SEED_LENGTHS) -> list:
    """Per-layer (r_k, r_v) with r_k drawn from {384, 448, 512, 576, 640} and r_v = budget - r_k."""
    g = torch.Generator().manual_seed(seed)
    choices = torch.tensor([384, 448, 512, 576, 640]) * budget // 1024
    idx = torch.randint(0, len(choices), (num_layers,), generator=g)
    return [(int(choices[i]), budget - int(choices[i])) for i in idx]


def spec_from_ranks(r_k: int, r_v: int, hidden: int = 1024, **kw) -> LayerSpec:
    base, extra = divmod(r_k, G)
    return LayerSpec(tuple(base + (1 if g < extra else 0) for g in range(G)), r_v, hidden, **kw)


def log_uniform_lengths(batch: int, lo: int, hi: int, seed: int = SEED_LENGTHS) -> list:
    g = torch.Generator().manual_seed(seed + 1000)
    u = torch.rand(batch, generator=g, dtype=torch.float64)
    return [int(round(math.exp(math.log(lo) + float(x) * (math.log(hi) - math.log(lo))))) for x in u]


def make_factors(spec: LayerSpec, seed: int = SEED_FACTORS):
    """(k_blocks [(VS_g, U_g)], (VS_v, U_v), k_norm weight [D]) fp32."""
    g = torch.Generator().manual_seed(seed)
    k_blocks = []
    for r in spec.k_ranks:
        VS = torch.randn(r, spec.hidden, generator=g) / math.sqrt(spec.hidden)
        U = torch.randn(D, r, generator=g) / math.sqrt(r)
        k_blocks.append((VS, U))
    VS_v = torch.randn(spec.v_rank, spec.hidden, generator=g) / math.sqrt(spec.hidden)
    U_v = torch.randn(G * D, spec.v_rank, generator=g) / math.sqrt(spec.v_rank)
    k_norm = torch.randn(D, generator=g) * spec.gain_std if spec.gain_std else torch.zeros(D)
    return k_blocks, (VS_v, U_v), k_norm


@dataclass
class LayerWeights:
    """What a latent export holds for one compressed layer (``latent_format.latent_tensors``)."""

    kv_latent_proj: torch.Tensor      # [pe_offset, hidden] BF16
    k_up: torch.Tensor                # [G, D, r_max] BF16
    v_up: torch.Tensor                # [G * D, r_v] BF16
    k_norm_weight: torch.Tensor       # [D] fp32 (zero-centred RMSNorm weight)
    layout: dict = field(default_factory=dict)


def make_layer(spec: LayerSpec, seed: int = SEED_FACTORS) -> LayerWeights:
    k_blocks, v_factors, k_norm = make_factors(spec, seed)
    proj, k_up, v_up, layout = latent_format.latent_tensors(k_blocks, v_factors, D, ROT, rope_align=spec.rope_align)
    return LayerWeights(proj, k_up, v_up, k_norm, layout)


def cos_sin_table(max_pos: int, rotary_dim: int = ROT, theta: float = THETA) -> torch.Tensor:
    """The model's NeoX cos/sin cache [max_pos, rot] in fp32 (cos half | sin half), computed on the CPU."""
    return latent_format.cos_sin_table(max_pos, rotary_dim, theta)


@dataclass
class PagedBatch:
    """Decode requests over a paged cache: ``seq_lens`` include this step's token (already written)."""

    cache: torch.Tensor               # [num_blocks, page, W] BF16 (possibly a strided per-layer view)
    block_table: torch.Tensor         # [B, max_pages] int32
    seq_lens: torch.Tensor            # [B] int32
    page: int
    owned: int                        # blocks owned by requests (the rest are poisoned)


def block_tables(seq_lens, page: int, extra_blocks: int = 0, seed: int = SEED_CACHE, min_pages: int = 1):
    """(block_table [B, max_pages] int32, num_blocks): every request gets ceil(L / page) physical blocks of a seeded
    random permutation; padding entries are 0."""
    pages = [max(-(-int(L) // page), 0) for L in seq_lens]
    owned = sum(pages)
    num_blocks = owned + extra_blocks
    g = torch.Generator().manual_seed(seed + 7)
    perm = torch.randperm(num_blocks, generator=g)[:owned]
    max_pages = max(max(pages, default=0), min_pages)
    bt = torch.zeros(len(pages), max_pages, dtype=torch.int32)
    i = 0
    for b, n in enumerate(pages):
        bt[b, :n] = perm[i:i + n].to(torch.int32)
        i += n
    return bt, num_blocks, owned


def latent_columns(layout: dict) -> torch.Tensor:
    """Boolean mask [W]: the columns that hold a latent coordinate (the rest are alignment gaps)."""
    W = layout["row_width"]
    m = torch.zeros(W, dtype=torch.bool)
    m[:layout["lk"]] = True
    m[layout["v_offset"]:layout["v_offset"] + layout["v_rank"]] = True
    return m


def fill_cache(cache: torch.Tensor, layout: dict, block_table: torch.Tensor, seq_lens, seed: int = SEED_CACHE,
               poison: bool = True) -> None:
    """N(0, 1) rows (zero gaps) in every block a request owns; NaN in every other block when ``poison``."""
    nb, page, W = cache.shape
    dev = cache.device
    gen = torch.Generator(device=dev).manual_seed(seed)
    mask = latent_columns(layout).to(dev)
    owned = torch.zeros(nb, dtype=torch.bool, device=dev)
    for b, L in enumerate(seq_lens):
        n = -(-int(L) // page)
        if n:
            owned[block_table[b, :n].long().to(dev)] = True
    step = max(1, (1 << 26) // max(1, page * W))       # bounded temporaries
    for i in range(0, nb, step):
        j = min(nb, i + step)
        x = torch.randn(j - i, page, W, generator=gen, device=dev, dtype=torch.bfloat16)
        x *= mask
        if poison:
            x[~owned[i:j]] = float("nan")
        cache[i:j] = x


def make_batch(layout: dict, seq_lens, page: int = 16, extra_blocks: int = 8, seed: int = SEED_CACHE,
               device="cpu", poison: bool = True) -> PagedBatch:
    bt, nb, owned = block_tables(seq_lens, page, extra_blocks, seed)
    cache = torch.empty(nb, page, layout["row_width"], dtype=torch.bfloat16, device=device)
    fill_cache(cache, layout, bt, seq_lens, seed, poison)
    return PagedBatch(cache, bt.to(device), torch.tensor(list(seq_lens), dtype=torch.int32, device=device), page,
                      owned)


def make_queries(batch: int, seed: int = SEED_QUERY, device="cpu") -> torch.Tensor:
    """q [B, H, D] BF16 ~ N(0, 1) (the normed, rotated query of the decode token)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(batch, H, D, generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)
