"""The attention block of a compressed layer as the model runs it (plugins/vllm_lrkv/vllm_lrkv/models/
qwen3_5_latent.py:98-217, ``LatentAttention`` + ``forward``), on this package's kernels:

    qg   = hidden @ q_gate_proj^T                         [T, 24 * 2 * 256]   belt_gemm_bf16 (tcgen05)
    q    = NeoX-RoPE(RMSNorm_{1 + w}(qg query halves))     belt_q_norm_rope    (the query side of the fused q-norm/RoPE)
    rows = the new tokens' cache rows from hidden            fused into the cache write (belt_latent_proj_rows_to_cache)
    attn = the backend's decode / prefill attention          ``latent_attention_step``
    attn = attn * sigmoid(qg gate halves)                    belt_gate_mul
    out  = attn @ o_proj^T                                   belt_gemm_bf16 (tcgen05)

One model copy per GPU (the reference refuses tensor parallelism, qwen3_5_latent.py:101-102). The weights are the
export's: ``q_gate_proj`` [24 * 512, hidden], ``o_proj`` [hidden, 24 * 256], ``q_norm`` / ``k_norm`` weights [256]
(zero-centred RMSNorm), ``kv_latent_proj`` [row_width, hidden], ``k_up`` / ``v_up`` (``derive_latent_tensors``).
"""

from __future__ import annotations

import torch

from . import _lib
from .decode import _stream_ptr
from .latent_backend import LatentAttentionImpl, LatentAttentionMetadata, latent_attention_step
from .latent_ops import linear
from .layer import derive_latent_tensors

H, D = 24, 256


def q_norm_rope(qg: torch.Tensor, norm_weight: torch.Tensor, eps: float, cos_sin: torch.Tensor,
                positions: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """q [T, 24, 256] BF16 from the query halves ``qg`` [T, 24, >= 256] (a view of q_gate_proj's output): zero-centred
    RMSNorm (weight 1 + ``norm_weight``) and the NeoX rotation of the first cos_sin.shape[1] channels at
    ``positions``, in fp32, rounded to BF16 once (``belt_q_norm_rope``)."""
    T = qg.shape[0]
    if out is None:
        out = torch.empty(T, H, D, dtype=torch.bfloat16, device=qg.device)
    if T == 0:
        return out
    if qg.dtype != torch.bfloat16 or qg.dim() != 3 or qg.shape[1] != H or qg.stride(2) != 1:
        raise ValueError("q_norm_rope: qg [T, 24, >= 256] BF16 with contiguous channels")
    if positions.dtype not in (torch.int32, torch.int64) or not positions.is_contiguous():
        raise ValueError("q_norm_rope: contiguous int32 / int64 positions")
    if cos_sin.dtype != torch.bfloat16 or not cos_sin.is_contiguous() or cos_sin.device != qg.device:
        raise ValueError("q_norm_rope: cos_sin [max_pos, rot] BF16 contiguous, on the query's device")
    w = norm_weight.detach().to(device=qg.device, dtype=torch.float32).contiguous()
    _lib.call("belt_q_norm_rope", qg.data_ptr(), T, qg.stride(0), qg.stride(1), w.data_ptr(), float(eps),
              cos_sin.data_ptr(), cos_sin.shape[0], cos_sin.shape[1], positions.data_ptr(),
              int(positions.dtype == torch.int64), out.data_ptr(), out.stride(0), out.stride(1),
              _stream_ptr(qg.device))
    return out


def gate_mul(attn: torch.Tensor, gate: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """attn * sigmoid(gate) for [T, 24, 256] BF16 views (``belt_gate_mul``); ``out`` may be ``attn``."""
    T = attn.shape[0]
    if out is None:
        out = torch.empty(T, H, D, dtype=torch.bfloat16, device=attn.device)
    if T == 0:
        return out
    for name, t in (("attn", attn), ("gate", gate), ("out", out)):
        if t.dtype != torch.bfloat16 or t.dim() != 3 or t.shape[1] != H or t.shape[2] < D or t.stride(2) != 1:
            raise ValueError(f"gate_mul: {name} [T, 24, 256] BF16 with contiguous channels")
    _lib.call("belt_gate_mul", attn.data_ptr(), attn.stride(0), attn.stride(1), gate.data_ptr(), gate.stride(0),
              gate.stride(1), T, out.data_ptr(), out.stride(0), out.stride(1), _stream_ptr(attn.device))
    return out


class LatentSelfAttention:
    """One compressed layer's attention block. ``latent`` is its ``LatentLayer`` (the backend reads it as
    ``layer.latent``); ``forward(positions, hidden, kv_cache, attn_metadata)`` -> [T, hidden] BF16."""

    def __init__(self, q_gate_proj: torch.Tensor, o_proj: torch.Tensor, q_norm_weight: torch.Tensor,
                 k_norm_weight: torch.Tensor, kv_latent_proj: torch.Tensor, k_up: torch.Tensor, v_up: torch.Tensor,
                 layout: dict, cos_sin: torch.Tensor, eps: float = 1e-6, device=None):
        device = torch.device(device) if device is not None else q_gate_proj.device
        bf = dict(device=device, dtype=torch.bfloat16)
        self.q_gate_proj = q_gate_proj.detach().to(**bf).contiguous()
        self.o_proj = o_proj.detach().to(**bf).contiguous()
        self.kv_latent_proj = kv_latent_proj.detach().to(**bf).contiguous()
        self.q_norm_weight = q_norm_weight.detach().to(device=device, dtype=torch.float32).contiguous()
        self.eps = float(eps)
        self.latent = derive_latent_tensors(k_up, v_up, k_norm_weight, layout, cos_sin, eps=eps, device=device)
        self.impl = LatentAttentionImpl(H, D, D ** -0.5, self.latent.num_kv_heads)

    def forward(self, positions: torch.Tensor, hidden: torch.Tensor, kv_cache: torch.Tensor,
                attn_metadata: LatentAttentionMetadata) -> torch.Tensor:
        T = hidden.shape[0]
        qg = linear(hidden, self.q_gate_proj).view(T, H, 2 * D)
        q = q_norm_rope(qg[:, :, :D], self.q_norm_weight, self.eps, self.latent.rope.cos_sin, positions)
        attn = torch.empty(T, H, D, dtype=torch.bfloat16, device=hidden.device)
        latent_attention_step(self.impl, self, q, hidden, self.kv_latent_proj, kv_cache, attn_metadata, attn)
        gate_mul(attn, qg[:, :, D:], out=attn)
        return linear(attn.view(T, H * D), self.o_proj)
