"""The tensor-core GEMM (``belt_gemm_bf16`` / ``latent_ops.linear``) against an fp32 product of the same BF16 operands.

Bound: the kernel accumulates in fp32 and rounds once to BF16, so every output is within one BF16 ulp of the fp32
product (the rounding itself is half an ulp; a different fp32 summation order can move it across a rounding boundary),
plus 1e-4 absolute for outputs that cancel to near zero (the fp32 summation error of K terms of size ~1 relative to an
output much smaller than them).
Shapes cover both column tiles (128 and 256), ragged M / N / K (the TMA zero fill and the masked epilogue), strided
rows, one-row products and the model's shapes (q_gate_proj, o_proj, kv_latent_proj of a prefill chunk).
"""

import pytest
import torch

from belt_b200 import latent_ops
from conftest import bf16_ulp_close

DEV = "cuda"


def test_linear_rejects_bad_operands():
    with pytest.raises(ValueError, match="\\[M, K\\] and \\[N, K\\]"):
        latent_ops.linear(torch.zeros(4, 8, dtype=torch.bfloat16), torch.zeros(5, 16, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="BF16"):
        latent_ops.linear(torch.zeros(4, 8), torch.zeros(5, 8))


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,pad", [
    (1, 256, 64, 0), (77, 300, 200, 0), (300, 520, 264, 8), (128, 12288, 1024, 0), (2048, 1024, 6144, 0),
    (8192, 1024, 1024, 0), (333, 1024, 1024, 16),
])
def test_gemm_matches_fp32(M, N, K, pad):
    g = torch.Generator().manual_seed(M * 7 + N * 3 + K)
    x = torch.randn(M, K + pad, generator=g).to(torch.bfloat16)[:, :K]
    w = (torch.randn(N, K, generator=g) / K ** 0.5).to(torch.bfloat16)
    out = latent_ops.linear(x.to(DEV), w.to(DEV))
    torch.cuda.synchronize()
    from belt_b200 import decode as dec
    dec.check_device_errors(DEV)
    assert out.shape == (M, N) and out.dtype == torch.bfloat16
    ref = x.float() @ w.float().T
    assert bf16_ulp_close(out.cpu(), ref, ulps=1, atol=1e-4)


@pytest.mark.gpu
def test_gemm_output_rows_at_a_stride():
    """The op writes its own [M, N] buffer; the C entry also takes a strided output (ldc > N)."""
    from belt_b200 import _lib
    M, N, K = 200, 384, 512
    g = torch.Generator().manual_seed(3)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(N, K, generator=g) / K ** 0.5).to(torch.bfloat16).to(DEV)
    big = torch.full((M, N + 64), 7.0, dtype=torch.bfloat16, device=DEV)
    _lib.call("belt_gemm_bf16", x.data_ptr(), M, K, K, w.data_ptr(), N, K, big.data_ptr(), N + 64, 0,
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert bf16_ulp_close(big[:, :N].cpu(), x.float().cpu() @ w.float().cpu().T, ulps=1, atol=1e-4)
    assert bool((big[:, N:] == 7.0).all())          # nothing written past the N columns of a row
