"""The tcgen05 / TMEM tensor-core GEMM (g4_gemm_bf16, the prefill's contraction engine)
against an fp32 PyTorch matmul of the same bf16 operands.

Shapes cover a single tile, the prefill's projection shapes (K = 2816, 2112, 704 k-blocks;
N = 2816, 4224 with a partial 256-wide tile), M = 1 (the LM head of the last prompt
position), ragged M / N / K tails that the TMA zero-fills, and row strides wider than K.
Tolerances: fp32 output within 1e-5 of the output's max magnitude (accumulation order
only); bf16 output within one bf16 rounding (2^-8 relative) of the fp32 reference.
"""
import pytest
import torch

from gemma4_b200 import _native as N

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

CASES = [  # M, N, K, lda_pad, c_f32
    (128, 256, 64, 0, 1),
    (300, 2816, 2816, 0, 1),
    (1, 4096, 2816, 0, 0),
    (257, 200, 704, 16, 1),
    (512, 4224, 2112, 0, 0),
    (77, 72, 1000, 8, 1),
    (1024, 1024, 4096, 0, 0),
]


@pytest.mark.parametrize("M,Nn,K,pad,f32", CASES)
def test_gemm_matches_fp32_matmul(M, Nn, K, pad, f32):
    g = torch.Generator(device=DEV).manual_seed(M * 131 + Nn + K)
    lda, ldb = K + pad, K + 2 * pad
    A = torch.randn(M, lda, device=DEV, generator=g).to(torch.bfloat16)
    B = torch.randn(Nn, ldb, device=DEV, generator=g).to(torch.bfloat16)
    C = torch.full((M, Nn), float("nan"), device=DEV, dtype=torch.float32 if f32 else torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    N.check(N.lib().g4_gemm_bf16(N.ptr(A), lda, N.ptr(B), ldb, N.ptr(C), Nn, M, Nn, K, f32, N.ptr(status),
                                 N.stream_handle()), "g4_gemm_bf16")
    torch.cuda.synchronize()
    assert int(status) == 0
    ref = A[:, :K].float() @ B[:, :K].float().T
    got = C.float()
    assert not torch.isnan(got).any()
    err = float((got - ref).abs().max()) / float(ref.abs().max())
    assert err <= (1e-5 if f32 else 2.0 ** -8), err
