"""The tcgen05 prefill GEMM (mq_gemm_bf16, through the C ABI) against a torch
fp32 reference of the same operation on the same bf16 inputs.

Tolerance: fp32 accumulation of bf16 products in both; differences come from
summation order only, so a relative error of 1e-4 of the output scale is
required (bf16 output: 1 ulp, 2^-8 relative)."""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from megaqwen_b200.build import LIB
    lib = ctypes.CDLL(str(LIB))
    lib.mq_gemm_bf16.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                 ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_void_p, ctypes.c_void_p]
    lib.mq_gemm_bf16.restype = ctypes.c_int
    return lib


def _gemm(lib, A, B, C, epi, B2=None):
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    M, K = A.shape
    N = B.shape[0]
    rc = lib.mq_gemm_bf16(A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0),
                          B2.data_ptr() if B2 is not None else None, C.data_ptr(), C.stride(0), M, N, K, epi,
                          err.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (200, 256, 1024), (2048, 1024, 3072), (16, 2048, 1024)])
def test_gemm_store_f32(M, N, K):
    lib = _lib()
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    B = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    C = torch.full((M, N), float("nan"), device="cuda")
    _gemm(lib, A, B, C, 0)
    ref = A.float() @ B.float().T
    scale = ref.abs().max().item()
    assert (C - ref).abs().max().item() <= 1e-4 * scale + 1e-6


def test_gemm_residual_add_and_gate_up():
    lib = _lib()
    g = torch.Generator(device="cuda").manual_seed(7)
    M, N, K = 300, 384, 1024
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    B = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    B2 = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    R = torch.randn(M, N, device="cuda", generator=g)
    C = R.clone()
    _gemm(lib, A, B, C, 1)
    ref = R + A.float() @ B.float().T
    assert (C - ref).abs().max().item() <= 1e-4 * ref.abs().max().item()
    act = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    _gemm(lib, A, B, act, 2, B2=B2)
    gte = A.float() @ B.float().T
    up = A.float() @ B2.float().T
    ref = torch.nn.functional.silu(gte) * up
    assert (act.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    _gemm(lib, A, B, out, 3)
    assert (out.float() - gte).abs().max().item() <= 1e-2 * gte.abs().max().item()


@pytest.mark.parametrize("M,N,K", [(9856, 1024, 2048), (16384, 1024, 3072)])
def test_pair_gemm_residual_add(M, N, K):
    """Shapes with enough 256 x 256 pair tiles for the CTA-pair (cta_group::2)
    GEMM: C += A . B^T against torch, ragged M included."""
    lib = _lib()
    g = torch.Generator(device="cuda").manual_seed(M + K)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    B = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    R = torch.randn(M, N, device="cuda", generator=g)
    C = R.clone()
    _gemm(lib, A, B, C, 1)
    ref = R + A.float() @ B.float().T
    assert (C - ref).abs().max().item() <= 1e-4 * ref.abs().max().item()


@pytest.mark.parametrize("M", [2048, 2000, 16384])
def test_gate_up_large(M):
    """gate/up + SiLU*mul at the prefill shapes (B = 1 and 8 x 2048 prompts,
    ragged M) against torch."""
    lib = _lib()
    N, K = 3072, 1024
    g = torch.Generator(device="cuda").manual_seed(M)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    B = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    B2 = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    act = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
    _gemm(lib, A, B, act, 2, B2=B2)
    ref = torch.nn.functional.silu(A.float() @ B.float().T) * (A.float() @ B2.float().T)
    assert (act.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()
