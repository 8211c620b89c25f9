"""tcgen05 GEMM through the C ABI against a plain PyTorch fp32 reference."""
import pytest
import torch

from specgrove_b200 import _lib
from specgrove_b200._lib import check, ptr, stream_ptr

pytestmark = pytest.mark.gpu


def gemm(a, b, out, epilogue, aux=None):
    st = _lib.load().sg_gemm_bf16(ptr(a), a.stride(0), ptr(b), b.stride(0), ptr(out), out.stride(0),
                                  a.shape[0], b.shape[0], a.shape[1], epilogue, ptr(aux),
                                  aux.stride(0) if aux is not None else 0, None, stream_ptr())
    check(st, "sg_gemm_bf16")


def ref_mm(a, b):
    return a.float() @ b.float().t()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (2048, 6144, 4096), (100, 512, 256), (257, 96, 192),
                                   (1, 4096, 4096), (512, 151936 // 4, 512)])
def test_store_f32(cuda_lib, M, N, K):
    torch.manual_seed(M + N + K)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    out = torch.full((M, N), float("nan"), device="cuda")
    gemm(a, b, out, _lib.SG_EPI_STORE_F32)
    ref = ref_mm(a, b)
    # fp32 accumulation in a different order: |err| << 1e-3 * sqrt(K)
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=2e-3 * (K / 64) ** 0.5)


@pytest.mark.parametrize("M,N,K", [(2048, 4096, 4096), (77, 1024, 128)])
def test_store_bf16(cuda_lib, M, N, K):
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16) * 0.1
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.1
    out = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
    gemm(a, b, out, _lib.SG_EPI_STORE_BF16)
    ref = ref_mm(a, b)
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2)


def test_residual_epilogue(cuda_lib):
    M, N, K = 300, 4096, 1024
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16) * 0.05
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    x = torch.randn(M, N, device="cuda")
    x0 = x.clone()
    xb = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
    gemm(a, b, x, _lib.SG_EPI_RESIDUAL, aux=xb)
    ref = x0 + ref_mm(a, b)
    torch.testing.assert_close(x, ref, rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(xb.float(), ref, rtol=8e-3, atol=1e-3)


def test_swiglu_epilogue(cuda_lib):
    M, I, K = 200, 512, 256
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16) * 0.1
    gate = torch.randn(I, K, device="cuda", dtype=torch.bfloat16) * 0.1
    up = torch.randn(I, K, device="cuda", dtype=torch.bfloat16) * 0.1
    w = torch.stack([gate.view(I // 128, 128, K), up.view(I // 128, 128, K)], dim=1).reshape(2 * I, K).contiguous()
    out = torch.empty((M, I), device="cuda", dtype=torch.bfloat16)
    gemm(a, w, out, _lib.SG_EPI_SWIGLU)
    g, u = ref_mm(a, gate), ref_mm(a, up)
    ref = torch.nn.functional.silu(g) * u
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-3)


def test_zero_rows_is_noop(cuda_lib):
    a = torch.empty((0, 64), device="cuda", dtype=torch.bfloat16)
    b = torch.randn(32, 64, device="cuda", dtype=torch.bfloat16)
    out = torch.empty((0, 32), device="cuda")
    assert _lib.load().sg_gemm_bf16(ptr(b), 64, ptr(b), 64, ptr(b), 32, 0, 32, 64, 1, None, 0, None,
                                    stream_ptr()) == 0
    with pytest.raises(_lib.SpecgroveError):
        bad = torch.randn(4, 100, device="cuda", dtype=torch.bfloat16)
        gemm(bad, torch.randn(32, 100, device="cuda", dtype=torch.bfloat16), torch.empty(4, 32, device="cuda"),
             _lib.SG_EPI_STORE_F32)
