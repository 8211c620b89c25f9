"""Stream-K wave tail of the tcgen05 GEMM (sg_gemm_bf16_ws) against a plain
PyTorch fp32 reference and against the unsplit kernel.  Shapes are chosen so
that the tiles leave a partial last wave (the split path) or fill no wave at
all; repeated calls check that the workspace flags reset themselves."""
import pytest
import torch

from specgrove_b200 import _lib
from specgrove_b200._lib import check, ptr, stream_ptr

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def workspace(cuda_lib):
    lib = _lib.load()
    nbytes = lib.sg_gemm_split_workspace_bytes()
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    check(lib.sg_gemm_split_workspace_init(ptr(ws), nbytes, stream_ptr()), "split workspace init")
    return ws


def gemm(a, b, out, epilogue, ws=None, aux=None):
    lib = _lib.load()
    if ws is None:
        st = lib.sg_gemm_bf16(ptr(a), a.stride(0), ptr(b), b.stride(0), ptr(out), out.stride(0), a.shape[0],
                              b.shape[0], a.shape[1], epilogue, ptr(aux), aux.stride(0) if aux is not None else 0,
                              None, stream_ptr())
    else:
        st = lib.sg_gemm_bf16_ws(ptr(a), a.stride(0), ptr(b), b.stride(0), ptr(out), out.stride(0), a.shape[0],
                                 b.shape[0], a.shape[1], epilogue, ptr(aux),
                                 aux.stride(0) if aux is not None else 0, None, ptr(ws), ws.numel(), stream_ptr())
    check(st, "gemm")


# (M, N, K): a 1.73-wave O projection, a 2.6-wave QKV, a long-K down
# projection, fewer tiles than SMs (config-3 rows), a single tile, ragged M.
SHAPES = [(2048, 4096, 4096), (2048, 6144, 4096), (2048, 4096, 12288), (512, 6144, 2560), (128, 256, 1024),
          (300, 2560, 4096)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_split_store_f32(workspace, M, N, K):
    torch.manual_seed(M * 7 + N + K)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    ref = a.float() @ b.float().t()
    whole = torch.empty((M, N), device="cuda")
    gemm(a, b, whole, _lib.SG_EPI_STORE_F32)
    for _ in range(3):  # flags must come back to zero after every call
        out = torch.full((M, N), float("nan"), device="cuda")
        gemm(a, b, out, _lib.SG_EPI_STORE_F32, ws=workspace)
        torch.testing.assert_close(out, ref, rtol=1e-4, atol=2e-3 * (K / 64) ** 0.5)
        # same products, partial sums added in another (fixed) order
        torch.testing.assert_close(out, whole, rtol=1e-5, atol=1e-3 * (K / 64) ** 0.5)
    again = torch.empty((M, N), device="cuda")
    gemm(a, b, again, _lib.SG_EPI_STORE_F32, ws=workspace)
    assert torch.equal(again, out), "split result is not reproducible"


def test_split_residual_and_swiglu(workspace):
    M, N, K = 2048, 4096, 4096
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16) * 0.05
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    x = torch.randn(M, N, device="cuda")
    ref = x + a.float() @ b.float().t()
    xb = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
    gemm(a, b, x, _lib.SG_EPI_RESIDUAL, ws=workspace, aux=xb)
    torch.testing.assert_close(x, ref, rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(xb.float(), ref, rtol=8e-3, atol=1e-3)
    I = 1408  # 2 * I / 256 = 11 n-tiles x 4 m-tiles = 44 tiles: fewer than the SMs
    w = torch.randn(2 * I, K, device="cuda", dtype=torch.bfloat16) * 0.05
    h = torch.empty((512, I), device="cuda", dtype=torch.bfloat16)
    gemm(a[:512], w, h, _lib.SG_EPI_SWIGLU, ws=workspace)
    acc = a[:512].float() @ w.float().t()
    blocks = acc.view(512, -1, 2, 128)
    gate, up = blocks[:, :, 0].reshape(512, I), blocks[:, :, 1].reshape(512, I)
    torch.testing.assert_close(h.float(), torch.nn.functional.silu(gate) * up, rtol=2e-2, atol=2e-2)


def test_small_workspace_falls_back(workspace):
    """A workspace below the required size runs the unsplit kernel."""
    M, N, K = 2048, 4096, 1024
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    out, whole = torch.empty((M, N), device="cuda"), torch.empty((M, N), device="cuda")
    gemm(a, b, whole, _lib.SG_EPI_STORE_F32)
    gemm(a, b, out, _lib.SG_EPI_STORE_F32, ws=workspace[:1024])
    assert torch.equal(out, whole)
