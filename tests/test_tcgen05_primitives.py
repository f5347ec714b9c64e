"""Known-answer checks of the sm_100a tensor-core building blocks the chunked
prefill is made of (tcgen05.mma operand layouts, TMEM operands, TMA tiles):
one CTA computes D = A @ B^T per layout mode and is compared with float64."""
import ctypes

import pytest
import torch

from fastaf_kernel_b200.build import SELFTEST_LIB_PATH

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _lib():
    lib = ctypes.CDLL(SELFTEST_LIB_PATH)
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    lib.gdn_selftest_umma.argtypes = [i32, vp, vp, vp, i32, i32, i32, i32, i32, vp, vp, vp]
    lib.gdn_selftest_umma.restype = i32
    return lib


def _run(mode, N, K, A=None, B=None, X=None, h=1):
    lib = _lib()
    D = torch.full((128, N), float("nan"), device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    T, H = (X.shape[0], X.shape[1]) if X is not None else (0, 0)
    ptr = lambda t: None if t is None else t.data_ptr()
    rc = lib.gdn_selftest_umma(mode, ptr(A), ptr(B), ptr(X), T, H, h, N, K, D.data_ptr(),
                               status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0, "an mbarrier wait timed out"
    return D.cpu().double()


def _rand(shape, g):
    return torch.randn(shape, generator=g).to(torch.bfloat16)


@pytest.mark.parametrize("mode", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("N,K", [(64, 64), (64, 128), (128, 64), (128, 128)])
def test_smem_and_tmem_operands(mode, N, K):
    g = torch.Generator().manual_seed(mode * 1000 + N + K)
    A, B = _rand((128, K), g), _rand((N, K), g)
    D = _run(mode, N, K, A.to(DEV), B.to(DEV))
    ref = A.double() @ B.double().T
    assert torch.allclose(D, ref, rtol=1e-5, atol=1e-4), (D - ref).abs().max()


def _x(g):
    return _rand((128, 3, 128), g)


def test_tma_kmajor_a():
    g = torch.Generator().manual_seed(5)
    X, B = _x(g), _rand((64, 128), g)
    D = _run(5, 64, 128, B=B.to(DEV), X=X.to(DEV), h=1)
    ref = X[:, 1, :].double() @ B.double().T
    assert torch.allclose(D, ref, rtol=1e-5, atol=1e-4), (D - ref).abs().max()


def test_tma_mnmajor_a():
    g = torch.Generator().manual_seed(6)
    X, B = _x(g), _rand((64, 64), g)
    D = _run(6, 64, 64, B=B.to(DEV), X=X.to(DEV), h=2)
    A = X[64:, 2, :].double().T                      # A[d][t] = X[64+t][h][d]
    ref = A @ B.double().T
    assert torch.allclose(D, ref, rtol=1e-5, atol=1e-4), (D - ref).abs().max()


def test_tma_mnmajor_b_with_tmem_a():
    g = torch.Generator().manual_seed(7)
    X, A = _x(g), _rand((128, 64), g)
    D = _run(7, 128, 64, A=A.to(DEV), X=X.to(DEV), h=0)
    Bm = X[64:, 0, :].double().T                     # B[d][t] = X[64+t][h][d]
    ref = A.double() @ Bm.T
    assert torch.allclose(D, ref, rtol=1e-5, atol=1e-4), (D - ref).abs().max()


def _roles_lib():
    lib = ctypes.CDLL(SELFTEST_LIB_PATH)
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    lib.gdn_selftest_roles.argtypes = [vp, vp, i32, i32, i32, i32, vp, vp, vp]
    lib.gdn_selftest_roles.restype = i32
    return lib


@pytest.mark.parametrize("N,K,a_col,d_col", [(64, 128, 192, 448), (128, 64, 0, 256),
                                             (64, 64, 384, 256), (128, 128, 320, 128)])
def test_warp_roles_full_tmem(N, K, a_col, d_col):
    """All 512 TMEM columns allocated by warp 0, MMAs issued by warp 0, the
    accumulator at a nonzero column, 32-column TMEM stores/loads by warps 4-7."""
    g = torch.Generator().manual_seed(N * 7 + K + a_col + d_col)
    A, B = _rand((128, K), g), _rand((N, K), g)
    D = torch.full((128, N), float("nan"), device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    Ad, Bd = A.to(DEV), B.to(DEV)   # keep the device copies alive across the launch
    rc = _roles_lib().gdn_selftest_roles(Ad.data_ptr(), Bd.data_ptr(), N, K, a_col, d_col,
                                         D.data_ptr(), status.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = A.double() @ B.double().T
    assert torch.allclose(D.cpu().double(), ref, rtol=1e-5, atol=1e-4)
