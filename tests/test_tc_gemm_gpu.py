"""p2cu_sgemm_tf32x3: the fp32-accurate tensor-core GEMM behind the encoder's attention products, against float64
numpy. Split-tf32 products keep a relative error of about 2^-21 per product, so the tolerance is written relative to
the sum of |a * b| over K (the scale of the rounding a float32 dot product itself incurs)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-6


@pytest.mark.parametrize("transB", [1, 0])
@pytest.mark.parametrize("M,N,K", [(128, 128, 32), (375, 375, 128), (200, 749, 128), (375, 128, 375), (7, 5, 3),
                                   (130, 129, 33)])
def test_sgemm_tf32x3_matches_float64(pkg, cuda, transB, M, N, K):
    import torch
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = (rng.standard_normal((N, K)) if transB else rng.standard_normal((K, N))).astype(np.float32)
    Ad, Bd = torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda)
    Cd = torch.full((M, N), np.nan, dtype=torch.float32, device=cuda)
    pkg.check(pkg.lib().p2cu_sgemm_tf32x3(transB, M, N, K, Ad.data_ptr(), K, Bd.data_ptr(), B.shape[1],
                                          Cd.data_ptr(), N, None))
    pkg.check_device()
    Bk = B.T if transB else B
    ref = A.astype(np.float64) @ Bk.astype(np.float64)
    scale = np.abs(A).astype(np.float64) @ np.abs(Bk).astype(np.float64)
    err = np.abs(Cd.cpu().numpy() - ref) / scale
    assert np.isfinite(Cd.cpu().numpy()).all()
    assert err.max() <= TOL, err.max()


@pytest.mark.parametrize("M,N,K,pad", [(375, 128, 375, 1), (200, 130, 100, 4), (129, 257, 48, 0), (64, 64, 17, 3)])
def test_sgemm_tf32x3_padded_rows(pkg, cuda, M, N, K, pad):
    """Row strides rounded up to 16 bytes (as the encoder's score and V^T rows are), K not a multiple of the 16-deep
    K step: the branch-free path for whole steps and the bounds-checked one for the last, partial step."""
    import torch
    rng = np.random.default_rng(M + N + K)
    ld = (K + pad + 3) & ~3
    A = rng.standard_normal((M, ld)).astype(np.float32)
    B = rng.standard_normal((N, ld)).astype(np.float32)
    A[:, K:] = np.nan   # past K: must not be read into the products
    B[:, K:] = np.nan
    Ad, Bd = torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda)
    Cd = torch.full((M, N), np.nan, dtype=torch.float32, device=cuda)
    pkg.check(pkg.lib().p2cu_sgemm_tf32x3(1, M, N, K, Ad.data_ptr(), ld, Bd.data_ptr(), ld, Cd.data_ptr(), N, None))
    pkg.check_device()
    a, b = A[:, :K].astype(np.float64), B[:, :K].astype(np.float64)
    ref = a @ b.T
    scale = np.abs(a) @ np.abs(b).T
    got = Cd.cpu().numpy()
    assert np.isfinite(got).all()
    assert (np.abs(got - ref) / scale).max() <= TOL
