"""p2cu_sgemm_fvb_noalloc: the five-value GEMM for callers that cannot allocate device memory.

A real-time audio thread cannot risk cudaMalloc (it may block and synchronise the whole device), and a host
application may hand this library a fixed memory budget. For them the GEMM's scratch (the int8 activations and, for K > 1024, the per-block partial results) lives in a
fixed device array inside the library. These tests call the entry point through the C ABI and compare it with the
workspace-taking entry point, p2cu_sgemm_fvb, bit for bit (the tolerance of every int8 GEMM test here), on two calls in
a row that leave different contents in the shared array. The file is named to be collected last.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _workspace_call(pkg, torch, dev, M, N, K, alpha, A_d, B, mode, beta, C0):
    C_d = torch.from_numpy(C0.copy()).to(dev)
    nws = max(pkg.workspace_bytes(M, N, K, mode), 16)
    ws = torch.empty(nws, dtype=torch.uint8, device=dev)
    pkg.sgemm_fvb(M, N, K, alpha, A_d.data_ptr(), K, B.struct, mode, beta, C_d.data_ptr(), N, ws.data_ptr(), nws)
    pkg.check_device()
    return C_d.cpu().numpy()


def _noalloc_call(pkg, torch, dev, M, N, K, alpha, A_d, B, mode, beta, C0):
    C_d = torch.from_numpy(C0.copy()).to(dev)
    pkg.sgemm_fvb_noalloc(M, N, K, alpha, A_d.data_ptr(), K, B.struct, mode, beta, C_d.data_ptr(), N)
    pkg.check_device()
    return C_d.cpu().numpy()


def test_noalloc_matches_workspace_entry_on_two_calls_in_a_row(pkg, synth, cuda):
    import torch
    from phonon2_b200.device import DeviceFiveValue
    cases = [(375, 4096, 1024, 0.5, 1.0, False),   # K > 1024: the per-block partials go through the fixed array
             (375, 1024, 4096, 1.0, 0.0, False),   # then a call that leaves other contents behind
             (200, 3072, 384, 1.0, 1.0, False),    # K > 1024 again over the stale bytes, other M and N
             (130, 2048, 512, 1.0, 0.0, True)]     # the tensor-memory kernel (value-index plane), K > 1024
    for i, (M, K, N, alpha, beta, vindex) in enumerate(cases):
        w = synth.five_value(K, N, seed=50 + i)
        B = DeviceFiveValue(w, cuda, vindex=vindex)
        A_d = torch.from_numpy(synth.activations(M, K, seed=60 + i)).to(cuda)
        C0 = np.random.default_rng(70 + i).standard_normal((M, N)).astype(np.float32)
        want = _workspace_call(pkg, torch, cuda, M, N, K, alpha, A_d, B, pkg.INT8W, beta, C0)
        got = _noalloc_call(pkg, torch, cuda, M, N, K, alpha, A_d, B, pkg.INT8W, beta, C0)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"call {i}: outputs differ"


def test_noalloc_refuses_shapes_beyond_its_array(pkg, synth, cuda):
    import torch
    from phonon2_b200.device import DeviceFiveValue
    M, K, N = 2048, 4096, 1024   # 8 MiB of int8 rows + 32 MiB of partials > the 16 MiB array
    assert pkg.workspace_bytes(M, N, K, pkg.INT8W) > pkg.NOALLOC_SCRATCH_BYTES
    B = DeviceFiveValue(synth.five_value(K, N, seed=1), cuda)
    A_d = torch.zeros((M, K), dtype=torch.float32, device=cuda)
    C_d = torch.zeros((M, N), dtype=torch.float32, device=cuda)
    with pytest.raises(pkg.Error) as e:
        pkg.sgemm_fvb_noalloc(M, N, K, 1.0, A_d.data_ptr(), K, B.struct, pkg.INT8W, 0.0, C_d.data_ptr(), N)
    assert e.value.code == pkg.P2CU_EINVAL and "fixed array" in str(e.value)
    pkg.check_device()


def test_noalloc_allocates_nothing(pkg, synth, cuda):
    """The property the entry point exists for: after a first call on the device, further calls - the split-K path,
    the tensor-memory kernel and the SIMT kernel (N % 128 != 0) - leave the device's free memory unchanged."""
    import torch
    from phonon2_b200.device import DeviceFiveValue
    cases = []
    for i, (M, K, N, vindex) in enumerate([(300, 4096, 1024, False), (375, 1024, 2048, True), (64, 1024, 144, False)]):
        B = DeviceFiveValue(synth.five_value(K, N, seed=80 + i), cuda, vindex=vindex)
        A_d = torch.from_numpy(synth.activations(M, K, seed=90 + i)).to(cuda)
        C_d = torch.zeros((M, N), dtype=torch.float32, device=cuda)
        cases.append((M, K, N, B, A_d, C_d))
    for (M, K, N, B, A_d, C_d) in cases:   # first calls: the array's address is looked up, kernels get configured
        pkg.sgemm_fvb_noalloc(M, N, K, 1.0, A_d.data_ptr(), K, B.struct, pkg.INT8W, 0.0, C_d.data_ptr(), N)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        for (M, K, N, B, A_d, C_d) in cases:
            pkg.sgemm_fvb_noalloc(M, N, K, 1.0, A_d.data_ptr(), K, B.struct, pkg.INT8W, 0.0, C_d.data_ptr(), N)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    pkg.check_device()
    assert free_after == free_before, (free_before, free_after)
