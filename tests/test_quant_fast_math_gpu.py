"""The opt-in quantisation rule of the reference as its Makefile builds it (-ffast-math), on the device.

With p2cu_set_quant_fast_math(1) every int8 path quantises as the reference's -ffast-math build does: scale =
amax * (1/127), the reciprocal 127 / amax, the K % 16 tail multiplied by it. The oracle restates that rule
(orc_quant_row_fast_math, pinned bit for bit against that build of the reference in tests/test_ref_neon.py); here the
device's quantiser, the fused producers' quantisation and the int8 GEMM entry points are held to it bit for bit, and
p2cu_sgemm_fvb end to end to the reference's -ffast-math build itself where that build is present. Each test restores
the default rule.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture
def fast_math(pkg):
    prev = pkg.set_quant_fast_math(True)
    try:
        yield
    finally:
        pkg.set_quant_fast_math(prev)


def _bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def _device_quant(pkg, torch, cuda, A):
    M, K = A.shape
    A_d = torch.from_numpy(np.ascontiguousarray(A, np.float32)).to(cuda)
    q_d = torch.empty((M, K), dtype=torch.int8, device=cuda)
    s_d = torch.empty(M, dtype=torch.float32, device=cuda)
    pkg.quant_rows(A_d.data_ptr(), M, K, K, q_d.data_ptr(), s_d.data_ptr())
    pkg.check_device()
    return q_d.cpu().numpy(), s_d.cpu().numpy()


@pytest.mark.parametrize("K", [20, 1000, 1002, 1024, 4100])
def test_quantiser_fast_math_bitwise(pkg, orc, synth, cuda, fast_math, K):
    """The register path (K % 4 == 0, K <= 4096) and the strided one, the edge rows (a value on each side of every
    rounding the two rules treat differently, a row whose reciprocal overflows, zeros, ties)."""
    import torch
    A = np.concatenate([synth.quantiser_edge_rows(K, seed=K), synth.activations(40, K, seed=K + 1)])
    q, s = _device_quant(pkg, torch, cuda, A)
    q_o, s_o = orc.quant_rows(A, fast_math=True)
    assert _bits_equal(s, s_o)
    assert np.array_equal(q, q_o)
    q_i, s_i = orc.quant_rows(A)
    assert not _bits_equal(s, s_i)   # the rule in force is not the IEEE one


def test_rule_is_restored_and_default_is_ieee(pkg, orc, synth, cuda):
    import torch
    assert not bool(pkg.lib().p2cu_quant_fast_math())
    A = synth.activations(64, 1024, seed=9)
    q, s = _device_quant(pkg, torch, cuda, A)
    q_o, s_o = orc.quant_rows(A)
    assert _bits_equal(s, s_o) and np.array_equal(q, q_o)


def test_fused_producers_quantise_by_the_rule(pkg, orc, cuda, fast_math):
    """LayerNorm + quantisation and SiLU + quantisation of the encoder: the quantised rows equal the rule applied to
    the same kernels' fp32 rows."""
    import torch
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((96, 1024)) * 2).astype(np.float32)
    g = (1 + 0.02 * rng.standard_normal(1024)).astype(np.float32)
    b = (0.02 * rng.standard_normal(1024)).astype(np.float32)
    xd, gd, bd = (torch.from_numpy(a).to(cuda) for a in (x, g, b))
    y = torch.empty((96, 1024), dtype=torch.float32, device=cuda)
    q = torch.empty((96, 1024), dtype=torch.int8, device=cuda)
    s = torch.empty(96, dtype=torch.float32, device=cuda)
    L = pkg.lib()
    pkg.check(L.p2cu_layer_norm_rows(xd.data_ptr(), gd.data_ptr(), bd.data_ptr(), y.data_ptr(), 96, 1024, None))
    pkg.check(L.p2cu_layer_norm_quant_rows(xd.data_ptr(), gd.data_ptr(), bd.data_ptr(), q.data_ptr(), s.data_ptr(),
                                           96, 1024, None))
    pkg.check_device()
    q_o, s_o = orc.quant_rows(y.cpu().numpy(), fast_math=True)
    assert _bits_equal(s.cpu().numpy(), s_o) and np.array_equal(q.cpu().numpy(), q_o)

    h = (rng.standard_normal((64, 4096)) * 3).astype(np.float32)
    hd = torch.from_numpy(h).to(cuda)
    hs = hd.clone()
    pkg.check(L.p2cu_swish(hs.data_ptr(), hs.numel(), None))
    q2 = torch.empty((64, 4096), dtype=torch.int8, device=cuda)
    s2 = torch.empty(64, dtype=torch.float32, device=cuda)
    pkg.check(L.p2cu_swish_quant_rows(hd.data_ptr(), q2.data_ptr(), s2.data_ptr(), 64, 4096, None))
    pkg.check_device()
    q_o, s_o = orc.quant_rows(hs.cpu().numpy(), fast_math=True)
    assert _bits_equal(s2.cpu().numpy(), s_o) and np.array_equal(q2.cpu().numpy(), q_o)


@pytest.mark.parametrize("mode", ["int8w", "int8"])
@pytest.mark.parametrize("M,K,N,alpha,beta", [(375, 1024, 1024, 1.0, 0.0), (38, 4096, 1024, 0.5, 1.0),
                                              (33, 1000, 256, 1.0, 1.0)])
def test_sgemm_fvb_matches_reference_fast_math_build(pkg, orc, synth, cuda, fast_math, mode, M, K, N, alpha, beta):
    """p2cu_sgemm_fvb from fp32 A against the reference's own p2_sgemm_fvb as its Makefile builds it: bit for bit,
    quantisation included, on rows that include the quantiser's edge rows."""
    import torch
    if not orc.ref_neon_available():
        pytest.skip("the reference's AArch64 build is not present")
    from phonon2_b200.device import DeviceFiveValue
    edge = synth.quantiser_edge_rows(K, seed=K)[: M // 2]
    A = np.concatenate([edge, synth.activations(M - edge.shape[0], K, seed=M)]).astype(np.float32)
    w = synth.five_value(K, N, seed=N + K)
    C0 = np.random.default_rng(M).standard_normal((M, N)).astype(np.float32)
    want = orc.neon_sgemm_fvb(orc.ref_neon(mode, fast_math=True), A, w, C0.copy(), alpha=alpha, beta=beta)
    B = DeviceFiveValue(w, cuda, vindex=(mode == "int8w"))
    pm = pkg.MODES[mode]
    A_d = torch.from_numpy(A).to(cuda)
    C_d = torch.from_numpy(C0.copy()).to(cuda)
    nws = max(pkg.workspace_bytes(M, N, K, pm), 16)
    ws = torch.empty(nws, dtype=torch.uint8, device=cuda)
    pkg.sgemm_fvb(M, N, K, alpha, A_d.data_ptr(), K, B.struct, pm, beta, C_d.data_ptr(), N, ws.data_ptr(), nws)
    pkg.check_device()
    got = C_d.cpu().numpy()
    assert _bits_equal(got, want), float(np.abs(got - want).max())
