"""The int8w GEMM with the weights in tensor memory (fv_gemm_t.cu), through the device C ABI: the value-index plane
(p2cu_fv_pack_vindex) against its numpy restatement, and every output bit for bit against the oracle, which runs the
reference's int8w arithmetic (csrc/blas.c:1222-1240, 1316-1366) in the reference's order.

A weight that carries `vindex` takes this kernel for int8w GEMMs with N % 128 == 0, K % 16 == 0 and M <= 1024.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# (M, K, N, alpha, beta, ldc_extra): the block's shapes at T = 375 (the positional projection at 2T - 1 rows), the
# short utterance (T = 38), one-row and ragged row counts around the tile sizes, K not a multiple of 128 or 1024,
# K > 1024 (per-block slices folded in order), beta outside {0, 1}, and C with a row stride above N.
SHAPES = [
    (375, 1024, 4096, 1.0, 0.0, 0),
    (375, 4096, 1024, 0.5, 1.0, 0),
    (375, 1024, 3072, 1.0, 0.0, 0),
    (749, 1024, 1024, 1.0, 0.0, 0),
    (375, 1024, 1024, 1.0, 1.0, 0),
    (375, 1024, 2048, 1.0, 0.0, 0),
    (38, 1024, 4096, 1.0, 0.0, 0),
    (38, 4096, 1024, 0.5, 1.0, 0),
    (1, 1024, 128, 1.0, 0.0, 0),
    (16, 1024, 256, 1.0, 0.0, 0),
    (17, 512, 256, 1.0, 0.0, 0),
    (127, 1024, 128, 1.0, 1.0, 0),
    (129, 2048, 256, 1.0, 1.0, 0),
    (200, 1040, 384, 1.0, 0.0, 0),
    (256, 96, 128, 1.0, 0.0, 0),
    (1000, 1024, 512, 2.0, 0.0, 0),
    (1024, 3000, 256, 1.0, 1.0, 0),
    (64, 4096, 128, 0.5, 0.5, 0),
    (100, 1024, 384, 1.0, 1.0, 40),
]


def _weight(pkg, torch, cuda, w):
    from phonon2_b200.device import DeviceFiveValue
    return DeviceFiveValue(w, cuda, vindex=True)


def _run(pkg, torch, cuda, B, A, alpha, beta, C0, ldc):
    M, K = A.shape
    N = B.N
    A_d = torch.from_numpy(A).to(cuda)
    Cfull = np.zeros((M, ldc), np.float32)
    Cfull[:, :N] = C0
    C_d = torch.from_numpy(Cfull).to(cuda)
    nws = max(pkg.workspace_bytes(M, N, K, pkg.INT8W), 16)
    ws = torch.empty(nws, dtype=torch.uint8, device=cuda)
    pkg.sgemm_fvb(M, N, K, alpha, A_d.data_ptr(), K, B.struct, pkg.INT8W, beta, C_d.data_ptr(), ldc, ws.data_ptr(),
                  nws)
    pkg.check_device()
    out = C_d.cpu().numpy()
    assert np.array_equal(out[:, N:], Cfull[:, N:]), "columns past N were written"
    return np.ascontiguousarray(out[:, :N])


def _report(got, want):
    bad = np.argwhere(got.view(np.uint32) != want.view(np.uint32))
    if len(bad) == 0:
        return "equal"
    i = tuple(bad[0])
    return f"{len(bad)} of {got.size} differ; first {i}: got {got[i]!r} want {want[i]!r}"


@pytest.mark.parametrize("K,N", [(1024, 4096), (4096, 1024), (1040, 384), (100, 128), (32, 16)])
def test_vindex_layout(pkg, orc, synth, cuda, K, N):
    import torch
    w = synth.five_value(K, N, seed=K + N)
    w["signs"] = w["signs"].copy()
    w["signs"][::5, ::3] |= 0x03   # some 2-bit codes 3 (unused by the converter; the reference reads them as sign +2)
    B = _weight(pkg, torch, cuda, w)
    torch.cuda.synchronize()
    got = B.vindex.cpu().numpy().view(np.uint32).reshape(-1, N, 4)
    assert np.array_equal(got, orc.vindex(w))


@pytest.mark.parametrize("M,K,N,alpha,beta,ldc_extra", SHAPES)
def test_tgemm_int8w_bitwise(pkg, orc, synth, cuda, M, K, N, alpha, beta, ldc_extra):
    import torch
    w = synth.five_value(K, N, seed=M + K + N + 11)
    A = synth.activations(M, K, seed=M * 7 + 3)
    C0 = np.random.default_rng(9).standard_normal((M, N)).astype(np.float32)
    B = _weight(pkg, torch, cuda, w)
    got = _run(pkg, torch, cuda, B, A, alpha, beta, C0, N + ldc_extra)
    want = orc.sgemm_i8(A, "int8w", C0.copy(), w=w, alpha=alpha, beta=beta)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), _report(got, want)


def test_tgemm_edge_weights_and_rows(pkg, orc, synth, cuda):
    """Columns whose clo is 0 and 127 (lo = 0 and lo = hi), zero columns, 2-bit codes 3, and the quantiser's edge
    rows."""
    import torch
    M, K, N = 40, 1024, 256
    w = synth.five_value(K, N, seed=21)
    w["lo"] = w["lo"].copy()
    w["lo"][:16] = 0.0
    w["lo"][16:32] = w["hi"][16:32]
    w["signs"] = w["signs"].copy()
    w["signs"][:, 8:12] = 0x55   # code 1 everywhere: zero weights in columns 32-47
    w["signs"][::7, 20:30] |= 0x03   # code 3 in some rows of columns 80-119
    A = np.concatenate([synth.quantiser_edge_rows(K, seed=K), synth.activations(M - 8, K, seed=6)])
    B = _weight(pkg, torch, cuda, w)
    got = _run(pkg, torch, cuda, B, A, 1.0, 0.0, np.zeros((M, N), np.float32), N)
    want = orc.sgemm_i8(A, "int8w", np.zeros((M, N), np.float32), w=w)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), _report(got, want)


def test_tgemm_equals_planes_and_codes(pkg, orc, synth, cuda):
    """The same product through the three int8w operand forms (planes, code cache, device layout) is bit-identical,
    and a weight carrying both the code cache and the device layout takes the device layout at few rows."""
    import torch
    from phonon2_b200.device import DeviceFiveValue
    M, K, N = 375, 1024, 2048
    w = synth.five_value(K, N, seed=31)
    A = synth.activations(M, K, seed=32)
    B = DeviceFiveValue(w, cuda, codes=True, vindex=True)
    A_d = torch.from_numpy(A).to(cuda)
    nws = pkg.workspace_bytes(M, N, K, pkg.INT8W)
    ws = torch.empty(nws, dtype=torch.uint8, device=cuda)
    outs = []
    for s in (B.variant(), B.variant(codes=True), B.variant(vindex=True), B.variant(codes=True, vindex=True)):
        C_d = torch.zeros((M, N), dtype=torch.float32, device=cuda)
        pkg.sgemm_fvb(M, N, K, 1.0, A_d.data_ptr(), K, s, pkg.INT8W, 0.0, C_d.data_ptr(), N, ws.data_ptr(), nws)
        pkg.check_device()
        outs.append(C_d.cpu().numpy())
    for o in outs[1:]:
        assert np.array_equal(o.view(np.uint32), outs[0].view(np.uint32))


def test_tgemm_q8a_repeat_and_graph(pkg, orc, synth, cuda):
    """Quantised rows in (p2cu_sgemm_fvb_q8a), the same call twice in a row and replayed from a CUDA graph."""
    import torch
    M, K, N = 375, 1024, 1024
    w = synth.five_value(K, N, seed=41)
    q, sc = orc.quant_rows(synth.activations(M, K, seed=42))
    B = _weight(pkg, torch, cuda, w)
    q_d, sc_d = torch.from_numpy(q).to(cuda), torch.from_numpy(sc).to(cuda)
    C_d = torch.zeros((M, N), dtype=torch.float32, device=cuda)
    want = orc.gemm_i8(q, sc, "int8w", np.zeros((M, N), np.float32), w=w)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for _ in range(2):
            pkg.sgemm_fvb_q8a(M, N, K, 1.0, q_d.data_ptr(), sc_d.data_ptr(), B.struct, pkg.INT8W, 0.0, C_d.data_ptr(),
                              N, 0, 0, s)
        s.synchronize()
        assert np.array_equal(C_d.cpu().numpy().view(np.uint32), want.view(np.uint32))
        C_d.zero_()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            pkg.sgemm_fvb_q8a(M, N, K, 1.0, q_d.data_ptr(), sc_d.data_ptr(), B.struct, pkg.INT8W, 0.0, C_d.data_ptr(),
                              N, 0, 0, s)
        g.replay()
        s.synchronize()
    pkg.check_device(s)
    assert np.array_equal(C_d.cpu().numpy().view(np.uint32), want.view(np.uint32))
