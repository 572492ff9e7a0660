"""The CPU checkers: pin the C restatement (oracle/fv_oracle.c) against phonon-2-c's own library compiled from its
sources (oracle/_ref), and check the restatement's int8 arithmetic against identities it must satisfy."""
import numpy as np
import pytest


def _ref_or_skip(orc):
    if not orc.ref_available():
        pytest.skip("reference library not built (its sources are absent on this machine)")


SHAPES = [(1, 64, 16), (7, 256, 64), (33, 1024, 128), (375, 1024, 512), (40, 4096, 128), (5, 100, 48)]


@pytest.mark.parametrize("M,K,N", SHAPES)
@pytest.mark.parametrize("alpha,beta", [(1.0, 0.0), (0.5, 1.0), (1.0, 0.5), (2.0, 1.0)])
def test_exact_restatement_matches_reference_bitwise(orc, synth, M, K, N, alpha, beta):
    """The exact path is one FMA chain per output in the reference (csrc/blas.c:155-181, 931-987): bit for bit."""
    _ref_or_skip(orc)
    w = synth.five_value(K, N, seed=M * 7 + K)
    A = synth.activations(M, K, seed=N)
    C0 = np.random.default_rng(3).standard_normal((M, N)).astype(np.float32)
    got = orc.gemm_exact(A, C0.copy(), w=w, alpha=alpha, beta=beta)
    want = orc.ref_sgemm_fvb(A, w, C0.copy(), alpha=alpha, beta=beta)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("M,K,N", [(9, 4096, 1024), (38, 1024, 640), (3, 64, 32)])
def test_exact_q8b_restatement_matches_reference_bitwise(orc, synth, M, K, N):
    _ref_or_skip(orc)
    t = synth.int8_table(K, N, seed=5)
    A = synth.activations(M, K, seed=6)
    got = orc.gemm_exact(A, np.zeros((M, N), np.float32), q8=t)
    want = orc.ref_sgemm_q8b(A, t, np.zeros((M, N), np.float32))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_reference_runs_exact_on_x86(orc):
    """On x86 the reference has no int8 path (csrc/blas.c:1021-1023, 1043-1045): it reports the exact mode."""
    _ref_or_skip(orc)
    assert orc.ref().p2_gemm_exact() == 1
    assert b"exact" in orc.ref().p2_gemm_mode()


def _exactly_quantised(M, K, seed):
    """Integer-valued rows in [-127, 127] with |max| = 127: the quantiser maps them to themselves with scale 1."""
    rng = np.random.default_rng(seed)
    A = rng.integers(-127, 128, size=(M, K)).astype(np.float32)
    A[:, 0] = 127.0
    return A


@pytest.mark.parametrize("mode", ["int8", "int8w"])
@pytest.mark.parametrize("K", [1024, 4096])
def test_int8_restatement_agrees_with_reference_exact_on_exact_inputs(orc, synth, mode, K):
    """Where quantisation is lossless, the int8 mode and the reference's exact path compute the same sums and may
    differ only by fp32 rounding (int8) or by rounding lo to the 127-step grid of hi (int8w, csrc/blas.c:1222)."""
    _ref_or_skip(orc)
    M, N = 24, 256
    w = synth.five_value(K, N, seed=11)
    A = _exactly_quantised(M, K, seed=12)
    q, s = orc.quant_rows(A)
    assert np.all(s == 1.0) and np.array_equal(q.astype(np.float32), A)
    got = orc.sgemm_i8(A, mode, np.zeros((M, N), np.float32), w=w)
    want = orc.ref_sgemm_fvb(A, w, np.zeros((M, N), np.float32))
    scale = np.abs(A).astype(np.float64) @ np.abs(synth.expand(w)).astype(np.float64)   # sum of |a w|
    err = np.abs(got.astype(np.float64) - want) / scale
    if mode == "int8":
        assert err.max() < 1e-6
    else:   # |lo - clo * hi / 127| <= hi / 254 per weight, relative to |w| >= lo >= hi / 4
        assert err.max() < 4.0 / 254


@pytest.mark.parametrize("K", [256, 1024, 3072])
def test_int8w_sum_is_the_two_plane_identity(orc, synth, K):
    """sum q * code == clo * sum q * S + (127 - clo) * sum q * T, exactly: the identity the GPU kernel uses."""
    M, N = 16, 128
    w = synth.five_value(K, N, seed=K)
    q, _ = orc.quant_rows(synth.activations(M, K, seed=1))
    accW, _ = orc.acc_blocks(q, "int8w", w=w)
    accS, accT = orc.acc_blocks(q, "int8", w=w)
    clo = np.array([orc.clo(l, h) for l, h in zip(w["lo"], w["hi"])], np.int64)
    assert np.array_equal(accW, clo * accS.astype(np.int64) + (127 - clo) * accT.astype(np.int64))


def test_int32_sums_restart_every_1024_rows(orc, synth):
    M, K, N = 4, 2500, 32
    w = synth.five_value(K, N, seed=2)
    q, _ = orc.quant_rows(synth.activations(M, K, seed=3))
    accS, accT = orc.acc_blocks(q, "int8", w=w)
    assert accS.shape == (3, M, N)
    S = np.sign(synth.expand(w)).astype(np.int64)
    for b, (k0, k1) in enumerate([(0, 1024), (1024, 2048), (2048, 2500)]):
        assert np.array_equal(accS[b], q[:, k0:k1].astype(np.int64) @ S[k0:k1])


def test_quantisation_contract(orc):
    rng = np.random.default_rng(0)
    A = (rng.standard_normal((64, 1024)) * rng.uniform(0.01, 100, (64, 1))).astype(np.float32)
    A[3] = 0.0                                          # an all-zero row: scale 1, codes 0
    A[5, :4] = [127.0, 0.5, 1.5, -2.5]                  # ties round to even at scale 1
    A[5, 4:] = 0.0
    q, s = orc.quant_rows(A)
    amax = np.abs(A).max(axis=1)
    assert s[3] == 1.0 and not q[3].any()
    assert np.array_equal(q[5, :4], np.array([127, 0, 2, -2], np.int8))
    nz = amax > 0
    assert np.array_equal(s[nz], (amax[nz] / np.float32(127.0)).astype(np.float32))
    assert np.abs(q.astype(np.int32)).max() <= 127


def test_clo_edges(orc):
    assert orc.clo(0.01, 0.0) == 0            # hi <= 0
    assert orc.clo(0.01, -1.0) == 0
    assert orc.clo(0.02, 0.01) == 127         # lo > hi clamps
    rng = np.random.default_rng(4)
    lo = rng.uniform(0.005, 0.02, 2000).astype(np.float32)
    hi = (lo * rng.uniform(1.0, 4.0, 2000)).astype(np.float32)
    # IEEE single: (127 * lo) / hi, rounded half to even (numpy float32 arithmetic is IEEE single precision)
    want = np.clip(np.rint((np.float32(127.0) * lo) / hi), 0, 127).astype(np.int64)
    got = np.array([orc.clo(float(a), float(b)) for a, b in zip(lo, hi)])
    assert np.array_equal(got, want)


def test_codes_plane_matches_identity(orc, synth):
    w = synth.five_value(64, 48, seed=9)
    codes = orc.fv_codes(w).astype(np.int32)
    S = np.sign(synth.expand(w)).astype(np.int32)
    flag = np.unpackbits(w["flags"], axis=1, bitorder="little").astype(bool)
    clo = np.array([orc.clo(l, h) for l, h in zip(w["lo"], w["hi"])], np.int32)
    assert np.array_equal(codes, S * np.where(flag, 127, clo[None, :]))


@pytest.mark.parametrize("K,N", [(1024, 256), (100, 32), (4096, 128)])
def test_vindex_restatement_decodes_to_the_codes(orc, synth, K, N):
    """The value-index plane (include/p2cuda.h p2cu_fv_pack_vindex, restated by oracle.vindex) decodes through the
    per-column palette to exactly the int8w codes (csrc/blas.c:1222-1240)."""
    w = synth.five_value(K, N, seed=K + 3)
    assert np.array_equal(orc.vindex_codes(orc.vindex(w), w), orc.fv_codes(w))


def test_vindex_code3_matches_reference_pack(orc, synth):
    """The unused 2-bit code 3 decodes as the reference's own code packer reads it (sign +2, product wrapping)."""
    if not orc.ref_neon_available():
        pytest.skip("the reference's AArch64 build is not built")
    w = synth.five_value(64, 32, seed=5)
    w["signs"] = w["signs"].copy()
    w["signs"][::3, ::2] |= 0x03
    ref = orc.neon_fv_pack_codes(orc.ref_neon("int8w"), w)
    assert np.array_equal(orc.vindex_codes(orc.vindex(w), w), ref)
