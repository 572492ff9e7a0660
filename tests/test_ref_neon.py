"""The int8 and int8w GEMMs pinned against phonon-2-c's own AArch64 code.

The reference's int8 paths (per-row quantisation, the S/T planes, the int8w code plane, SDOT over 1024-row K blocks
and the blockwise epilogue; csrc/blas.c:1068-1447) compile only for AArch64 with dot products. oracle/Makefile
compiles that very blas.c for this x86 host with the AArch64 macros defined and the NEON intrinsics modelled in C
(oracle/neon_emu/arm_neon.h), twice: with IEEE arithmetic (what the C source says) and with the reference's own
-ffast-math flags. These tests hold the C restatement (oracle/fv_oracle.c) - which the GPU tests compare the kernels
with bit for bit - to the reference's code:
  * IEEE build: quantised rows and scales, the int32 accumulators, the int8w codes and every fp32 output bit for bit;
  * -ffast-math build: the compiler turns `amax / 127.0f` (csrc/blas.c:1120) into `amax * (1/127)`, which moves the
    scale of about one row in twenty by one ulp and, rarely, one quantised value by one step; on identical quantised
    rows its outputs are still bit for bit those of the restatement, and end to end, on rows it quantises alike,
    they stay within the 1e-5 relative bound that applies to fp32 outputs.
"""
import numpy as np
import pytest


@pytest.fixture(scope="module")
def neon(orc):
    if not orc.ref_neon_available():
        pytest.skip("the reference's AArch64 build is not present (its sources are absent on this machine)")
    return orc


def _bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def _special_rows(K, seed):
    """Rows that reach the quantiser's edge cases: zeros (scale 1), one large value, exact halves after scaling
    (ties to even), values far below the row maximum, denormals, negative extremes."""
    rng = np.random.default_rng(seed)
    rows = [np.zeros(K, np.float32)]
    r = np.zeros(K, np.float32); r[K // 2] = 3.0e7; rows.append(r)
    r = (np.arange(K) % 9 - 4).astype(np.float32) + 0.5; r[0] = 127.0; rows.append(r)       # scale 1: x.5 ties
    r = (np.arange(K) % 7 - 3).astype(np.float32) * 0.5; r[-1] = -127.0; rows.append(r)
    r = rng.standard_normal(K).astype(np.float32) * 1e-3; r[1] = 50.0; rows.append(r)
    r = np.full(K, 1e-40, np.float32); r[2] = -1e-39; rows.append(r)                          # denormals
    r = rng.standard_normal(K).astype(np.float32); r[3] = -np.float32(np.abs(r).max() * 2); rows.append(r)
    return np.stack(rows)


def test_aarch64_build_reports_its_int8_modes(neon):
    assert neon.ref_neon("int8").p2_gemm_mode() == b"int8 dot products, exact weights"
    assert neon.ref_neon("int8w").p2_gemm_mode() == b"int8 dot products, int8 weights"
    assert neon.ref_neon("exact").p2_gemm_mode() == b"fp32 expansion (exact)"


@pytest.mark.parametrize("K", [16, 20, 1024, 1028, 4096])
def test_quantiser_matches_reference_bitwise(neon, synth, K):
    """csrc/blas.c:1114-1144 (the 16-wide NEON loop, and its scalar tail when K % 16 != 0) against the restatement."""
    A = np.concatenate([synth.activations(60, K, seed=K), _special_rows(K, seed=K + 1),
                        synth.quantiser_edge_rows(K, seed=K + 2)])
    q, s = neon.neon_quant_rows(neon.ref_neon("int8w"), A)
    q_o, s_o = neon.quant_rows(A)
    assert np.array_equal(q, q_o)
    assert _bits_equal(s, s_o)


def test_quantiser_under_fast_math_takes_the_reciprocal_of_127(neon, synth):
    """The reference as its Makefile builds it: amax * (1/127) for the scale; quantised values within one step."""
    K = 1024
    A = np.concatenate([synth.activations(4000, K, seed=3), _special_rows(K, seed=4)])
    q, s = neon.neon_quant_rows(neon.ref_neon("int8w", fast_math=True), A)
    amax = np.abs(A).max(axis=1)
    recip = np.where(amax > 0, amax * (np.float32(1) / np.float32(127)), np.float32(1)).astype(np.float32)
    assert _bits_equal(s, recip)
    q_o, s_o = neon.quant_rows(A)
    moved = q.astype(np.int32) - q_o.astype(np.int32)
    assert np.abs(moved).max() <= 1
    assert np.count_nonzero(moved) <= 1e-5 * moved.size
    assert 0 < np.count_nonzero(s.view(np.uint32) != s_o.view(np.uint32)) < 0.1 * len(s)


@pytest.mark.parametrize("K", [1024, 4096, 1000, 100, 36])
def test_fast_math_quantiser_restatement_matches_reference_build(neon, synth, K):
    """The opt-in rule (orc_quant_row_fast_math; on the device p2cu_set_quant_fast_math) against the reference's
    -ffast-math build itself: every scale and every quantised value bit for bit, ragged tails and edge rows included
    (the denormal row, whose reciprocal overflows, among them). The rule it pins: scale = amax * (1/127), the 16-wide
    loop's reciprocal 127 / amax, the tail multiplied by it too."""
    A = np.concatenate([synth.activations(3000, K, seed=K), _special_rows(K, seed=K + 1),
                        synth.quantiser_edge_rows(K, seed=K)])
    q, s = neon.neon_quant_rows(neon.ref_neon("int8w", fast_math=True), A)
    q_o, s_o = neon.quant_rows(A, fast_math=True)
    assert _bits_equal(s, s_o)
    assert np.array_equal(q, q_o)
    # and it is a different rule from the IEEE one: some rows' scales and values move
    q_i, s_i = neon.quant_rows(A)
    assert not _bits_equal(s_i, s_o)


def _unit_quanta(M, K, seed):
    q = np.random.default_rng(seed).integers(-127, 128, size=(M, K)).astype(np.int8)
    return q, np.ones(M, np.float32)


@pytest.mark.parametrize("K", [64, 1024, 2048])
def test_int32_accumulators_match_reference(neon, synth, K):
    """The SDOT sums themselves (csrc/blas.c:1257-1282), read through the reference's own epilogue with unit factors:
    a_scale = alpha = 1 and per-column factors of exactly 1 make each K block's output (float)acc, exact below 2^24.
      int8 table: scale 1 (csrc/blas.c:1335);  int8 two planes: lo = 1, hi = 1 gives accS, lo = 0, hi = 1 gives accT
      (c1 = lo, c2 = hi - lo; csrc/blas.c:1329-1333, 1362);  int8w: hi = 127 makes c1 = hi * (1/127) = 1 and
      clo = lo for integer lo (csrc/blas.c:1319-1328)."""
    M, N = 37, 64
    q, ones = _unit_quanta(M, K, seed=K)
    nblk = (K + 1023) // 1024

    def blocks_summed(acc):
        out = np.zeros(acc.shape[1:], np.float32)
        for b in range(nblk):
            out = (out + acc[b].astype(np.float32)).astype(np.float32)
        return out

    t = synth.int8_table(K, N, seed=1)
    t = dict(t, scales=np.ones(N, np.float32))
    got = neon.neon_sgemm_q8b_q8a(neon.ref_neon("int8"), q, ones, t, np.zeros((M, N), np.float32))
    accS, _ = neon.acc_blocks(q, "q8b", q8=t)
    assert np.array_equal(got, blocks_summed(accS))

    w = synth.five_value(K, N, seed=2)
    accS, accT = neon.acc_blocks(q, "int8", w=w)
    L = neon.ref_neon("int8")
    w_s = dict(w, lo=np.ones(N, np.float32), hi=np.ones(N, np.float32))
    assert np.array_equal(neon.neon_sgemm_fvb_q8a(L, q, ones, w_s, np.zeros((M, N), np.float32)), blocks_summed(accS))
    w_t = dict(w, lo=np.zeros(N, np.float32), hi=np.ones(N, np.float32))
    assert np.array_equal(neon.neon_sgemm_fvb_q8a(L, q, ones, w_t, np.zeros((M, N), np.float32)), blocks_summed(accT))

    lo = np.random.default_rng(3).integers(0, 128, size=N).astype(np.float32)
    w_c = dict(w, lo=lo, hi=np.full(N, 127.0, np.float32))
    accC, _ = neon.acc_blocks(q, "int8w", w=w_c)
    got = neon.neon_sgemm_fvb_q8a(neon.ref_neon("int8w"), q, ones, w_c, np.zeros((M, N), np.float32))
    assert np.array_equal(got, blocks_summed(accC))


@pytest.mark.parametrize("fast_math", [False, True], ids=["ieee", "fast_math"])
@pytest.mark.parametrize("mode", ["int8", "int8w", "q8b"])
@pytest.mark.parametrize("M,K,N,alpha,beta", [(375, 1024, 4096, 1.0, 0.0), (77, 4096, 1024, 0.5, 1.0),
                                               (13, 1028, 48, 1.0, 0.25), (1, 2048, 16, 2.0, 1.0)])
def test_gemm_on_identical_quantised_rows_matches_reference_bitwise(neon, synth, fast_math, mode, M, K, N, alpha,
                                                                    beta):
    """p2_sgemm_fvb_q8a / p2_sgemm_q8b_q8a (csrc/blas.c:1430-1446) on the same int8 rows and scales: the planes or codes
    expanded, the blockwise int32 sums and the fp32 epilogue in K-block order, against the restatement."""
    L = neon.ref_neon("int8w" if mode == "int8w" else "int8", fast_math=fast_math)
    A = synth.activations(M, K, seed=M + K)
    q, s = neon.quant_rows(A)
    C0 = np.random.default_rng(N).standard_normal((M, N)).astype(np.float32)
    if mode == "q8b":
        t = synth.int8_table(K, N, seed=4)
        got = neon.neon_sgemm_q8b_q8a(L, q, s, t, C0.copy(), alpha=alpha, beta=beta)
        want = neon.gemm_i8(q, s, "q8b", C0.copy(), q8=t, alpha=alpha, beta=beta)
    else:
        w = synth.five_value(K, N, seed=5)
        got = neon.neon_sgemm_fvb_q8a(L, q, s, w, C0.copy(), alpha=alpha, beta=beta)
        want = neon.gemm_i8(q, s, mode, C0.copy(), w=w, alpha=alpha, beta=beta)
    assert _bits_equal(got, want)


@pytest.mark.parametrize("mode", ["int8", "int8w"])
@pytest.mark.parametrize("M,K,N,alpha,beta", [(375, 1024, 4096, 1.0, 0.0), (749, 1024, 1024, 1.0, 0.0),
                                               (375, 4096, 1024, 0.5, 1.0), (38, 1024, 3072, 1.0, 0.0),
                                               (5, 1028, 32, 1.0, 0.5), (13, 1000, 48, 1.0, 0.0),
                                               (77, 2056, 144, 0.5, 1.0)])
def test_sgemm_fvb_end_to_end_matches_reference(neon, synth, mode, M, K, N, alpha, beta):
    """p2_sgemm_fvb in the int8 modes (csrc/blas.c:1481-1499: quantise, then the int8 GEMM) on fp32 activations:
    bit for bit against the IEEE build, the first rows being the quantiser's edge cases (synth.quantiser_edge_rows);
    against the -ffast-math build within 1e-5 of the largest output on every row both quantise alike."""
    w = synth.five_value(K, N, seed=7)
    A = np.concatenate([synth.quantiser_edge_rows(K, seed=K)[:M], synth.activations(max(M - 8, 0), K, seed=8)])[:M]
    C0 = np.random.default_rng(9).standard_normal((M, N)).astype(np.float32)
    want = neon.sgemm_i8(A, mode, C0.copy(), w=w, alpha=alpha, beta=beta)
    got = neon.neon_sgemm_fvb(neon.ref_neon(mode), A, w, C0.copy(), alpha=alpha, beta=beta)
    assert _bits_equal(got, want)
    # The -ffast-math build on N(0, 1) rows (the edge rows sit on rounding boundaries on purpose): its scale
    # amax * (1/127) can move a code by one step (about one in a million); rows it quantises to the same codes
    # differ only through that scale's last bit.
    A = synth.activations(M, K, seed=10)
    want = neon.sgemm_i8(A, mode, C0.copy(), w=w, alpha=alpha, beta=beta)
    L_fm = neon.ref_neon(mode, fast_math=True)
    same = np.all(neon.neon_quant_rows(L_fm, A)[0] == neon.quant_rows(A)[0], axis=1)
    assert np.count_nonzero(~same) <= max(1, 0.01 * M)
    got_fm = neon.neon_sgemm_fvb(L_fm, A, w, C0.copy(), alpha=alpha, beta=beta)
    assert np.max(np.abs(got_fm - want)[same]) <= 1e-5 * np.max(np.abs(want))


@pytest.mark.parametrize("fast_math", [False, True], ids=["ieee", "fast_math"])
@pytest.mark.parametrize("K,N", [(1024, 4096), (4096, 1024), (64, 16)])
def test_code_plane_matches_reference(neon, synth, fast_math, K, N):
    """p2_fv_pack_codes (csrc/blas.c:1372-1400): sign * (flag ? 127 : clo), clo = round(127 * lo / hi)."""
    w = synth.five_value(K, N, seed=K + N)
    got = neon.neon_fv_pack_codes(neon.ref_neon("int8w", fast_math=fast_math), w)
    assert np.array_equal(got, neon.fv_codes(w))


@pytest.mark.parametrize("M,K,N,alpha,beta", [(375, 1024, 512, 1.0, 0.0), (40, 4096, 128, 0.5, 1.0),
                                               (5, 100, 48, 1.0, 0.5)])
def test_exact_path_is_the_same_on_both_isas(neon, synth, M, K, N, alpha, beta):
    """The exact path (fp32 expansion, one FMA chain per output) gives the same bits from the reference's NEON
    branches as from its AVX2 build (and so as from the restatement), as its cross-platform check expects."""
    if not neon.ref_available():
        pytest.skip("reference x86 library not built")
    w = synth.five_value(K, N, seed=M + N)
    A = synth.activations(M, K, seed=K)
    C0 = np.random.default_rng(1).standard_normal((M, N)).astype(np.float32)
    x86 = neon.ref_sgemm_fvb(A, w, C0.copy(), alpha=alpha, beta=beta)
    arm = neon.neon_sgemm_fvb(neon.ref_neon("exact"), A, w, C0.copy(), alpha=alpha, beta=beta)
    assert _bits_equal(arm, x86)
    assert _bits_equal(arm, neon.gemm_exact(A, C0.copy(), w=w, alpha=alpha, beta=beta))


# ---- the encoder as the reference's AArch64 build runs it ----------------------------------------------------------

@pytest.fixture(scope="module")
def enc_model(pkg):
    from phonon2_b200 import model as M
    return M.SyntheticModel(seed=7)


def _rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


def test_aarch64_encoder_exact_mode_matches_x86_build(neon, enc_model):
    """p2_encoder in exact mode through the reference's NEON branches (LayerNorm, softmax, the polynomial exp, SiLU,
    the depthwise convolution; csrc/tensor_ops.c, csrc/encoder.c) against its x86 build, which the device encoder's
    exact-mode tests use: within the same 1e-4 of the largest output."""
    from phonon2_b200 import model as M
    mel = M.mel(300, seed=11)
    arm = neon.ref_neon_encoder(enc_model.struct, mel, "exact")
    x86 = neon.ref_encoder(enc_model.struct, mel, "exact")
    assert arm.shape == (38, 640)
    assert _rel(arm, x86) <= 1e-4


@pytest.mark.parametrize("mode", ["int8w", "int8"])
def test_aarch64_int8_encoder_is_within_the_envelope_of_the_int8_oracle(neon, enc_model, mode):
    """The device's int8 encoder is tested against the reference's encoder sources run with the restated int8 GEMMs
    on their x86 branches (libphonon2_ref_i8.so): within twice that oracle's distance from exact mode, correlation
    above 0.999. The reference's own AArch64 int8 encoder - its NEON branches and its int8 GEMMs - is a second valid
    int8 encoder, and it meets the same criterion against that oracle (measured: 1.2-1.45 times the distance,
    correlation 0.9993-0.9994): an ulp before a quantiser flips a code, and 24 blocks carry such flips."""
    from phonon2_b200 import model as M
    mel = M.mel(300, seed=11)
    arm = neon.ref_neon_encoder(enc_model.struct, mel, mode)
    oracle = neon.ref_encoder(enc_model.struct, mel, mode)
    exact = neon.ref_encoder(enc_model.struct, mel, "exact")
    noise = _rel(oracle, exact)
    assert 1e-3 < noise < 0.1
    assert _rel(arm, oracle) <= 2 * noise and _rel(arm, exact) <= 2 * noise
    assert np.corrcoef(arm.ravel(), oracle.ravel())[0, 1] > 0.999


@pytest.mark.parametrize("beta", [0.0, 1.0, 0.5])
def test_alpha_zero_only_scales_c(neon, synth, beta):
    """alpha == 0: the reference's q8a entry points only apply beta to C (csrc/blas.c:1433, 1442): zeros for beta 0
    (a memset, so +0 everywhere), C unchanged for 1, C * beta otherwise."""
    M, K, N = 9, 1024, 64
    q, s = neon.quant_rows(synth.activations(M, K, seed=1))
    w = synth.five_value(K, N, seed=2)
    C0 = np.random.default_rng(3).standard_normal((M, N)).astype(np.float32)
    got = neon.neon_sgemm_fvb_q8a(neon.ref_neon("int8w"), q, s, w, C0.copy(), alpha=0.0, beta=beta)
    want = neon.gemm_i8(q, s, "int8w", C0.copy(), w=w, alpha=0.0, beta=beta)
    assert _bits_equal(got, want)
    assert _bits_equal(want, np.zeros_like(C0) if beta == 0.0 else (C0 * np.float32(beta)).astype(np.float32))
