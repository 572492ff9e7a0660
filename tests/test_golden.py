"""The C restatement (oracle/fv_oracle.c) against golden vectors from phonon-2-c's own code (tests/golden/gemm.npz,
written by tests/golden/make_golden.py from the reference's x86 build and its AArch64 int8 code). Needs no reference
sources: the vectors are committed, the inputs are regenerated from their seeds and checked against stored SHA-256s."""
import sys
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import make_golden as mg  # noqa: E402


@pytest.fixture(scope="module")
def golden():
    with np.load(GOLDEN / "gemm.npz") as z:
        return {k: z[k] for k in z.files}


def _bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("case", mg.GEMM_CASES, ids=[c[0] for c in mg.GEMM_CASES])
def test_gemm_restatement_matches_golden(orc, synth, golden, case):
    name, mode, M, K, N, alpha, beta, wseed, aseed, edge = case
    w, A, C0 = mg.gemm_inputs(synth, mode, M, K, N, wseed, aseed, edge)
    assert list(golden[f"{name}/sha"]) == [mg.weight_sha(w), mg.sha(A), mg.sha(C0)], "regenerated inputs drifted"
    if mode == "exact" or K % 4:   # the reference quantises only whole quads; other K run its exact path
        got = orc.gemm_exact(A, C0.copy(), w=w, alpha=alpha, beta=beta)
    elif mode == "q8b":
        got = orc.sgemm_i8(A, "q8b", C0.copy(), q8=w, alpha=alpha, beta=beta)
    else:
        got = orc.sgemm_i8(A, mode, C0.copy(), w=w, alpha=alpha, beta=beta)
    assert _bits_equal(got, golden[f"{name}/out"])


@pytest.mark.parametrize("K", mg.QUANT_K)
def test_quantiser_restatement_matches_golden(orc, synth, golden, K):
    A = mg.quant_input(synth, K)
    assert golden[f"quant{K}/sha"][0] == mg.sha(A)
    q, s = orc.quant_rows(A)
    assert np.array_equal(q, golden[f"quant{K}/q"])
    assert _bits_equal(s, golden[f"quant{K}/scales"])


@pytest.mark.parametrize("K,N", mg.CODES)
def test_code_plane_restatement_matches_golden(orc, synth, golden, K, N):
    w = synth.five_value(K, N, seed=K + N)
    assert golden[f"codes{K}x{N}/sha"][0] == mg.weight_sha(w)
    assert np.array_equal(orc.fv_codes(w), golden[f"codes{K}x{N}"])


def test_encoder_golden_inputs_regenerate(pkg):
    """The encoder vectors' model and log-mel input regenerate from their seeds (tests/test_golden_gpu.py compares
    the device encoder with them)."""
    from phonon2_b200 import model as M
    with np.load(GOLDEN / "encoder.npz") as z:
        stored = list(z["sha"])
        shapes = [z[k].shape for k in ("exact", "int8w", "int8")]
    model = M.SyntheticModel(seed=mg.ENCODER_SEED)
    mel = M.mel(mg.ENCODER_MEL_FRAMES, seed=mg.ENCODER_MEL_SEED)
    assert stored == [mg.sha(*(model.arrays[k] for k in sorted(model.arrays))), mg.sha(mel)]
    assert shapes == [(M.frames_after_subsampling(mg.ENCODER_MEL_FRAMES), 640)] * 3


def test_decoder_and_mel_golden_inputs_regenerate(pkg):
    """The decoder and log-mel vectors' inputs regenerate from their seeds (tests/test_golden_gpu.py compares the
    device's decoder and front end with them)."""
    from phonon2_b200 import model as M
    with np.load(GOLDEN / "decoder.npz") as z:
        assert z["joint/sha"][0] == mg.sha(*(a for pair in mg.joint_inputs() for a in pair))
        for T in mg.DECODE_T:
            assert z[f"tokens{T}/sha"][0] == mg.sha(mg.decode_frames(T))
            assert z[f"tokens{T}"].shape[1] == 3 and len(z[f"tokens{T}"]) > 0
    with np.load(GOLDEN / "mel.npz") as z:
        assert z["sha"][0] == mg.sha(M.audio(mg.MEL_SAMPLES, seed=mg.MEL_SAMPLES))
        assert z["mel"].shape == (mg.MEL_SAMPLES // 160, 128)


def test_golden_vectors_regenerate_from_the_reference(orc, tmp_path):
    """Where the reference's builds are present, writing the vectors again gives the committed ones exactly: the
    generator, the seeds and the reference's results have not drifted."""
    if not (orc.ref_available() and orc.ref_neon_available()):
        pytest.skip("the reference's builds are not present")
    mg.main(tmp_path)
    for name in ("gemm", "encoder", "decoder", "mel"):
        with np.load(GOLDEN / f"{name}.npz") as want, np.load(tmp_path / f"{name}.npz") as got:
            assert sorted(want.files) == sorted(got.files), name
            for k in want.files:
                assert np.array_equal(want[k], got[k]), f"{name}: {k}"
