"""The device against golden vectors from phonon-2-c's own code (tests/golden/, written by tests/golden/make_golden.py
from the reference's x86 build and its AArch64 int8 code), with no oracle in the loop: the GEMMs, the quantiser and
the int8w code plane bit for bit; the encoder in exact mode within 1e-4 of the largest output, and in the int8 modes
within the statistical envelope of the encoder tests (twice the reference's own int8-vs-exact distance, correlation
above 0.999; see tests/test_encoder_gpu.py); the decoder's joint logits bit for bit and its greedy tokens equal; the
log-mel features within 1e-4 absolute."""
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
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
def test_device_gemm_matches_golden(pkg, synth, cuda, golden, case):
    import torch
    from phonon2_b200.device import DeviceFiveValue
    name, mode, M, K, N, alpha, beta, wseed, aseed, edge = case
    w, A, C0 = mg.gemm_inputs(synth, mode, M, K, N, wseed, aseed, edge)
    m = pkg.INT8 if mode == "q8b" else pkg.MODES[mode]
    A_d = torch.from_numpy(A).to(cuda)
    C_d = torch.from_numpy(C0.copy()).to(cuda)
    nws = max(pkg.workspace_bytes(M, N, K, m), 16)
    ws = torch.empty(nws, dtype=torch.uint8, device=cuda)
    if mode == "q8b":
        B_d = torch.from_numpy(w["q8"]).to(cuda)
        s_d = torch.from_numpy(w["scales"]).to(cuda)
        pkg.sgemm_q8b(M, N, K, alpha, A_d.data_ptr(), K, B_d.data_ptr(), s_d.data_ptr(), N, m, beta, C_d.data_ptr(),
                      N, ws.data_ptr(), nws)
    else:
        B = DeviceFiveValue(w, cuda)
        pkg.sgemm_fvb(M, N, K, alpha, A_d.data_ptr(), K, B.struct, m, beta, C_d.data_ptr(), N, ws.data_ptr(), nws)
    pkg.check_device()
    assert _bits_equal(C_d.cpu().numpy(), golden[f"{name}/out"])


@pytest.mark.parametrize("K", mg.QUANT_K)
def test_device_quantiser_matches_golden(pkg, synth, cuda, golden, K):
    import torch
    A = mg.quant_input(synth, K)
    M = A.shape[0]
    A_d = torch.from_numpy(A).to(cuda)
    q_d = torch.empty((M, K), dtype=torch.int8, device=cuda)
    s_d = torch.empty(M, dtype=torch.float32, device=cuda)
    pkg.quant_rows(A_d.data_ptr(), M, K, K, q_d.data_ptr(), s_d.data_ptr())
    pkg.check_device()
    assert np.array_equal(q_d.cpu().numpy(), golden[f"quant{K}/q"])
    assert _bits_equal(s_d.cpu().numpy(), golden[f"quant{K}/scales"])


@pytest.mark.parametrize("K,N", mg.CODES)
def test_device_code_plane_matches_golden(synth, cuda, golden, K, N):
    import torch
    from phonon2_b200.device import DeviceFiveValue
    B = DeviceFiveValue(synth.five_value(K, N, seed=K + N), cuda, codes=True)
    torch.cuda.synchronize()
    assert np.array_equal(B.codes.cpu().numpy(), golden[f"codes{K}x{N}"])


def _rel(got, ref):
    return float(np.abs(got - ref).max() / np.abs(ref).max())


def test_device_encoder_matches_golden(pkg, cuda):
    import torch
    from phonon2_b200 import model as M
    from phonon2_b200.device import device_view
    with np.load(GOLDEN / "encoder.npz") as z:
        gold = {k: z[k] for k in ("exact", "int8w", "int8")}
    model = M.SyntheticModel(seed=mg.ENCODER_SEED)
    mel = M.mel(mg.ENCODER_MEL_FRAMES, seed=mg.ENCODER_MEL_SEED)
    dev = pkg.DeviceModel(model.struct)
    try:
        out = {}
        for mode in ("exact", "int8w", "int8"):
            enc = pkg.Encoder(dev, [mel.shape[0]], pkg.MODES[mode], 0, 8)
            device_view(enc.mel_ptr, mel.shape).copy_(torch.from_numpy(mel))
            enc.run()
            pkg.check_device()
            out[mode] = device_view(enc.out_ptr, (enc.total_frames, 640)).cpu().numpy()
            enc.close()
    finally:
        dev.close()
    assert _rel(out["exact"], gold["exact"]) <= 1e-4
    for mode in ("int8w", "int8"):
        noise = _rel(gold[mode], gold["exact"])
        assert 1e-3 < noise < 0.1
        assert _rel(out[mode], gold[mode]) <= 2 * noise
        assert np.corrcoef(out[mode].ravel(), gold[mode].ravel())[0, 1] > 0.999


@pytest.fixture(scope="module")
def model7(pkg):
    from phonon2_b200 import model as M
    return M.SyntheticModel(seed=mg.ENCODER_SEED)


def test_device_joint_matches_golden(pkg, cuda, model7):
    """p2_joint bit for bit: the dot products in the reference's order (csrc/tensor_ops.c:66-96)."""
    with np.load(GOLDEN / "decoder.npz") as z:
        want = z["joint"]
    for i, (enc, dec) in enumerate(mg.joint_inputs()):
        got = np.zeros(8198, np.float32)
        pkg.host_joint(model7.struct, enc, dec, got)
        assert _bits_equal(got, want[i])


@pytest.mark.parametrize("T", mg.DECODE_T)
def test_device_greedy_decode_matches_golden(pkg, cuda, model7, T):
    """p2_greedy_decode: the same tokens (id, frame, duration) as the reference's."""
    with np.load(GOLDEN / "decoder.npz") as z:
        want = z[f"tokens{T}"]
    assert np.array_equal(pkg.host_greedy_decode(model7.struct, mg.decode_frames(T)), want)


def test_device_mel_matches_golden(pkg, cuda):
    """p2_mel_spectrogram within 1e-4 (absolute, on features normalised to unit variance) of the reference's."""
    from phonon2_b200 import model as M
    with np.load(GOLDEN / "mel.npz") as z:
        want = z["mel"]
    got = pkg.host_mel_spectrogram(M.audio(mg.MEL_SAMPLES, seed=mg.MEL_SAMPLES))
    err = np.abs(got - want)
    print(f"mel: max |device - golden| {err.max():.2e}, median {np.median(err):.2e}")
    assert got.shape == want.shape and err.max() <= 1e-4 and np.median(err) <= 2e-5
