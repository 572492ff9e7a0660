"""The log-mel front end on the device against phonon-2-c's own p2_mel_spectrogram (csrc/mel.c), through the C ABI.

Oracle: the reference library compiled from its sources (oracle/_ref/libphonon2_ref.so). Tolerance: the features are
normalised per bin (mean 0, std 1); the device's FFT takes exact twiddles where the reference advances them by a
recurrence, and its logf is CUDA's, so the two agree to a few 1e-6 in most bins and to MEL_TOL (absolute) in all. A batch
of windows is compared bit for bit with each window computed alone, and the audio -> tokens pipeline with mel -> tokens.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MEL_TOL = 1e-3


@pytest.mark.parametrize("n", [320, 321, 3200, 16000, 48123, 480000])
def test_mel_matches_reference(pkg, orc, cuda, n):
    from phonon2_b200 import model as M
    a = M.audio(n, seed=n)
    got = pkg.host_mel_spectrogram(a)
    ref = orc.ref_mel_spectrogram(a)
    assert got.shape == ref.shape == (n // 160, 128)
    err = np.abs(got - ref)
    print(f"n={n}: max |device - reference| {err.max():.2e}, mean {err.mean():.2e}")
    assert err.max() <= MEL_TOL, err.max()
    assert np.median(err) <= 2e-5


def test_mel_too_short(pkg, cuda):
    with pytest.raises(pkg.Error):
        pkg.host_mel_spectrogram(np.zeros(319, np.float32))


def test_mel_batch_equals_single_windows(pkg, cuda):
    import torch
    from phonon2_b200 import model as M
    lengths = [48000, 320, 33333, 160 * 700 + 17]
    audios = [M.audio(n, seed=i + 1) for i, n in enumerate(lengths)]
    x = torch.from_numpy(np.concatenate(audios)).to(cuda)
    frames = [n // 160 for n in lengths]
    out = torch.empty((sum(frames), 128), device=cuda)
    plan = pkg.Mel(len(lengths), sum(lengths))
    plan.run(x.data_ptr(), lengths, out.data_ptr())
    pkg.check_device()
    got = out.cpu().numpy()
    offs = np.cumsum([0] + frames)
    for i, a in enumerate(audios):
        one = pkg.host_mel_spectrogram(a)
        assert np.array_equal(got[offs[i]:offs[i + 1]].view(np.uint32), one.view(np.uint32)), i
    plan.close()


def test_transcribe_audio_equals_transcribe_mel(pkg, cuda):
    """Audio -> tokens on the device (mel, encoder, decoder) equals mel -> tokens on p2_mel_spectrogram's features."""
    from phonon2_b200 import model as M
    sm = M.SyntheticModel(seed=1)
    audios = [M.audio(n, seed=100 + n) for n in (48000, 16000 * 5 + 77, 160 * 400)]
    got = pkg.host_transcribe_audio_windows(sm.struct, audios, devices=[0, 0])
    mels = [pkg.host_mel_spectrogram(a) for a in audios]
    want = pkg.host_transcribe_windows(sm.struct, mels, devices=[0])
    for g, w in zip(got, want):
        assert np.array_equal(g, w)
