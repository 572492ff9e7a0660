"""The greedy TDT decoder on the device against phonon-2-c's own decoder (csrc/decoder.c), through the C ABI.

Oracle: p2_greedy_decode, p2_decoder_step and p2_joint of phonon-2-c compiled from its sources
(oracle/_ref/libphonon2_ref.so). Parity:
  * p2_joint: bit for bit (the same dot-product order, csrc/tensor_ops.c:66-96, the same adds);
  * p2_decoder_step: within 2e-6 relative (the LSTM cell's expf / tanhf come from different math libraries, each
    within an ulp or two of the exact values);
  * p2_greedy_decode: identical token lists (id, frame, duration) - greedy decisions are argmaxes, which the ulp-level
    differences of the LSTM cell do not move except at exact near-ties, which these seeded inputs do not contain.
The decoder alone runs on Gaussian frames (about one token every two frames). The encoder -> decoder pipelines run the
speech-like synthetic model (model.SPEECH_ATTN_OUT_GAIN), on which greedy decoding emits about one token per encoder
frame, and ask for at least T / 4 tokens per window besides the equality, so no comparison is between empty lists.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model(pkg):
    from phonon2_b200 import model as M
    return M.SyntheticModel(seed=1)


@pytest.fixture(scope="module")
def dev_model(pkg, cuda, model):
    d = pkg.DeviceModel(model.struct)
    yield d
    d.close()


@pytest.fixture(scope="module")
def speech(pkg):
    from phonon2_b200 import model as M
    return M.SyntheticModel(seed=1, attn_out_gain=M.SPEECH_ATTN_OUT_GAIN)


@pytest.fixture(scope="module")
def dev_speech(pkg, cuda, speech):
    d = pkg.DeviceModel(speech.struct)
    yield d
    d.close()


def _frames(T, seed):
    return np.random.default_rng(seed).standard_normal((T, 640), dtype=np.float32)


def test_joint_bitwise(pkg, orc, cuda, model):
    rng = np.random.default_rng(3)
    for _ in range(3):
        enc = rng.standard_normal(640, dtype=np.float32)
        dec = (rng.standard_normal(640) * 0.5).astype(np.float32)
        dec[:40] = -enc[:40]   # sums of exactly zero
        got = np.zeros(8198, np.float32)
        pkg.host_joint(model.struct, enc, dec, got)
        ref = orc.ref_joint(model.struct, enc, dec)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_decoder_step_matches_reference(pkg, orc, cuda, model):
    state_ref = np.zeros((2, 2, 640), np.float32)
    dec_ref = np.zeros(640, np.float32)
    for tok in (8192, 17, 4000, 8191, 0):
        state = state_ref.copy()
        dec = np.zeros(640, np.float32)
        pkg.host_decoder_step(model.struct, tok, state, dec)
        orc.ref_decoder_step(model.struct, tok, state_ref, dec_ref)
        np.testing.assert_allclose(state, state_ref, rtol=2e-6, atol=2e-7)
        np.testing.assert_allclose(dec, dec_ref, rtol=2e-6, atol=2e-7)


@pytest.mark.parametrize("T", [1, 7, 38, 375])
def test_greedy_decode_matches_reference(pkg, orc, cuda, model, T):
    enc = _frames(T, seed=T)
    got = pkg.host_greedy_decode(model.struct, enc)
    ref = orc.ref_greedy_decode(model.struct, enc)
    assert len(ref) > 0 or T < 7
    assert np.array_equal(got, ref), (len(got), len(ref))


def test_greedy_decode_empty(pkg, orc, cuda, model):
    got = pkg.host_greedy_decode(model.struct, np.zeros((0, 640), np.float32))
    assert got.shape == (0, 3)


def test_max_symbols_rule(pkg, orc, cuda, model):
    """Frames on which the decoder keeps emitting with duration 0 hit the max-symbols guard (csrc/decoder.c:132-134):
    a large frame along the head's direction of one token with its duration-0 logit raised."""
    from phonon2_b200 import model as M
    hw = model.arrays["joint.head.weight"]
    enc = _frames(20, seed=5) * 0.1
    enc[3:6] += 40 * np.maximum(hw[123], 0) + 40 * np.maximum(hw[8193], 0)   # token 123, duration 0
    ref = orc.ref_greedy_decode(model.struct, enc)
    got = pkg.host_greedy_decode(model.struct, enc)
    assert np.array_equal(got, ref)
    per_frame = np.bincount(ref[:, 1], minlength=20) if len(ref) else np.zeros(20, int)
    assert per_frame.max() == M.MAX_SYMBOLS, per_frame


def test_batched_decode_matches_reference(pkg, orc, cuda, model, dev_model):
    """One launch over windows of different lengths (one of them empty) gives each window the reference's tokens."""
    import torch
    lengths = [375, 0, 38, 1, 200, 77, 3, 150, 90, 12, 301, 64, 5, 9, 33, 120, 250, 18, 44]   # > 16: two groups
    encs = [_frames(T, seed=100 + i) for i, T in enumerate(lengths)]
    stacked = torch.from_numpy(np.concatenate(encs)).to(cuda)
    dec = pkg.Decoder(dev_model, len(lengths), sum(lengths))
    dec.decode(stacked.data_ptr(), lengths)
    got = dec.read()
    for i, e in enumerate(encs):
        ref = orc.ref_greedy_decode(model.struct, e) if len(e) else np.zeros((0, 3), np.int32)
        assert np.array_equal(got[i], ref), (i, len(got[i]), len(ref))
    # the device lists agree with the read
    from phonon2_b200.device import device_view
    offs = device_view(pkg.lib().p2cu_decoder_offsets(dec.ptr), (len(lengths) + 1,), torch.int32).cpu().numpy()
    toks = device_view(pkg.lib().p2cu_decoder_tokens(dec.ptr), (int(offs[-1]), 3), torch.int32).cpu().numpy()
    assert np.array_equal(toks, np.concatenate(got))
    # a second decode on the same plan (state reset between launches)
    dec.decode(stacked.data_ptr(), lengths)
    again = dec.read()
    assert all(np.array_equal(a, g) for a, g in zip(again, got))
    dec.close()


def test_transcribe_windows_matches_encoder_then_reference_decoder(pkg, orc, cuda, speech):
    """p2_b200_transcribe_windows (encoder and decoder on the device, frames never leave it) equals the reference's
    decoder run on p2_b200_encode_windows' frames, window by window. GPU 0 is named twice: two host threads."""
    from phonon2_b200 import model as M
    mels = [M.mel(n, seed=n) for n in (300, 251, 333, 17, 290)]
    got = pkg.host_transcribe_windows(speech.struct, mels, devices=[0, 0])
    frames = pkg.host_encode_windows(speech.struct, mels, devices=[0, 0])
    for g, f in zip(got, frames):
        ref = orc.ref_greedy_decode(speech.struct, f)
        assert len(ref) >= len(f) // 4, (len(ref), len(f))
        assert np.array_equal(g, ref)


@pytest.mark.parametrize("mel_frames", [[300], [3000], [600, 311]])
def test_exact_pipeline_matches_reference(pkg, orc, cuda, speech, dev_speech, mel_frames):
    """Exact-mode encoder plan then the device decoder, against the reference's p2_encoder then p2_greedy_decode:
    identical token lists (id, frame, duration) of at least T / 4 tokens per window, at T' = 38 (a 3 s utterance),
    T' = 375 (a 30 s window) and two windows batched."""
    import torch
    from phonon2_b200 import model as M
    from phonon2_b200.device import device_view
    mels = [M.mel(n, seed=40 + n) for n in mel_frames]
    enc = pkg.Encoder(dev_speech, [m.shape[0] for m in mels], pkg.EXACT)
    stacked = np.ascontiguousarray(np.concatenate(mels), np.float32)
    device_view(enc.mel_ptr, stacked.shape).copy_(torch.from_numpy(stacked))
    enc.run()
    dec = pkg.Decoder(dev_speech, len(mels), enc.total_frames)
    dec.decode(enc.out_ptr, enc.frames)
    got = dec.read()
    for mel, g in zip(mels, got):
        ref_frames = orc.ref_encoder(speech.struct, mel, "exact")
        ref = orc.ref_greedy_decode(speech.struct, ref_frames)
        assert len(ref) >= len(ref_frames) // 4, (len(ref), len(ref_frames))
        assert len(set(ref[:, 0].tolist())) > 1
        assert np.array_equal(g, ref), (len(g), len(ref))
    dec.close()
    enc.close()


def test_decoder_argument_errors(pkg, cuda, model, dev_model):
    from phonon2_b200 import model as M
    bare = M.SyntheticModel(seed=2, decoder=False)
    dm = pkg.DeviceModel(bare.struct)
    with pytest.raises(pkg.Error):
        pkg.Decoder(dm, 1, 10)   # uploaded without decoder tables
    dm.close()
    with pytest.raises(pkg.Error):
        pkg.Decoder(dev_model, 513, 10)
    dec = pkg.Decoder(dev_model, 2, 100)
    with pytest.raises(pkg.Error):
        dec.decode(0, [50, 60])          # NULL frames
    import torch
    buf = torch.zeros((200, 640), device=cuda)
    with pytest.raises(pkg.Error):
        dec.decode(buf.data_ptr(), [50, 60, 1])   # three windows on a two-window plan
    with pytest.raises(pkg.Error):
        dec.decode(buf.data_ptr(), [80, 60])      # 140 frames on a 100-frame plan
    with pytest.raises(pkg.Error):
        dec.step(8193, buf.data_ptr(), buf.data_ptr())   # token outside the vocabulary
    dec.close()
    assert pkg.lib().p2_greedy_decode(C.addressof(bare.struct), None, 0, C.byref(C.c_void_p())) == -1
