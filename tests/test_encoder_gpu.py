"""The encoder on the device against phonon-2-c's own encoder, through the C ABI.

Oracles: exact mode is phonon-2-c's p2_encoder compiled from its sources (oracle/_ref/libphonon2_ref.so, whose x86
build is the exact path); the int8 modes are the same encoder sources with the int8 GEMM entry points restated
(oracle/_ref/libphonon2_ref_i8.so), so the reference's int8 control flow - rows quantised as they are produced,
residuals added in the GEMM epilogues - runs on x86; and, where it is built, the reference's own AArch64 build of
the encoder and its int8 GEMMs (oracle/_ref/libphonon2_ref_neon.so, through oracle/neon_emu).

Tolerances. The five-value GEMMs are bit-exact (tests/test_gemm_gpu.py); the encoder as a whole cannot be, because the
compiled reference's LayerNorm takes 1/sqrt from an approximate reciprocal square root refined by one Newton step and
some of its exps from a vectorised libm, both host-CPU specific. So:
  * exact mode: max |device - reference| <= 1e-4 * max |reference| over the [T', 640] output (the north star's 1e-4);
  * int8 modes: statistical (see the test's docstring): an ulp-level difference before a quantiser can move one int8
    value by a whole step, which the following layers carry and multiply;
  * the row ops: allclose at a few fp32 ulp, quantised rows equal except for rare one-step differences.
Batched windows are compared bit for bit with the same windows run one at a time (every GEMM is row-independent and
every cross-row op stops at window edges).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

EXACT_TOL = 1e-4


@pytest.fixture(scope="module")
def model(pkg):
    from phonon2_b200 import model as M
    return M.SyntheticModel(seed=7)


@pytest.fixture(scope="module")
def dev_model(pkg, cuda, model):
    d = pkg.DeviceModel(model.struct)
    yield d
    d.close()


def _run(pkg, torch, dev_model, mels, mode, chunk=0, overlap=8):
    """One plan over the windows `mels`: the per-window [T', 640] outputs."""
    from phonon2_b200.device import device_view
    enc = pkg.Encoder(dev_model, [m.shape[0] for m in mels], mode, chunk, overlap)
    stacked = np.ascontiguousarray(np.concatenate(mels), np.float32)
    device_view(enc.mel_ptr, stacked.shape).copy_(torch.from_numpy(stacked))
    enc.run()
    pkg.check_device()
    out = device_view(enc.out_ptr, (enc.total_frames, 640)).cpu().numpy()
    offs = np.cumsum([0] + enc.frames)
    res = [out[offs[i]:offs[i + 1]] for i in range(len(mels))]
    enc.close()
    return res


def _rel(got, ref):
    return float(np.abs(got - ref).max() / np.abs(ref).max())


def _elementwise_rel(got, ref):
    """Percentiles (50, 99, 99.9, 100) of |got - ref| / |ref| over the outputs with |ref| >= 1 % of max |ref| (an
    element-wise relative error is meaningless at values near zero), and the share of outputs that covers."""
    big = np.abs(ref) >= 1e-2 * np.abs(ref).max()
    r = np.abs(got - ref)[big] / np.abs(ref)[big]
    return [float(np.percentile(r, q)) for q in (50, 99, 99.9, 100)], float(big.mean())


# ---- the row ops against the reference's own functions -------------------------------------------------------------

def test_layer_norm_rows(pkg, orc, cuda):
    import torch
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((300, 1024)) * 3 + 0.5).astype(np.float32)
    g = (1 + 0.02 * rng.standard_normal(1024)).astype(np.float32)
    b = (0.02 * rng.standard_normal(1024)).astype(np.float32)
    xd, gd, bd = (torch.from_numpy(a).to(cuda) for a in (x, g, b))
    out = torch.empty_like(xd)
    pkg.check(pkg.lib().p2cu_layer_norm_rows(xd.data_ptr(), gd.data_ptr(), bd.data_ptr(), out.data_ptr(), 300, 1024,
                                             None))
    ref = orc.ref_layer_norm_rows(x, g, b)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=2e-6, atol=2e-6)
    # in place (p2_layer_norm_rows_inplace)
    pkg.check(pkg.lib().p2cu_layer_norm_rows(xd.data_ptr(), gd.data_ptr(), bd.data_ptr(), xd.data_ptr(), 300, 1024,
                                             None))
    assert np.array_equal(xd.cpu().numpy(), out.cpu().numpy())


def _quant_close(q, s, rq, rs):
    np.testing.assert_allclose(s, rs, rtol=2e-6)
    d = np.abs(q.astype(np.int32) - rq.astype(np.int32))
    assert d.max() <= 1 and (d != 0).mean() < 1e-3, (d.max(), (d != 0).mean())


def test_layer_norm_quant_rows(pkg, orc, cuda):
    import torch
    rng = np.random.default_rng(2)
    x = (rng.standard_normal((200, 1024)) * 2).astype(np.float32)
    g = (1 + 0.02 * rng.standard_normal(1024)).astype(np.float32)
    b = (0.02 * rng.standard_normal(1024)).astype(np.float32)
    xd, gd, bd = (torch.from_numpy(a).to(cuda) for a in (x, g, b))
    q = torch.empty((200, 1024), dtype=torch.int8, device=cuda)
    s = torch.empty(200, dtype=torch.float32, device=cuda)
    pkg.check(pkg.lib().p2cu_layer_norm_quant_rows(xd.data_ptr(), gd.data_ptr(), bd.data_ptr(), q.data_ptr(),
                                                   s.data_ptr(), 200, 1024, None))
    rq, rs = orc.ref_layer_norm_quant_rows(x, g, b)
    _quant_close(q.cpu().numpy(), s.cpu().numpy(), rq, rs)


def test_swish_and_swish_quant(pkg, orc, cuda):
    import torch
    rng = np.random.default_rng(3)
    h = (rng.standard_normal((64, 4096)) * 4).astype(np.float32)
    hd = torch.from_numpy(h.copy()).to(cuda)
    pkg.check(pkg.lib().p2cu_swish(hd.data_ptr(), h.size, None))
    np.testing.assert_allclose(hd.cpu().numpy(), orc.ref_swish(h), rtol=1e-6, atol=1e-7)
    hd = torch.from_numpy(h).to(cuda)
    q = torch.empty((64, 4096), dtype=torch.int8, device=cuda)
    s = torch.empty(64, dtype=torch.float32, device=cuda)
    pkg.check(pkg.lib().p2cu_swish_quant_rows(hd.data_ptr(), q.data_ptr(), s.data_ptr(), 64, 4096, None))
    rq, rs = orc.ref_swish_quant_rows(h)
    _quant_close(q.cpu().numpy(), s.cpu().numpy(), rq, rs)


@pytest.mark.parametrize("length", [375, 38, 64, 7])
def test_softmax_rows(pkg, orc, cuda, length):
    import torch
    x = (np.random.default_rng(length).standard_normal((96, length)) * 4).astype(np.float32)
    xd = torch.from_numpy(x.copy()).to(cuda)
    pkg.check(pkg.lib().p2cu_softmax_rows(xd.data_ptr(), 96, length, None))
    np.testing.assert_allclose(xd.cpu().numpy(), orc.ref_softmax_rows(x), rtol=2e-6, atol=1e-8)


@pytest.mark.parametrize("T", [375, 38, 7, 13, 1])
def test_depthwise_conv1d(pkg, orc, cuda, T):
    import torch
    rng = np.random.default_rng(T)
    Cn = 1024
    x = rng.standard_normal((T, Cn)).astype(np.float32)   # time-major
    w = (rng.standard_normal((Cn, 9)) / 3).astype(np.float32)
    b = (0.02 * rng.standard_normal(Cn)).astype(np.float32)
    xd, wd, bd = (torch.from_numpy(a).to(cuda) for a in (x, w, b))
    out = torch.empty_like(xd)
    pkg.check(pkg.lib().p2cu_depthwise_conv1d_rows(xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), out.data_ptr(), Cn,
                                                   T, None))
    ref = orc.ref_depthwise_conv1d(x.T, w, b).T
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-6, atol=1e-6)


# ---- the encoder ---------------------------------------------------------------------------------------------------

@pytest.mark.parametrize("n_mel", [300, 3000])   # config 4 (T' = 38) and config 2 (T' = 375)
def test_encoder_exact_matches_reference(pkg, orc, cuda, model, dev_model, n_mel):
    import torch
    from phonon2_b200 import model as M
    mel = M.mel(n_mel, seed=n_mel)
    got, = _run(pkg, torch, dev_model, [mel], pkg.EXACT)
    ref = orc.ref_encoder(model.struct, mel, "exact")
    assert got.shape == ref.shape == (M.frames_after_subsampling(n_mel), 640)
    pct, share = _elementwise_rel(got, ref)
    print(f"exact T'={got.shape[0]}: normwise {_rel(got, ref):.2e}; element-wise relative p50 {pct[0]:.2e} "
          f"p99 {pct[1]:.2e} p99.9 {pct[2]:.2e} max {pct[3]:.2e} over {100 * share:.1f} % of the outputs")
    assert _rel(got, ref) <= EXACT_TOL, _rel(got, ref)


@pytest.mark.parametrize("mode", ["int8w", "int8"])
def test_encoder_int8_matches_reference_control_flow(pkg, orc, cuda, model, dev_model, mode):
    """Statistical parity: quantisation makes the int8 encoder sensitive to ulp-level differences before a quantiser
    (one flipped rounding moves an activation by a whole step, and 24 blocks carry and multiply such steps), so two
    valid int8 encoders - the reference built on two different CPUs, for one - agree only to about the size of the
    quantisation noise itself. The device's int8 output must sit within that envelope of the reference's int8 output
    (the distance between the reference's int8 and exact outputs), and correlate with it almost perfectly."""
    import torch
    from phonon2_b200 import model as M
    mel = M.mel(300, seed=11)
    got, = _run(pkg, torch, dev_model, [mel], pkg.MODES[mode])
    ref = orc.ref_encoder(model.struct, mel, mode)
    exact = orc.ref_encoder(model.struct, mel, "exact")
    noise = _rel(ref, exact)
    print(f"{mode}: device vs reference {_rel(got, ref):.3e}, device vs exact {_rel(got, exact):.3e}, "
          f"reference int8 vs exact {noise:.3e}, corr {np.corrcoef(got.ravel(), ref.ravel())[0, 1]:.6f}")
    assert noise < 0.1
    assert _rel(got, ref) <= 2 * noise and _rel(got, exact) <= 2 * noise
    assert np.corrcoef(got.ravel(), ref.ravel())[0, 1] > 0.999
    if orc.ref_neon_available():   # the reference's own AArch64 int8 encoder (oracle/neon_emu), same envelope
        arm = orc.ref_neon_encoder(model.struct, mel, mode)
        print(f"{mode}: device vs the reference's AArch64 build {_rel(got, arm):.3e}, "
              f"corr {np.corrcoef(got.ravel(), arm.ravel())[0, 1]:.6f}")
        assert _rel(got, arm) <= 2 * noise
        assert np.corrcoef(got.ravel(), arm.ravel())[0, 1] > 0.999


def test_encoder_int8w_config2_window(pkg, orc, cuda, model, dev_model):
    """The same statistical parity on one 30 s window (3000 mel frames, T' = 375), int8w, against
    both int8 oracles: the restated-GEMM control flow and the reference's own AArch64 build."""
    import torch
    from phonon2_b200 import model as M
    mel = M.mel(3000, seed=12)
    got, = _run(pkg, torch, dev_model, [mel], pkg.INT8W)
    exact = orc.ref_encoder(model.struct, mel, "exact")
    refs = [orc.ref_encoder(model.struct, mel, "int8w")]
    if orc.ref_neon_available():
        refs.append(orc.ref_neon_encoder(model.struct, mel, "int8w"))
    noise = _rel(refs[0], exact)
    assert got.shape == (375, 640) and 1e-3 < noise < 0.1
    assert _rel(got, exact) <= 2 * noise
    for ref in refs:
        print(f"T'=375 int8w: device vs reference {_rel(got, ref):.3e} (noise {noise:.3e}), "
              f"corr {np.corrcoef(got.ravel(), ref.ravel())[0, 1]:.6f}")
        assert _rel(got, ref) <= 2 * noise
        assert np.corrcoef(got.ravel(), ref.ravel())[0, 1] > 0.999


@pytest.mark.parametrize("mode", ["int8w", "exact"])
def test_windows_batched_equal_windows_alone(pkg, cuda, dev_model, mode):
    import torch
    from phonon2_b200 import model as M
    mels = [M.mel(n, seed=n) for n in (300, 251, 333, 17)]
    together = _run(pkg, torch, dev_model, mels, pkg.MODES[mode])
    for mel, got in zip(mels, together):
        alone, = _run(pkg, torch, dev_model, [mel], pkg.MODES[mode])
        assert np.array_equal(got.view(np.uint32), alone.view(np.uint32))


def test_chunked_encoder_matches_reference(pkg, orc, cuda, model, dev_model):
    import torch
    from phonon2_b200 import model as M
    mel = M.mel(4500, seed=3)   # T' = 563 > 500: the reference chunks (400 frames + 8 of context each side)
    ref = orc.ref_encoder(model.struct, mel, "exact")
    got, = _run(pkg, torch, dev_model, [mel], pkg.EXACT, chunk=400, overlap=8)
    assert _rel(got, ref) <= EXACT_TOL, _rel(got, ref)
    full, = _run(pkg, torch, dev_model, [mel], pkg.EXACT)
    assert _rel(full, ref) > 10 * EXACT_TOL   # the chunk boundaries do change the result


def test_host_entry_point_matches_plan(pkg, cuda, model, dev_model):
    """p2_encoder (host pointers, the reference's signature) gives the plan's output bit for bit."""
    import torch
    from phonon2_b200 import model as M
    mel = M.mel(300, seed=21)
    got = pkg.host_encoder(model.struct, mel)
    mode = pkg.MODES["int8w"]   # the host entry's default mode (P2_GEMM unset)
    plan, = _run(pkg, torch, dev_model, [mel], mode)
    assert np.array_equal(got.view(np.uint32), plan.view(np.uint32))


def test_encoder_argument_errors(pkg, cuda, dev_model):
    with pytest.raises(pkg.Error):
        pkg.Encoder(dev_model, [0], pkg.INT8W)
    with pytest.raises(pkg.Error):
        pkg.Encoder(dev_model, [300], 7)


def test_failed_gpu_share_is_rerun_on_another(pkg, cuda, model, monkeypatch):
    """Failure detection on the host, no GPU disturbed: P2_B200_FAIL_SLOT=0 makes the first GPU's share report a
    failure before it runs anything; the batched entry points hand its windows to the other GPU of the list (GPU 0
    named twice: two host threads), and every window's frames and tokens equal those of a run without the failure, bit
    for bit. With one GPU listed, no GPU is left to take the share over and the call fails."""
    from phonon2_b200 import model as M
    mels = [M.mel(n, seed=n) for n in (300, 251, 333, 17)]
    want = pkg.host_encode_windows(model.struct, mels, devices=[0, 0])
    want_tok = pkg.host_transcribe_windows(model.struct, mels, devices=[0, 0])
    monkeypatch.setenv("P2_B200_FAIL_SLOT", "0")
    got = pkg.host_encode_windows(model.struct, mels, devices=[0, 0])
    for g, w in zip(got, want):
        assert np.array_equal(g.view(np.uint32), w.view(np.uint32))
    got_tok = pkg.host_transcribe_windows(model.struct, mels, devices=[0, 0])
    assert all(np.array_equal(g, w) for g, w in zip(got_tok, want_tok))
    with pytest.raises(pkg.Error):
        pkg.host_encode_windows(model.struct, mels, devices=[0])


def test_encode_windows_spread_over_devices(pkg, cuda, model):
    """p2_b200_encode_windows gives every window exactly what p2_encoder gives it. The device list names GPU 0 twice,
    so the sharding, the per-GPU threads and the per-GPU plan cache run on a one-GPU box too."""
    from phonon2_b200 import model as M
    mels = [M.mel(n, seed=n) for n in (300, 251, 333, 17, 290)]
    got = pkg.host_encode_windows(model.struct, mels, devices=[0, 0])
    again = pkg.host_encode_windows(model.struct, mels, devices=[0, 0])   # from the cached plans
    for mel, g, a in zip(mels, got, again):
        one = pkg.host_encoder(model.struct, mel)
        assert np.array_equal(g.view(np.uint32), one.view(np.uint32))
        assert np.array_equal(a.view(np.uint32), one.view(np.uint32))


@pytest.mark.parametrize("path", ["tc_fused", "tc", "simt", "fused"])
def test_attention_paths_match_reference(pkg, orc, cuda, model, dev_model, path, monkeypatch):
    """Each attention implementation (the fused tensor-core kernel, the tensor-core products with the scores in
    device memory, SIMT grouped GEMMs, the fused SIMT kernel) gives the exact-mode encoder within 1e-4 of the
    reference (P2CU_ATTN chooses; the plan reads it)."""
    import torch
    from phonon2_b200 import model as M
    monkeypatch.setenv("P2CU_ATTN", path)
    mel = M.mel(1000, seed=9)   # T' = 125
    got, = _run(pkg, torch, dev_model, [mel], pkg.EXACT)
    ref = orc.ref_encoder(model.struct, mel, "exact")
    assert _rel(got, ref) <= EXACT_TOL, _rel(got, ref)
