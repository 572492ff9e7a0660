"""The segmenter's decisions (segment.cu, host code) against phonon-2-c's own csrc/segment.c compiled from its sources
(oracle/_ref/libphonon2_ref.so), given the same block RMS - the reference's p2_block_rms - so that the comparison is of
the decision logic alone: where a window ends (p2_first_cut, and p2_plan_windows by chaining it), where a quiet window
is split (p2_split_point), the speech gate and share, and the engine's dropout test (csrc/engine.c:224-251, restated in
the oracle over the reference's energy functions). The device block RMS and the scheduling are covered by
tests/test_long_audio_gpu.py."""
import ctypes as C

import numpy as np
import pytest

SR = 16000


@pytest.fixture(scope="module")
def ref(orc):
    if not orc.ref_available():
        pytest.skip("oracle/_ref/libphonon2_ref.so not built")
    return orc


def speechy(seconds: float, seed: int, pause_lo=0.05, pause_hi=1.4) -> np.ndarray:
    from phonon2_b200 import model as M
    return M.audio_with_pauses(seconds, seed, pause_lo, pause_hi)


def _f(a):
    a = np.ascontiguousarray(a, np.float32)
    return a, a.ctypes.data


CASES = [(36.0, 1), (47.5, 2), (95.0, 3), (181.3, 4), (70.0, 5)]


@pytest.mark.parametrize("seconds,seed", CASES)
@pytest.mark.parametrize("window_max", ["", "20", "35.37"])
def test_first_cut_and_plan(pkg, ref, monkeypatch, seconds, seed, window_max):
    if window_max:
        monkeypatch.setenv("P2_WINDOW_MAX", window_max)
    else:
        monkeypatch.delenv("P2_WINDOW_MAX", raising=False)
    L = pkg.lib()
    x = speechy(seconds, seed)
    single = L.p2cu_seg_window_max_samples(SR)
    plan, start = [], 0
    while True:
        rest = x[start:]
        if rest.shape[0] > single:
            rms, p = _f(ref.ref_block_rms(rest[:single]))
            cut = L.p2cu_seg_first_cut(p, rms.shape[0], rest.shape[0], SR)
        else:
            cut = L.p2cu_seg_first_cut(None, 0, rest.shape[0], SR)
        assert cut == ref.ref_first_cut(rest), (start, cut)
        plan.append((start, start + cut))
        if start + cut >= x.shape[0]:
            break
        start += cut
    assert plan == ref.ref_plan_windows(x)


def test_first_cut_without_pause(pkg, ref):
    """No block quiet enough in the band (steady loud signal): the cut falls on the target, 30 s."""
    L = pkg.lib()
    t = np.arange(40 * SR) / SR
    x = (0.5 * np.sin(2 * np.pi * 220 * t)).astype(np.float32)
    rms, p = _f(ref.ref_block_rms(x[: L.p2cu_seg_window_max_samples(SR)]))
    cut = L.p2cu_seg_first_cut(p, rms.shape[0], x.shape[0], SR)
    assert cut == ref.ref_first_cut(x) == 30 * SR


@pytest.mark.parametrize("seed", range(12))
def test_split_point(pkg, ref, seed):
    L = pkg.lib()
    rng = np.random.default_rng(100 + seed)
    x = speechy(rng.uniform(12.0, 36.0), seed, pause_hi=rng.uniform(0.1, 1.5))
    if seed == 0:
        x[:] = 0.3   # nothing quiet: the middle
    rms, p = _f(ref.ref_block_rms(x))
    got = L.p2cu_seg_split_point(p, rms.shape[0], x.shape[0], SR)
    assert got == ref.ref_split_point(x)


@pytest.mark.parametrize("seed", range(8))
def test_speech_gate_and_share(pkg, ref, seed):
    L = pkg.lib()
    rng = np.random.default_rng(200 + seed)
    x = speechy(rng.uniform(3.0, 40.0), seed)
    rms, p = _f(ref.ref_block_rms(x))
    gate = L.p2cu_seg_speech_gate(p, rms.shape[0])
    assert np.float32(gate) == np.float32(ref.ref_speech_gate(rms))
    for _ in range(20):
        a, b = sorted(int(v) for v in rng.integers(0, x.shape[0] + 2000, 2))
        assert (np.float32(L.p2cu_seg_speech_share(p, rms.shape[0], SR, a, b, C.c_float(gate))) ==
                np.float32(ref.ref_speech_share(rms, a, b, gate)))
    assert L.p2cu_seg_speech_gate(p, 0) == pytest.approx(0.004)


def _tokens(rng, n_samples, density):
    """Sorted synthetic tokens (id, frame, duration) over a window with about `density` tokens per second in runs."""
    frames = n_samples // 1280
    out, f = [], 0
    while f < frames:
        if rng.random() < 0.15:
            f += int(rng.integers(10, 60))     # a gap of 0.8-4.8 s
            continue
        d = int(rng.integers(0, 5))
        out.append((int(rng.integers(0, 8192)), f, d))
        f += max(d, 1) + (int(rng.integers(0, 8)) if rng.random() < 1.0 / max(density, 0.1) else 0)
    return np.array(out, np.int32).reshape(-1, 3)


@pytest.mark.parametrize("seed", range(16))
def test_dropped_out(pkg, ref, seed):
    L = pkg.lib()
    rng = np.random.default_rng(300 + seed)
    x = speechy(rng.uniform(10.0, 36.0), seed)
    toks = _tokens(rng, x.shape[0], rng.uniform(0.5, 4.0))
    if seed == 0:
        toks = toks[:0]
    rms, p = _f(ref.ref_block_rms(x))
    tk = np.ascontiguousarray(toks)
    gf, gt, sp = C.c_int(-1), C.c_int(-1), C.c_float(-1)
    got = L.p2cu_seg_dropped_out(p, rms.shape[0], x.shape[0], tk.ctypes.data, tk.shape[0], C.byref(gf), C.byref(gt),
                                 C.byref(sp))
    want = ref.ref_dropped_out(x, toks)
    assert bool(got) == (want is not None)
    if want is not None:
        assert (gf.value, gt.value) == want[:2] and np.float32(sp.value) == np.float32(want[2])
    has_gap = L.p2cu_seg_long_gap(tk.ctypes.data, tk.shape[0], x.shape[0])
    assert has_gap or not got


def test_long_gap_edges(pkg):
    """A stretch of exactly 2 s counts, one sample less does not; a duration of 0 advances one frame."""
    L = pkg.lib()
    t = np.array([[5, 25, 0]], np.int32)    # 25 frames = 32000 samples: a 2 s stretch before it
    assert L.p2cu_seg_long_gap(t.ctypes.data, 1, 32000 + 1280 + 31999) == 1
    t = np.array([[5, 24, 0], [6, 25, 0]], np.int32)
    assert L.p2cu_seg_long_gap(t.ctypes.data, 2, 25 * 1280 + 1280 + 31999) == 0
    assert L.p2cu_seg_long_gap(t.ctypes.data, 2, 25 * 1280 + 1280 + 32000) == 1
    assert L.p2cu_seg_long_gap(None, 0, 31999) == 0
    assert L.p2cu_seg_long_gap(None, 0, 32000) == 1


def _scene(parts, seed):
    """Audio from (kind, seconds) parts - "speech" (tokens every 2-6 frames), "silent" speech (no tokens), "pause"
    (low noise) or "tone" (a steady loud tone) - and its tokens (id, frame, duration)."""
    from phonon2_b200 import model as M
    rng = np.random.default_rng(seed)
    audio, toks, n = [], [], 0
    for kind, sec in parts:
        k = int(sec * SR)
        if kind in ("speech", "silent"):
            audio.append(M.audio(k, int(rng.integers(1 << 30))) * rng.uniform(0.3, 1.0))
            if kind == "speech":
                f = (n + 1279) // 1280
                while (f + 1) * 1280 < n + k:
                    d = int(rng.integers(0, 3))
                    toks.append((int(rng.integers(0, 8192)), f, d))
                    f += max(d, 1) + int(rng.integers(1, 5))
        elif kind == "pause":
            audio.append((rng.standard_normal(k) * 0.0005).astype(np.float32))
        else:
            audio.append((0.4 * np.sin(2 * np.pi * 440 * np.arange(k) / SR)).astype(np.float32))
        n += k
    return np.concatenate(audio).astype(np.float32), np.array(toks, np.int32).reshape(-1, 3)


SCENES = {
    "quiet over speech": ([("speech", 4), ("silent", 3.5), ("speech", 3), ("pause", 0.5), ("speech", 3)], True),
    "real pauses": ([("speech", 3), ("pause", 2.6), ("speech", 4), ("pause", 3.1), ("speech", 2.5)], False),
    "tone": ([("speech", 3), ("pause", 1), ("speech", 2), ("tone", 3.5), ("speech", 4)], False),
    "dense": ([("speech", 5), ("pause", 0.8), ("speech", 6), ("pause", 1.2), ("speech", 4)], False),
    "quiet at the end": ([("speech", 5), ("pause", 1.0), ("speech", 3), ("silent", 4)], True),
    "quiet from the start": ([("silent", 3), ("speech", 4), ("pause", 1.0), ("speech", 6)], True),
}


@pytest.mark.parametrize("name", list(SCENES))
def test_dropped_out_scenes(pkg, ref, name):
    """Stretches without tokens over speech (a dropout), over real pauses and over a steady tone (not one)."""
    L = pkg.lib()
    parts, expect = SCENES[name]
    x, toks = _scene(parts, len(name))
    rms, p = _f(ref.ref_block_rms(x))
    got = L.p2cu_seg_dropped_out(p, rms.shape[0], x.shape[0], toks.ctypes.data, toks.shape[0], None, None, None)
    want = ref.ref_dropped_out(x, toks)
    assert bool(got) == (want is not None) == expect
