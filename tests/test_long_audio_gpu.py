"""Long audio on the device against phonon-2-c's own segmenter and engine (oracle/_ref/libphonon2_ref.so, compiled from
its sources): the block RMS kernel against p2_block_rms, p2_b200_plan_windows / p2_b200_split_point against
p2_plan_windows / p2_split_point, and p2_b200_transcribe_long - every split depth's windows decoded as one batch -
against the reference's p2_transcribe on the same model (a model directory in the reference's format, the decoder
tables as its loader expands them) in exact mode: the same segments (start, end, token ranges), the same tokens (id,
frame in the whole audio, duration) and the same encoder frame count, with the re-decode recursion two levels deep."""
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
SR = 16000


@pytest.fixture(scope="module")
def ref(orc):
    if not orc.ref_available():
        pytest.skip("oracle/_ref/libphonon2_ref.so not built")
    return orc


def test_block_rms_matches_reference(pkg, ref, cuda):
    import torch
    from phonon2_b200 import model as M
    x = M.audio_with_pauses(40.0, 11)
    x[5000:5100] = 0.0
    dx = torch.from_numpy(x).to(cuda)
    rng = np.random.default_rng(3)
    spans = [(0, x.shape[0]), (0, 799), (1, 800), (123457, 801), (400, 0), (17, 5 * SR + 3)]
    spans += [(int(a), int(rng.integers(0, x.shape[0] - a))) for a in rng.integers(0, x.shape[0] - 1, 40)]
    starts = np.array([s for s, _ in spans], np.int64)
    lens = np.array([n for _, n in spans], np.int32)
    L = pkg.lib()
    nb = [L.p2cu_seg_blocks(int(n), SR) for n in lens]
    out = torch.full((sum(nb),), -1.0, device=cuda)
    import ctypes as C
    rc = L.p2cu_block_rms(dx.data_ptr(), starts.ctypes.data_as(C.POINTER(C.c_longlong)),
                          lens.ctypes.data_as(C.POINTER(C.c_int)), len(spans), SR, out.data_ptr(), None)
    assert rc == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    at, diff, total = 0, 0, 0
    for (s, n), k in zip(spans, nb):
        want = ref.ref_block_rms(x[s:s + n])
        assert want.shape[0] == k
        g = got[at:at + k]
        # the same double sum in another order: equal floats but for (very rare) one-ulp ties
        ulps = np.abs(g.view(np.int32).astype(np.int64) - want.view(np.int32).astype(np.int64))
        assert ulps.max(initial=0) <= 1
        diff += int((ulps > 0).sum())
        total += k
        at += k
    assert diff <= max(1, total // 10000)


@pytest.mark.parametrize("seconds,seed", [(36.0, 1), (95.0, 3), (181.3, 4), (300.0, 9)])
def test_plan_windows_matches_reference(pkg, ref, cuda, seconds, seed):
    from phonon2_b200 import model as M
    x = M.audio_with_pauses(seconds, seed)
    assert pkg.host_plan_windows(x) == ref.ref_plan_windows(x)


def test_plan_windows_window_max(pkg, ref, cuda, monkeypatch):
    from phonon2_b200 import model as M
    x = M.audio_with_pauses(120.0, 8)
    for v in ("20", "35.37", "60"):
        monkeypatch.setenv("P2_WINDOW_MAX", v)
        assert pkg.host_plan_windows(x) == ref.ref_plan_windows(x)
    monkeypatch.delenv("P2_WINDOW_MAX")
    assert pkg.host_plan_windows(x[:100]) == [(0, 100)]
    assert pkg.host_plan_windows(x[:0]) == []


@pytest.mark.parametrize("seed", range(6))
def test_split_point_matches_reference(pkg, ref, cuda, seed):
    from phonon2_b200 import model as M
    rng = np.random.default_rng(seed)
    x = M.audio_with_pauses(rng.uniform(12.0, 36.0), 50 + seed, pause_hi=rng.uniform(0.1, 1.5))
    assert pkg.host_split_point(x) == ref.ref_split_point(x)


# ---- the scheduling, end to end ---------------------------------------------------------------------------------

CHILD = r"""
import json, os, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
import __graft_entry__ as ge
pkg = ge.load_package()
from oracle import weights_file as wf
from phonon2_b200 import model as M
m = wf.as_loaded(M.SyntheticModel(seed=1))
jobs = json.load(open(sys.argv[2]))
res = []
for job in jobs:
    for k in ("P2_SEGMENT", "P2_REDECODE"):
        os.environ.pop(k, None)
    os.environ.update(job["env"])
    x = np.load(job["audio"])
    wins, frames = pkg.host_transcribe_long(m.struct, x, devices=job["devices"])
    res.append({"windows": [{"start": w["start"], "end": w["end"], "depth": w["depth"],
                             "encoder_frames": w["encoder_frames"], "tokens": w["tokens"].tolist()} for w in wins],
                "frames": frames})
json.dump(res, open(sys.argv[3], "w"))
"""


def _cases():
    from phonon2_b200 import model as M
    x_nan = M.audio_with_pauses(20.0, 21)
    x_nan[::997] = np.nan
    x_nan[5] = np.inf
    return {
        "pauses 70 s": (M.audio_with_pauses(70.0, 5), {}, [0]),
        "syllables 70 s": (M.audio(70 * SR, seed=70), {}, [0]),
        "syllables 70 s, GPU 0 twice": (M.audio(70 * SR, seed=70), {}, [0, 0]),
        "pauses 70 s, no re-decode": (M.audio_with_pauses(70.0, 5), {"P2_REDECODE": "0"}, [0]),
        "pauses 45 s, not segmented": (M.audio_with_pauses(45.0, 6), {"P2_SEGMENT": "off"}, [0]),
        "non-finite samples": (x_nan, {}, [0]),
        "shorter than a frame": (M.audio(1000, seed=1), {}, [0]),
        "empty": (np.zeros(0, np.float32), {}, [0]),
        "empty, not segmented": (np.zeros(0, np.float32), {"P2_SEGMENT": "0"}, [0]),
    }


@pytest.fixture(scope="module")
def long_runs(pkg, ref, cuda, tmp_path_factory):
    """Every case through p2_b200_transcribe_long in a child process with P2_GEMM=exact (the GEMM mode is read once
    per process), and through the reference's p2_transcribe here."""
    from oracle import weights_file as wf
    from phonon2_b200 import model as M
    d = tmp_path_factory.mktemp("long")
    model_dir = wf.write_model_dir(M.SyntheticModel(seed=1), d / "model")
    cases = _cases()
    assert list(cases) == CASE_NAMES
    jobs = []
    for i, (name, (x, env, devs)) in enumerate(cases.items()):
        np.save(d / f"a{i}.npy", x)
        jobs.append({"audio": str(d / f"a{i}.npy"), "env": env, "devices": devs})
    (d / "jobs.json").write_text(json.dumps(jobs))
    env = dict(os.environ, P2_GEMM="exact")
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), str(d / "jobs.json"), str(d / "out.json")], env=env,
                       capture_output=True, text=True, timeout=1200)
    assert r.returncode == 0, r.stderr[-3000:]
    ours = json.loads((d / "out.json").read_text())
    refs = {}
    for name, (x, env_case, _) in cases.items():
        saved = {k: os.environ.get(k) for k in ("P2_SEGMENT", "P2_REDECODE")}
        try:
            for k in saved:
                os.environ.pop(k, None)
            os.environ.update(env_case)
            refs[name] = ref.ref_transcribe(model_dir, x)
        finally:
            for k, v in saved.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v
    return {name: (cases[name][0], ours[i], refs[name]) for i, name in enumerate(cases)}


CASE_NAMES = ["pauses 70 s", "syllables 70 s", "syllables 70 s, GPU 0 twice", "pauses 70 s, no re-decode",
              "pauses 45 s, not segmented", "non-finite samples", "shorter than a frame", "empty",
              "empty, not segmented"]


@pytest.mark.parametrize("name", CASE_NAMES)
def test_transcribe_long_matches_reference_engine(long_runs, name):
    x, ours, want = long_runs[name]
    wins = ours["windows"]
    # the windows as the reference's segments: start and end in seconds, token ranges
    segs, toks = [], []
    for w in wins:
        off = int(w["start"] / 1280.0 + 0.5)
        segs.append((np.float32(w["start"] / SR), np.float32(w["end"] / SR), len(toks), len(w["tokens"])))
        toks += [(t[0], t[1] + off, t[2]) for t in w["tokens"]]
    assert len(segs) == len(want["segments"])
    for g, r in zip(segs, want["segments"]):
        assert (g[0], g[1], g[2], g[3]) == (np.float32(r[0]), np.float32(r[1]), r[2], r[3])
    assert np.array_equal(np.array(toks, np.int32).reshape(-1, 3), want["tokens"])
    assert ours["frames"] == want["encoder_frames"]
    # the windows tile the audio, in order
    if wins:
        assert wins[0]["start"] == 0 and wins[-1]["end"] == x.shape[0]
        assert all(a["end"] == b["start"] for a, b in zip(wins, wins[1:]))


def test_transcribe_long_recursion_depth(long_runs):
    """The cases exercise the recursion: windows split once and twice, and not at all without re-decoding."""
    depths = {name: {w["depth"] for w in long_runs[name][1]["windows"]} for name in long_runs}
    assert 2 in depths["syllables 70 s"]
    assert depths["pauses 70 s, no re-decode"] == {0}
    assert depths["pauses 45 s, not segmented"] == {2}
