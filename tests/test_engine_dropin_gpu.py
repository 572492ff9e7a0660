"""The drop-in, end to end: phonon-2-c's own command-line program (csrc/main.c over engine.c, segment.c, wav.c, ...)
built twice by oracle/Makefile - on the reference's own sources (_ref/phonon2_cpu), and without blas.c, encoder.c,
decoder.c and mel.c, linked against libphonon2_b200.so (_ref/phonon2_b200) - transcribes the same WAV files with the
same synthetic model directory (oracle/weights_file.py; the speech-like model, model.SPEECH_ATTN_OUT_GAIN, on which
greedy decoding emits tokens). In exact mode (P2_GEMM=exact) the token ids must be identical and at least one per four
encoder frames: the engine's segmentation into windows, its dropout check and re-decodes, and the detokeniser run in
the reference's C either way, while log-mel, encoder and decoder run on the GPU in the second program.
"""
import os
import subprocess
import time
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
CPU_BIN = ROOT / "oracle" / "_ref" / "phonon2_cpu"
B200_BIN = ROOT / "oracle" / "_ref" / "phonon2_b200"


@pytest.fixture(scope="module")
def model_dir(pkg, tmp_path_factory):
    from oracle import weights_file as wf
    from phonon2_b200 import model as M
    d = tmp_path_factory.mktemp("model")
    wf.write_model_dir(M.SyntheticModel(seed=1, attn_out_gain=M.SPEECH_ATTN_OUT_GAIN), d)
    return d


def _run(binary, model_dir, wav, env_extra):
    env = dict(os.environ)
    env.update(env_extra)
    t = time.perf_counter()
    r = subprocess.run([str(binary), "--quiet", "--tokens", str(model_dir), str(wav)], capture_output=True, text=True,
                       env=env, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stdout.split(), time.perf_counter() - t


@pytest.mark.skipif(not (CPU_BIN.exists() and B200_BIN.exists()), reason="oracle/_ref programs not built")
@pytest.mark.parametrize("seconds", [3, 70])
def test_reference_program_on_library_matches_reference(pkg, cuda, model_dir, tmp_path, seconds):
    from oracle import weights_file as wf
    from phonon2_b200 import model as M
    wav = tmp_path / f"audio{seconds}.wav"
    wf.write_wav16(wav, M.audio(16000 * seconds, seed=seconds))
    want, t_cpu = _run(CPU_BIN, model_dir, wav, {})
    got, t_gpu = _run(B200_BIN, model_dir, wav, {"P2_GEMM": "exact"})
    print(f"{seconds} s: reference {t_cpu:.1f} s, reference program on the library {t_gpu:.1f} s (exact mode, "
          f"including start-up and weight upload); {len(want)} tokens")
    encoder_frames = M.frames_after_subsampling(seconds * 100)
    assert len(want) >= encoder_frames // 4, (len(want), encoder_frames)
    assert got == want


@pytest.mark.skipif(not B200_BIN.exists(), reason="oracle/_ref programs not built")
def test_reference_program_on_library_int8w(pkg, cuda, model_dir, tmp_path):
    """The default int8w mode through the same program: it runs and yields a transcript (the int8 encoder differs from
    the exact one by the quantisation, so no token equality is asked)."""
    from oracle import weights_file as wf
    from phonon2_b200 import model as M
    wav = tmp_path / "audio.wav"
    wf.write_wav16(wav, M.audio(16000 * 40, seed=4))
    tokens, _ = _run(B200_BIN, model_dir, wav, {"P2_GEMM": "int8w"})
    assert all(t.isdigit() for t in tokens)


BATCHED_BIN = ROOT / "oracle" / "_ref" / "phonon2_b200_batched"


@pytest.mark.skipif(not (CPU_BIN.exists() and BATCHED_BIN.exists()), reason="oracle/_ref programs not built")
def test_reference_engine_batched_over_gpu_slots(pkg, cuda, model_dir, tmp_path):
    """The reference's program with its engine edited as INTEGRATION.md describes
    (phonon-2-c_b200/integration/engine_gpu_windows.patch: p2_transcribe hands the recording to
    p2_b200_transcribe_long, which decodes every window - and every re-decode depth - as one batch spread over the
    GPUs) on two device slots (P2_DEVICES=0,0: GPU 0 listed twice, so each slot's share runs as its own batch, as on
    two GPUs): the same token ids as the unmodified program on the CPU, exact mode, and the library's log says that
    the 70 s recording's windows went over both slots."""
    from oracle import weights_file as wf
    from phonon2_b200 import model as M
    wav = tmp_path / "audio70.wav"
    wf.write_wav16(wav, M.audio(16000 * 70, seed=70))
    want, _ = _run(CPU_BIN, model_dir, wav, {})
    env = dict(os.environ, P2_GEMM="exact", P2_DEVICES="0,0")
    r = subprocess.run([str(BATCHED_BIN), "--tokens", str(model_dir), str(wav)], capture_output=True, text=True,
                       env=env, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "over 2 GPU slot(s) of 2 listed" in r.stderr, r.stderr[-2000:]
    assert len(want) >= M.frames_after_subsampling(70 * 100) // 4
    assert r.stdout.split() == want


@pytest.mark.skipif(not (CPU_BIN.exists() and B200_BIN.exists()), reason="oracle/_ref programs not built")
def test_stream_through_library_matches_reference(pkg, cuda, model_dir):
    """p2_stream_* (csrc/engine.c:364-497) through the reference's program linked against the library: 16-bit PCM
    on stdin (--stream --json), the engine cutting windows as the audio arrives and decoding each on the GPU. Exact
    mode: the same segments, words and times as the unmodified program on the CPU (the reference's own check of
    --stream, tests/check.py:142-189, compares the stream with the batch windows the same way)."""
    from phonon2_b200 import model as M
    x = M.audio(16000 * 75, seed=75)
    pcm = (np.clip(x, -1.0, 1.0) * 32767.0).astype("<i2").tobytes()
    out = []
    for binary, extra in ((CPU_BIN, {}), (B200_BIN, {"P2_GEMM": "exact"})):
        env = dict(os.environ, **extra)
        r = subprocess.run([str(binary), "--quiet", "--stream", "--json", str(model_dir)], input=pcm,
                           capture_output=True, env=env, timeout=900)
        assert r.returncode == 0, r.stderr[-2000:]
        out.append(r.stdout.decode().strip().splitlines())
    want, got = out
    assert len(want) >= 2, want   # 75 s: at least two finished windows
    assert got == want
