"""CPU checks of the encoder's test infrastructure: the ctypes P2Model mirror against the C header, and the reference
encoder oracles (phonon-2-c's own p2_encoder, and the same sources with the int8 GEMMs restated)."""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def _c_layout(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(r'''
#include <stdio.h>
#include <stddef.h>
#include "phonon2.h"
int main(void) {
    printf("%zu %zu %zu %zu %zu %zu %zu %zu %zu %zu\n", sizeof(Weight), offsetof(Weight, f32), offsetof(Weight, codes),
           sizeof(SubsamplingWeights), sizeof(ConformerBlock), offsetof(ConformerBlock, mha),
           offsetof(ConformerBlock, conv), sizeof(EncoderWeights), sizeof(DecoderWeights), sizeof(P2Model));
    return 0;
}
''')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    return [int(v) for v in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]


def test_model_struct_layout_matches_header(pkg, tmp_path):
    from phonon2_b200 import model as M
    want = _c_layout(tmp_path)
    got = [C.sizeof(M.Weight), M.Weight.f32.offset, M.Weight.codes.offset, C.sizeof(M.SubsamplingWeights),
           C.sizeof(M.ConformerBlock), M.ConformerBlock.mha.offset, M.ConformerBlock.conv.offset,
           C.sizeof(M.EncoderWeights), C.sizeof(M.DecoderWeights), C.sizeof(M.P2Model)]
    assert got == want


def test_synthetic_model_shapes_and_seed(pkg):
    from phonon2_b200 import model as M
    a, b = M.SyntheticModel(seed=3), M.SyntheticModel(seed=3)
    w = a.struct.enc.blocks[5].ff1.linear2_w
    assert (w.kind, w.K, w.N) == (M.W_FV, 4096, 1024)
    assert a.struct.enc.projector_w.kind == M.W_I8 and a.struct.enc.projector_w.N == 640
    name = "layers.5.feed_forward1.linear2.weight"
    assert np.array_equal(a.five_value(name)["signs"], b.five_value(name)["signs"])
    assert a.nbytes > 225e6   # 226.5 MB of planes plus the rest
    assert M.frames_after_subsampling(3000) == 375 and M.frames_after_subsampling(300) == 38


@pytest.fixture(scope="module")
def small_model(pkg):
    from phonon2_b200 import model as M
    return M.SyntheticModel(seed=5)


def test_reference_encoder_runs(orc, small_model):
    from phonon2_b200 import model as M
    mel = M.mel(300, seed=1)
    out = orc.ref_encoder(small_model.struct, mel, "exact")
    assert out.shape == (38, 640) and np.isfinite(out).all() and 0.1 < out.std() < 10


def test_int8_oracle_in_exact_mode_is_the_reference(orc, small_model):
    """With the shim in exact mode every GEMM forwards to the reference's own code: bit-identical outputs."""
    from phonon2_b200 import model as M
    mel = M.mel(120, seed=2)
    ref = orc.ref_encoder(small_model.struct, mel, "exact")
    L = orc.ref_i8()
    L.orc_shim_set_mode(1)
    out, n = C.c_void_p(), C.c_int()
    assert L.p2_encoder(C.addressof(small_model.struct), np.ascontiguousarray(mel), mel.shape[0], C.byref(out),
                        C.byref(n)) == 0
    got = np.ctypeslib.as_array(C.cast(out, C.POINTER(C.c_float)), shape=(n.value, 640)).copy()
    orc._libc.free(out)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("mode", ["int8w", "int8"])
def test_int8_oracle_tracks_exact(orc, small_model, mode):
    """The int8 control flow differs from exact only by quantisation: a few percent of the output's range."""
    from phonon2_b200 import model as M
    mel = M.mel(120, seed=3)
    ex = orc.ref_encoder(small_model.struct, mel, "exact")
    i8 = orc.ref_encoder(small_model.struct, mel, mode)
    rel = np.abs(i8 - ex).max() / np.abs(ex).max()
    assert 1e-4 < rel < 0.1, rel
