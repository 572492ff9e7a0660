"""The reference-facing ABI (include/blas.h): phonon-2-c's own function names on host pointers, run on the GPU.

Mirrors how the reference's callers use it (csrc/tensor_ops.c:30-63, csrc/encoder.c, csrc/bench_gemm.c): plain host
arrays in, results in host memory when the call returns. The GEMM mode comes from P2_GEMM / P2_EXACT, read once per
process as in the reference (csrc/blas.c:1027-1047), so each non-default mode runs in a child process.
"""
import ctypes as C
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _bits_equal(a, b):
    return np.array_equal(np.ascontiguousarray(a).view(np.uint32), np.ascontiguousarray(b).view(np.uint32))


def test_default_mode_is_int8w(pkg, cuda):
    assert b"int8 weights" in pkg.lib().p2_gemm_mode()
    assert pkg.lib().p2_gemm_exact() == 0


@pytest.mark.parametrize("M,K,N,alpha,beta", [(375, 1024, 4096, 1.0, 0.0), (375, 4096, 1024, 0.5, 1.0),
                                              (17, 1024, 640, 1.0, 0.0), (749, 1024, 1024, 1.0, 0.0)])
def test_p2_sgemm_fvb_int8w(pkg, orc, synth, cuda, M, K, N, alpha, beta):
    w = synth.five_value(K, N, seed=K + N)
    A = synth.activations(M, K, seed=M)
    C0 = np.random.default_rng(1).standard_normal((M, N)).astype(np.float32)
    got = pkg.host_sgemm_fvb(A, w, C0.copy(), alpha=alpha, beta=beta)
    want = orc.sgemm_i8(A, "int8w", C0.copy(), w=w, alpha=alpha, beta=beta)
    assert _bits_equal(got, want)
    again = pkg.host_sgemm_fvb(A, w, C0.copy(), alpha=alpha, beta=beta)   # the weight is now resident
    assert _bits_equal(again, want)


@pytest.mark.parametrize("M,K,N,alpha,beta", [(13, 1028, 48, 1.0, 0.0), (5, 100, 16, 0.5, 1.0)])
def test_p2_sgemm_fvb_any_reference_shape(pkg, orc, synth, cuda, M, K, N, alpha, beta):
    """Every shape the reference's int8 path takes (N % 16 == 0, K % 4 == 0), not only the tensor-core ones."""
    w = synth.five_value(K, N, seed=K + N)
    A = synth.activations(M, K, seed=M)
    C0 = np.random.default_rng(1).standard_normal((M, N)).astype(np.float32)
    got = pkg.host_sgemm_fvb(A, w, C0.copy(), alpha=alpha, beta=beta)
    want = orc.sgemm_i8(A, "int8w", C0.copy(), w=w, alpha=alpha, beta=beta)
    assert _bits_equal(got, want)


def test_strided_host_arrays(pkg, orc, synth, cuda):
    """lda > K and ldc > N, as the reference's row-major contract allows (csrc/blas.h:24-29)."""
    M, K, N = 40, 1024, 256
    w = synth.five_value(K, N, seed=2)
    big_A = synth.activations(M, K + 64, seed=3)
    A = big_A[:, :K]
    C_big = np.random.default_rng(4).standard_normal((M, N + 32)).astype(np.float32)
    want = orc.sgemm_i8(np.ascontiguousarray(A), "int8w", np.ascontiguousarray(C_big[:, :N]).copy(), w=w, beta=1.0)
    out = C_big.copy()
    pkg.host_sgemm_fvb(A, w, out[:, :N], beta=1.0)
    assert _bits_equal(np.ascontiguousarray(out[:, :N]), want)
    assert _bits_equal(out[:, N:], C_big[:, N:])   # columns beyond N untouched


def _pinned(a):
    """A page-locked copy of a float32 array (torch's pinned allocator), as a numpy view."""
    import torch
    t = torch.empty(a.shape, dtype=torch.float32, pin_memory=True)
    t.numpy()[...] = a
    return t, t.numpy()


@pytest.mark.parametrize("M,K,N,alpha,beta", [(520, 1024, 512, 1.0, 1.0), (375, 4096, 1024, 0.5, 1.0),
                                              (375, 1024, 4096, 1.0, 0.0), (192, 1024, 256, 1.0, 0.0)])
def test_page_locked_buffers(pkg, orc, synth, cuda, M, K, N, alpha, beta):
    """Page-locked A and C (as the bench's end-to-end leg passes them), ldc > N with the columns beyond N untouched;
    K > 1024 (the K-block workspace), alpha 1/2, beta 0 and 1."""
    w = synth.five_value(K, N, seed=11)
    A = synth.activations(M, K, seed=12)
    C_big = np.random.default_rng(13).standard_normal((M, N + 32)).astype(np.float32)
    ta, pa = _pinned(A)
    tc, pc = _pinned(C_big)
    pkg.host_sgemm_fvb(pa, w, pc[:, :N], alpha=alpha, beta=beta)
    want = orc.sgemm_i8(A, "int8w", np.ascontiguousarray(C_big[:, :N]).copy(), w=w, alpha=alpha, beta=beta)
    assert _bits_equal(np.ascontiguousarray(pc[:, :N]), want)
    assert _bits_equal(pc[:, N:], C_big[:, N:])


def test_quant_prepare_row_gemm(pkg, orc, synth, cuda):
    """p2_quant_prepare / p2_quant_row / p2_sgemm_fvb_q8a as csrc/encoder.c:330-348 drives them."""
    M, K, N = 375, 1024, 2048
    w = synth.five_value(K, N, seed=5)
    A = synth.activations(M, K, seed=6)
    qa = pkg.QuantA()
    assert pkg.lib().p2_quant_prepare(C.byref(qa), M, K) == 0
    for m in range(M):
        pkg.lib().p2_quant_row(C.byref(qa), m, A[m].ctypes.data)
    out = np.zeros((M, N), np.float32)
    b = pkg.host_five_value(w)
    pkg.lib().p2_sgemm_fvb_q8a(M, N, K, 1.0, C.byref(qa), C.byref(b), 0.0, out.ctypes.data, N)
    want = orc.sgemm_i8(A, "int8w", np.zeros((M, N), np.float32), w=w)
    assert _bits_equal(out, want)


def test_fv_pack_codes_round_trip(pkg, orc, synth, cuda):
    """p2_fv_pack_codes returns the int8w codes (row-major here) and passing them back selects the code plane."""
    K, N, M = 1024, 1024, 64
    w = synth.five_value(K, N, seed=7)
    b = pkg.host_five_value(w)
    ptr = pkg.lib().p2_fv_pack_codes(C.byref(b), K, N)
    assert ptr
    codes = np.ctypeslib.as_array((C.c_int8 * (K * N)).from_address(ptr)).reshape(K, N).copy()
    assert np.array_equal(codes, orc.fv_codes(w))
    b.codes = ptr
    A = synth.activations(M, K, seed=8)
    got = pkg.host_sgemm_fvb(A, w, np.zeros((M, N), np.float32), fvb=b)
    want = orc.sgemm_i8(A, "int8w", np.zeros((M, N), np.float32), w=w)
    assert _bits_equal(got, want)
    C.CDLL(None).free(C.c_void_p(ptr))


def test_p2_sgemm_q8b(pkg, orc, synth, cuda):
    M, K, N = 375, 4096, 1024
    t = synth.int8_table(K, N, seed=9)
    A = synth.activations(M, K, seed=10)
    got = pkg.host_sgemm_q8b(A, t, np.zeros((M, N), np.float32))
    want = orc.sgemm_i8(A, "q8b", np.zeros((M, N), np.float32), q8=t)
    assert _bits_equal(got, want)


def test_p2_sgemm_nn_matches_reference(pkg, orc, cuda):
    if not orc.ref_available():
        pytest.skip("reference library not built")
    rng = np.random.default_rng(11)
    for (M, N, K) in [(256, 3000, 256), (48, 384, 128)]:   # the subsampling 1x1 conv and an attention head shape
        A = rng.standard_normal((M, K)).astype(np.float32)
        B = rng.standard_normal((K, N)).astype(np.float32)
        got = pkg.host_sgemm(False, False, A, B, np.zeros((M, N), np.float32))
        want = orc.ref_sgemm(False, False, A, B, np.zeros((M, N), np.float32))
        assert _bits_equal(got, want)


CHILD = r"""
import json, sys
import numpy as np
sys.path.insert(0, {root!r})
import __graft_entry__ as ge
pkg, orc = ge.load_package(), ge.load_oracle()
from phonon2_b200 import synth
M, K, N = 200, 2048, 512
w = synth.five_value(K, N, seed=12)
A = synth.activations(M, K, seed=13)
got = pkg.host_sgemm_fvb(A, w, np.zeros((M, N), np.float32))
mode = {mode!r}
if mode == "exact":
    want = orc.gemm_exact(A, np.zeros((M, N), np.float32), w=w)
else:
    want = orc.sgemm_i8(A, mode, np.zeros((M, N), np.float32), w=w)
qa = pkg.QuantA()
print(json.dumps({{"equal": bool(np.array_equal(got.view(np.uint32), want.view(np.uint32))),
                  "mode": pkg.lib().p2_gemm_mode().decode(), "exact": pkg.lib().p2_gemm_exact(),
                  "prepare": pkg.lib().p2_quant_prepare(__import__("ctypes").byref(qa), M, K)}}))
"""


@pytest.mark.parametrize("env,mode,exact,prepare", [({"P2_GEMM": "int8"}, "int8", 0, 0),
                                                    ({"P2_GEMM": "exact"}, "exact", 1, -1),
                                                    ({"P2_GEMM": "int8", "P2_EXACT": "1"}, "exact", 1, -1)])
def test_mode_from_environment(cuda, env, mode, exact, prepare):
    e = dict(os.environ, **env)
    out = subprocess.run([sys.executable, "-c", CHILD.format(root=str(ROOT), mode=mode)], env=e, capture_output=True,
                         text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    r = json.loads(out.stdout.strip().splitlines()[-1])
    assert r["equal"] and r["exact"] == exact and r["prepare"] == prepare, r
