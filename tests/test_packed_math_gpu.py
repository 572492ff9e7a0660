"""The packed fp32x2 arithmetic of the encoder's row kernels (phonon-2-c_b200/csrc/numerics.cuh) gives the bits of
the scalar forms it replaces, over every fp32 input.

SiLU + quantise and the depthwise convolution compute two values per packed add / multiply / FMA (sm_100's
.f32x2 forms) and take 1 / (1 + e) from a packed Markstein correction of the hardware reciprocal estimate; the
polynomial exp of the reference's vector loop (csrc/tensor_ops.c:154-172) reads k = rint(x log2 e) off
x log2 e + 1.5 * 2^23. p2cu_probe_packed_math (the test-only probes library) runs each against its scalar form on
all 2^32 bit patterns (the reciprocal on every d in [1, 2^126), the range SiLU gives it) and counts mismatches.
"""
import ctypes as C
import pathlib

import pytest

PROBES = pathlib.Path(__file__).resolve().parents[1] / "phonon-2-c_b200" / "libphonon2_probes.so"
NAMES = ["exp_poly vs the rintf form", "exp_poly2 vs exp_poly", "swish2 vs swish1", "f2_fma vs fmaf",
         "rcp2_ge1 vs __frcp_rn"]


@pytest.mark.gpu
def test_packed_math_bit_identical(cuda):
    assert PROBES.exists(), "libphonon2_probes.so is not built"
    L = C.CDLL(str(PROBES))
    L.p2cu_probes_last_error.restype = C.c_char_p
    bad = (C.c_ulonglong * 5)()
    rc = L.p2cu_probe_packed_math(bad)
    assert rc == 0, L.p2cu_probes_last_error().decode()
    got = dict(zip(NAMES, list(bad)))
    print(got)
    assert all(v == 0 for v in got.values()), got
