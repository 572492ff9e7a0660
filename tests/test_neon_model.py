"""Known answers for oracle/neon_emu/arm_neon.h, the C model of the NEON intrinsics through which the reference's
AArch64 code is compiled on x86 (tests/test_ref_neon.py). Each case is the instruction's architectural result for
inputs that reach its edges: ties to even and saturation in FCVTNS, truncation in FCVTZS, NaN handling, out-of-range
table indices (TBL), negative and large shift counts (USHL), the ST4 interleave, SDOT by lane, signed zeros in
FMAX / FMIN, the FADDP pairing, wrap-around integer lanes."""
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

PROGRAM = r"""
#include <stdio.h>
#include <math.h>
#include "arm_neon.h"

static void f4(const char *name, float32x4_t v) { printf("%s %a %a %a %a\n", name, v[0], v[1], v[2], v[3]); }
static void i4(const char *name, int32x4_t v) { printf("%s %d %d %d %d\n", name, v[0], v[1], v[2], v[3]); }
static void b16(const char *name, const void *p) {
    const unsigned char *b = p; printf("%s", name);
    for (int i = 0; i < 16; i++) printf(" %d", (int)(signed char)b[i]);
    printf("\n");
}

int main(void) {
    float32x4_t t1 = {0.5f, 1.5f, 2.5f, -0.5f}, t2 = {-1.5f, -2.5f, 3.5f, 0.49999997f};
    i4("cvtn_ties", vcvtnq_s32_f32(t1));
    i4("cvtn_ties2", vcvtnq_s32_f32(t2));
    float32x4_t sat = {3e9f, -3e9f, NAN, INFINITY};
    i4("cvtn_sat", vcvtnq_s32_f32(sat));
    float32x4_t tz = {1.9f, -1.9f, NAN, -INFINITY};
    i4("cvtz", vcvtq_s32_f32(tz));
    float32x4_t rn = {0.5f, 1.5f, -2.5f, 2.7f};
    f4("rndn", vrndnq_f32(rn));
    float32x4_t z1 = {0.0f, -0.0f, 1.0f, -3.0f}, z2 = {-0.0f, 0.0f, 2.0f, -4.0f};
    f4("max", vmaxq_f32(z1, z2));
    f4("min", vminq_f32(z1, z2));
    float32x4_t m4 = {1.0f, 7.0f, -2.0f, 3.0f};
    printf("maxv %a\n", vmaxvq_f32(m4));
    float32x4_t s4 = {1.0f, 0x1p-24f, 0x1p-24f, 0x1p-24f};
    printf("addv %a\n", vaddvq_f32(s4));          /* (1 + 2^-24) + (2^-24 + 2^-24) = 1 + 2^-23 */
    float32x4_t fa = {1.0f, 1.0f, 1.0f, 1.0f}, fb = {0x1.000002p0f, 3.0f, 0.0f, -1.0f};
    f4("fma", vfmaq_f32(vdupq_n_f32(-1.0f), fb, fa));
    f4("abs_neg", vabsq_f32(vnegq_f32(z1)));

    int32x4_t big = {70000, -70000, 127, -129};
    int16x4_t n16 = vqmovn_s32(big);
    printf("qmovn32 %d %d %d %d\n", n16[0], n16[1], n16[2], n16[3]);
    int16x8_t w = vcombine_s16(n16, n16);
    int8x8_t n8 = vqmovn_s16(w);
    printf("qmovn16 %d %d %d %d\n", n8[0], n8[1], n8[2], n8[3]);

    uint8x16_t tab; for (int i = 0; i < 16; i++) tab[i] = (uint8_t)(100 + i);
    uint8x16_t idx = {0, 15, 16, 255, 3, 3, 200, 1, 0, 0, 0, 0, 0, 0, 0, 17};
    uint8x16_t tb = vqtbl1q_u8(tab, idx);
    b16("tbl", &tb);
    uint8x16_t sv = vdupq_n_u8(0xB4);
    int8x16_t sh = {0, 1, -1, 2, -2, 7, -7, 8, -8, 9, -9, 3, -3, 127, -128, -6};
    uint8x16_t shl = vshlq_u8(sv, sh);
    b16("ushl", &shl);

    int8x16x4_t q4;
    for (int j = 0; j < 4; j++) for (int i = 0; i < 16; i++) q4.val[j][i] = (int8_t)(10 * j + i);
    int8_t out[64];
    vst4q_s8(out, q4);
    b16("st4_0", out); b16("st4_1", out + 16);

    int8x16_t a, b;
    for (int i = 0; i < 16; i++) { a[i] = (int8_t)(i - 8); b[i] = (int8_t)(127 - 17 * i); }
    i4("sdot_l0", vdotq_laneq_s32(vdupq_n_s32(1), a, b, 0));
    i4("sdot_l3", vdotq_laneq_s32(vdupq_n_s32(0), a, b, 3));
    int8x16_t m1 = vdupq_n_s8(-128), m2 = vdupq_n_s8(2);
    int8x16_t mul = vmulq_s8(m1, m2), neg = vnegq_s8(m1), sub = vsubq_s8(m1, vdupq_n_s8(1));
    printf("wrap %d %d %d\n", mul[0], neg[0], sub[0]);
    int8x16_t tst1 = {1, 2, 0, -1}, tst2 = {1, 1, -1, 0};
    uint8x16_t ts = vtstq_s8(tst1, tst2);
    printf("tst %d %d %d %d\n", ts[0], ts[1], ts[2], ts[3]);
    uint8x16_t msk = {0xFF, 0x0F, 0x00, 0xF0};
    int8x16_t s1 = vdupq_n_s8(0x55), s2 = vdupq_n_s8((int8_t)0xAA);
    int8x16_t bs = vbslq_s8(msk, s1, s2);
    printf("bsl %d %d %d %d\n", (uint8_t)bs[0], (uint8_t)bs[1], (uint8_t)bs[2], (uint8_t)bs[3]);
    int32x4_t sl = {1, -1, 0x40000000, 127};
    i4("shl_n", vshlq_n_s32(sl, 23));
    return 0;
}
"""

WANT = {
    "cvtn_ties": "0 2 2 0",
    "cvtn_ties2": "-2 -2 4 0",
    "cvtn_sat": "2147483647 -2147483648 0 2147483647",
    "cvtz": "1 -1 0 -2147483648",
    "rndn": "0x0p+0 0x1p+1 -0x1p+1 0x1.8p+1",
    "max": "0x0p+0 0x0p+0 0x1p+1 -0x1.8p+1",
    "min": "-0x0p+0 -0x0p+0 0x1p+0 -0x1p+2",
    "maxv": "0x1.cp+2",
    "addv": "0x1.000002p+0",
    "fma": "0x1p-23 0x1p+1 -0x1p+0 -0x1p+1",
    "abs_neg": "0x0p+0 0x0p+0 0x1p+0 0x1.8p+1",
    "qmovn32": "32767 -32768 127 -129",
    "qmovn16": "127 -128 127 -128",
    "tbl": "100 115 0 0 103 103 0 101 100 100 100 100 100 100 100 0",
    # 0xB4 = 180: << 1 = 0x68, >> 1 = 0x5A, << 2 = 0xD0, >> 2 = 0x2D, << 7 = 0x00, >> 7 = 1, |count| >= 8 gives 0
    "ushl": "-76 104 90 -48 45 0 1 0 0 0 0 -96 22 0 0 2",
    "st4_0": "0 10 20 30 1 11 21 31 2 12 22 32 3 13 23 33",
    "st4_1": "4 14 24 34 5 15 25 35 6 16 26 36 7 17 27 37",
    "wrap": "0 -128 127",
    "tst": "255 0 0 0",
    "bsl": "85 165 170 90",
    "shl_n": "8388608 -8388608 0 1065353216",
}


def _sdot_expected(lane, acc):
    a = [i - 8 for i in range(16)]
    b = [((127 - 17 * i + 128) % 256) - 128 for i in range(16)]
    return " ".join(str(acc + sum(a[4 * i + t] * b[4 * lane + t] for t in range(4))) for i in range(4))


WANT["sdot_l0"] = _sdot_expected(0, 1)
WANT["sdot_l3"] = _sdot_expected(3, 0)


@pytest.fixture(scope="module")
def results(tmp_path_factory):
    d = tmp_path_factory.mktemp("neon_model")
    src = d / "known.c"
    src.write_text(PROGRAM)
    exe = d / "known"
    subprocess.run(["gcc", "-O2", "-std=gnu11", "-fno-fast-math", "-ffp-contract=off", "-march=x86-64-v2", "-mfma",
                    f"-I{ROOT / 'oracle' / 'neon_emu'}", str(src), "-o", str(exe), "-lm"], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return dict(line.split(" ", 1) for line in out.strip().splitlines())


@pytest.mark.parametrize("name", sorted(WANT))
def test_known_answer(results, name):
    assert results[name] == WANT[name]
