"""Seeded synthetic five-value weights and activations, in the layouts phonon-2-c stores them.

The five-value operand follows the reference's on-disk planes (csrc/blas.h:38-45, convert_weights.py:114-125):
``signs`` [K, N/4] uint8 with the 2-bit code (sign + 1) of column n at bits 2*(n % 4), ``flags`` [K, N/8] uint8 with
bit n % 8 set when |w| = hi[n], and fp32 ``lo``/``hi`` [N] that hold fp16 values (fermion_container.py:33-34; the
exact-mode expansion relies on that, csrc/blas.c:838-840).

Distribution: P(0) = 1/3 and P(+-lo) = P(+-hi) = 1/6 (each sign equally likely); lo ~ U(0.005, 0.02) and
hi = lo * U(2, 4) per output column, both rounded to fp16 (magnitudes of the size the reference's converter writes).
"""
from __future__ import annotations

import numpy as np

# The 81 bytes whose four 2-bit fields are all valid codes (0, 1, 2); drawing one uniformly draws four independent
# uniform codes, i.e. P(-1) = P(0) = P(+1) = 1/3 per weight.
_VALID_SIGN_BYTES = np.array(
    [a | (b << 2) | (c << 4) | (d << 6) for a in range(3) for b in range(3) for c in range(3) for d in range(3)],
    dtype=np.uint8)


def five_value(K: int, N: int, seed: int) -> dict:
    """A [K, N] five-value weight as the reference stores it."""
    if N % 16:
        raise ValueError(f"N = {N} is not a multiple of 16")
    rng = np.random.default_rng(seed)
    signs = _VALID_SIGN_BYTES[rng.integers(0, 81, size=(K, N // 4))]
    flags = rng.integers(0, 256, size=(K, N // 8), dtype=np.uint8)
    lo = rng.uniform(0.005, 0.02, N).astype(np.float16).astype(np.float32)
    hi = (lo.astype(np.float64) * rng.uniform(2.0, 4.0, N)).astype(np.float16).astype(np.float32)
    return {"signs": np.ascontiguousarray(signs), "flags": np.ascontiguousarray(flags), "lo": lo, "hi": hi,
            "K": K, "N": N}


def int8_table(K: int, N: int, seed: int) -> dict:
    """A [K, N] int8 weight table with one fp32 scale per column (csrc/phonon2.h:110-126, kind P2_W_I8)."""
    rng = np.random.default_rng(seed)
    q8 = rng.integers(-31, 32, size=(K, N), dtype=np.int8)   # the container holds int6 values
    scales = rng.uniform(0.001, 0.01, N).astype(np.float32)
    return {"q8": q8, "scales": scales, "K": K, "N": N}


def activations(M: int, K: int, seed: int) -> np.ndarray:
    """fp32 N(0, 1) activations [M, K]."""
    return np.random.default_rng(seed).standard_normal((M, K), dtype=np.float32)


def quantiser_edge_rows(K: int, seed: int) -> np.ndarray:
    """fp32 rows [8, K] that reach the edges of the reference's per-row quantiser (csrc/blas.c:1114-1144).

    Rows 0-3: the largest magnitude fixed at the first value, every other value placed where x * (1 / scale) and
    x / scale round to different integers (near a half of the quantisation step), so the 16-wide loop (reciprocal)
    and the scalar tail of the last K % 16 values (division) give visibly different codes. Row 4: all zeros
    (scale 1). Row 5: a maximum of 2e-37, so that 1 / scale overflows to infinity (x * inf saturates to +127 or -128,
    0 * inf is NaN and converts to 0). Row 6: one large value among small ones. Row 7: exact halves at scale 1
    (ties to even)."""
    rng = np.random.default_rng(seed)
    f32 = np.float32
    rows = np.zeros((8, K), f32)
    for r in range(4):
        amax = f32(rng.uniform(0.5, 8.0))
        scale = f32(amax / f32(127))
        inv = f32(f32(1) / scale)
        picked = []
        barren = 0
        while len(picked) < K - 1:
            n = rng.integers(-126, 126, 4096)
            x = ((n + 0.5) * np.float64(scale)).astype(f32)
            x = np.concatenate([x, np.nextafter(x, f32(np.inf)), np.nextafter(x, f32(-np.inf))]).astype(f32)
            split = np.rint((x * inv).astype(f32)) != np.rint((x / scale).astype(f32))
            found = x[split & (np.abs(x) < amax)].tolist()
            picked.extend(found)
            barren = 0 if found else barren + 1
            if barren == 16 and not picked:   # a scale whose reciprocal never rounds apart: draw another
                amax = f32(rng.uniform(0.5, 8.0))
                scale = f32(amax / f32(127))
                inv = f32(f32(1) / scale)
                barren = 0
        rows[r, 0] = amax if r % 2 == 0 else -amax
        rows[r, 1:] = np.asarray(picked[:K - 1], f32)
    rows[5] = (rng.uniform(-2e-37, 2e-37, K)).astype(f32)
    rows[5, 0] = f32(2e-37)
    rows[5, 1:K:7] = 0.0
    rows[6] = (rng.standard_normal(K) * 1e-3).astype(f32)
    rows[6, K // 2] = f32(3.0e4)
    rows[7] = ((np.arange(K) % 9) - 4).astype(f32) + f32(0.5)
    rows[7, 0] = f32(127.0)
    return rows


def expand(w: dict) -> np.ndarray:
    """The exact fp32 weight [K, N], {0, +-lo, +-hi}, for reading results (not for the measured path)."""
    K, N = w["K"], w["N"]
    codes = np.stack([(w["signs"] >> (2 * j)) & 3 for j in range(4)], axis=-1).reshape(K, N).astype(np.int8) - 1
    flag = np.unpackbits(w["flags"], axis=1, bitorder="little").astype(bool)
    return codes.astype(np.float32) * np.where(flag, w["hi"][None, :], w["lo"][None, :])


# The GEMM shapes of one FastConformer block (csrc/phonon2.h:73-78, weights.c:459-494; qkv is stored fused as the
# converter writes it, convert_weights.py:185). (name, K, N, alpha, beta, rows) with rows relative to T frames:
# the positional projection runs over the 2T - 1 relative positions (csrc/encoder.c:498-500).
BLOCK_SHAPES = (
    ("ff1.linear1", 1024, 4096, 1.0, 0.0, "T"),
    ("ff1.linear2", 4096, 1024, 0.5, 1.0, "T"),
    ("qkv", 1024, 3072, 1.0, 0.0, "T"),
    ("pos", 1024, 1024, 1.0, 0.0, "2T-1"),
    ("out", 1024, 1024, 1.0, 1.0, "T"),
    ("pw1", 1024, 2048, 1.0, 0.0, "T"),
    ("pw2", 1024, 1024, 1.0, 1.0, "T"),
    ("ff2.linear1", 1024, 4096, 1.0, 0.0, "T"),
    ("ff2.linear2", 4096, 1024, 0.5, 1.0, "T"),
)


def block_rows(spec: str, T: int) -> int:
    return T if spec == "T" else 2 * T - 1
