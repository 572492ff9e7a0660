"""Writes the golden vectors under tests/golden/ from phonon-2-c's own code, compiled here from its sources.

Run on a machine that has the reference sources and oracle/_ref built (``__graft_entry__.build()``):

    python tests/golden/make_golden.py [output directory, default tests/golden]

Sources of the values (the libraries oracle/Makefile builds):
  * exact mode: ``_ref/libphonon2_ref.so``, the reference's x86 build (its only x86 GEMM path);
  * int8 / int8w modes and the quantiser: ``_ref/libphonon2_ref_neon.so``, the reference's AArch64 code (csrc/blas.c
    with its dot-product branches, csrc/tensor_ops.c and csrc/encoder.c with their NEON branches) compiled for x86
    through the intrinsic model in oracle/neon_emu, with IEEE arithmetic.

Inputs are not stored: they are regenerated from seeds by phonon2_b200.synth / .model, and a SHA-256 of each input is
stored beside the outputs so that a reader can tell regenerated inputs from drifted ones. Files:
  * gemm.npz    - per case ``<case>/out`` (fp32 C), ``<case>/spec`` (M, K, N, seeds, alpha, beta), ``<case>/sha``;
                  quantiser cases ``quant<K>/q``, ``/scales``; int8w code planes ``codes<K>x<N>``.
  * encoder.npz - p2_encoder's [T', 640] output on a 3 s synthetic log-mel (300 frames) with SyntheticModel(seed=7),
                  exact (x86 build) and int8w / int8 (AArch64 build).
  * decoder.npz - with the same model: p2_joint's 8198 logits for two (encoder frame, decoder output) pairs, and
                  p2_greedy_decode's tokens (id, frame, duration) over N(0, 1) frames of 38 and 375 rows.
  * mel.npz     - p2_mel_spectrogram's [100, 128] features of 1 s of synthetic speech (model.audio).
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

import __graft_entry__ as ge  # noqa: E402

# (name, mode, M, K, N, alpha, beta, weight seed, activation seed, edge rows first)
GEMM_CASES = [
    ("exact_fvb_16x1024x128", "exact", 16, 1024, 128, 1.0, 0.0, 101, 201, False),
    ("exact_fvb_9x4096x64", "exact", 9, 4096, 64, 0.5, 1.0, 102, 202, False),
    ("exact_fvb_5x100x48", "exact", 5, 100, 48, 1.0, 0.5, 103, 203, False),
    ("int8w_fvb_16x1024x128", "int8w", 16, 1024, 128, 1.0, 0.0, 104, 204, True),
    ("int8w_fvb_9x4096x64", "int8w", 9, 4096, 64, 0.5, 1.0, 105, 205, False),
    ("int8w_fvb_13x1028x48", "int8w", 13, 1028, 48, 1.0, 0.25, 106, 206, True),
    ("int8_fvb_16x1024x128", "int8", 16, 1024, 128, 1.0, 0.0, 107, 207, True),
    ("int8_fvb_9x4096x64", "int8", 9, 4096, 64, 0.5, 1.0, 108, 208, False),
    ("int8_fvb_13x1028x48", "int8", 13, 1028, 48, 1.0, 0.25, 109, 209, True),
    ("int8_q8b_7x2048x128", "q8b", 7, 2048, 128, 1.0, 0.0, 110, 210, False),
    ("int8w_fvb_5x1022x48", "int8w", 5, 1022, 48, 1.0, 0.5, 111, 211, False),   # K % 4 != 0: the exact path
]
QUANT_K = (20, 1024, 1028)
CODES = ((256, 128), (64, 48))
ENCODER_SEED, ENCODER_MEL_FRAMES, ENCODER_MEL_SEED = 7, 300, 11
DECODE_T = (38, 375)
MEL_SAMPLES = 16000


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def gemm_inputs(synth, mode, M, K, N, wseed, aseed, edge):
    """The seeded inputs of one case: (weight dict, A [M, K], C0 [M, N])."""
    w = synth.int8_table(K, N, seed=wseed) if mode == "q8b" else synth.five_value(K, N, seed=wseed)
    A = synth.activations(M, K, seed=aseed)
    if edge:
        e = synth.quantiser_edge_rows(K, seed=aseed)
        A[:min(M, len(e))] = e[:min(M, len(e))]
    C0 = np.random.default_rng(aseed + 1).standard_normal((M, N)).astype(np.float32)
    return w, A, C0


def weight_sha(w) -> str:
    keys = ("q8", "scales") if "q8" in w else ("signs", "flags", "lo", "hi")
    return sha(*(w[k] for k in keys))


def quant_input(synth, K):
    return np.concatenate([synth.quantiser_edge_rows(K, seed=K), synth.activations(8, K, seed=K + 1)])


def joint_inputs():
    """Two (encoder frame, decoder output) pairs; the second's first 40 products cancel exactly."""
    rng = np.random.default_rng(3)
    pairs = []
    for i in range(2):
        enc = rng.standard_normal(640, dtype=np.float32)
        dec = (rng.standard_normal(640) * 0.5).astype(np.float32)
        if i == 1:
            dec[:40] = -enc[:40]
        pairs.append((enc, dec))
    return pairs


def decode_frames(T):
    return np.random.default_rng(T).standard_normal((T, 640), dtype=np.float32)


def main(out_dir: Path = HERE) -> None:
    out_dir = Path(out_dir)
    ge.load_package()
    orc = ge.load_oracle()
    from phonon2_b200 import synth, model as M
    if not (orc.ref_available() and orc.ref_neon_available()):
        raise SystemExit("oracle/_ref is not built (the reference sources are needed): run __graft_entry__.build()")

    g = {}
    for name, mode, m, k, n, alpha, beta, wseed, aseed, edge in GEMM_CASES:
        w, A, C0 = gemm_inputs(synth, mode, m, k, n, wseed, aseed, edge)
        if mode == "exact":
            out = orc.ref_sgemm_fvb(A, w, C0.copy(), alpha=alpha, beta=beta)
        elif mode == "q8b":
            out = C0.copy()
            orc.ref_neon("int8").p2_sgemm_q8b(m, n, k, alpha, A, k, w["q8"], w["scales"], n, beta, out, n)
        else:
            out = orc.neon_sgemm_fvb(orc.ref_neon(mode), A, w, C0.copy(), alpha=alpha, beta=beta)
        g[f"{name}/out"] = out
        g[f"{name}/spec"] = np.array([m, k, n, wseed, aseed, int(edge)], np.int64)
        g[f"{name}/ab"] = np.array([alpha, beta], np.float32)
        g[f"{name}/sha"] = np.array([weight_sha(w), sha(A), sha(C0)])
    for k in QUANT_K:
        A = quant_input(synth, k)
        q, s = orc.neon_quant_rows(orc.ref_neon("int8w"), A)
        g[f"quant{k}/q"], g[f"quant{k}/scales"], g[f"quant{k}/sha"] = q, s, np.array([sha(A)])
    for k, n in CODES:
        w = synth.five_value(k, n, seed=k + n)
        g[f"codes{k}x{n}"] = orc.neon_fv_pack_codes(orc.ref_neon("int8w"), w)
        g[f"codes{k}x{n}/sha"] = np.array([weight_sha(w)])
    np.savez_compressed(out_dir / "gemm.npz", **g)

    model = M.SyntheticModel(seed=ENCODER_SEED)
    mel = M.mel(ENCODER_MEL_FRAMES, seed=ENCODER_MEL_SEED)
    e = {"exact": orc.ref_encoder(model.struct, mel, "exact"),
         "int8w": orc.ref_neon_encoder(model.struct, mel, "int8w"),
         "int8": orc.ref_neon_encoder(model.struct, mel, "int8"),
         "sha": np.array([sha(*(model.arrays[k] for k in sorted(model.arrays))), sha(mel)])}
    np.savez_compressed(out_dir / "encoder.npz", **e)

    d = {"joint": np.stack([orc.ref_joint(model.struct, enc, dec) for enc, dec in joint_inputs()]),
         "joint/sha": np.array([sha(*(a for pair in joint_inputs() for a in pair))])}
    for T in DECODE_T:
        frames = decode_frames(T)
        d[f"tokens{T}"] = orc.ref_greedy_decode(model.struct, frames)
        d[f"tokens{T}/sha"] = np.array([sha(frames)])
    np.savez_compressed(out_dir / "decoder.npz", **d)

    audio = M.audio(MEL_SAMPLES, seed=MEL_SAMPLES)
    np.savez_compressed(out_dir / "mel.npz", mel=orc.ref_mel_spectrogram(audio), sha=np.array([sha(audio)]))
    print("wrote", *(out_dir / f for f in ("gemm.npz", "encoder.npz", "decoder.npz", "mel.npz")))


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else HERE)
