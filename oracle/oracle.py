"""ctypes access to the CPU checkers. TEST INFRASTRUCTURE ONLY.

Three libraries, all built by oracle/Makefile (``__graft_entry__.build()`` runs it):
  * ``liboracle.so``             - fv_oracle.c, the C restatement of the reference's GEMM arithmetic;
  * ``_ref/libphonon2_ref.so``    - phonon-2-c's own library compiled from its sources (exact mode on x86);
  * ``_ref/libphonon2_ref_i8.so`` - the same, with its int8 GEMM entry points supplied by ref_int8_blas.c (the
    restatement), so that the reference's own encoder runs its int8 control flow on x86.

  * ``_ref/libphonon2_ref_neon.so`` (IEEE arithmetic) and ``_ref/libphonon2_ref_neon_fm.so`` (the reference's own
    -ffast-math flags) - phonon-2-c's blas.c compiled as for AArch64 with dot products, its NEON intrinsics modelled
    in C by ``neon_emu/arm_neon.h``: the reference's own int8 and int8w GEMM code running on x86.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU legs import this module; the product never does.
"""
from __future__ import annotations

import atexit
import ctypes as C
import os
import shutil
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libphonon2_ref.so"
REF_I8_SO = HERE / "_ref" / "libphonon2_ref_i8.so"
REF_NEON_SO = HERE / "_ref" / "libphonon2_ref_neon.so"
REF_NEON_FM_SO = HERE / "_ref" / "libphonon2_ref_neon_fm.so"

MODE_INT8, MODE_INT8W, MODE_Q8B = 0, 2, 8
_MODES = {"int8": MODE_INT8, "int8w": MODE_INT8W}

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")

_lib = None
_ref = None
_ref_i8 = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            raise RuntimeError(f"{ORACLE_SO} is not built (run __graft_entry__.build())")
        L = C.CDLL(str(ORACLE_SO))
        L.orc_quant_rows.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, _i8p, _f32p]
        L.orc_quant_rows_fast_math.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, _i8p, _f32p]
        L.orc_clo.argtypes = [C.c_float, C.c_float]
        L.orc_clo.restype = C.c_int
        L.orc_fv_codes.argtypes = [_u8p, _u8p, _f32p, _f32p, C.c_int, C.c_int, _i8p]
        L.orc_acc_blocks.argtypes = [C.c_int, C.c_int, C.c_int, _i8p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                     C.c_void_p, C.c_void_p, C.c_int, _i32p, C.c_void_p]
        common = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_float,
                  _f32p, C.c_int]
        L.orc_gemm_i8.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, _i8p, _f32p, C.c_int] + common
        L.orc_gemm_exact.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, _f32p, C.c_int] + common
        L.orc_sgemm_i8.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, _f32p, C.c_int, C.c_int] + common
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _fv_args(w):
    if w is None:
        return [None] * 4
    return [_ptr(w["signs"]), _ptr(w["flags"]), _ptr(w["lo"]), _ptr(w["hi"])]


def quant_rows(A: np.ndarray, fast_math: bool = False):
    """The reference's per-row quantiser restated (orc_quant_row), or with fast_math what its -ffast-math build
    computes (orc_quant_row_fast_math): (q [M, K] int8, scales [M])."""
    M, K = A.shape
    q = np.empty((M, K), np.int8)
    s = np.empty(M, np.float32)
    fn = lib().orc_quant_rows_fast_math if fast_math else lib().orc_quant_rows
    fn(np.ascontiguousarray(A, np.float32), M, K, K, q, s)
    return q, s


def clo(lo: float, hi: float) -> int:
    return lib().orc_clo(lo, hi)


def fv_codes(w) -> np.ndarray:
    K, N = w["K"], w["N"]
    out = np.empty((K, N), np.int8)
    lib().orc_fv_codes(w["signs"], w["flags"], w["lo"], w["hi"], K, N, out)
    return out


def vindex(w) -> np.ndarray:
    """The value-index plane p2cu_fv_pack_vindex writes (include/p2cuda.h), restated with numpy: uint32
    [ceil(K / 32), N, 4]; word [kc, n, v] holds the 4-bit indices of K rows 32 kc + 8 v .. + 7 of column n at bits 4 t,
    from the reference's 2-bit code and flag (csrc/blas.h:38-45): code 1 -> 0, code 2 -> 1 / 3, code 0 -> 2 / 4,
    code 3 -> 5 / 6 (flag 0 / 1); rows past K -> 0. A layout of this build, not of the reference; only the tests use
    this function."""
    K, N = int(w["K"]), int(w["N"])
    codes = ((w["signs"][:, :, None] >> (2 * np.arange(4, dtype=np.uint8))) & 3).reshape(K, N).astype(np.uint32)
    flags = ((w["flags"][:, :, None] >> np.arange(8, dtype=np.uint8)) & 1).reshape(K, N).astype(np.uint32)
    idx = np.select([codes == 1, codes == 2, codes == 0], [np.zeros_like(flags), 1 + 2 * flags, 2 + 2 * flags], 5 + flags)
    kc = (K + 31) // 32
    idx = np.concatenate([idx, np.zeros((kc * 32 - K, N), np.uint32)]).astype(np.uint32).reshape(kc, 4, 8, N)
    words = (idx << (4 * np.arange(8, dtype=np.uint32))[None, None, :, None]).sum(axis=2, dtype=np.uint64)
    return np.ascontiguousarray(words.astype(np.uint32).transpose(0, 2, 1))                # [kc, N, 4]


def vindex_codes(vi: np.ndarray, w) -> np.ndarray:
    """The int8w codes [K, N] the tensor-memory GEMM decodes from the value-index plane: per column n the palette
    bytes {0, clo, -clo, 127, -127, 2 clo, -2} (mod 256) selected by each 4-bit index, as the kernel's byte permute
    does (fv_gemm_t.cu), restated with numpy so a CPU test can hold it to the reference's codes (csrc/blas.c:1222-1240,
    whose sign * magnitude product wraps for the unused code 3)."""
    K, N = int(w["K"]), int(w["N"])
    clo_n = np.array([clo(float(a), float(b)) for a, b in zip(w["lo"], w["hi"])], np.int64)
    palette = np.stack([np.zeros(N, np.int64), clo_n, -clo_n, np.full(N, 127), np.full(N, -127), 2 * clo_n,
                        np.full(N, 254), np.zeros(N, np.int64)])                          # [8, N]
    palette = (palette & 0xFF).astype(np.uint8).view(np.int8)
    words = vi.reshape(-1, N, 4).transpose(0, 2, 1)                                     # [kc, 4, N]
    idx = (words[:, :, None, :] >> (4 * np.arange(8, dtype=np.uint32))[None, None, :, None]) & 0xF
    idx = idx.reshape(-1, N)[:K].astype(np.int64)
    return np.take_along_axis(palette, idx & 7, axis=0)


def acc_blocks(q: np.ndarray, mode: str, w=None, q8=None):
    """int32 accumulators per 1024-row K block: (accS, accT) as [nblk, M, N] (accT None unless mode 'int8')."""
    M, K = q.shape
    N = w["N"] if w is not None else q8["N"]
    nblk = (K + 1023) // 1024
    accS = np.empty((nblk, M, N), np.int32)
    accT = np.empty((nblk, M, N), np.int32) if mode == "int8" else None
    m = MODE_Q8B if mode == "q8b" else _MODES[mode]
    lib().orc_acc_blocks(M, N, K, np.ascontiguousarray(q), m, *_fv_args(w),
                         _ptr(q8["q8"]) if q8 else None, N, accS, _ptr(accT))
    return accS, accT


def gemm_i8(q, a_scales, mode, out, w=None, q8=None, alpha=1.0, beta=0.0):
    """In place on out [M, N]: the int8 GEMM on pre-quantised rows with the reference epilogue."""
    M, K = q.shape
    N = out.shape[1]
    m = MODE_Q8B if mode == "q8b" else _MODES[mode]
    lib().orc_gemm_i8(M, N, K, alpha, np.ascontiguousarray(q), np.ascontiguousarray(a_scales), m, *_fv_args(w),
                      _ptr(q8["q8"]) if q8 else None, _ptr(q8["scales"]) if q8 else None, N, beta, out, N)
    return out


def sgemm_i8(A, mode, out, w=None, q8=None, alpha=1.0, beta=0.0):
    """In place on out: quantise fp32 A per row, then the int8 GEMM (p2_sgemm_fvb / p2_sgemm_q8b in int8 modes)."""
    M, K = A.shape
    N = out.shape[1]
    m = MODE_Q8B if mode == "q8b" else _MODES[mode]
    lib().orc_sgemm_i8(M, N, K, alpha, np.ascontiguousarray(A, np.float32), K, m, *_fv_args(w),
                       _ptr(q8["q8"]) if q8 else None, _ptr(q8["scales"]) if q8 else None, N, beta, out, N)
    return out


def gemm_exact(A, out, w=None, q8=None, alpha=1.0, beta=0.0):
    """In place on out: the exact path, one FMA chain per output (p2_sgemm_fvb / p2_sgemm_q8b in exact mode)."""
    M, K = A.shape
    N = out.shape[1]
    lib().orc_gemm_exact(M, N, K, alpha, np.ascontiguousarray(A, np.float32), K, *_fv_args(w),
                         _ptr(q8["q8"]) if q8 else None, _ptr(q8["scales"]) if q8 else None, N, beta, out, N)
    return out


# ---- the reference library ---------------------------------------------------------------------------------------

class FiveValueB(C.Structure):
    """The reference's FiveValueB (csrc/blas.h:38-45)."""
    _fields_ = [("signs", C.c_void_p), ("flags", C.c_void_p), ("lo", C.c_void_p), ("hi", C.c_void_p),
                ("codes", C.c_void_p)]


def ref_available() -> bool:
    return REF_SO.exists()


def ref() -> C.CDLL:
    """phonon-2-c compiled from source. Exact mode on x86 (its int8 paths need AArch64 dot products)."""
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            raise RuntimeError(f"{REF_SO} is not built (needs the reference sources; run __graft_entry__.build())")
        L = C.CDLL(str(REF_SO))
        L.p2_sgemm_fvb.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, _f32p, C.c_int, C.POINTER(FiveValueB),
                                   C.c_float, _f32p, C.c_int]
        L.p2_sgemm_q8b.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, _f32p, C.c_int, _i8p, _f32p, C.c_int,
                                   C.c_float, _f32p, C.c_int]
        L.p2_sgemm.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, _f32p, C.c_int, _f32p,
                               C.c_int, C.c_float, _f32p, C.c_int]
        L.p2_gemm_mode.restype = C.c_char_p
        L.p2_gemm_exact.restype = C.c_int
        L.p2_pool.restype = C.c_void_p
        L.p2_pool_nthreads.argtypes = [C.c_void_p]
        L.p2_pool_nthreads.restype = C.c_int
        _ref = L
    return _ref


def ref_threads() -> int:
    L = ref()
    return L.p2_pool_nthreads(L.p2_pool())


def ref_sgemm_fvb(A, w, out, alpha=1.0, beta=0.0):
    """The reference's p2_sgemm_fvb on host arrays, in place on C."""
    M, K = A.shape
    N = out.shape[1]
    b = FiveValueB(_ptr(w["signs"]).value, _ptr(w["flags"]).value, _ptr(w["lo"]).value, _ptr(w["hi"]).value, None)
    ref().p2_sgemm_fvb(M, N, K, alpha, np.ascontiguousarray(A, np.float32), K, C.byref(b), beta, out, N)
    return out


def ref_sgemm_q8b(A, q8, out, alpha=1.0, beta=0.0):
    M, K = A.shape
    N = out.shape[1]
    ref().p2_sgemm_q8b(M, N, K, alpha, np.ascontiguousarray(A, np.float32), K, q8["q8"], q8["scales"], N, beta, out, N)
    return out


def ref_sgemm(transA, transB, A, B, out, alpha=1.0, beta=0.0):
    """The reference's fp32 p2_sgemm (P2Trans 111 = no transpose, 112 = transpose), in place on out."""
    M, N = out.shape
    K = A.shape[0] if transA else A.shape[1]
    ref().p2_sgemm(112 if transA else 111, 112 if transB else 111, M, N, K, alpha, np.ascontiguousarray(A), A.shape[1],
                   np.ascontiguousarray(B), B.shape[1], beta, out, N)
    return out


# ---- the reference's AArch64 int8 GEMM code, compiled for x86 through the NEON model -------------------------------

class QuantA(C.Structure):
    """The reference's QuantA (csrc/phonon2.h:432-436)."""
    _fields_ = [("q", C.c_void_p), ("scales", C.c_void_p), ("M", C.c_int), ("K", C.c_int)]


_neon = {}


def ref_neon_available() -> bool:
    return REF_NEON_SO.exists() and REF_NEON_FM_SO.exists()


def ref_neon(mode: str, fast_math: bool = False) -> C.CDLL:
    """phonon-2-c's blas.c built as for AArch64 with dot products (oracle/Makefile, oracle/neon_emu/arm_neon.h), in GEMM
    mode `mode` ('int8', 'int8w' or 'exact'); `fast_math` picks the build with the reference's own -ffast-math flags.

    The reference reads P2_GEMM once per process (csrc/blas.c:1029-1053), so each mode gets its own copy of the library
    file, loaded and initialised with P2_GEMM set to that mode (a second dlopen of one path would share its state)."""
    key = (mode, fast_math)
    if key in _neon:
        return _neon[key]
    src = REF_NEON_FM_SO if fast_math else REF_NEON_SO
    if not src.exists():
        raise RuntimeError(f"{src} is not built (needs the reference sources; run __graft_entry__.build())")
    tmp = tempfile.mkdtemp(prefix="p2_ref_neon_")
    atexit.register(shutil.rmtree, tmp, True)   # the mapping stays valid after the file is unlinked
    copy = Path(tmp) / f"{src.stem}_{mode}.so"
    shutil.copyfile(src, copy)
    saved = {k: os.environ.get(k) for k in ("P2_GEMM", "P2_EXACT")}
    os.environ["P2_GEMM"] = mode
    os.environ.pop("P2_EXACT", None)
    try:
        L = C.CDLL(str(copy))
        L.p2_gemm_mode.restype = C.c_char_p
        L.p2_gemm_mode()                      # the mode is read now, under this P2_GEMM
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    L.p2_sgemm_fvb.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, _f32p, C.c_int, C.POINTER(FiveValueB),
                               C.c_float, _f32p, C.c_int]
    L.p2_sgemm_q8b.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, _f32p, C.c_int, _i8p, _f32p, C.c_int,
                               C.c_float, _f32p, C.c_int]
    L.p2_sgemm.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, _f32p, C.c_int, _f32p,
                           C.c_int, C.c_float, _f32p, C.c_int]
    L.p2_quant_prepare.argtypes = [C.POINTER(QuantA), C.c_int, C.c_int]
    L.p2_quant_prepare.restype = C.c_int
    L.p2_quant_row.argtypes = [C.POINTER(QuantA), C.c_int, _f32p]
    L.p2_sgemm_fvb_q8a.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, C.POINTER(QuantA), C.POINTER(FiveValueB),
                                   C.c_float, _f32p, C.c_int]
    L.p2_sgemm_q8b_q8a.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, C.POINTER(QuantA), _i8p, _f32p, C.c_int,
                                   C.c_float, _f32p, C.c_int]
    L.p2_fv_pack_codes.argtypes = [C.POINTER(FiveValueB), C.c_int, C.c_int]
    L.p2_fv_pack_codes.restype = C.c_void_p
    _neon[key] = L
    return L


def _fv_struct(w, codes=None):
    return FiveValueB(_ptr(w["signs"]).value, _ptr(w["flags"]).value, _ptr(w["lo"]).value, _ptr(w["hi"]).value,
                      None if codes is None else _ptr(codes).value)


def neon_quant_rows(L, A: np.ndarray):
    """The reference's own quantiser (p2_quant_prepare + p2_quant_row, csrc/blas.c:1114-1187) on the rows of A:
    returns (q [M, K] int8 row-major, scales [M]), read out of its tile layout [Mp/4][K/4][4 rows][4 k]."""
    A = np.ascontiguousarray(A, np.float32)
    M, K = A.shape
    qa = QuantA()
    if L.p2_quant_prepare(C.byref(qa), M, K) != 0:
        raise RuntimeError("p2_quant_prepare refused (exact mode, or K % 4 != 0)")
    for m in range(M):
        L.p2_quant_row(C.byref(qa), m, A[m])
    Mp = (M + 3) // 4 * 4
    tiles = np.ctypeslib.as_array(C.cast(qa.q, C.POINTER(C.c_int8)), shape=(Mp * K,))
    q = tiles.reshape(Mp // 4, K // 4, 4, 4).transpose(0, 2, 1, 3).reshape(Mp, K)[:M].copy()
    scales = np.ctypeslib.as_array(C.cast(qa.scales, C.POINTER(C.c_float)), shape=(M,)).copy()
    return q, scales


def neon_quanta(L, q: np.ndarray, scales: np.ndarray):
    """A QuantA of the reference holding the given quantised rows (its own buffer from p2_quant_prepare, filled in
    its tile layout), so that its GEMMs run on exactly these activations. Valid until the next prepare."""
    M, K = q.shape
    qa = QuantA()
    if L.p2_quant_prepare(C.byref(qa), M, K) != 0:
        raise RuntimeError("p2_quant_prepare refused (exact mode, or K % 4 != 0)")
    Mp = (M + 3) // 4 * 4
    qp = np.zeros((Mp, K), np.int8)
    qp[:M] = q
    tiles = np.ctypeslib.as_array(C.cast(qa.q, C.POINTER(C.c_int8)), shape=(Mp * K,))
    tiles[:] = qp.reshape(Mp // 4, 4, K // 4, 4).transpose(0, 2, 1, 3).reshape(-1)
    np.ctypeslib.as_array(C.cast(qa.scales, C.POINTER(C.c_float)), shape=(M,))[:] = scales
    return qa


def neon_sgemm_fvb(L, A, w, out, alpha=1.0, beta=0.0):
    M, K = A.shape
    b = _fv_struct(w)
    L.p2_sgemm_fvb(M, out.shape[1], K, alpha, np.ascontiguousarray(A, np.float32), K, C.byref(b), beta, out,
                   out.shape[1])
    return out


def neon_sgemm_fvb_q8a(L, q, scales, w, out, alpha=1.0, beta=0.0):
    M, K = q.shape
    qa = neon_quanta(L, q, scales)
    b = _fv_struct(w)
    L.p2_sgemm_fvb_q8a(M, out.shape[1], K, alpha, C.byref(qa), C.byref(b), beta, out, out.shape[1])
    return out


def neon_sgemm_q8b_q8a(L, q, scales, q8, out, alpha=1.0, beta=0.0):
    M, K = q.shape
    N = out.shape[1]
    qa = neon_quanta(L, q, scales)
    L.p2_sgemm_q8b_q8a(M, N, K, alpha, C.byref(qa), np.ascontiguousarray(q8["q8"]), q8["scales"], N, beta, out, N)
    return out


def neon_fv_pack_codes(L, w) -> np.ndarray:
    """The reference's p2_fv_pack_codes (csrc/blas.c:1372-1400) as a row-major [K, N] int8 plane, read out of its
    panel layout [N/16][K/4][16 columns][4 k]."""
    K, N = w["K"], w["N"]
    b = _fv_struct(w)
    p = L.p2_fv_pack_codes(C.byref(b), K, N)
    if not p:
        raise RuntimeError("p2_fv_pack_codes returned NULL")
    try:
        raw = np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_int8)), shape=(K * N,)).copy()
    finally:
        C.CDLL(None).free(C.c_void_p(p))
    return raw.reshape(N // 16, K // 4, 16, 4).transpose(1, 3, 0, 2).reshape(K, N)


def ref_neon_encoder(model_struct, mel: np.ndarray, mode: str = "int8w") -> np.ndarray:
    """phonon-2-c's p2_encoder as its AArch64 build runs it (the NEON branches of csrc/encoder.c and csrc/tensor_ops.c,
    the int8 GEMMs of csrc/blas.c; compiled here through oracle/neon_emu), in GEMM mode `mode`: [T', 640]."""
    L = ref_neon(mode)
    if not hasattr(L, "_enc_ready"):
        L.p2_encoder.argtypes = [C.c_void_p, _f32p, C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_int)]
        L.p2_encoder.restype = C.c_int
        C.c_int.in_dll(L, "p2_verbose").value = 0
        L._enc_ready = True
    mel = np.ascontiguousarray(mel, np.float32)
    out, n = C.c_void_p(), C.c_int()
    if L.p2_encoder(C.addressof(model_struct), mel, mel.shape[0], C.byref(out), C.byref(n)) != 0:
        raise RuntimeError("reference p2_encoder (AArch64 build) failed")
    try:
        return np.ctypeslib.as_array(C.cast(out, C.POINTER(C.c_float)), shape=(n.value, 640)).copy()
    finally:
        _libc.free(out)


def _encoder_lib(path):
    L = C.CDLL(str(path))
    L.p2_encoder.argtypes = [C.c_void_p, _f32p, C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_int)]
    L.p2_encoder.restype = C.c_int
    L.p2_encoder_chunked.argtypes = L.p2_encoder.argtypes
    L.p2_encoder_chunked.restype = C.c_int
    C.c_int.in_dll(L, "p2_verbose").value = 0
    return L


def ref_i8() -> C.CDLL:
    """The reference's encoder with the restated int8 GEMMs (see ref_int8_blas.c)."""
    global _ref_i8
    if _ref_i8 is None:
        if not REF_I8_SO.exists():
            raise RuntimeError(f"{REF_I8_SO} is not built (needs the reference sources; run __graft_entry__.build())")
        L = _encoder_lib(REF_I8_SO)
        L.orc_shim_set_mode.argtypes = [C.c_int]
        _ref_i8 = L
    return _ref_i8


_libc = C.CDLL(None)
_libc.free.argtypes = [C.c_void_p]


def ref_encoder(model_struct, mel: np.ndarray, mode: str = "exact", chunked: bool = False) -> np.ndarray:
    """phonon-2-c's p2_encoder (csrc/encoder.c:753-761) on a P2Model (ctypes struct) and mel [n, 128]: [T', 640].

    mode "exact" runs the reference library as built (its x86 path is exact); "int8" / "int8w" run its encoder with
    the restated int8 GEMMs (libphonon2_ref_i8.so)."""
    if mode == "exact":
        L = ref()
        if not hasattr(L, "_enc_ready"):
            L.p2_encoder.argtypes = [C.c_void_p, _f32p, C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_int)]
            L.p2_encoder.restype = C.c_int
            L.p2_encoder_chunked.argtypes = L.p2_encoder.argtypes
            L.p2_encoder_chunked.restype = C.c_int
            C.c_int.in_dll(L, "p2_verbose").value = 0
            L._enc_ready = True
    else:
        L = ref_i8()
        L.orc_shim_set_mode({"int8": 0, "int8w": 2}[mode])
    mel = np.ascontiguousarray(mel, np.float32)
    out, n = C.c_void_p(), C.c_int()
    fn = L.p2_encoder_chunked if chunked else L.p2_encoder
    rc = fn(C.addressof(model_struct), mel, mel.shape[0], C.byref(out), C.byref(n))
    if rc != 0:
        raise RuntimeError(f"reference p2_encoder returned {rc}")
    try:
        return np.ctypeslib.as_array(C.cast(out, C.POINTER(C.c_float)), shape=(n.value, 640)).copy()
    finally:
        _libc.free(out)


def _ref_decoder():
    L = ref()
    if not hasattr(L, "_dec_ready"):
        L.p2_greedy_decode.argtypes = [C.c_void_p, _f32p, C.c_int, C.POINTER(C.c_void_p)]
        L.p2_greedy_decode.restype = C.c_int
        L.p2_decoder_step.argtypes = [C.c_void_p, C.c_int, _f32p, _f32p]
        L.p2_decoder_step.restype = None
        L.p2_joint.argtypes = [C.c_void_p, _f32p, _f32p, _f32p]
        L.p2_joint.restype = None
        L._dec_ready = True
    return L


def ref_greedy_decode(model_struct, enc: np.ndarray) -> np.ndarray:
    """phonon-2-c's p2_greedy_decode (csrc/decoder.c:100-141) on frames [T, 640]: int32 [n, 3] (id, frame, duration)."""
    L = _ref_decoder()
    enc = np.ascontiguousarray(enc, np.float32)
    out = C.c_void_p()
    n = L.p2_greedy_decode(C.addressof(model_struct), enc, enc.shape[0], C.byref(out))
    try:
        if n <= 0:
            return np.zeros((0, 3), np.int32)
        return np.ctypeslib.as_array(C.cast(out, C.POINTER(C.c_int)), shape=(n, 3)).copy()
    finally:
        _libc.free(out)


def ref_decoder_step(model_struct, token: int, state: np.ndarray, dec_out: np.ndarray) -> None:
    """phonon-2-c's p2_decoder_step (csrc/decoder.c:62-74): state float32 [2, 2, 640] (h, c) in place, dec_out [640]."""
    _ref_decoder().p2_decoder_step(C.addressof(model_struct), token, state, dec_out)


def ref_joint(model_struct, enc_t: np.ndarray, dec_out: np.ndarray) -> np.ndarray:
    """phonon-2-c's p2_joint (csrc/decoder.c:78-88): logits float32 [8198]."""
    logits = np.zeros(8198, np.float32)
    _ref_decoder().p2_joint(C.addressof(model_struct), np.ascontiguousarray(enc_t, np.float32),
                            np.ascontiguousarray(dec_out, np.float32), logits)
    return logits


def ref_mel_spectrogram(audio: np.ndarray) -> np.ndarray:
    """phonon-2-c's p2_mel_spectrogram (csrc/mel.c:158-217) on 16 kHz audio: [n // 160, 128] normalised log-mel."""
    L = ref()
    if not hasattr(L, "_mel_ready"):
        L.p2_mel_spectrogram.argtypes = [_f32p, C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_int)]
        L.p2_mel_spectrogram.restype = C.c_int
        L._mel_ready = True
    audio = np.ascontiguousarray(audio, np.float32)
    out, n = C.c_void_p(), C.c_int()
    if L.p2_mel_spectrogram(audio, audio.shape[0], C.byref(out), C.byref(n)) != 0:
        raise RuntimeError("reference p2_mel_spectrogram failed")
    try:
        return np.ctypeslib.as_array(C.cast(out, C.POINTER(C.c_float)), shape=(n.value, 128)).copy()
    finally:
        _libc.free(out)


class _QuantA(C.Structure):   # csrc/phonon2.h:432-436
    _fields_ = [("q", C.c_void_p), ("scales", C.c_void_p), ("M", C.c_int), ("K", C.c_int)]


def _rows_fn(L, name, argtypes):
    fn = getattr(L, name)
    fn.argtypes = argtypes
    fn.restype = None
    return fn


def ref_layer_norm_rows(x, gamma, beta):
    """The reference's p2_layer_norm_rows (csrc/tensor_ops.c:298-303)."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    _rows_fn(ref(), "p2_layer_norm_rows", [_f32p, _f32p, _f32p, _f32p, C.c_int, C.c_int])(
        x, np.ascontiguousarray(gamma, np.float32), np.ascontiguousarray(beta, np.float32), out, x.shape[0],
        x.shape[1])
    return out


def ref_softmax_rows(x):
    """The reference's p2_softmax_rows (csrc/tensor_ops.c:424-428), on a copy."""
    x = np.array(x, np.float32, order="C")
    _rows_fn(ref(), "p2_softmax_rows", [_f32p, C.c_int, C.c_int])(x, x.shape[0], x.shape[1])
    return x


def ref_swish(x):
    """The reference's p2_swish (csrc/tensor_ops.c:481-490), on a copy."""
    x = np.array(x, np.float32, order="C")
    _rows_fn(ref(), "p2_swish", [_f32p, C.c_int])(x, x.size)
    return x


def ref_depthwise_conv1d(x_ct, w, b):
    """The reference's p2_depthwise_conv1d with kernel 9 (csrc/tensor_ops.c:644-649) on channel-major x [C, T]."""
    x_ct = np.ascontiguousarray(x_ct, np.float32)
    Cn, T = x_ct.shape
    out = np.empty_like(x_ct)
    _rows_fn(ref(), "p2_depthwise_conv1d", [_f32p, _f32p, C.c_void_p, _f32p, C.c_int, C.c_int, C.c_int])(
        x_ct, np.ascontiguousarray(w, np.float32), None if b is None else np.ascontiguousarray(b, np.float32).ctypes.data,
        out, Cn, T, 9)
    return out


def _ref_quant_rows(name, x, *extra):
    L = ref_i8()
    L.orc_shim_set_mode(2)
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.shape
    qa = _QuantA()
    L.p2_quant_prepare.argtypes = [C.POINTER(_QuantA), C.c_int, C.c_int]
    if L.p2_quant_prepare(C.byref(qa), M, K) != 0:
        raise RuntimeError("p2_quant_prepare declined")
    fn = getattr(L, name)
    fn.restype = None
    if extra:
        fn.argtypes = [_f32p, _f32p, _f32p, C.POINTER(_QuantA), C.c_int, C.c_int]
        fn(x, np.ascontiguousarray(extra[0], np.float32), np.ascontiguousarray(extra[1], np.float32), C.byref(qa), M, K)
    else:
        fn.argtypes = [_f32p, C.POINTER(_QuantA), C.c_int, C.c_int]
        fn(x, C.byref(qa), M, K)
    q = np.ctypeslib.as_array(C.cast(qa.q, C.POINTER(C.c_int8)), shape=(M, K)).copy()
    sc = np.ctypeslib.as_array(C.cast(qa.scales, C.POINTER(C.c_float)), shape=(M,)).copy()
    return q, sc


def ref_layer_norm_quant_rows(x, gamma, beta):
    """The reference's p2_layer_norm_quant_rows (csrc/tensor_ops.c:329-350), quantiser restated."""
    return _ref_quant_rows("p2_layer_norm_quant_rows", x, gamma, beta)


def ref_swish_quant_rows(h):
    """The reference's p2_swish_quant_rows (csrc/tensor_ops.c:492-511), quantiser restated."""
    return _ref_quant_rows("p2_swish_quant_rows", h)


def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---- the segmenter and the engine (csrc/segment.c, csrc/engine.c), for the long-audio scheduling ---------------------

def _seg_ready(L):
    if hasattr(L, "_seg_ready"):
        return
    L.p2_block_rms.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int)]
    L.p2_block_rms.restype = C.c_void_p
    L.p2_speech_gate.argtypes = [C.c_void_p, C.c_int]
    L.p2_speech_gate.restype = C.c_float
    L.p2_speech_share.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
    L.p2_speech_share.restype = C.c_float
    L.p2_first_cut.argtypes = [C.c_void_p, C.c_int, C.c_int]
    L.p2_first_cut.restype = C.c_int
    L.p2_split_point.argtypes = [C.c_void_p, C.c_int, C.c_int]
    L.p2_split_point.restype = C.c_int
    L.p2_plan_windows.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_void_p)]
    L.p2_plan_windows.restype = C.c_int
    L._seg_ready = True


def ref_block_rms(audio: np.ndarray) -> np.ndarray:
    """phonon-2-c's p2_block_rms (csrc/segment.c:158-162) on 16 kHz audio: 50 ms block RMS, float32."""
    L = ref()
    _seg_ready(L)
    x = np.ascontiguousarray(audio, np.float32)
    nb = C.c_int()
    p = L.p2_block_rms(x.ctypes.data, x.shape[0], 16000, C.byref(nb))
    if not p:
        return np.zeros(0, np.float32)
    try:
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_float)), shape=(nb.value,)).copy()
    finally:
        _libc.free(p)


def ref_speech_gate(rms: np.ndarray) -> float:
    """p2_speech_gate (csrc/segment.c:164-177)."""
    L = ref()
    _seg_ready(L)
    r = np.ascontiguousarray(rms, np.float32)
    return float(L.p2_speech_gate(r.ctypes.data, r.shape[0]))


def ref_speech_share(rms: np.ndarray, frm: int, to: int, gate: float) -> float:
    """p2_speech_share (csrc/segment.c:179-184) at 16 kHz."""
    L = ref()
    _seg_ready(L)
    r = np.ascontiguousarray(rms, np.float32)
    return float(L.p2_speech_share(r.ctypes.data, r.shape[0], 16000, frm, to, gate))


def ref_first_cut(audio: np.ndarray) -> int:
    """p2_first_cut (csrc/segment.c:90-118) at 16 kHz."""
    L = ref()
    _seg_ready(L)
    x = np.ascontiguousarray(audio, np.float32)
    return int(L.p2_first_cut(x.ctypes.data, x.shape[0], 16000))


def ref_split_point(audio: np.ndarray) -> int:
    """p2_split_point (csrc/segment.c:142-151) at 16 kHz."""
    L = ref()
    _seg_ready(L)
    x = np.ascontiguousarray(audio, np.float32)
    return int(L.p2_split_point(x.ctypes.data, x.shape[0], 16000))


def ref_plan_windows(audio: np.ndarray) -> list[tuple[int, int]]:
    """p2_plan_windows (csrc/segment.c:120-140) at 16 kHz: [(start, end), ...]."""
    L = ref()
    _seg_ready(L)
    x = np.ascontiguousarray(audio, np.float32)
    out = C.c_void_p()
    n = L.p2_plan_windows(x.ctypes.data, x.shape[0], 16000, C.byref(out))
    if n <= 0:
        return []
    try:
        w = np.ctypeslib.as_array(C.cast(out, C.POINTER(C.c_int)), shape=(n, 2)).copy()
    finally:
        _libc.free(out)
    return [(int(a), int(b)) for a, b in w]


def ref_dropped_out(audio: np.ndarray, tokens: np.ndarray):
    """The engine's dropout test (csrc/engine.c:224-251; a static function there, restated here over the reference's
    own p2_block_rms / p2_speech_gate / p2_speech_share): (gap_from, gap_to, speech share) of the first stretch of
    2 s or more without a token whose speech share lies in [0.40, 0.90], or None. tokens: int [k, 3] (id, frame,
    duration) with frames relative to the window's start."""
    frame, min_gap, n = 160 * 8, 32000, int(audio.shape[0])
    rms, gate, prev = None, 0.0, 0
    for i in range(len(tokens) + 1):
        cur = int(tokens[i][1]) * frame if i < len(tokens) else n
        cur = min(cur, n)
        if cur - prev >= min_gap:
            if rms is None:
                rms = ref_block_rms(audio)
                if rms.shape[0] == 0:
                    return None
                gate = ref_speech_gate(rms)
            s = ref_speech_share(rms, prev, cur, gate)
            if np.float32(0.40) <= np.float32(s) <= np.float32(0.90):
                return prev, cur, s
        if i < len(tokens):
            d = int(tokens[i][2])
            prev = cur + (d if d > 0 else 1) * frame
    return None


class _P2Token(C.Structure):
    _fields_ = [("id", C.c_int), ("frame", C.c_int), ("duration", C.c_int)]


class _P2Segment(C.Structure):   # csrc/phonon2.h:249-257
    _fields_ = [("start", C.c_float), ("end", C.c_float), ("text", C.c_char_p), ("first_word", C.c_int),
                ("n_words", C.c_int), ("first_token", C.c_int), ("n_tokens", C.c_int)]


class _P2Result(C.Structure):   # csrc/phonon2.h:259-270
    _fields_ = [("text", C.c_char_p), ("words", C.c_void_p), ("n_words", C.c_int),
                ("tokens", C.POINTER(_P2Token)), ("n_tokens", C.c_int), ("segments", C.POINTER(_P2Segment)),
                ("n_segments", C.c_int), ("encoder_frames", C.c_int), ("duration_seconds", C.c_float),
                ("t_mel", C.c_double), ("t_encoder", C.c_double), ("t_decoder", C.c_double)]


def ref_transcribe(model_dir, audio: np.ndarray, sample_rate: int = 16000) -> dict:
    """phonon-2-c's engine end to end (p2_engine_open on a model directory, p2_transcribe; csrc/engine.c:293-357):
    {"tokens": int [k, 3] (id, frame in the whole audio, duration), "segments": [(start_s, end_s, first_token,
    n_tokens), ...], "encoder_frames": int}. The GEMM mode follows P2_GEMM (exact on x86)."""
    L = ref()
    if not hasattr(L, "_engine_ready"):
        L.p2_engine_open.argtypes = [C.c_char_p]
        L.p2_engine_open.restype = C.c_void_p
        L.p2_engine_close.argtypes = [C.c_void_p]
        L.p2_transcribe.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.POINTER(_P2Result)]
        L.p2_transcribe.restype = C.c_int
        L.p2_result_free.argtypes = [C.POINTER(_P2Result)]
        L._engine_ready = True
    C.c_int.in_dll(L, "p2_verbose").value = 0
    e = L.p2_engine_open(str(model_dir).encode())
    if not e:
        raise RuntimeError(f"p2_engine_open({model_dir}) failed")
    x = np.ascontiguousarray(audio, np.float32)
    r = _P2Result()
    try:
        if L.p2_transcribe(e, x.ctypes.data, x.shape[0], sample_rate, C.byref(r)) != 0:
            raise RuntimeError("reference p2_transcribe failed")
        toks = np.array([(r.tokens[i].id, r.tokens[i].frame, r.tokens[i].duration) for i in range(r.n_tokens)],
                        np.int32).reshape(-1, 3)
        segs = [(r.segments[i].start, r.segments[i].end, r.segments[i].first_token, r.segments[i].n_tokens)
                for i in range(r.n_segments)]
        out = {"tokens": toks, "segments": segs, "encoder_frames": int(r.encoder_frames)}
        L.p2_result_free(C.byref(r))
        return out
    finally:
        L.p2_engine_close(e)
