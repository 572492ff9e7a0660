"""phonon2_b200 - Python access to libphonon2_b200.so, the B200 build of phonon-2-c's five-value GEMM.

The library is C: ``include/blas.h`` (the reference's host-pointer GEMM ABI) and ``include/p2cuda.h`` (device
pointers, explicit streams and workspaces). This module binds both with ctypes for tests, the benchmark and Python
callers; it adds no arithmetic of its own. Loading fails loudly when the library has not been built: there is no
CPU fallback.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libphonon2_b200.so"

# GEMM modes (include/p2cuda.h), numbered as the reference's internal enum (csrc/blas.c:1027).
INT8, EXACT, INT8W = 0, 1, 2
MODES = {"int8": INT8, "exact": EXACT, "int8w": INT8W}

P2CU_OK, P2CU_EINVAL, P2CU_ECUDA, P2CU_EDEVICE, P2CU_EUNSUPPORTED = 0, -1, -2, -3, -4


class Error(RuntimeError):
    """A P2CU_E* return code, with the library's message."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"p2cu error {code}: {msg}")
        self.code = code


class P2cuFiveValue(C.Structure):
    """include/p2cuda.h P2cuFiveValue: a five-value weight resident on the device."""
    _fields_ = [("signs", C.c_void_p), ("flags", C.c_void_p), ("lo", C.c_void_p), ("hi", C.c_void_p),
                ("codes", C.c_void_p), ("K", C.c_int), ("N", C.c_int), ("vindex", C.c_void_p)]


class FiveValueB(C.Structure):
    """include/blas.h FiveValueB (the reference's csrc/blas.h:38-45): host pointers."""
    _fields_ = [("signs", C.c_void_p), ("flags", C.c_void_p), ("lo", C.c_void_p), ("hi", C.c_void_p),
                ("codes", C.c_void_p)]


class QuantA(C.Structure):
    """include/phonon2.h QuantA (the reference's csrc/phonon2.h:432-436)."""
    _fields_ = [("q", C.c_void_p), ("scales", C.c_void_p), ("M", C.c_int), ("K", C.c_int)]


_lib = None
_vp, _i, _f, _sz = C.c_void_p, C.c_int, C.c_float, C.c_size_t

# (name, restype, argtypes) of every exported function, in the order of include/p2cuda.h then include/blas.h.
SIGNATURES = {
    "p2cu_last_error": (C.c_char_p, []),
    "p2cu_check_device": (_i, [_vp]),
    "p2cu_quant_rows": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp]),
    "p2cu_set_quant_fast_math": (_i, [_i]),
    "p2cu_quant_fast_math": (_i, []),
    "p2cu_sgemm_fvb_q8a": (_i, [_i, _i, _i, _f, _vp, _vp, C.POINTER(P2cuFiveValue), _i, _f, _vp, _i, _vp, _sz,
                                _vp]),
    "p2cu_sgemm_q8b_q8a": (_i, [_i, _i, _i, _f, _vp, _vp, _vp, _vp, _i, _f, _vp, _i, _vp, _sz, _vp]),
    "p2cu_q8a_workspace_bytes": (_sz, [_i, _i, _i]),
    "p2cu_gemm_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "p2cu_sgemm_fvb": (_i, [_i, _i, _i, _f, _vp, _i, C.POINTER(P2cuFiveValue), _i, _f, _vp, _i, _vp, _sz, _vp]),
    "p2cu_sgemm_q8b": (_i, [_i, _i, _i, _f, _vp, _i, _vp, _vp, _i, _i, _f, _vp, _i, _vp, _sz, _vp]),
    "p2cu_sgemm": (_i, [_i, _i, _i, _i, _i, _f, _vp, _i, _vp, _i, _f, _vp, _i, _vp]),
    "p2cu_fv_pack_codes": (_i, [C.POINTER(P2cuFiveValue), _vp, _vp]),
    "p2cu_fv_vindex_bytes": (_sz, [_i, _i]),
    "p2cu_fv_pack_vindex": (_i, [C.POINTER(P2cuFiveValue), _vp, _vp]),
    "p2cu_sgemm_fvb_noalloc": (_i, [_i, _i, _i, _f, _vp, _i, C.POINTER(P2cuFiveValue), _i, _f, _vp, _i, _vp]),
    "p2cu_layer_norm_rows": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp]),
    "p2cu_layer_norm_quant_rows": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _vp]),
    "p2cu_swish": (_i, [_vp, _sz, _vp]),
    "p2cu_swish_quant_rows": (_i, [_vp, _vp, _vp, _i, _i, _vp]),
    "p2cu_softmax_rows": (_i, [_vp, _i, _i, _vp]),
    "p2cu_depthwise_conv1d_rows": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp]),
    "p2cu_sgemm_tf32x3": (_i, [_i, _i, _i, _i, _vp, _i, _vp, _i, _vp, _i, _vp]),
    "p2cu_rel_attention_ws_bytes": (_sz, [_i, C.POINTER(_i)]),
    "p2cu_rel_attention": (_i, [_vp, _vp, _vp, _vp, C.POINTER(_i), _i, _i, _vp, _vp, _sz, _vp]),
    "p2cu_model_upload": (_i, [_vp, _i, C.POINTER(_vp)]),
    "p2cu_model_free": (None, [_vp]),
    "p2cu_model_bytes": (_sz, [_vp]),
    "p2cu_encoder_create": (_i, [_vp, C.POINTER(_i), _i, _i, _i, _i, C.POINTER(_vp)]),
    "p2cu_encoder_destroy": (None, [_vp]),
    "p2cu_encoder_frames": (_i, [_vp, _i]),
    "p2cu_encoder_mel": (_vp, [_vp]),
    "p2cu_encoder_out": (_vp, [_vp]),
    "p2cu_encoder_run": (_i, [_vp, _vp]),
    "p2cu_decoder_create": (_i, [_vp, _i, _i, C.POINTER(_vp)]),
    "p2cu_decoder_destroy": (None, [_vp]),
    "p2cu_decode": (_i, [_vp, _vp, C.POINTER(_i), _i, _vp]),
    "p2cu_decoder_read": (_i, [_vp, C.POINTER(_i), _vp, _i, _vp]),
    "p2cu_decoder_tokens": (_vp, [_vp]),
    "p2cu_decoder_offsets": (_vp, [_vp]),
    "p2cu_decoder_step": (_i, [_vp, _i, _vp, _vp, _vp]),
    "p2cu_joint": (_i, [_vp, _vp, _vp, _vp, _vp]),
    "p2cu_mel_create": (_i, [_i, C.c_longlong, C.POINTER(_vp)]),
    "p2cu_mel_destroy": (None, [_vp]),
    "p2cu_mel_frames": (_i, [C.c_longlong]),
    "p2cu_mel_run": (_i, [_vp, _vp, C.POINTER(C.c_longlong), _i, _vp, _vp]),
    "p2cu_block_rms": (_i, [_vp, C.POINTER(C.c_longlong), C.POINTER(_i), _i, _i, _vp, _vp]),
    "p2cu_seg_block": (_i, [_i]),
    "p2cu_seg_blocks": (_i, [_i, _i]),
    "p2cu_seg_window_max_samples": (_i, [_i]),
    "p2cu_seg_first_cut": (_i, [_vp, _i, _i, _i]),
    "p2cu_seg_split_point": (_i, [_vp, _i, _i, _i]),
    "p2cu_seg_speech_gate": (_f, [_vp, _i]),
    "p2cu_seg_speech_share": (_f, [_vp, _i, _i, _i, _i, _f]),
    "p2cu_seg_long_gap": (_i, [_vp, _i, _i]),
    "p2cu_seg_dropped_out": (_i, [_vp, _i, _i, _vp, _i, C.POINTER(_i), C.POINTER(_i), C.POINTER(_f)]),
    "p2cu_probe_wait_timeout": (_i, [C.c_uint, C.POINTER(C.c_double)]),
    # include/phonon2.h: the reference's encoder and decoder entry points
    "p2_encoder": (_i, [_vp, _vp, _i, C.POINTER(_vp), C.POINTER(_i)]),
    "p2_encoder_chunked": (_i, [_vp, _vp, _i, C.POINTER(_vp), C.POINTER(_i)]),
    "p2_b200_encode_windows": (_i, [_vp, _vp, C.POINTER(_i), _i, C.POINTER(_i), _i, _vp]),
    "p2_decoder_step": (None, [_vp, _i, _vp, _vp]),
    "p2_joint": (None, [_vp, _vp, _vp, _vp]),
    "p2_greedy_decode": (_i, [_vp, _vp, _i, C.POINTER(_vp)]),
    "p2_b200_transcribe_windows": (_i, [_vp, _vp, C.POINTER(_i), _i, C.POINTER(_i), _i, C.POINTER(_vp),
                                        C.POINTER(_i)]),
    "p2_mel_spectrogram": (_i, [_vp, _i, C.POINTER(_vp), C.POINTER(_i)]),
    "p2_b200_transcribe_audio_windows": (_i, [_vp, _vp, C.POINTER(C.c_longlong), _i, C.POINTER(_i), _i,
                                              C.POINTER(_vp), C.POINTER(_i)]),
    "p2_b200_plan_windows": (_i, [_vp, _i, _i, C.POINTER(_vp)]),
    "p2_b200_split_point": (_i, [_vp, _i, _i]),
    "p2_b200_transcribe_long": (_i, [_vp, _vp, _i, C.POINTER(_i), _i, C.POINTER(_vp), C.POINTER(_i),
                                     C.POINTER(C.c_longlong)]),
    "p2_b200_windows_free": (None, [_vp, _i]),
    # include/blas.h: the reference's host-pointer ABI
    "p2_sgemm": (None, [_i, _i, _i, _i, _i, _f, _vp, _i, _vp, _i, _f, _vp, _i]),
    "p2_sgemm_st": (None, [_i, _i, _i, _i, _i, _f, _vp, _i, _vp, _i, _f, _vp, _i]),
    "p2_fv_pack_codes": (_vp, [C.POINTER(FiveValueB), _i, _i]),
    "p2_sgemm_q8b": (None, [_i, _i, _i, _f, _vp, _i, _vp, _vp, _i, _f, _vp, _i]),
    "p2_sgemm_fvb": (None, [_i, _i, _i, _f, _vp, _i, C.POINTER(FiveValueB), _f, _vp, _i]),
    "p2_gemm_mode": (C.c_char_p, []),
    "p2_gemm_exact": (_i, []),
    "p2_quant_prepare": (_i, [C.POINTER(QuantA), _i, _i]),
    "p2_quant_row": (None, [C.POINTER(QuantA), _i, _vp]),
    "p2_sgemm_fvb_q8a": (None, [_i, _i, _i, _f, C.POINTER(QuantA), C.POINTER(FiveValueB), _f, _vp, _i]),
    "p2_sgemm_q8b_q8a": (None, [_i, _i, _i, _f, C.POINTER(QuantA), _vp, _vp, _i, _f, _vp, _i]),
    "p2_b200_set_device": (_i, [_i]),
    "p2_b200_release_weights": (None, []),
}

P2_NO_TRANS, P2_TRANS = 111, 112


def lib() -> C.CDLL:
    """The loaded library (raises when it is missing: build it with __graft_entry__.build())."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is not built; run __graft_entry__.build() (no CPU fallback exists)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().p2cu_last_error().decode()


def check(rc: int) -> None:
    if rc != P2CU_OK:
        raise Error(rc, last_error())


def five_value_struct(signs: int, flags: int, lo: int, hi: int, K: int, N: int, codes: int | None = None):
    """A P2cuFiveValue from device addresses."""
    return P2cuFiveValue(signs, flags, lo, hi, codes, K, N)


def workspace_bytes(M: int, N: int, K: int, mode: int) -> int:
    """Workspace of sgemm_fvb / sgemm_q8b (quantised activations plus K-block slices)."""
    return int(lib().p2cu_gemm_workspace_bytes(M, N, K, mode))


def q8a_workspace_bytes(M: int, N: int, K: int) -> int:
    """Workspace of sgemm_fvb_q8a / sgemm_q8b_q8a (K-block slices when K > 1024)."""
    return int(lib().p2cu_q8a_workspace_bytes(M, N, K))


def stream_ptr(stream) -> int | None:
    """A cudaStream_t value from a torch stream (or None for the legacy default stream)."""
    return None if stream is None else int(stream.cuda_stream)


# ---- device-pointer calls (addresses are ints, e.g. torch's data_ptr()) ----------------------------------------------

def quant_rows(A: int, M: int, K: int, lda: int, q: int, scales: int, stream=None) -> None:
    check(lib().p2cu_quant_rows(A, M, K, lda, q, scales, stream_ptr(stream)))


def set_quant_fast_math(on: bool) -> bool:
    """p2cu_set_quant_fast_math: the quantisation rule of every int8 path from now on (False: the reference's C
    source, IEEE; True: its -ffast-math build's arithmetic). Returns the previous rule."""
    return bool(lib().p2cu_set_quant_fast_math(1 if on else 0))


def sgemm_fvb(M, N, K, alpha, A, lda, B: P2cuFiveValue, mode, beta, Cp, ldc, workspace, ws_bytes, stream=None):
    check(lib().p2cu_sgemm_fvb(M, N, K, alpha, A, lda, C.byref(B), mode, beta, Cp, ldc, workspace, ws_bytes,
                               stream_ptr(stream)))


def sgemm_fvb_noalloc(M, N, K, alpha, A, lda, B: P2cuFiveValue, mode, beta, Cp, ldc, stream=None):
    """p2cu_sgemm_fvb with its scratch in the library's fixed device array (no workspace, no allocation)."""
    check(lib().p2cu_sgemm_fvb_noalloc(M, N, K, alpha, A, lda, C.byref(B), mode, beta, Cp, ldc, stream_ptr(stream)))


NOALLOC_SCRATCH_BYTES = 16 << 20   # P2CU_NOALLOC_SCRATCH_BYTES in include/p2cuda.h


def sgemm_fvb_q8a(M, N, K, alpha, q, a_scales, B: P2cuFiveValue, mode, beta, Cp, ldc, workspace=None, ws_bytes=0,
                  stream=None):
    check(lib().p2cu_sgemm_fvb_q8a(M, N, K, alpha, q, a_scales, C.byref(B), mode, beta, Cp, ldc, workspace, ws_bytes,
                                   stream_ptr(stream)))


def sgemm_q8b(M, N, K, alpha, A, lda, B, scales, ldb, mode, beta, Cp, ldc, workspace, ws_bytes, stream=None):
    check(lib().p2cu_sgemm_q8b(M, N, K, alpha, A, lda, B, scales, ldb, mode, beta, Cp, ldc, workspace, ws_bytes,
                               stream_ptr(stream)))


def sgemm_q8b_q8a(M, N, K, alpha, q, a_scales, B, scales, ldb, beta, Cp, ldc, workspace=None, ws_bytes=0,
                  stream=None):
    check(lib().p2cu_sgemm_q8b_q8a(M, N, K, alpha, q, a_scales, B, scales, ldb, beta, Cp, ldc, workspace, ws_bytes,
                                   stream_ptr(stream)))


def sgemm(transA, transB, M, N, K, alpha, A, lda, B, ldb, beta, Cp, ldc, stream=None):
    check(lib().p2cu_sgemm(int(transA), int(transB), M, N, K, alpha, A, lda, B, ldb, beta, Cp, ldc,
                           stream_ptr(stream)))


def fv_pack_codes(B: P2cuFiveValue, codes: int, stream=None) -> None:
    check(lib().p2cu_fv_pack_codes(C.byref(B), codes, stream_ptr(stream)))


def fv_vindex_bytes(K: int, N: int) -> int:
    return int(lib().p2cu_fv_vindex_bytes(K, N))


def fv_pack_vindex(B: P2cuFiveValue, vindex: int, stream=None) -> None:
    """The weight's value-index plane (include/p2cuda.h p2cu_fv_pack_vindex), read by the tensor-memory GEMM."""
    check(lib().p2cu_fv_pack_vindex(C.byref(B), vindex, stream_ptr(stream)))


def check_device(stream=None) -> None:
    check(lib().p2cu_check_device(stream_ptr(stream)))


# ---- the reference's host-pointer ABI (include/blas.h), on numpy arrays -------------------------------------------

def _addr(a) -> int:
    return a.ctypes.data


def host_five_value(w: dict, codes: int | None = None) -> FiveValueB:
    """A FiveValueB over host arrays in synth.five_value layout (the arrays must outlive every call using it)."""
    return FiveValueB(_addr(w["signs"]), _addr(w["flags"]), _addr(w["lo"]), _addr(w["hi"]), codes)


def host_sgemm_fvb(A, w: dict, out, alpha=1.0, beta=0.0, fvb: FiveValueB | None = None):
    """p2_sgemm_fvb on host arrays, in place on `out` (float32 [M, N])."""
    M, K = A.shape
    N = out.shape[1]
    b = fvb if fvb is not None else host_five_value(w)
    lib().p2_sgemm_fvb(M, N, K, alpha, _addr(A), A.strides[0] // 4, C.byref(b), beta, _addr(out), out.strides[0] // 4)
    return out


def host_sgemm_q8b(A, t: dict, out, alpha=1.0, beta=0.0):
    M, K = A.shape
    N = out.shape[1]
    lib().p2_sgemm_q8b(M, N, K, alpha, _addr(A), A.strides[0] // 4, _addr(t["q8"]), _addr(t["scales"]),
                       t["q8"].strides[0], beta, _addr(out), out.strides[0] // 4)
    return out


def host_sgemm(transA, transB, A, B, out, alpha=1.0, beta=0.0):
    M, N = out.shape
    K = A.shape[0] if transA else A.shape[1]
    lib().p2_sgemm(P2_TRANS if transA else P2_NO_TRANS, P2_TRANS if transB else P2_NO_TRANS, M, N, K, alpha,
                   _addr(A), A.strides[0] // 4, _addr(B), B.strides[0] // 4, beta, _addr(out), out.strides[0] // 4)
    return out


# ---- the encoder (include/p2cuda.h device plans, include/phonon2.h host entry) --------------------------------------

class DeviceModel:
    """p2cu_model_upload: a P2Model's encoder weights (and decoder tables, when it has them) on the current device."""

    def __init__(self, model_struct, codes: bool = False):
        self.ptr = C.c_void_p()
        check(lib().p2cu_model_upload(C.addressof(model_struct), 1 if codes else 0, C.byref(self.ptr)))

    @property
    def nbytes(self) -> int:
        return lib().p2cu_model_bytes(self.ptr)

    def close(self) -> None:
        if self.ptr:
            lib().p2cu_model_free(self.ptr)
            self.ptr = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Encoder:
    """p2cu_encoder_create: a plan (buffers + captured graph) for a batch of windows of n_frames mel frames each."""

    def __init__(self, model: DeviceModel, n_frames, mode: int = INT8W, chunk: int = 0, overlap: int = 8):
        self.model = model   # keeps the weights alive
        self.n_frames = [int(n) for n in n_frames]
        arr = (C.c_int * len(self.n_frames))(*self.n_frames)
        self.ptr = C.c_void_p()
        check(lib().p2cu_encoder_create(model.ptr, arr, len(self.n_frames), mode, chunk, overlap, C.byref(self.ptr)))
        L = lib()
        self.frames = [L.p2cu_encoder_frames(self.ptr, w) for w in range(len(self.n_frames))]
        self.total_frames = L.p2cu_encoder_frames(self.ptr, -1)
        self.mel_ptr = L.p2cu_encoder_mel(self.ptr)
        self.out_ptr = L.p2cu_encoder_out(self.ptr)

    def run(self, stream=None) -> None:
        check(lib().p2cu_encoder_run(self.ptr, stream_ptr(stream)))

    def close(self) -> None:
        if self.ptr:
            lib().p2cu_encoder_destroy(self.ptr)
            self.ptr = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def host_encoder(model_struct, mel, chunked: bool = False):
    """p2_encoder (or p2_encoder_chunked) on a host mel array [n_frames, 128]: the [T', 640] frames as numpy."""
    import numpy as _np
    mel = _np.ascontiguousarray(mel, dtype=_np.float32)
    out = C.c_void_p()
    n = C.c_int()
    fn = lib().p2_encoder_chunked if chunked else lib().p2_encoder
    rc = fn(C.addressof(model_struct), mel.ctypes.data, mel.shape[0], C.byref(out), C.byref(n))
    if rc != 0:
        raise Error(rc, "p2_encoder failed (see stderr)")
    try:
        res = _np.ctypeslib.as_array(C.cast(out, C.POINTER(C.c_float)), shape=(n.value, 640)).copy()
    finally:
        C.CDLL(None).free(out)
    return res


def host_encode_windows(model_struct, mels, devices=None):
    """p2_b200_encode_windows: a list of host mel arrays [n_i, 128] -> their [T'_i, 640] frames, spread over
    `devices` (all visible GPUs when None)."""
    import numpy as _np
    from .model import frames_after_subsampling
    frames = [int(m.shape[0]) for m in mels]
    stacked = _np.ascontiguousarray(_np.concatenate(mels), dtype=_np.float32)
    T = [frames_after_subsampling(n) for n in frames]
    out = _np.empty((sum(T), 640), _np.float32)
    fr = (C.c_int * len(frames))(*frames)
    devs = None if not devices else (C.c_int * len(devices))(*devices)
    rc = lib().p2_b200_encode_windows(C.addressof(model_struct), stacked.ctypes.data, fr, len(frames), devs,
                                      len(devices) if devices else 0, out.ctypes.data)
    if rc != 0:
        raise Error(rc, "p2_b200_encode_windows failed (see stderr)")
    offs = _np.cumsum([0] + T)
    return [out[offs[i]:offs[i + 1]] for i in range(len(mels))]


# ---- the greedy TDT decoder (include/p2cuda.h device plans, include/phonon2.h host entry) ----------------------------

def _tokens_array(ptr, n: int):
    """n P2Tokens at ptr as an int32 [n, 3] array (id, frame, duration), copied."""
    import numpy as _np
    if n <= 0:
        return _np.zeros((0, 3), _np.int32)
    return _np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_int)), shape=(n, 3)).copy()


class Decoder:
    """p2cu_decoder_create: state and token buffers for up to max_windows windows of max_frames frames together."""

    def __init__(self, model: DeviceModel, max_windows: int, max_frames: int):
        self.model = model
        self.ptr = C.c_void_p()
        check(lib().p2cu_decoder_create(model.ptr, max_windows, max_frames, C.byref(self.ptr)))
        self.n_windows = 0

    def decode(self, enc_ptr: int, n_frames, stream=None) -> None:
        """p2cu_decode over device frames at enc_ptr ([sum n_frames, 640]), asynchronous on `stream`."""
        fr = [int(n) for n in n_frames]
        arr = (C.c_int * len(fr))(*fr)
        check(lib().p2cu_decode(self.ptr, enc_ptr, arr, len(fr), stream_ptr(stream)))
        self.n_windows = len(fr)

    def read(self, stream=None):
        """p2cu_decoder_read: per-window int32 [n_i, 3] token arrays (id, frame, duration)."""
        import numpy as _np
        offs = (C.c_int * (self.n_windows + 1))()
        total = lib().p2cu_decoder_read(self.ptr, offs, None, 0, stream_ptr(stream))
        check(min(total, 0))
        toks = _np.zeros((max(total, 1), 3), _np.int32)
        if total > 0:
            got = lib().p2cu_decoder_read(self.ptr, offs, toks.ctypes.data, total, stream_ptr(stream))
            check(min(got, 0))
        return [toks[offs[i]:offs[i + 1]].copy() for i in range(self.n_windows)]

    def step(self, token: int, state_ptr: int, dec_ptr: int, stream=None) -> None:
        check(lib().p2cu_decoder_step(self.ptr, token, state_ptr, dec_ptr, stream_ptr(stream)))

    def joint(self, enc_ptr: int, dec_ptr: int, logits_ptr: int, stream=None) -> None:
        check(lib().p2cu_joint(self.ptr, enc_ptr, dec_ptr, logits_ptr, stream_ptr(stream)))

    def close(self) -> None:
        if self.ptr:
            lib().p2cu_decoder_destroy(self.ptr)
            self.ptr = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def host_greedy_decode(model_struct, enc):
    """p2_greedy_decode on host frames [T, 640]: int32 [n, 3] tokens (id, frame, duration)."""
    import numpy as _np
    enc = _np.ascontiguousarray(enc, dtype=_np.float32)
    out = C.c_void_p()
    n = lib().p2_greedy_decode(C.addressof(model_struct), enc.ctypes.data, enc.shape[0], C.byref(out))
    if n < 0:
        raise Error(n, "p2_greedy_decode failed (see stderr)")
    try:
        return _tokens_array(out, n)
    finally:
        C.CDLL(None).free(out)


def host_decoder_step(model_struct, token: int, state, dec_out) -> None:
    """p2_decoder_step on host arrays: state float32 [2, 2, 640] (h then c) updated in place, dec_out [640]."""
    lib().p2_decoder_step(C.addressof(model_struct), token, state.ctypes.data, dec_out.ctypes.data)


def host_joint(model_struct, enc_t, dec_out, logits) -> None:
    """p2_joint on host arrays: logits float32 [8198]."""
    lib().p2_joint(C.addressof(model_struct), enc_t.ctypes.data, dec_out.ctypes.data, logits.ctypes.data)


def host_transcribe_windows(model_struct, mels, devices=None):
    """p2_b200_transcribe_windows: a list of host mel arrays [n_i, 128] -> per-window int32 [k, 3] tokens, encoder
    and decoder on the device, windows spread over `devices` (all visible GPUs when None)."""
    import numpy as _np
    frames = [int(m.shape[0]) for m in mels]
    stacked = _np.ascontiguousarray(_np.concatenate(mels), dtype=_np.float32)
    fr = (C.c_int * len(frames))(*frames)
    devs = None if not devices else (C.c_int * len(devices))(*devices)
    toks = (C.c_void_p * len(frames))()
    counts = (C.c_int * len(frames))()
    rc = lib().p2_b200_transcribe_windows(C.addressof(model_struct), stacked.ctypes.data, fr, len(frames), devs,
                                          len(devices) if devices else 0, toks, counts)
    if rc != 0:
        raise Error(rc, "p2_b200_transcribe_windows failed (see stderr)")
    res = []
    libc = C.CDLL(None)
    for i in range(len(frames)):
        res.append(_tokens_array(toks[i], counts[i]))
        if toks[i]:
            libc.free(C.c_void_p(toks[i]))
    return res


# ---- the log-mel front end (include/p2cuda.h device plan, include/phonon2.h host entry) -----------------------------

class Mel:
    """p2cu_mel_create: tables for up to max_windows windows of max_samples samples together."""

    def __init__(self, max_windows: int, max_samples: int):
        self.ptr = C.c_void_p()
        check(lib().p2cu_mel_create(max_windows, max_samples, C.byref(self.ptr)))

    def run(self, audio_ptr: int, n_samples, mel_ptr: int, stream=None) -> None:
        ns = (C.c_longlong * len(n_samples))(*[int(n) for n in n_samples])
        check(lib().p2cu_mel_run(self.ptr, audio_ptr, ns, len(n_samples), mel_ptr, stream_ptr(stream)))

    def close(self) -> None:
        if self.ptr:
            lib().p2cu_mel_destroy(self.ptr)
            self.ptr = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def mel_frames(n_samples: int) -> int:
    return lib().p2cu_mel_frames(n_samples)


def host_mel_spectrogram(audio):
    """p2_mel_spectrogram on host audio (16 kHz float32): the [n // 160, 128] features as numpy."""
    import numpy as _np
    audio = _np.ascontiguousarray(audio, dtype=_np.float32)
    out = C.c_void_p()
    n = C.c_int()
    rc = lib().p2_mel_spectrogram(audio.ctypes.data, audio.shape[0], C.byref(out), C.byref(n))
    if rc != 0:
        raise Error(rc, "p2_mel_spectrogram failed (see stderr)")
    try:
        return _np.ctypeslib.as_array(C.cast(out, C.POINTER(C.c_float)), shape=(n.value, 128)).copy()
    finally:
        C.CDLL(None).free(out)


def host_transcribe_audio_windows(model_struct, audios, devices=None):
    """p2_b200_transcribe_audio_windows: a list of host audio arrays (16 kHz) -> per-window int32 [k, 3] tokens."""
    import numpy as _np
    ns = [int(a.shape[0]) for a in audios]
    stacked = _np.ascontiguousarray(_np.concatenate(audios), dtype=_np.float32)
    na = (C.c_longlong * len(ns))(*ns)
    devs = None if not devices else (C.c_int * len(devices))(*devices)
    toks = (C.c_void_p * len(ns))()
    counts = (C.c_int * len(ns))()
    rc = lib().p2_b200_transcribe_audio_windows(C.addressof(model_struct), stacked.ctypes.data, na, len(ns), devs,
                                                len(devices) if devices else 0, toks, counts)
    if rc != 0:
        raise Error(rc, "p2_b200_transcribe_audio_windows failed (see stderr)")
    res = []
    libc = C.CDLL(None)
    for i in range(len(ns)):
        res.append(_tokens_array(toks[i], counts[i]))
        if toks[i]:
            libc.free(C.c_void_p(toks[i]))
    return res


# ---- long audio: the segmenter's decisions and the batched re-decode scheduling ----------------------------------------

class P2B200Window(C.Structure):   # include/phonon2.h
    _fields_ = [("start", C.c_int), ("end", C.c_int), ("depth", C.c_int), ("encoder_frames", C.c_int),
                ("tokens", C.c_void_p), ("n_tokens", C.c_int)]


def host_plan_windows(audio):
    """p2_b200_plan_windows on 16 kHz float32 audio: a list of (start, end) sample pairs."""
    import numpy as _np
    x = _np.ascontiguousarray(audio, dtype=_np.float32)
    out = C.c_void_p()
    n = lib().p2_b200_plan_windows(x.ctypes.data, int(x.shape[0]), 16000, C.byref(out))
    if n <= 0:
        return []
    w = _np.ctypeslib.as_array(C.cast(out, C.POINTER(C.c_int)), shape=(n, 2)).copy()
    C.CDLL(None).free(out)
    return [(int(a), int(b)) for a, b in w]


def host_split_point(audio) -> int:
    """p2_b200_split_point on 16 kHz float32 audio."""
    import numpy as _np
    x = _np.ascontiguousarray(audio, dtype=_np.float32)
    return int(lib().p2_b200_split_point(x.ctypes.data, int(x.shape[0]), 16000))


def host_transcribe_long(model_struct, audio, devices=None):
    """p2_b200_transcribe_long: 16 kHz audio -> (list of dicts with start, end, depth, encoder_frames and int32 [k, 3]
    tokens (frames relative to the window's start), in the reference's segment order; total encoder frames)."""
    import numpy as _np
    x = _np.ascontiguousarray(audio, dtype=_np.float32)
    devs = None if not devices else (C.c_int * len(devices))(*devices)
    out = C.c_void_p()
    n = C.c_int()
    frames = C.c_longlong()
    rc = lib().p2_b200_transcribe_long(C.addressof(model_struct), x.ctypes.data, int(x.shape[0]), devs,
                                       len(devices) if devices else 0, C.byref(out), C.byref(n), C.byref(frames))
    if rc != 0:
        raise Error(rc, "p2_b200_transcribe_long failed (see stderr)")
    res = []
    if n.value > 0:
        arr = C.cast(out, C.POINTER(P2B200Window * n.value)).contents
        for w in arr:
            res.append({"start": w.start, "end": w.end, "depth": w.depth, "encoder_frames": w.encoder_frames,
                        "tokens": _tokens_array(w.tokens, w.n_tokens)})
    lib().p2_b200_windows_free(out, n.value)
    return res, frames.value
