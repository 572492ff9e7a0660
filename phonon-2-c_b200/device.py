"""Device-memory plumbing for Python callers of libphonon2_b200.so: torch allocates and moves bytes, the library
computes. Nothing here does arithmetic on the data."""
from __future__ import annotations

import numpy as np
import torch

from . import P2cuFiveValue, five_value_struct


class DeviceFiveValue:
    """A five-value weight (synth.five_value layout) copied to the device once, with its P2cuFiveValue view."""

    def __init__(self, w: dict, device="cuda", codes: bool = False, stream=None, vindex: bool = False):
        self.K, self.N = int(w["K"]), int(w["N"])
        self.signs = torch.from_numpy(np.ascontiguousarray(w["signs"])).to(device)
        self.flags = torch.from_numpy(np.ascontiguousarray(w["flags"])).to(device)
        self.lo = torch.from_numpy(np.ascontiguousarray(w["lo"])).to(device)
        self.hi = torch.from_numpy(np.ascontiguousarray(w["hi"])).to(device)
        self.codes = None
        self.vindex = None
        self.struct = five_value_struct(self.signs.data_ptr(), self.flags.data_ptr(), self.lo.data_ptr(),
                                        self.hi.data_ptr(), self.K, self.N)
        if codes:
            self.pack_codes(stream)
        if vindex:
            self.pack_vindex(stream)

    def pack_codes(self, stream=None) -> None:
        from . import fv_pack_codes
        self.codes = torch.empty((self.K, self.N), dtype=torch.int8, device=self.signs.device)
        fv_pack_codes(self.struct, self.codes.data_ptr(), stream)
        self.struct.codes = self.codes.data_ptr()

    def pack_vindex(self, stream=None) -> None:
        from . import fv_pack_vindex, fv_vindex_bytes
        self.vindex = torch.empty(fv_vindex_bytes(self.K, self.N) // 4, dtype=torch.int32, device=self.signs.device)
        fv_pack_vindex(self.struct, self.vindex.data_ptr(), stream)
        self.struct.vindex = self.vindex.data_ptr()

    def without_codes(self) -> P2cuFiveValue:
        s = P2cuFiveValue.from_buffer_copy(self.struct)
        s.codes = None
        return s

    def variant(self, codes: bool = False, vindex: bool = False) -> P2cuFiveValue:
        """A view of the weight with only the chosen optional layouts (the planes are always there)."""
        s = P2cuFiveValue.from_buffer_copy(self.struct)
        s.codes = s.codes if codes else None
        s.vindex = s.vindex if vindex else None
        return s

    @property
    def plane_bytes(self) -> int:
        return self.signs.numel() + self.flags.numel() + 4 * (self.lo.numel() + self.hi.numel())


class _CudaArray:
    """A raw device pointer presented through __cuda_array_interface__ (no copy, no ownership)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


def device_view(ptr: int, shape, dtype=torch.float32, device="cuda"):
    """A torch tensor over device memory the library owns (a plan's input or output buffer); valid while it lives."""
    typestr = {torch.float32: "<f4", torch.int8: "|i1", torch.uint8: "|u1", torch.int32: "<i4"}[dtype]
    return torch.as_tensor(_CudaArray(ptr, shape, typestr), device=device)
