"""Read-only checkpoint mappings (mapped_file.nim) over libbybycuda's bybycu_map_file.

The mapping is the source of residentUploadQ4Mapped / sessionUploadPrivatePtr: device copies
are made straight from its pages by the library's staging engine."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from . import _lib
from ._lib import call


@dataclass
class MappedReadOnlyFile:
    """mapped_file.nim:5-8: the mapped bytes (`data` is the address) and their count."""
    data: int = 0
    size: int = 0
    _handle: int = 0

    def view(self, offset: int = 0, nbytes: int | None = None):
        """A read-only numpy view of [offset, offset + nbytes) of the mapping (valid until
        unmapReadOnlyFile)."""
        import numpy as np
        n = self.size - offset if nbytes is None else nbytes
        if offset < 0 or n < 0 or offset + n > self.size:
            raise _lib.BybyCudaError(_lib.ERR_RANGE, "mapping view outside the file")
        buf = (C.c_uint8 * n).from_address(self.data + offset)
        a = np.frombuffer(buf, dtype=np.uint8)
        a.flags.writeable = False
        return a


def openReadOnlyMapping(path: str) -> MappedReadOnlyFile:
    """mapped_file.nim:10-13."""
    data, size, handle = C.c_void_p(), C.c_int64(), C.c_void_p()
    call("bybycu_map_file", str(path).encode(), C.byref(data), C.byref(size), C.byref(handle))
    return MappedReadOnlyFile(data.value or 0, size.value, handle.value or 0)


def unmapReadOnlyFile(mapping: MappedReadOnlyFile) -> None:
    """mapped_file.nim:15-19."""
    if mapping.data:
        call("bybycu_unmap_file", C.c_void_p(mapping._handle))
        mapping.data = 0
        mapping.size = 0
        mapping._handle = 0


__all__ = ["MappedReadOnlyFile", "openReadOnlyMapping", "unmapReadOnlyFile"]
