"""Checkpoint tensor index and content fingerprints (probe_weights.nim, probe_data.nim) over
libbybycuda's bybycu_checkpoint_index / bybycu_fingerprint."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

from . import _lib
from ._lib import call


@dataclass
class ProbeTensor:
    """probe_weights.nim:5-9."""
    name: str = ""
    shape: list = field(default_factory=list)
    offset: int = 0
    bytes: int = 0
    kind: int = 0
    scaleOffset: int = 0
    scales: int = 0
    groupSize: int = 0
    eb: int = 0
    mb: int = 0
    source: str = ""
    dtype: str = ""


def probeTensorIndex(path: str) -> list[ProbeTensor]:
    """probe_weights.nim:29-104: the tensors of a NIMQ2 / NIMQ3 / NIMBIN / .safetensors file
    from its headers."""
    n = C.c_int(0)
    call("bybycu_checkpoint_index", str(path).encode(), None, 0, C.byref(n))
    arr = (_lib.TensorInfo * max(1, n.value))()
    call("bybycu_checkpoint_index", str(path).encode(), arr, n.value, C.byref(n))
    out = []
    for t in arr[:n.value]:
        if t.name_len >= 256:
            raise _lib.BybyCudaError(_lib.ERR_RANGE, f"tensor name of {t.name_len} bytes in {path}")
        out.append(ProbeTensor(t.name.decode(errors="replace"), [int(d) for d in t.shape[:t.rank]], t.offset,
                               t.bytes, t.kind, t.scale_offset, t.scales, t.group_size, t.eb, t.mb, str(path),
                               t.dtype.decode()))
    return out


def fingerprint(data: int, nbytes: int) -> str:
    """probe_data.nim:11-17 over `nbytes` at host address `data`."""
    buf = C.create_string_buffer(32)
    call("bybycu_fingerprint", C.c_void_p(data), int(nbytes), buf, 32)
    return buf.value.decode()


def fingerprintFile(path: str, offset: int, nbytes: int) -> str:
    """probe_data.nim:19-33: the same identity read from a file range."""
    from .mapped_file import openReadOnlyMapping, unmapReadOnlyFile
    m = openReadOnlyMapping(path)
    try:
        if offset < 0 or nbytes < 0 or offset + nbytes > m.size:
            raise _lib.BybyCudaError(_lib.ERR_RANGE, f"fingerprint range outside file: {path}")
        return fingerprint(m.data + offset, nbytes)
    finally:
        unmapReadOnlyFile(m)


def matchProbeTensor(index: list[ProbeTensor], path: str, nbytes: int, fp: str) -> int:
    """probe_weights.nim:107-115: the one tensor of `nbytes` whose fingerprint is `fp` (no
    fingerprint: size alone); -1 when none, -2 when ambiguous (fails closed)."""
    result = -1
    for i, t in enumerate(index):
        if t.bytes != nbytes:
            continue
        source = t.source or path
        if fp and fingerprintFile(source, t.offset, nbytes) != fp:
            continue
        if result >= 0:
            return -2
        result = i
    return result


__all__ = ["ProbeTensor", "probeTensorIndex", "fingerprint", "fingerprintFile", "matchProbeTensor"]
