"""TEST INFRASTRUCTURE ONLY: a pure-Python restatement of the reference's checkpoint tensor
index and content fingerprint, the checker for the library's bybycu_checkpoint_index and
bybycu_fingerprint.

* ``probe_tensor_index`` follows probeTensorIndex (probe_weights.nim:29-104) step by step:
  the same reads, seeks, limits and error messages for .safetensors, NIMBIN, NIMQ2 and NIMQ3.
* ``fingerprint`` follows fingerprint / fingerprintOffsets (probe_data.nim:4-17).

Parity for these two is unpinned: the reference ships no checkpoint fixtures or golden
fingerprints, so the restatement itself is the specification the tests hold the library to.
The ``write_*`` helpers build synthetic checkpoints in the reference's layouts for the tests.

Only ``tests/`` imports this module; the product never does.
"""
from __future__ import annotations

import json
import os
import struct


class CheckpointError(IOError):
    pass


def _i32(f) -> int:
    b = f.read(4)
    if len(b) != 4:
        raise CheckpointError("truncated checkpoint header")
    return struct.unpack("<i", b)[0]


def _i64_count(f) -> int:
    b = f.read(8)
    if len(b) != 8:
        raise CheckpointError("truncated checkpoint header")
    v = struct.unpack("<q", b)[0]
    if v < 0:
        raise CheckpointError("invalid checkpoint element count")
    return v


def _string(f) -> str:
    n = _i32(f)
    if n < 0 or n > 1 << 24:
        raise CheckpointError("invalid checkpoint string length")
    b = f.read(n)
    if len(b) != n:
        raise CheckpointError("truncated checkpoint string")
    return b.decode("latin-1")


def probe_tensor_index(path: str) -> list[dict]:
    """probe_weights.nim:29-104.  Each tensor: name, shape, offset, bytes, kind, scale_offset,
    scales, group_size, eb, mb, dtype."""
    out = []
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        if path.endswith(".safetensors"):
            hb = f.read(8)
            if len(hb) != 8:
                raise CheckpointError("invalid safetensors header")
            header_bytes = struct.unpack("<Q", hb)[0]
            if header_bytes > 1 << 28:
                raise CheckpointError("invalid safetensors header")
            text = f.read(header_bytes)
            if len(text) != header_bytes:
                raise CheckpointError("truncated safetensors header")
            try:
                header = json.loads(text)
            except ValueError:
                raise CheckpointError("invalid safetensors header")
            for name, item in header.items():
                if name == "__metadata__":
                    continue
                o0, o1 = item["data_offsets"]
                out.append(dict(name=name, shape=list(item["shape"]), offset=8 + header_bytes + o0, bytes=o1 - o0,
                                kind=0 if item["dtype"] == "F32" else -1, scale_offset=0, scales=0, group_size=0,
                                eb=0, mb=0, dtype=item["dtype"]))
        else:
            prefix = f.read(8)
            if len(prefix) != 8:
                raise CheckpointError("truncated checkpoint header")
            f.seek(0)
            if prefix.startswith(b"NIMBIN"):
                f.seek(8)
                meta = _i32(f)
                if meta < 0 or meta > 1_000_000:
                    raise CheckpointError("invalid .bin metadata")
                for _ in range(meta):
                    _string(f)
                    _string(f)
                count = _i32(f)
                if count < 0 or count > 1_000_000:
                    raise CheckpointError("invalid tensor count")
                for _ in range(count):
                    name = _string(f)
                    rank = _i32(f)
                    if rank < 0 or rank > 8:
                        raise CheckpointError("invalid tensor rank")
                    shape = [_i32(f) for _ in range(rank)]
                    elems = _i64_count(f)
                    if elems > size // 4:
                        raise CheckpointError("invalid .bin tensor element count")
                    off = f.tell()
                    out.append(dict(name=name, shape=shape, offset=off, bytes=elems * 4, kind=0, scale_offset=0,
                                    scales=0, group_size=0, eb=0, mb=0, dtype=""))
                    f.seek(off + elems * 4)
            else:
                magic = _string(f)
                alignment = 0
                if magic == "NIMQ3":
                    alignment = _i32(f)
                    if alignment < 64 or alignment > 1 << 24:
                        raise CheckpointError("invalid NIMQ3 alignment")
                    f.seek(alignment)
                elif magic != "NIMQ2":
                    raise CheckpointError("unsupported checkpoint format: " + magic)
                for _ in range(5):
                    _i32(f)
                count = _i32(f)
                if count < 0 or count > 1_000_000:
                    raise CheckpointError("invalid tensor count")
                for _ in range(count):
                    name = _string(f)
                    k = f.read(1)
                    if len(k) != 1:
                        raise CheckpointError("truncated tensor kind")
                    rank = _i32(f)
                    if rank < 0 or rank > 8:
                        raise CheckpointError("invalid tensor rank")
                    shape = [_i32(f) for _ in range(rank)]
                    scales = _i32(f)
                    if scales < 0:
                        raise CheckpointError("invalid tensor scale count")
                    scale_offset = f.tell()
                    f.seek(scale_offset + scales * 8)
                    group, eb, mb, nbytes = _i32(f), _i32(f), _i32(f), _i32(f)
                    if nbytes < 0:
                        raise CheckpointError("checkpoint tensor outside file: " + name)
                    if alignment > 0:
                        at = f.tell()
                        f.seek(at + (alignment - at % alignment) % alignment)
                    off = f.tell()
                    out.append(dict(name=name, shape=shape, offset=off, bytes=nbytes, kind=k[0],
                                    scale_offset=scale_offset, scales=scales, group_size=group, eb=eb, mb=mb,
                                    dtype=""))
                    f.seek(off + nbytes)
    for t in out:
        if t["offset"] < 0 or t["bytes"] < 0 or t["offset"] + t["bytes"] > size:
            raise CheckpointError("checkpoint tensor outside file: " + t["name"])
    return out


def fingerprint_offsets(nbytes: int) -> list[int]:
    """probe_data.nim:4-9."""
    r = []
    if nbytes <= 0:
        return r
    width = min(64, nbytes)
    for i in range(5):
        off = (nbytes - width) * i // 4
        if off not in r:
            r.append(off)
    return r


def fingerprint(data: bytes) -> str:
    """probe_data.nim:11-17."""
    n = len(data)
    h = 0xcbf29ce484222325
    mask = (1 << 64) - 1
    for i in range(8):
        h = ((h ^ ((n >> (8 * i)) & 255)) * 0x100000001b3) & mask
    for off in fingerprint_offsets(n):
        for j in range(min(64, n)):
            h = ((h ^ data[off + j]) * 0x100000001b3) & mask
    return "sample1-%016x" % h


# ---- synthetic checkpoints in the reference's layouts ---------------------------------

def _s(b: bytes) -> bytes:
    return struct.pack("<i", len(b)) + b


def write_safetensors(path: str, tensors: list[tuple[str, str, list, bytes]], metadata=None) -> None:
    """tensors: (name, dtype, shape, payload)."""
    header, off = {}, 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, dtype, shape, payload in tensors:
        header[name] = {"dtype": dtype, "shape": shape, "data_offsets": [off, off + len(payload)]}
        off += len(payload)
    text = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for *_, payload in tensors:
            f.write(payload)


def write_nimbin(path: str, meta: list[tuple[str, str]], tensors: list[tuple[str, list, bytes]]) -> None:
    """tensors: (name, shape, fp32 payload)."""
    with open(path, "wb") as f:
        f.write(b"NIMBIN\0\0")
        f.write(struct.pack("<i", len(meta)))
        for k, v in meta:
            f.write(_s(k.encode()) + _s(v.encode()))
        f.write(struct.pack("<i", len(tensors)))
        for name, shape, payload in tensors:
            f.write(_s(name.encode()) + struct.pack("<i", len(shape)))
            for d in shape:
                f.write(struct.pack("<i", d))
            f.write(struct.pack("<q", len(payload) // 4))
            f.write(payload)


def write_nimq(path: str, tensors: list[dict], version: int = 2, alignment: int = 0) -> None:
    """tensors: dicts with name, kind, shape, scales (list of float), group_size, eb, mb,
    payload.  version 3 pads the header to `alignment` and every payload to a multiple of it."""
    with open(path, "wb") as f:
        if version == 3:
            f.write(_s(b"NIMQ3") + struct.pack("<i", alignment))
            f.write(b"\0" * (alignment - f.tell()))
        else:
            f.write(_s(b"NIMQ2"))
        f.write(struct.pack("<5i", 1, 2, 3, 4, 5))
        f.write(struct.pack("<i", len(tensors)))
        for t in tensors:
            f.write(_s(t["name"].encode()) + bytes([t["kind"]]) + struct.pack("<i", len(t["shape"])))
            for d in t["shape"]:
                f.write(struct.pack("<i", d))
            f.write(struct.pack("<i", len(t["scales"])))
            for v in t["scales"]:
                f.write(struct.pack("<d", v))
            f.write(struct.pack("<4i", t["group_size"], t["eb"], t["mb"], len(t["payload"])))
            if alignment:
                f.write(b"\0" * ((alignment - f.tell() % alignment) % alignment))
            f.write(t["payload"])
