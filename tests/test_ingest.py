"""Weight ingestion on the host (no GPU): the checkpoint tensor index, the content fingerprint
and the read-only mappings of libbybycuda.so against the Python restatement in
oracle/checkpoint.py (probe_weights.nim:29-115, probe_data.nim:4-33, mapped_file.nim).

Checked: every field of every tensor for NIMQ2, NIMQ3 (alignment padding), NIMBIN and
.safetensors files (metadata skipped, key order kept, \\u-escaped names, non-F32 dtypes);
each error the reference raises, with its message; fingerprints for sizes around the 64-byte
sample width; matchProbeTensor's size / fingerprint / ambiguity rules.
"""
import json
import os
import struct

import numpy as np
import pytest

from bybylang_b200 import _lib
from bybylang_b200.mapped_file import openReadOnlyMapping, unmapReadOnlyFile
from bybylang_b200.probe_weights import fingerprint, fingerprintFile, matchProbeTensor, probeTensorIndex
from oracle import checkpoint as OC

FIELDS = ("name", "shape", "offset", "bytes", "kind", "scale_offset", "scales", "group_size", "eb", "mb", "dtype")


def lib_index(path):
    return [dict(name=t.name, shape=t.shape, offset=t.offset, bytes=t.bytes, kind=t.kind, scale_offset=t.scaleOffset,
                 scales=t.scales, group_size=t.groupSize, eb=t.eb, mb=t.mb, dtype=t.dtype)
            for t in probeTensorIndex(str(path))]


def assert_same_index(path):
    want = OC.probe_tensor_index(str(path))
    got = lib_index(path)
    assert len(got) == len(want)
    for g, w in zip(got, want):
        for f in FIELDS:
            assert g[f] == w[f], (f, g, w)
    return got


def rnd(n, seed):
    return np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8).tobytes()


def nimq_tensors(seed=0):
    return [
        dict(name="layers.0.wq", kind=4, shape=[64, 32], scales=[0.5, 0.25, 1.5], group_size=32, eb=2, mb=1,
             payload=rnd(1024, seed)),
        dict(name="layers.0.norm", kind=0, shape=[64], scales=[], group_size=0, eb=8, mb=23, payload=rnd(256, seed + 1)),
        dict(name="empty", kind=7, shape=[0, 5], scales=[2.0], group_size=16, eb=4, mb=3, payload=b""),
        dict(name="odd", kind=255, shape=[3, 3, 3], scales=[1.0] * 5, group_size=8, eb=1, mb=2, payload=rnd(77, seed + 2)),
    ]


@pytest.mark.parametrize("version,alignment", [(2, 0), (3, 64), (3, 4096)])
def test_nimq_index(tmp_path, version, alignment):
    p = tmp_path / f"m{version}.nimq"
    OC.write_nimq(str(p), nimq_tensors(), version=version, alignment=alignment)
    got = assert_same_index(p)
    assert [t["name"] for t in got] == ["layers.0.wq", "layers.0.norm", "empty", "odd"]
    if alignment:
        assert all(t["offset"] % alignment == 0 for t in got)
    raw = open(p, "rb").read()
    assert raw[got[0]["offset"]:got[0]["offset"] + 1024] == nimq_tensors()[0]["payload"]
    assert struct.unpack("<3d", raw[got[0]["scale_offset"]:got[0]["scale_offset"] + 24]) == (0.5, 0.25, 1.5)


def test_nimbin_index(tmp_path):
    p = tmp_path / "m.bin"
    a = np.arange(12, dtype=np.float32).tobytes()
    OC.write_nimbin(str(p), [("arch", "llama"), ("dim", "64")],
                    [("tok_embeddings", [3, 4], a), ("scalar", [], np.float32([7]).tobytes()), ("none", [0], b"")])
    got = assert_same_index(p)
    assert got[0]["shape"] == [3, 4] and got[0]["bytes"] == 48 and got[2]["bytes"] == 0


def test_safetensors_index(tmp_path):
    p = tmp_path / "m.safetensors"
    OC.write_safetensors(str(p), [
        ("model.layers.0.w", "U8", [16, 8], rnd(128, 3)),
        ("model.layers.0.scales", "F32", [16, 1], rnd(64, 4)),
        ("café.\U0001F600", "BF16", [2, 2, 2], rnd(16, 5)),
        ("zero", "F32", [0], b""),
    ], metadata={"format": "pt"})
    got = assert_same_index(p)
    assert [t["kind"] for t in got] == [-1, 0, -1, 0]
    assert got[2]["name"] == "café.\U0001F600" and got[2]["dtype"] == "BF16"


def _expect_error(path, msg, code=None):
    with pytest.raises(OC.CheckpointError) as e:
        OC.probe_tensor_index(str(path))
    assert msg in str(e.value)
    with pytest.raises(_lib.BybyCudaError) as e2:
        probeTensorIndex(str(path))
    assert msg in str(e2.value), str(e2.value)
    if code is not None:
        assert e2.value.code == code


def test_index_errors(tmp_path):
    # truncated prefix
    p = tmp_path / "short.nimq"
    p.write_bytes(b"NIM")
    _expect_error(p, "truncated checkpoint header")
    # unknown magic
    p = tmp_path / "magic.nimq"
    p.write_bytes(struct.pack("<i", 5) + b"NIMQ9" + b"\0" * 32)
    _expect_error(p, "unsupported checkpoint format: NIMQ9")
    # NIMQ3 alignment below 64
    p = tmp_path / "align.nimq"
    p.write_bytes(struct.pack("<i", 5) + b"NIMQ3" + struct.pack("<i", 32) + b"\0" * 64)
    _expect_error(p, "invalid NIMQ3 alignment")
    # negative tensor count
    p = tmp_path / "count.nimq"
    p.write_bytes(struct.pack("<i", 5) + b"NIMQ2" + struct.pack("<6i", 0, 0, 0, 0, 0, -1))
    _expect_error(p, "invalid tensor count")
    # rank 9
    p = tmp_path / "rank.nimq"
    p.write_bytes(struct.pack("<i", 5) + b"NIMQ2" + struct.pack("<6i", 0, 0, 0, 0, 0, 1) + struct.pack("<i", 1) + b"a"
                  + b"\x01" + struct.pack("<i", 9) + b"\0" * 64)
    _expect_error(p, "invalid tensor rank")
    # negative scale count
    p = tmp_path / "scales.nimq"
    p.write_bytes(struct.pack("<i", 5) + b"NIMQ2" + struct.pack("<6i", 0, 0, 0, 0, 0, 1) + struct.pack("<i", 1) + b"a"
                  + b"\x01" + struct.pack("<ii", 1, 4) + struct.pack("<i", -2) + b"\0" * 64)
    _expect_error(p, "invalid tensor scale count")
    # a payload running past the end of the file
    p = tmp_path / "trunc.nimq"
    OC.write_nimq(str(p), nimq_tensors())
    raw = p.read_bytes()
    p.write_bytes(raw[:-10])
    _expect_error(p, "checkpoint tensor outside file: odd", _lib.ERR_RANGE)
    # string length out of range
    p = tmp_path / "str.nimq"
    p.write_bytes(struct.pack("<i", 1 << 25) + b"\0" * 16)
    _expect_error(p, "invalid checkpoint string length")
    # NIMBIN: element count beyond the file
    p = tmp_path / "big.bin"
    p.write_bytes(b"NIMBIN\0\0" + struct.pack("<ii", 0, 1) + struct.pack("<i", 1) + b"t" + struct.pack("<i", 1)
                  + struct.pack("<i", 4) + struct.pack("<q", 1 << 20))
    _expect_error(p, "invalid .bin tensor element count")
    # NIMBIN: metadata count
    p = tmp_path / "meta.bin"
    p.write_bytes(b"NIMBIN\0\0" + struct.pack("<i", -1) + b"\0" * 8)
    _expect_error(p, "invalid .bin metadata")
    # safetensors: oversized header, bad JSON, offsets past the end
    p = tmp_path / "big.safetensors"
    p.write_bytes(struct.pack("<Q", (1 << 28) + 1) + b"{}")
    _expect_error(p, "invalid safetensors header")
    p = tmp_path / "bad.safetensors"
    text = b'{"a": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]'
    p.write_bytes(struct.pack("<Q", len(text)) + text + b"\0" * 4)
    _expect_error(p, "invalid safetensors header")
    p = tmp_path / "past.safetensors"
    text = json.dumps({"a": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}).encode()
    p.write_bytes(struct.pack("<Q", len(text)) + text + b"\0" * 8)
    _expect_error(p, "checkpoint tensor outside file: a", _lib.ERR_RANGE)


def test_index_capacity_protocol(tmp_path):
    import ctypes as C
    p = tmp_path / "m.nimq"
    OC.write_nimq(str(p), nimq_tensors())
    n = C.c_int(-1)
    lib = _lib.load()
    assert lib.bybycu_checkpoint_index(str(p).encode(), None, 0, C.byref(n)) == 0 and n.value == 4
    arr = (_lib.TensorInfo * 2)()
    assert lib.bybycu_checkpoint_index(str(p).encode(), arr, 2, C.byref(n)) == 0 and n.value == 4
    assert arr[1].name == b"layers.0.norm"
    assert lib.bybycu_checkpoint_index(b"/nonexistent/x.nimq", None, 0, C.byref(n)) == _lib.ERR_ARGS


@pytest.mark.parametrize("n", [0, 1, 63, 64, 65, 100, 255, 1000, 4103])
def test_fingerprint(n):
    data = rnd(n, n)
    buf = np.frombuffer(data, np.uint8) if n else np.zeros(1, np.uint8)
    assert fingerprint(buf.ctypes.data, n) == OC.fingerprint(data)


def test_mapping_and_fingerprint_file(tmp_path):
    p = tmp_path / "blob"
    data = rnd(1 << 20, 9)
    p.write_bytes(data)
    m = openReadOnlyMapping(str(p))
    try:
        assert m.size == len(data)
        assert m.view().tobytes() == data
        assert m.view(12345, 100).tobytes() == data[12345:12445]
        assert fingerprint(m.data + 777, 5000) == OC.fingerprint(data[777:5777])
    finally:
        unmapReadOnlyFile(m)
    assert m.data == 0
    assert fingerprintFile(str(p), 777, 5000) == OC.fingerprint(data[777:5777])
    with pytest.raises(_lib.BybyCudaError):
        fingerprintFile(str(p), len(data) - 10, 20)
    with pytest.raises(_lib.BybyCudaError):
        openReadOnlyMapping(str(tmp_path / "missing"))
    (tmp_path / "empty").write_bytes(b"")
    with pytest.raises(_lib.BybyCudaError):
        openReadOnlyMapping(str(tmp_path / "empty"))


def test_match_probe_tensor(tmp_path):
    p = tmp_path / "m.safetensors"
    a, b, c = rnd(256, 1), rnd(256, 2), rnd(128, 3)
    OC.write_safetensors(str(p), [("a", "U8", [256], a), ("b", "U8", [256], b), ("c", "U8", [128], c)])
    idx = probeTensorIndex(str(p))
    assert matchProbeTensor(idx, str(p), 128, "") == 2
    assert matchProbeTensor(idx, str(p), 256, "") == -2          # equal sizes: ambiguous, fails closed
    assert matchProbeTensor(idx, str(p), 256, OC.fingerprint(b)) == 1
    assert matchProbeTensor(idx, str(p), 256, OC.fingerprint(c + c)) == -1
    assert matchProbeTensor(idx, str(p), 64, "") == -1
