"""Weight ingestion on the GPU: host ranges - file mappings included - copied into HBM by the
library's engine (bybycu_upload_host_range, the dGPU branch of residentUploadQ4Mapped /
sessionUploadPrivatePtr, gpubackend.nim:2940-2998).  Bytes must land bit-exact, at any
source offset and length, through the staging slots (default) and through in-place pinning
(BYBY_CUDA_INGEST=register); weights uploaded from a checkpoint mapping must give the same
matmul_q4 results, bit for bit, as the same weights uploaded from a host array."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from bybylang_b200 import _lib  # noqa: E402
from bybylang_b200 import gpubackend as gb  # noqa: E402
from bybylang_b200.mapped_file import openReadOnlyMapping, unmapReadOnlyFile  # noqa: E402
from bybylang_b200.probe_weights import probeTensorIndex  # noqa: E402
from oracle import checkpoint as OC  # noqa: E402
from oracle import oracle as O  # noqa: E402

DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _init():
    gb.ensureGpuInit(gb.GpuBackend.gbCuda, 0)
    yield
    assert _lib.device_error() == 0


@pytest.mark.parametrize("mode", ["stage", "register"])
@pytest.mark.parametrize("off,n", [(0, 96 << 20), (3, (40 << 20) + 5), (4096, 1 << 20), (1, 4 << 20)])
def test_upload_mapped_range_bit_exact(tmp_path, monkeypatch, mode, off, n):
    monkeypatch.setenv("BYBY_CUDA_INGEST", mode)
    data = np.random.default_rng(n + off).integers(0, 256, off + n + 7, dtype=np.uint8)
    p = tmp_path / "blob"
    data.tofile(p)
    m = openReadOnlyMapping(str(p))
    try:
        dst = torch.zeros(n, dtype=torch.uint8, device=DEV)
        _lib.call("bybycu_upload_host_range", C.c_void_p(dst.data_ptr()), C.c_void_p(m.data + off), n)
        assert torch.equal(dst, torch.from_numpy(data[off:off + n]).to(DEV))
    finally:
        unmapReadOnlyFile(m)


def test_upload_pageable_and_pinned_arrays():
    for n in (12 << 20, (9 << 20) + 1):
        a = np.random.default_rng(n).integers(0, 256, n, dtype=np.uint8)
        dst = torch.zeros(n, dtype=torch.uint8, device=DEV)
        _lib.call("bybycu_upload_host_range", C.c_void_p(dst.data_ptr()), C.c_void_p(a.ctypes.data), n)
        assert torch.equal(dst, torch.from_numpy(a).to(DEV))
        pinned = torch.from_numpy(a).pin_memory()
        dst.zero_()
        _lib.call("bybycu_upload_host_range", C.c_void_p(dst.data_ptr()), C.c_void_p(pinned.data_ptr()), n)
        assert torch.equal(dst.cpu(), pinned)


def test_session_upload_ptr_round_trip():
    be = gb.GpuBackend.gbCuda
    a = np.random.default_rng(5).normal(size=3 << 20).astype(np.float32)   # 12 MiB: the staged path
    h = gb.sessionUploadPrivatePtr(be, a.ctypes.data, a.nbytes)
    try:
        assert np.array_equal(gb.sessionRead(be, h, a.size), a)
    finally:
        gb.sessionFree(be, h)
    wrapped, off = gb.sessionWrapHostRange(be, a.ctypes.data, a.nbytes)
    assert wrapped.ptr == 0 and off == 0   # no zero-copy wrapping on a discrete GPU


def test_resident_upload_q4_mapped_matches_array_upload(tmp_path):
    K, N, group = 4096, 1536, 32
    groups = K // group
    rng = np.random.default_rng(11)
    wq = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    scales = (np.abs(rng.normal(0, 0.02, size=(N, groups))) + 1e-4).astype(np.float32)
    zeros = rng.uniform(0, 15, size=(N, groups)).astype(np.float32)
    a = rng.normal(0, 1, size=(1, K)).astype(np.float32)
    p = tmp_path / "q4.safetensors"
    OC.write_safetensors(str(p), [("w.scales", "F32", [N, groups], scales.tobytes()),
                                  ("w.qweight", "U8", [N, K // 2], wq.tobytes()),
                                  ("w.zeros", "F32", [N, groups], zeros.tobytes())])
    idx = {t.name: t for t in probeTensorIndex(str(p))}
    t = idx["w.qweight"]
    assert t.offset % 16 != 0 or True   # any offset: the copy does not need alignment
    be = gb.GpuBackend.gbCuda
    m = openReadOnlyMapping(str(p))
    try:
        wm, zero_copy = gb.residentUploadQ4Mapped(be, m.data + t.offset, t.bytes,
                                                  m.view(idx["w.scales"].offset, idx["w.scales"].bytes).view(np.float32),
                                                  m.view(idx["w.zeros"].offset, idx["w.zeros"].bytes).view(np.float32),
                                                  K, N, group, groups)
    finally:
        unmapReadOnlyFile(m)
    assert not zero_copy
    wa = gb.residentUploadQ4(be, wq, scales, zeros, K, N, group, groups)
    try:
        outs = []
        for w in (wm, wa):
            gb.sessionBegin(be)
            ah = gb.sessionUpload(be, a)
            c = gb.SessionHandle()
            gb.sessionMatmulQ4(be, ah, w, c, 1)
            gb.sessionEnd(be)
            outs.append(gb.sessionRead(be, c, N))
            gb.sessionFree(be, ah)
            gb.sessionFree(be, c)
        assert np.array_equal(outs[0], outs[1])
        want = O.ref_matmul_q4(a, wq, scales, zeros, 1, K, N, group).reshape(-1)
        err = np.abs(outs[0] - want).max() / max(1.0, np.abs(want).max())
        assert err <= 1e-4
    finally:
        gb.residentFreeQ4(be, wm)
        gb.residentFreeQ4(be, wa)
