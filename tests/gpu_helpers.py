"""Helpers shared by the GPU parity tests (device copies, C-ABI calls, tolerance checks)."""
import numpy as np
import torch

from bybylang_b200 import _lib
from bybylang_b200 import gpubackend as gb

DEV = "cuda:0"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def run(fmt, M, K, N, x, packed, *, scale_base=0, lut=None, route=_lib.ROUTE_AUTO, out_dtype=torch.float32):
    out = torch.full((M, N), float("nan"), dtype=out_dtype, device=DEV)
    gb.tile_gemm(fmt, x, packed, out, M=M, K=K, N=N, scale_base=scale_base, lut=lut, route=route)
    torch.cuda.synchronize()
    return out


def q4_slot(p, s):
    """Nibbles then fp16 scales at a 16-byte aligned scale_base, as one device uint8 slot."""
    nb = p.size
    sb = (nb + 15) // 16 * 16
    blob = np.zeros(sb + s.size * 2, np.uint8)
    blob[:nb] = p.ravel()
    blob[sb:] = np.ascontiguousarray(s, np.uint16).view(np.uint8).ravel()
    return dev(blob), sb


def peak_err(want, got):
    """The reference test's metric: max|diff| / max(1, max|ref|)."""
    want = np.asarray(want, np.float64)
    got = np.asarray(got, np.float64)
    return float(np.abs(want - got).max()) / max(1.0, float(np.abs(want).max()))


def assert_close(want, got, peak_tol, elem_tol=None, what=""):
    want = np.asarray(want, np.float64)
    got = np.asarray(got, np.float64)
    assert np.isfinite(got).all(), what
    d = np.abs(want - got)
    peak = max(1.0, float(np.abs(want).max()))
    assert d.max() <= peak_tol * peak, f"{what}: max|diff| {d.max():.3e} peak {peak:.3f}"
    if elem_tol is not None:
        assert (d <= elem_tol * np.maximum(1.0, np.abs(want))).all(), f"{what}: per-element"


def elem_err(want, got):
    """The reference gate's metric (vulkan_driver.nim:2752-2754), worst element:
    max |got - want| / max(1, |want|)."""
    want = np.asarray(want, np.float64)
    got = np.asarray(got, np.float64)
    return float((np.abs(got - want) / np.maximum(1.0, np.abs(want))).max())
