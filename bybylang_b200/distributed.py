"""Column sharding of the tile GEMM across GPUs (one process per GPU).

The reference splits independent work over worker processes by ``partition``
(distributed.nim:109-135: largest remainder over the devices' weights) and gathers their text
results through pipes (distributed.nim:304-375).  Here each rank owns a contiguous column range
of W (rows of the packed layout) chosen by the same largest-remainder rule over blocks of 64
columns, computes its slice of out[M, N] on its own GPU, and the slices are exchanged on the
device:

* ``exchange="peer"`` - libbybycuda's own exchange: the slice is stored into every rank's
  output over NVLink peer pointers (CUDA IPC, no multicast objects) and a bounded device-side
  wait on per-rank counters completes the gather;
* ``exchange="nccl"`` - the baseline: an NCCL all-gather through torch.distributed.

torch.distributed is the plumbing (rank discovery, the IPC-handle exchange, NCCL); the math and
the peer exchange are the library's.
"""
from __future__ import annotations

import ctypes as C
import math

from . import _lib
from ._lib import BybyCudaError, call, check, load
from .gpubackend import _dtype_code, _ptr, _stream_ptr
from .session_vm import TileFormatQ4B32

SHARD_ALIGN = 64   # the tile width of the reference's tile GEMM (tile_gemm.nim:44)


def partition(length: int, world: int, ratios=None) -> list[int]:
    """distributed.nim:109-135: floor of length * w / total, then the largest remainders get
    one more each (first index first on ties)."""
    if world < 1:
        raise ValueError("Process group has no devices")
    if length < 0:
        raise ValueError("Length must be non-negative")
    ws = list(ratios) if ratios else [1.0] * world
    total = sum(ws)
    out, rem, assigned = [], [], 0
    for w in ws:
        exact = float(length) * (w / total)
        out.append(int(math.floor(exact)))
        rem.append(exact - out[-1])
        assigned += out[-1]
    while assigned < length:
        best = -1
        for i, r in enumerate(rem):
            if ws[i] > 0 and (best < 0 or r > rem[best]):
                best = i
        if best < 0:
            break
        out[best] += 1
        rem[best] = -1.0
        assigned += 1
    return out


def shard_range(N: int, world: int, rank: int, align: int = SHARD_ALIGN) -> tuple[int, int]:
    """The column range of `rank` (libbybycuda's bybycu_shard_range)."""
    n0, n1 = C.c_int(0), C.c_int(0)
    call("bybycu_shard_range", N, world, rank, align, C.byref(n0), C.byref(n1))
    return n0.value, n1.value


class PeerBuffers:
    """An fp32 output buffer [M, N] and a signal array on every rank, with every rank's
    buffers mapped on every other rank through CUDA IPC."""

    def __init__(self, M: int, N: int, world: int, rank: int, group=None):
        import torch
        import torch.distributed as dist
        self.M, self.N, self.world, self.rank = M, N, world, rank
        dev = torch.device("cuda", torch.cuda.current_device())
        self.out = torch.zeros(M, N, dtype=torch.float32, device=dev)
        self.signal = torch.zeros(64, dtype=torch.int32, device=dev)   # world counters used
        torch.cuda.synchronize()
        # each handle names the whole allocation; the offset locates the tensor inside it
        h_out, h_sig = C.create_string_buffer(64), C.create_string_buffer(64)
        o_out, o_sig = C.c_int64(0), C.c_int64(0)
        call("bybycu_ipc_handle", C.c_void_p(self.out.data_ptr()), h_out, C.byref(o_out))
        call("bybycu_ipc_handle", C.c_void_p(self.signal.data_ptr()), h_sig, C.byref(o_sig))
        mine = (bytes(h_out.raw), o_out.value, bytes(h_sig.raw), o_sig.value)
        allh = [None] * world
        dist.all_gather_object(allh, mine, group=group)
        self._opened = []
        outs, sigs = [], []
        for r in range(world):
            if r == rank:
                outs.append(self.out.data_ptr())
                sigs.append(self.signal.data_ptr())
                continue
            po, ps = C.c_void_p(), C.c_void_p()
            call("bybycu_ipc_open", C.c_char_p(allh[r][0]), allh[r][1], C.byref(po))
            call("bybycu_ipc_open", C.c_char_p(allh[r][2]), allh[r][3], C.byref(ps))
            self._opened += [po.value, ps.value]
            outs.append(po.value)
            sigs.append(ps.value)
        self.peer_out = (C.c_void_p * world)(*outs)
        self.peer_sig = (C.POINTER(C.c_uint32) * world)(*[C.cast(C.c_void_p(p), C.POINTER(C.c_uint32))
                                                          for p in sigs])
        self.epoch = 0

    def close(self):
        for p in self._opened:
            load().bybycu_ipc_close(C.c_void_p(p))
        self._opened = []


class ShardedQ4B32:
    """One rank's column shard of a Q4B32 weight [N, K] and the gathered GEMM."""

    def __init__(self, nibbles_full, scales_full, *, world: int, rank: int, align: int = SHARD_ALIGN):
        from .gpubackend import Q4B32Weights
        self.N, half = nibbles_full.shape
        self.K = half * 2
        self.world, self.rank = world, rank
        self.n0, self.n1 = shard_range(self.N, world, rank, align)
        self.local = Q4B32Weights(nibbles_full[self.n0:self.n1], scales_full[self.n0:self.n1]) \
            if self.n1 > self.n0 else None

    def gemm_local(self, x, out_slice, *, route: int = _lib.ROUTE_AUTO, stream=None):
        """This rank's slice out[:, n0:n1) into a contiguous [M, n1 - n0] buffer."""
        if self.local is not None:
            self.local.matmul(x, out=out_slice, route=route, stream=stream)
        return out_slice

    def gemm_allgather_peer(self, x, bufs: PeerBuffers, stream=None):
        """The slice, stored into every rank's bufs.out over NVLink, then the bounded wait."""
        bufs.epoch += 1
        M = x.shape[0]
        loc = self.local
        check(load().bybycu_tile_gemm_allgather(
            TileFormatQ4B32, M, self.K, self.N, self.n0, self.n1, _ptr(x), _dtype_code(x),
            _ptr(loc.packed) if loc else C.c_void_p(0), loc.packed.numel() if loc else 0,
            loc.scale_base if loc else 0, None, 0, 0, C.c_void_p(bufs.out.data_ptr()), bufs.peer_out,
            bufs.peer_sig, self.world, self.rank, bufs.epoch, _stream_ptr(stream)))
        return bufs.out

    def gemm_allgather_split(self, x, bufs: PeerBuffers, signal_bufs: PeerBuffers = None, stream=None):
        """Split phase: the slice goes into `bufs` (alternate two PeerBuffers between calls)
        and the launch does not wait for the other ranks; the next split call, or
        allgather_wait, completes it.  The signal array is `signal_bufs`' (default: bufs'),
        shared by both buffer sets."""
        sig = (signal_bufs or bufs)
        sig.epoch += 1
        M = x.shape[0]
        loc = self.local
        check(load().bybycu_tile_gemm_allgather_split(
            TileFormatQ4B32, M, self.K, self.N, self.n0, self.n1, _ptr(x), _dtype_code(x),
            _ptr(loc.packed) if loc else C.c_void_p(0), loc.packed.numel() if loc else 0,
            loc.scale_base if loc else 0, None, 0, 0, C.c_void_p(bufs.out.data_ptr()), bufs.peer_out,
            sig.peer_sig, self.world, self.rank, sig.epoch, _stream_ptr(stream)))
        return bufs.out

    def allgather_wait(self, signal_bufs: PeerBuffers, stream=None):
        """Completes the last split-phase call (bybycu_allgather_wait)."""
        check(load().bybycu_allgather_wait(signal_bufs.peer_sig, self.world, self.rank, signal_bufs.epoch,
                                           _stream_ptr(stream)))

    def gemm_allgather_nccl(self, x, slice_buf, gathered, group=None):
        """The baseline: compute the padded slice, NCCL all-gather, reorder to [M, N]."""
        import torch
        import torch.distributed as dist
        M = x.shape[0]
        width = slice_buf.shape[1]
        if self.local is not None:
            part = self.local.matmul(x)                   # contiguous [M, n1 - n0]
            slice_buf[:, :self.n1 - self.n0].copy_(part)
        dist.all_gather_into_tensor(gathered, slice_buf, group=group)
        parts = gathered.view(self.world, M, width)
        cols = [shard_range(self.N, self.world, r) for r in range(self.world)]
        return torch.cat([parts[r, :, :b - a] for r, (a, b) in enumerate(cols)], dim=1)
