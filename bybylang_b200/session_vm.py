"""Micro-VM program words of the tile-GEMM path, mirroring micro_kernel/session_vm.nim and the
shape helpers of micro_kernel/tile_gemm.nim.

Names keep the reference's spelling so that callers and tests read alike.  Format 2 (Q4B32:
signed int4 nibbles in the tile layout + one fp16 scale per 32-value block) is new here; its
weight slot holds the nibble bytes [N, K/2] followed, at byte ``scaleBase``, by the scales as
IEEE halves [N, K/32].
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

# opcodes (session_vm.nim:10-118) that this path uses
OP_NOP = 0x00
OP_HALT = 0x01
OP_BARRIER_TG = 0x50
OP_Q4_COOP_GEMM = 0xAA
OP_Q4_GEMV = 0xAB
OP_FP4_COOP_GEMM = 0xAC
OP_TILE_GEMM = 0xB0
OP_TILE_ZERO = 0xB1
OP_TILE_K_BEGIN = 0xB2
OP_TILE_K_END = 0xB3
OP_TILE_LOAD_A = 0xB4
OP_TILE_DECODE_FP4 = 0xB5
OP_TILE_MMA = 0xB6
OP_TILE_STORE = 0xB7
OP_TILE_LOAD_B_F16 = 0xB8

TileFormatFp4Km = 0
TileFormatF16 = 1
TileFormatQ4B32 = 2

TileGemmThreads = 128
TileGemmCols = 64
TileGemmRowTiles = (64, 32, 16)
Q4CoopRowTiles = (64, 32, 16)


def _reg_field(r: int, low: int, high: int) -> int:
    return ((r & 0x1F) << low) | (((r >> 5) & 0x7) << high)


def pack1(op: int, a: int) -> int:
    """session_vm.nim:213-214."""
    return (op & 0xFF) | _reg_field(a, 8, 23)


def vmRegA(w: int) -> int:
    """session_vm.nim:216."""
    return ((w >> 8) & 0x1F) | (((w >> 23) & 0x7) << 5)


def opImmediateWords(op: int) -> int:
    """session_vm.nim:351-356 for the ops of this path (the shape ops carry five words)."""
    return 5 if op in (OP_Q4_COOP_GEMM, OP_Q4_GEMV, OP_FP4_COOP_GEMM, OP_TILE_GEMM) else 0


@dataclass
class VmProgram:
    words: list = field(default_factory=list)

    def emit(self, w: int) -> None:
        self.words.append(int(w) & 0xFFFFFFFF)

    def emitHalt(self) -> None:
        self.emit(OP_HALT)

    def emitTileGemm(self, fmt: int, M: int, K: int, N: int, scaleBase: int, lutBase: int) -> None:
        """session_vm.nim:379-381."""
        self.emit(pack1(OP_TILE_GEMM, fmt))
        for v in (M, K, N, scaleBase, lutBase):
            self.emit(v)

    def emitFp4CoopGemm(self, M: int, K: int, N: int, groupSize: int, nGroups: int) -> None:
        """session_vm.nim:373-377."""
        self.emit(OP_FP4_COOP_GEMM)
        for v in (M, K, N, groupSize, nGroups):
            self.emit(v)

    def emitQ4Gemv(self, M: int, K: int, N: int, groupSize: int, nGroups: int) -> None:
        """session_vm.nim:418-420."""
        self.emit(OP_Q4_GEMV)
        for v in (M, K, N, groupSize, nGroups):
            self.emit(v)

    def emitQ4CoopGemm(self, M: int, K: int, N: int, groupSize: int, nGroups: int) -> None:
        """session_vm.nim:368-370."""
        self.emit(OP_Q4_COOP_GEMM)
        for v in (M, K, N, groupSize, nGroups):
            self.emit(v)

    def array(self) -> np.ndarray:
        return np.asarray(self.words, dtype=np.uint32)


def _tile_body(p: VmProgram, weight_op: int) -> VmProgram:
    for op in (OP_TILE_ZERO, OP_TILE_K_BEGIN, OP_TILE_LOAD_A, weight_op, OP_BARRIER_TG, OP_TILE_MMA,
               OP_BARRIER_TG, OP_TILE_K_END, OP_TILE_STORE, OP_HALT):
        p.emit(op)
    return p


def buildFp4TileGemmProgram(M: int, K: int, N: int, scaleBase: int, lutBase: int) -> VmProgram:
    """session_vm.nim:383-399."""
    p = VmProgram()
    p.emitTileGemm(TileFormatFp4Km, M, K, N, scaleBase, lutBase)
    return _tile_body(p, OP_TILE_DECODE_FP4)


def buildF16TileGemmProgram(M: int, K: int, N: int) -> VmProgram:
    """session_vm.nim:401-416."""
    p = VmProgram()
    p.emitTileGemm(TileFormatF16, M, K, N, 0, 0)
    return _tile_body(p, OP_TILE_LOAD_B_F16)


def buildQ4B32TileGemmProgram(M: int, K: int, N: int, scaleBase: int) -> VmProgram:
    """Format 2: the FP4-KM program shape with the Q4B32 weight format (no table)."""
    p = VmProgram()
    p.emitTileGemm(TileFormatQ4B32, M, K, N, scaleBase, 0)
    return _tile_body(p, OP_TILE_DECODE_FP4)


def fp4CoopLutWord(K: int, N: int) -> int:
    """session_vm.nim:447-450."""
    return (N * (K // 2) + N * (K // 32) + 3) // 4


def fp4CoopSupported(K: int, N: int, groupSize: int, nGroups: int) -> bool:
    """session_vm.nim:442-445."""
    return K > 0 and K % 64 == 0 and N >= 16 and groupSize == 32 and nGroups == K // 32


def fp4TileProgram(p: VmProgram) -> VmProgram:
    """tile_gemm.nim:55-66: the legacy one-blob shape op expands to a tile program."""
    w = p.words
    if w and (w[0] & 0xFF) == OP_TILE_GEMM:
        return p
    if len(w) == 7 and (w[0] & 0xFF) == OP_FP4_COOP_GEMM and w[6] == OP_HALT:
        M, K, N = w[1], w[2], w[3]
        if w[4] != 32 or K % 32 != 0 or w[5] != K // 32:
            raise ValueError("FP4 cooperative micro-kernel needs group 32 and K/32 groups")
        return buildFp4TileGemmProgram(M, K, N, N * (K // 2), fp4CoopLutWord(K, N))
    raise ValueError("not an FP4-KM tile GEMM micro-kernel program")


@dataclass
class TileGemmShape:
    format: int
    M: int
    K: int
    N: int
    scaleBase: int
    lutBase: int


def tileGemmShape(p: VmProgram) -> TileGemmShape:
    """tile_gemm.nim:68-80, with format 2 accepted."""
    q = fp4TileProgram(p)
    if len(q.words) < 6:
        raise ValueError("truncated tile GEMM header")
    w = q.words
    s = TileGemmShape(vmRegA(w[0]), w[1], w[2], w[3], w[4], w[5])
    if s.format not in (TileFormatFp4Km, TileFormatF16, TileFormatQ4B32):
        raise ValueError(f"tile GEMM weight format {s.format} is not supported (0 = FP4-KM, 1 = FP16, 2 = Q4B32)")
    if s.K <= 0 or s.K % 32 != 0 or s.N <= 0:
        raise ValueError(f"unsupported tile GEMM shape K={s.K} N={s.N}")
    return s


def tileGemmRowTile(rows: int) -> int:
    """tile_gemm.nim:88-90."""
    return 16 if rows <= 16 else 32 if rows <= 32 else 64


def tileGemmGroups(rows: int, N: int, rowTile: int) -> int:
    """tile_gemm.nim:92-94."""
    return ((rows + rowTile - 1) // rowTile) * ((N + TileGemmCols - 1) // TileGemmCols)


def q4CoopRowTile(rows: int, N: int, computeUnits: int = 0, perUnit: int = 2) -> int:
    """session_vm.nim:452-464."""
    units = computeUnits if computeUnits > 0 else 64
    cols = (N + 63) // 64
    for bm in (64, 32):
        if rows > bm // 2 and ((rows + bm - 1) // bm) * cols >= perUnit * units:
            return bm
    return 16


def tileWeightBytes(fmt: int, K: int, N: int) -> int:
    """Bytes of the packed weight slot of one op (tryTileGemm's size check,
    backends/vulkan/vulkan_driver.nim:2617-2619, with format 2 added)."""
    if fmt == TileFormatF16:
        return N * K * 2
    if fmt == TileFormatQ4B32:
        return N * (K // 2) + N * (K // 32) * 2
    return N * (K // 2) + N * (K // 32)
