"""Host-side logic of the path (no GPU): program words, shape helpers, backend parsing, the
weight layout and the column partition - including across two gloo ranks."""
import os

import numpy as np
import pytest

from bybylang_b200 import distributed as D
from bybylang_b200 import formats as F
from bybylang_b200 import gpubackend as gb
from bybylang_b200 import session_vm as sv


def test_program_words_match_reference_builders(oracle_mod):
    O = oracle_mod
    # buildFp4TileGemmProgram words (session_vm.nim:383-399)
    assert sv.buildFp4TileGemmProgram(0, 64, 16, 512, 0).words == list(O.fp4_tile_program(0, 64, 16, 512))
    assert sv.buildF16TileGemmProgram(5, 128, 96).words == list(O.f16_tile_program(5, 128, 96))
    assert sv.buildQ4B32TileGemmProgram(0, 64, 16, 512).words[0] == 0xB0 | (2 << 8)
    assert sv.buildFp4TileGemmProgram(0, 4096, 4096, 4096 * 2048, 0).words == \
        [0xB0, 0, 4096, 4096, 8388608, 0, 0xB1, 0xB2, 0xB4, 0xB5, 0x50, 0xB6, 0x50, 0xB3, 0xB7, 0x01]


def test_legacy_expansion_and_shape_checks():
    legacy = sv.VmProgram()
    legacy.emitFp4CoopGemm(37, 256, 80, 32, 8)
    legacy.emitHalt()
    t = sv.fp4TileProgram(legacy)
    s = sv.tileGemmShape(t)
    assert (s.format, s.M, s.K, s.N, s.scaleBase, s.lutBase) == (0, 37, 256, 80, 80 * 128, sv.fp4CoopLutWord(256, 80))
    bad = sv.VmProgram()
    bad.emitTileGemm(5, 1, 64, 16, 0, 0)
    with pytest.raises(ValueError, match="format 5 is not supported"):
        sv.tileGemmShape(bad)
    bad2 = sv.VmProgram()
    bad2.emitTileGemm(0, 1, 48, 16, 0, 0)
    with pytest.raises(ValueError, match="K=48"):
        sv.tileGemmShape(bad2)
    assert sv.tileGemmRowTile(1) == 16 and sv.tileGemmRowTile(17) == 32 and sv.tileGemmRowTile(70) == 64
    assert sv.tileGemmGroups(2048, 4096, 64) == 32 * 64
    assert sv.q4CoopRowTile(2048, 4096, 148) == 64 and sv.q4CoopRowTile(5, 96) == 16
    assert sv.vmRegA(sv.pack1(0xB0, 200)) == 200


def test_backend_parsing_and_fallback_policy():
    assert gb.parseBackend("cuda") == gb.GpuBackend.gbCuda
    assert gb.parseBackend(" Vulkan ") == gb.GpuBackend.gbVulkan
    assert gb.normalizeBackend(gb.GpuBackend.gbCuda) == gb.GpuBackend.gbCuda
    with pytest.raises(ValueError, match="unknown BybyLang backend"):
        gb.parseBackend("opencl")
    with pytest.raises(gb.BybyCudaError, match="fallback is forbidden"):
        gb.handleGpuFailure(gb.GpuBackend.gbCuda, "sessionEnd", RuntimeError("x"))
    with pytest.raises(gb.BybyCudaError, match="not provided"):
        gb.sessionBegin(gb.GpuBackend.gbVulkan)


def test_pack_layout_matches_oracle(oracle_mod):
    O = oracle_mod
    p, s = O.gen_q4b32(40, 320)
    q = F.unpack_q4b32(p)
    assert np.array_equal(F.pack_q4b32(q), p)
    import torch
    assert torch.equal(F.pack_q4b32(torch.from_numpy(q)), torch.from_numpy(p))
    assert torch.equal(F.unpack_q4b32(torch.from_numpy(p)), torch.from_numpy(q))
    # element k = 32g + j: low nibble of byte 16g + j (j < 16), high nibble of byte 16g + j - 16
    w = O.dequant_q4b32(p, s, 40, 320)
    assert np.array_equal(w, q.astype(np.float32) * O.f16_to_f32(np.repeat(s, 32, axis=1)))
    assert F.q4b32_weight_bytes(11008, 4096) == 25362432


@pytest.mark.parametrize("N,world", [(11008, 8), (4096, 3), (128256, 8), (130, 4), (64, 8), (0, 2), (11008, 7)])
def test_partition_matches_library(N, world):
    blocks = -(-N // 64)
    parts = D.partition(blocks, world)
    assert sum(parts) == blocks and max(parts) - min(parts) <= 1
    start = 0
    prev_end = 0
    for r in range(world):
        n0, n1 = D.shard_range(N, world, r)
        assert n0 == min(N, start * 64) and n1 == min(N, (start + parts[r]) * 64)
        assert n0 == prev_end
        prev_end = n1
        start += parts[r]
    assert prev_end == N


def test_partition_weighted_like_reference():
    # distributed.nim:109-135 with unequal ratios: floor then largest remainders
    assert D.partition(10, 3, [1.0, 1.0, 2.0]) == [3, 2, 5]
    assert D.partition(7, 2, [3.0, 1.0]) == [5, 2]
    with pytest.raises(ValueError):
        D.partition(-1, 2)


def _gloo_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from bybylang_b200 import distributed as DD
        mine = DD.shard_range(128256, world, rank)
        allr = [None] * world
        dist.all_gather_object(allr, mine)
        q.put((rank, allr))
    finally:
        dist.destroy_process_group()


def test_shards_agree_across_gloo_ranks():
    import multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] == res[1]
    (a0, b0), (a1, b1) = res[0]
    assert a0 == 0 and b0 == a1 and b1 == 128256 and b0 % 64 == 0
