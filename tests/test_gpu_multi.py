"""Column sharding over two GPUs (one process per GPU).  After the device-side all-gather
(bybycu_tile_gemm_allgather over CUDA IPC peer pointers) every rank holds, bit for bit, the
concatenation of the ranks' own shard GEMMs - the transport is exact - and that result matches
the single-GPU GEMM within the route's tolerance (a shard may pick another tiling of the same
sums than the full-width call).  The split-phase form (bybycu_tile_gemm_allgather_split over
two alternating buffer sets, completed by bybycu_allgather_wait) and the NCCL all-gather
variant are checked the same way.  Skipped with fewer than two GPUs."""
import os
import socket
from datetime import timedelta

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# GEMV (fused gather) at M = 1, 4, 16; tensor-core GEMM with one round of tiles (the copy
# kernel gathers) at M = 64 over ragged 256-row tiles and at M = 300 over three token tiles;
# tensor-core GEMM with more tiles than CTA pairs (the gather fused into its epilogue)
CASES = [(1, 4096, 11008), (4, 4096, 1000), (16, 2048, 4160), (64, 4096, 4160), (300, 1024, 512),
         (128, 1024, 40960)]


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import torch.distributed as dist
        from bybylang_b200 import _lib
        from bybylang_b200 import gpubackend as gb
        from bybylang_b200.distributed import PeerBuffers, ShardedQ4B32, shard_range
        from bybylang_b200.formats import synthetic_q4b32, synthetic_x
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        gb.ensureGpuInit(gb.GpuBackend.gbCuda, rank)
        results = []
        for (M, K, N) in CASES:
            nib, sc = synthetic_q4b32(N, K, seed=5 + N, device=dev)
            x = synthetic_x(M, K, seed=6 + M, device=dev)
            full = gb.Q4B32Weights(nib, sc, device=dev).matmul(x)
            sh = ShardedQ4B32(nib, sc, world=world, rank=rank)
            # the exact expectation: every rank's own shard result, gathered by NCCL
            width = max(b - a for a, b in (shard_range(N, world, r) for r in range(world)))
            slice_buf = torch.zeros(M, width, dtype=torch.float32, device=dev)
            gathered = torch.empty(world * M * width, dtype=torch.float32, device=dev)
            expect = sh.gemm_allgather_nccl(x, slice_buf, gathered)
            torch.cuda.synchronize()
            bufs = PeerBuffers(M, N, world, rank)
            exact, nan, maxd = True, 0, 0.0
            for _ in range(3):   # three epochs back to back
                bufs.out.fill_(float("nan"))
                torch.cuda.synchronize()
                dist.barrier()
                out = sh.gemm_allgather_peer(x, bufs)
                torch.cuda.synchronize()
                exact &= bool(torch.equal(out, expect))
                nan = max(nan, int(torch.isnan(out).sum()))
                maxd = max(maxd, float((out - expect).abs().nan_to_num(float("inf")).max()))
            # split phase: calls alternate between two buffer sets (one signal array), no
            # launch waits at its end; the next call or allgather_wait completes each one
            bufs_b = PeerBuffers(M, N, world, rank)
            for _ in range(2):
                for b in (bufs, bufs_b):
                    b.out.fill_(float("nan"))
                torch.cuda.synchronize()
                dist.barrier()
                sh.gemm_allgather_split(x, bufs, bufs)
                sh.gemm_allgather_split(x, bufs_b, bufs)
                sh.allgather_wait(bufs)
                torch.cuda.synchronize()
                for b in (bufs, bufs_b):
                    exact &= bool(torch.equal(b.out, expect))
                    nan = max(nan, int(torch.isnan(b.out).sum()))
            peak = max(1.0, float(full.abs().max()))
            rel = float((expect - full).abs().max()) / peak
            results.append((M, K, N, exact, nan, maxd, rel, _lib.device_error()))
            dist.barrier()
            bufs_b.close()
            bufs.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, results, None))
    except Exception as e:   # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


def test_allgather_over_two_gpus_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in procs:
            rank, results, err = q.get(timeout=300)
            got[rank] = (results, err)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, (results, err) in sorted(got.items()):
        assert err is None, f"rank {rank}: {err}"
        for (M, K, N, exact, nan, maxd, rel, dev_err) in results:
            what = f"rank {rank} M={M} K={K} N={N}"
            assert exact, f"{what}: peer all-gather != gathered shards ({nan} NaN, max diff {maxd:.3e})"
            # GEMV routes (M <= 16): 1e-4 of the peak; tensor-core route: 1e-3 (fp16 weights)
            assert rel <= (1e-4 if M <= 16 else 1e-3), f"{what}: shards vs one GPU {rel:.3e}"
            assert dev_err == 0, f"{what}: device error {dev_err}"
    assert sorted(got) == [0, 1]
