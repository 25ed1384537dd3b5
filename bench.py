"""Benchmark of the Q4B32 tile-GEMM path on B200 (one JSON line on rank 0).

Workload (a "step"): one decode GEMV of BASELINE config C2 - x bf16 [1, 4096] ~N(0,1),
Q4B32 weights [11008, 4096] (int4 uniform [-8, 7], one fp16 scale |N(0, 0.02)| per 32-block),
fp32 out - through libbybycuda's GEMV route.  Algorithmic bytes per step: 25,362,432 weight +
8,192 x + 44,032 out = 25,414,656 B.

* value       whole-job GB/s with inputs resident in HBM: K steps replayed from a CUDA graph
              over 20 rotating weight copies (507 MB > 4x the 126 MB L2, so every step reads
              its weights from HBM), timed with CUDA events on the launching stream.
* e2e         the same metric through bybycu_tile_gemm_host with pinned HOST x and out
              (H2D of x, the kernel, D2H of out, stream sync - every step).
* roofline    algorithmic bytes per launch / average launch duration vs measured HBM peak.
* cpu_baseline  the reference's own CPU C (oracle/_ref: OP_TILE_GEMM through
              nimf_cpu_vm_run_slots, single-threaded as the reference is) on the same shape.
* prefill     config C3 (M=2048, K=N=4096) TFLOP/s when the tensor-core route is present.
* f16_decode  format 1 (fp16 weights) at the C2 shape through the tile GEMM's decode route.
* q4_asym_decode  the asymmetric Q4 data of the reference's matmul_q4 (interleaved nibbles, fp32
              scales and zero points per 32-block, fp32 x) at the C2 shape through
              bybycu_matmul_q4's decode kernel: GB/s of its 0.75 B/weight, rotating sets > 4x L2.
* q4_asym_prefill  the asymmetric Q4 data at the C3 shape through bybycu_matmul_q4's
              tensor-core route, TFLOP/s.
* decode_x_f32  the headline step with fp32 activations (the session API's type).
* ingest      GB/s of a 1 GiB file mapping copied into HBM by bybycu_upload_host_range (the copy
              of residentUploadQ4Mapped), host clock, beside a plain pageable copy.

N > 1 GPUs (torchrun, one process per GPU): weak scaling.  Each rank owns an 11008-column
shard of a [11008*N, 4096] Q4B32 projection and every step ends with the device-side
all-gather of the fp32 output slices over NVLink (bybycu_tile_gemm_allgather: one launch, the
GEMV stores to the peers itself); value = all ranks' bytes / max-over-ranks time.  e2e at N > 1:
upload x, the gathered GEMV, download the whole [1, 11008*N] output, sync - on every rank.

`--impl reference` times the reference's CPU implementation (oracle/_ref, column-sharded over
all host threads) on the same workload and prints the same line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time
import warnings

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q4 GEMM: decode GB/s vs HBM peak; prefill TFLOP/s; at 1/2/4/8 B200"
M_DEC, K_DEC, N_DEC = 1, 4096, 11008
W_BYTES = N_DEC * (K_DEC // 2) + N_DEC * (K_DEC // 32) * 2
STEP_BYTES = W_BYTES + M_DEC * K_DEC * 2 + M_DEC * N_DEC * 4
L2_BYTES = 126 * 1024 * 1024
SEED = 2463534242


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def profiled_traffic(summary: str):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of the bench kernel,
    from the committed ncu summary under profiles/ (one `--set full` capture)."""
    try:
        with open(os.path.join(ROOT, "profiles", summary)) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return int(line.split(":", 1)[1])
    except (OSError, ValueError):
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.samples = []
        self.proc = None
        self.window = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), line.strip()))

    def mark(self, t0, t1):
        self.window = (t0, t1)

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        for t, line in self.samples:
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9:
                continue
            rows.append((t, p))
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        inside = [r for r in rows if self.window and self.window[0] <= r[0] <= self.window[1]]
        use = inside or rows
        sm = [float(p[1]) for _, p in use if p[1].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for _, p in use:
            for name, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(use[0][1][2]) if use[0][1][2].replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(use),
                "window": "timed" if inside else "run"}


def cpu_baseline(threads: int, min_seconds: float):
    """The reference's own CPU C on the decode workload (kind "reference"), else the port."""
    import numpy as np
    from oracle import oracle as O
    p, s = O.gen_q4b32(N_DEC, K_DEC, seed=SEED)
    x = O.bf16_to_f32(O.gen_x_bf16(M_DEC, K_DEC, seed=SEED + 2))
    pal = s.ravel()[:256].copy()
    s = pal[(np.arange(s.size) * 7919) % 256].reshape(s.shape)   # <= 256 scales: the VM's table
    blob, table = O.q4b32_to_fp4km(p, s, N_DEC, K_DEC)
    if O.ref_available():
        kind = "reference"
        fn = lambda: O.ref_tile_gemm(x, blob, table, M_DEC, K_DEC, N_DEC, threads=threads)  # noqa: E731
        what = "OP_TILE_GEMM via nimf_cpu_vm_run_slots (oracle/_ref, reference C unchanged)"
    else:
        kind = "port"
        fn = lambda: O.tile_gemm_q4b32(x, p, s, M_DEC, K_DEC, N_DEC, threads=threads)  # noqa: E731
        what = "q4_oracle.c restatement of cpu_vm.c:605-626"
    fn()
    reps, t0 = 0, time.perf_counter()
    while True:
        fn()
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    per = el / reps
    return {"value": round(STEP_BYTES / per / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": f"full decode GEMV (M=1, K=4096, N=11008) x {reps} runs, {what}; "
                      f"{per * 1e3:.1f} ms per run", "seconds_per_step": per}


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    from oracle import oracle as O
    base = cpu_baseline(threads, 0.0)   # inputs + warm check
    import numpy as np
    p, s = O.gen_q4b32(N_DEC, K_DEC, seed=SEED)
    x = O.bf16_to_f32(O.gen_x_bf16(M_DEC, K_DEC, seed=SEED + 2))
    pal = s.ravel()[:256].copy()
    s = pal[(np.arange(s.size) * 7919) % 256].reshape(s.shape)
    blob, table = O.q4b32_to_fp4km(p, s, N_DEC, K_DEC)
    run = (lambda: O.ref_tile_gemm(x, blob, table, M_DEC, K_DEC, N_DEC, threads=threads)) if O.ref_available() \
        else (lambda: O.tile_gemm_q4b32(x, p, s, M_DEC, K_DEC, N_DEC, threads=threads))
    for _ in range(args.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    el = time.perf_counter() - t0
    v = STEP_BYTES * args.steps / el / 1e9
    line = {"metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": "decode GEMV C2: M=1 K=4096 N=11008 Q4B32 (x widened to fp32)",
                       "cpu_threads": threads},
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": threads, "kind": base["kind"],
                             "sample": f"{args.steps} full decode GEMVs, column-sharded over {threads} threads "
                                       "(the distributed.nim split)"},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-q4asym", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        return reference_arm(args)
    args.warmup = max(args.warmup, 3)

    import torch
    import torch.distributed as dist
    import numpy as np
    from bybylang_b200 import _lib
    from bybylang_b200 import gpubackend as gb
    from bybylang_b200.formats import synthetic_q4b32, synthetic_x

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        # NCCL may print its version banner on stdout while the communicator comes up; send
        # that to stderr so that stdout carries the one JSON line
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
            dist.barrier()
        finally:
            os.dup2(saved, 1)
            os.close(saved)
    gb.ensureGpuInit(gb.GpuBackend.gbCuda, local)
    dev = torch.device("cuda", local)
    hbm_peak, tc_peak, peak_kind = peaks()

    # ---- resident inputs: rotating weight copies
    copies = max(2, -(-4 * L2_BYTES // W_BYTES))
    weights = []
    for c in range(copies):
        nib, sc = synthetic_q4b32(N_DEC, K_DEC, seed=SEED + 1000 * rank + c, device=dev)
        weights.append(gb.Q4B32Weights(nib, sc, device=dev))
    x = synthetic_x(M_DEC, K_DEC, seed=SEED + 2, device=dev)
    N_total = N_DEC * world
    stream = torch.cuda.Stream(device=dev)

    if world > 1:
        from bybylang_b200.distributed import PeerBuffers
        bufs = PeerBuffers(M_DEC, N_total, world, rank)
        n0, n1 = rank * N_DEC, (rank + 1) * N_DEC
        lib = _lib.load()

        def launch(i):
            w = weights[i % copies]
            _lib.check(lib.bybycu_tile_gemm_allgather(
                2, M_DEC, K_DEC, N_total, n0, n1, C.c_void_p(x.data_ptr()), _lib.DT_BF16,
                C.c_void_p(w.packed.data_ptr()), w.packed.numel(), w.scale_base, None, 0, 0,
                C.c_void_p(bufs.out.data_ptr()), bufs.peer_out, bufs.peer_sig, world, rank, 0,
                C.c_void_p(stream.cuda_stream)))
        launches_per_step = 1   # the GEMV stores to the peers and waits in the same launch
    else:
        outs = [torch.empty(M_DEC, N_DEC, dtype=torch.float32, device=dev) for _ in range(copies)]

        def launch(i):
            w = weights[i % copies]
            gb.tile_gemm(2, x, w.packed, outs[i % copies], M=M_DEC, K=K_DEC, N=N_DEC, scale_base=w.scale_base,
                         route=_lib.ROUTE_GEMV, stream=stream)
        launches_per_step = 1

    # ---- capture one graph over all copies; replay it
    with torch.cuda.stream(stream):
        for i in range(copies):
            launch(i)
    stream.synchronize()
    if world > 1:
        dist.barrier()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(copies):
            launch(i)
    reps_w = -(-args.warmup // copies)
    reps_t = -(-args.steps // copies)
    steps = reps_t * copies
    with torch.cuda.stream(stream):
        for _ in range(reps_w):
            graph.replay()
    stream.synchronize()
    assert _lib.device_error() == 0

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.time()
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(reps_t):
            graph.replay()
    e1.record(stream)
    stream.synchronize()
    w1 = time.time()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.mark(w0, w1)
    time.sleep(0.25)
    sampler.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    assert _lib.device_error() == 0
    per_launch_ms = ms / steps
    value = STEP_BYTES * world * steps / (ms / 1e3) / 1e9
    achieved = STEP_BYTES / (per_launch_ms / 1e3) / 1e9

    # ---- e2e through the C-ABI host entry (N = 1), host buffers, copies inside the timed region
    e2e = None
    if world > 1:
        # every step on every rank: pinned x -> device (bybycu_upload), the sharded GEMV with its
        # device all-gather, the gathered [1, N_total] output -> pinned host (bybycu_download),
        # stream sync; the max over ranks of the host-timed loop
        lib = _lib.load()
        xh = x.cpu().pin_memory()
        oh = torch.empty(M_DEC, N_total, dtype=torch.float32).pin_memory()
        xd = torch.empty_like(x)
        sp = C.c_void_p(stream.cuda_stream)
        x_bytes, o_bytes = M_DEC * K_DEC * 2, M_DEC * N_total * 4

        def e2e_step(i):
            w = weights[i % copies]
            _lib.check(lib.bybycu_upload(C.c_void_p(xd.data_ptr()), C.c_void_p(xh.data_ptr()), x_bytes, sp))
            _lib.check(lib.bybycu_tile_gemm_allgather(
                2, M_DEC, K_DEC, N_total, n0, n1, C.c_void_p(xd.data_ptr()), _lib.DT_BF16,
                C.c_void_p(w.packed.data_ptr()), w.packed.numel(), w.scale_base, None, 0, 0,
                C.c_void_p(bufs.out.data_ptr()), bufs.peer_out, bufs.peer_sig, world, rank, 0, sp))
            _lib.check(lib.bybycu_download(C.c_void_p(oh.data_ptr()), C.c_void_p(bufs.out.data_ptr()), o_bytes, sp))
            _lib.check(lib.bybycu_synchronize(sp))
        for i in range(max(args.warmup, 20)):
            e2e_step(i)
        n_e2e = min(steps, 5000)
        dist.barrier()
        t0 = time.perf_counter()
        for i in range(n_e2e):
            e2e_step(i)
        el = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
        dist.all_reduce(el, op=dist.ReduceOp.MAX)
        el = float(el.item())
        e2e = {"value": round(STEP_BYTES * world * n_e2e / el / 1e9, 2), "unit": "GB/s",
               "h2d_bytes_per_step": x_bytes * world, "d2h_bytes_per_step": o_bytes * world,
               "steps": n_e2e, "us_per_step": round(el / n_e2e * 1e6, 2),
               "api": "bybycu_upload + bybycu_tile_gemm_allgather + bybycu_download + bybycu_synchronize "
                      "(C ABI) on every rank, pinned host x/out, max over ranks"}
    if world == 1:
        lib = _lib.load()
        xh = x.cpu().pin_memory()
        oh = torch.empty(M_DEC, N_DEC, dtype=torch.float32).pin_memory()
        xd = torch.empty_like(x)
        od = torch.empty(M_DEC, N_DEC, dtype=torch.float32, device=dev)
        sp = C.c_void_p(stream.cuda_stream)

        def e2e_step(i):
            w = weights[i % copies]
            _lib.check(lib.bybycu_tile_gemm_host(2, M_DEC, K_DEC, N_DEC, C.c_void_p(xh.data_ptr()), _lib.DT_BF16,
                                                 C.c_void_p(w.packed.data_ptr()), w.packed.numel(), w.scale_base,
                                                 None, 0, 0, C.c_void_p(oh.data_ptr()), _lib.DT_F32,
                                                 C.c_void_p(xd.data_ptr()), C.c_void_p(od.data_ptr()),
                                                 _lib.ROUTE_GEMV, sp))
        for i in range(max(args.warmup, 20)):
            e2e_step(i)
        n_e2e = min(steps, 5000)
        t0 = time.perf_counter()
        for i in range(n_e2e):
            e2e_step(i)
        el = time.perf_counter() - t0
        e2e = {"value": round(STEP_BYTES * n_e2e / el / 1e9, 2), "unit": "GB/s",
               "h2d_bytes_per_step": M_DEC * K_DEC * 2, "d2h_bytes_per_step": M_DEC * N_DEC * 4,
               "steps": n_e2e, "us_per_step": round(el / n_e2e * 1e6, 2),
               "api": "bybycu_tile_gemm_host (C ABI), pinned host x/out"}

    # ---- prefill (config C3) when the tensor-core route exists
    prefill = None
    if world == 1 and not args.no_prefill:
        Mp, Kp, Np = 2048, 4096, 4096
        try:
            if gb.route_for(2, Mp, Kp, Np) == _lib.ROUTE_TC:
                # rotating (weights, activations, output) sets larger than 4x L2 together, so each
                # call reads its inputs from HBM; calls run back to back on one stream
                per_set = W_BYTES * Np // N_DEC + Mp * Kp * 2 + Mp * Np * 2
                n_sets = max(2, -(-4 * L2_BYTES // per_set))
                sets = []
                for c in range(n_sets):
                    nib, sc = synthetic_q4b32(Np, Kp, seed=SEED + 7 + c, device=dev)
                    sets.append((gb.Q4B32Weights(nib, sc, device=dev),
                                 synthetic_x(Mp, Kp, seed=SEED + 100 + c, device=dev),
                                 torch.empty(Mp, Np, dtype=torch.bfloat16, device=dev)))
                with torch.cuda.stream(stream):
                    for i in range(2 * n_sets):
                        wp, xp, op = sets[i % n_sets]
                        wp.matmul(xp, op, route=_lib.ROUTE_TC, stream=stream)
                stream.synchronize()
                reps = 10 * n_sets
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                with torch.cuda.stream(stream):
                    for i in range(reps):
                        wp, xp, op = sets[i % n_sets]
                        wp.matmul(xp, op, route=_lib.ROUTE_TC, stream=stream)
                b.record(stream)
                stream.synchronize()
                assert _lib.device_error() == 0
                t = a.elapsed_time(b) / reps
                tf = 2.0 * Mp * Np * Kp / (t / 1e3) / 1e12
                prefill = {"value": round(tf, 2), "unit": "TFLOP/s", "workload": "C3 M=2048 K=N=4096 Q4B32, x bf16, bf16 out",
                           "ms_per_call": round(t, 5), "calls": reps,
                           "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": tc_peak, "unit": "TFLOP/s",
                                        "frac": round(tf / tc_peak, 4), "peak_kind": peak_kind,
                                        "traffic": profiled_traffic("tc_gemm_prefill_c3.md"),
                                        "traffic_source": "ncu --set full, one gemm_kernel launch: "
                                                          "profiles/tc_gemm_prefill_c3.md"},
                           "includes": "fp16 staging pass + tcgen05 GEMM (2 launches per call)",
                           "l2": f"inputs larger than L2: {n_sets} rotating (W, x, out) sets ({n_sets * per_set >> 20} MiB), "
                                 "back-to-back calls, CUDA events on the launching stream"}
        except _lib.BybyCudaError as e:
            prefill = {"error": str(e)}

    # ---- asymmetric Q4 prefill at the C3 shape: bybycu_matmul_q4's tensor-core route
    q4asym_prefill = None
    if world == 1 and not args.no_prefill and not args.no_q4asym:
        Mp, Kp, Np = 2048, 4096, 4096
        try:
            Gp = Kp // 32
            per_set = Np * Kp // 2 + 2 * Np * Gp * 4 + Mp * Kp * 4 + Mp * Np * 4
            n_sets = max(2, -(-4 * L2_BYTES // per_set))
            gen = torch.Generator(device=dev).manual_seed(SEED + 51)
            asets = []
            for c in range(n_sets):
                wq = torch.randint(0, 256, (Np, Kp // 2), dtype=torch.uint8, device=dev, generator=gen)
                sc = torch.rand(Np, Gp, device=dev, generator=gen) * 0.02 + 1e-4
                zp = torch.rand(Np, Gp, device=dev, generator=gen) * 15
                asets.append((wq, sc, zp, torch.randn(Mp, Kp, device=dev, generator=gen),
                              torch.empty(Mp, Np, device=dev)))
            lib = _lib.load()

            def asym_call(i):
                wq, sc, zp, xa, oa = asets[i % n_sets]
                _lib.check(lib.bybycu_matmul_q4(C.c_void_p(xa.data_ptr()), C.c_void_p(wq.data_ptr()),
                                                C.c_void_p(sc.data_ptr()), C.c_void_p(zp.data_ptr()),
                                                C.c_void_p(oa.data_ptr()), Mp, Kp, Np, 32, Gp, _lib.ROUTE_TC,
                                                C.c_void_p(stream.cuda_stream)))
            for i in range(2 * n_sets):
                asym_call(i)
            stream.synchronize()
            reps = 10 * n_sets
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for i in range(reps):
                asym_call(i)
            b.record(stream)
            stream.synchronize()
            assert _lib.device_error() == 0
            t = a.elapsed_time(b) / reps
            tf = 2.0 * Mp * Np * Kp / (t / 1e3) / 1e12
            q4asym_prefill = {"value": round(tf, 2), "unit": "TFLOP/s",
                              "workload": "asymmetric Q4 prefill M=2048 K=N=4096 (group 32), x fp32, out fp32",
                              "ms_per_call": round(t, 5), "calls": reps,
                              "frac": round(tf / tc_peak, 4), "peak_kind": peak_kind,
                              "includes": "fp16 staging pass + tcgen05 GEMM (2 launches per call)",
                              "l2": f"inputs larger than L2: {n_sets} rotating sets, back-to-back calls"}
            del asets
        except _lib.BybyCudaError as e:
            q4asym_prefill = {"error": str(e)}

    # ---- asymmetric Q4 decode (the matmul_q4 data: interleaved nibbles, fp32 scales and zero
    # points per 32-block, fp32 x) at the C2 shape, through bybycu_matmul_q4's decode kernel
    q4asym = None
    if world == 1 and not args.no_q4asym:
        try:
            G = K_DEC // 32
            wbytes = N_DEC * K_DEC // 2 + N_DEC * G * 8
            abytes = wbytes + K_DEC * 4 + N_DEC * 4
            n_sets = max(2, -(-4 * L2_BYTES // wbytes))
            gen = torch.Generator(device=dev).manual_seed(SEED + 31)
            qsets = []
            for c in range(n_sets):
                wq = torch.randint(0, 256, (N_DEC, K_DEC // 2), dtype=torch.uint8, device=dev, generator=gen)
                sc = torch.rand(N_DEC, G, device=dev, generator=gen) * 0.02 + 1e-4
                zp = torch.rand(N_DEC, G, device=dev, generator=gen) * 15
                qsets.append((gb.Q4AsymWeights(wq, sc, zp, K_DEC), torch.empty(1, N_DEC, device=dev)))
            xa = torch.randn(1, K_DEC, device=dev, generator=gen)
            with torch.cuda.stream(stream):
                for wqs, o in qsets:
                    wqs.matmul(xa, o, route=_lib.ROUTE_GEMV, stream=stream)
            stream.synchronize()
            qgraph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(qgraph, stream=stream):
                for wqs, o in qsets:
                    wqs.matmul(xa, o, route=_lib.ROUTE_GEMV, stream=stream)
            reps = max(20, min(reps_t, 4000 // n_sets))
            with torch.cuda.stream(stream):
                for _ in range(3):
                    qgraph.replay()
            stream.synchronize()
            qa, qb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            qa.record(stream)
            with torch.cuda.stream(stream):
                for _ in range(reps):
                    qgraph.replay()
            qb.record(stream)
            stream.synchronize()
            assert _lib.device_error() == 0
            t_us = qa.elapsed_time(qb) * 1e3 / (reps * n_sets)
            gbs = abytes / (t_us * 1e-6) / 1e9
            q4asym = {"value": round(gbs, 2), "unit": "GB/s", "us_per_launch": round(t_us, 3),
                      "workload": "asymmetric Q4 decode M=1 K=4096 N=11008 (nibbles, fp32 scales + zero "
                                  "points per 32-block, x fp32, out fp32)",
                      "algorithmic_bytes": abytes, "launches": reps * n_sets,
                      "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": hbm_peak, "unit": "GB/s",
                                   "frac": round(gbs / hbm_peak, 4), "peak_kind": peak_kind},
                      "l2": f"inputs larger than L2: {n_sets} rotating weight sets, CUDA graph replay"}
            # the fused gate/up form of the same data (a Llama FFN's first half): RMSNorm of x,
            # silu(gate) * up, residual, one launch over two 11008 x 4096 matrices per step
            gamma = torch.rand(1, K_DEC, device=dev, generator=gen) + 0.5
            resid = torch.randn(1, N_DEC, device=dev, generator=gen)
            pairs = [(qsets[2 * i][0], qsets[2 * i + 1][0], torch.empty(1, N_DEC, device=dev),
                      torch.empty(1, N_DEC, device=dev)) for i in range(n_sets // 2)]
            fgraph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                for wg, wu, o0, o1 in pairs:
                    gb.matmul_q4_fused(1, xa, [wg, wu], [o0, o1], res=resid, gamma=gamma, eps=1e-5, stream=stream)
            stream.synchronize()
            with torch.cuda.graph(fgraph, stream=stream):
                for wg, wu, o0, o1 in pairs:
                    gb.matmul_q4_fused(1, xa, [wg, wu], [o0, o1], res=resid, gamma=gamma, eps=1e-5, stream=stream)
            with torch.cuda.stream(stream):
                for _ in range(3):
                    fgraph.replay()
            stream.synchronize()
            fa, fb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            fa.record(stream)
            with torch.cuda.stream(stream):
                for _ in range(reps):
                    fgraph.replay()
            fb.record(stream)
            stream.synchronize()
            assert _lib.device_error() == 0
            f_us = fa.elapsed_time(fb) * 1e3 / (reps * len(pairs))
            fbytes = 2 * wbytes + 2 * K_DEC * 4 + 2 * N_DEC * 4
            q4asym["fused_gate_up"] = {
                "value": round(fbytes / (f_us * 1e-6) / 1e9, 2), "unit": "GB/s", "us_per_launch": round(f_us, 3),
                "workload": "fused decode GEMV mode 1: RMSNorm(x), silu(x.Wg) * (x.Wu) + residual, "
                            "Wg, Wu 11008 x 4096 asymmetric Q4, one launch",
                "algorithmic_bytes": fbytes,
                "roofline": {"bound": "hbm", "achieved": round(fbytes / (f_us * 1e-6) / 1e9, 2), "peak": hbm_peak,
                             "unit": "GB/s", "frac": round(fbytes / (f_us * 1e-6) / 1e9 / hbm_peak, 4),
                             "peak_kind": peak_kind}}
            del qgraph, fgraph
        except _lib.BybyCudaError as e:
            q4asym = {"error": str(e)}

    # ---- format 1 (fp16 weights, 2 B per weight) decode at the C2 shape, through the tile GEMM's
    # decode route
    f16dec = None
    if world == 1 and not args.no_q4asym:
        try:
            fbytes = N_DEC * K_DEC * 2
            n_sets = max(2, -(-4 * L2_BYTES // fbytes))
            gen = torch.Generator(device=dev).manual_seed(SEED + 41)
            hsets = [((torch.randn(N_DEC, K_DEC, device=dev, generator=gen) * 0.05).half().view(torch.uint8),
                      torch.empty(1, N_DEC, device=dev)) for _ in range(n_sets)]

            def f16_launch(i):
                wh, o = hsets[i % n_sets]
                gb.tile_gemm(1, x, wh, o, M=1, K=K_DEC, N=N_DEC, route=_lib.ROUTE_GEMV, stream=stream)
            with torch.cuda.stream(stream):
                for i in range(n_sets):
                    f16_launch(i)
            stream.synchronize()
            hgraph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(hgraph, stream=stream):
                for i in range(n_sets):
                    f16_launch(i)
            reps = max(20, min(reps_t, 2000 // n_sets))
            with torch.cuda.stream(stream):
                for _ in range(3):
                    hgraph.replay()
            stream.synchronize()
            ha, hb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ha.record(stream)
            with torch.cuda.stream(stream):
                for _ in range(reps):
                    hgraph.replay()
            hb.record(stream)
            stream.synchronize()
            assert _lib.device_error() == 0
            h_us = ha.elapsed_time(hb) * 1e3 / (reps * n_sets)
            hbytes = fbytes + K_DEC * 2 + N_DEC * 4
            f16dec = {"value": round(hbytes / (h_us * 1e-6) / 1e9, 2), "unit": "GB/s", "us_per_launch": round(h_us, 3),
                      "workload": "format 1 (fp16 weights) decode M=1 K=4096 N=11008, x bf16, out fp32",
                      "algorithmic_bytes": hbytes,
                      "roofline": {"bound": "hbm", "achieved": round(hbytes / (h_us * 1e-6) / 1e9, 2),
                                   "peak": hbm_peak, "unit": "GB/s",
                                   "frac": round(hbytes / (h_us * 1e-6) / 1e9 / hbm_peak, 4), "peak_kind": peak_kind},
                      "l2": f"inputs larger than L2: {n_sets} rotating weight sets, CUDA graph replay"}
            del hgraph, hsets
        except _lib.BybyCudaError as e:
            f16dec = {"error": str(e)}

    # ---- the C2 decode with fp32 activation rows (the reference's own activation type)
    dec32 = None
    if world == 1 and not args.no_q4asym:
        try:
            x32 = x.float().contiguous()

            def launch32(i):
                w = weights[i % copies]
                gb.tile_gemm(2, x32, w.packed, outs[i % copies], M=M_DEC, K=K_DEC, N=N_DEC,
                             scale_base=w.scale_base, route=_lib.ROUTE_GEMV, stream=stream)
            g32 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g32, stream=stream):
                for i in range(copies):
                    launch32(i)
            reps = max(20, min(reps_t, 4000 // copies))
            with torch.cuda.stream(stream):
                for _ in range(3):
                    g32.replay()
            stream.synchronize()
            da, db = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            da.record(stream)
            with torch.cuda.stream(stream):
                for _ in range(reps):
                    g32.replay()
            db.record(stream)
            stream.synchronize()
            assert _lib.device_error() == 0
            d_us = da.elapsed_time(db) * 1e3 / (reps * copies)
            dbytes = W_BYTES + K_DEC * 4 + N_DEC * 4
            dec32 = {"value": round(dbytes / (d_us * 1e-6) / 1e9, 2), "unit": "GB/s", "us_per_launch": round(d_us, 3),
                     "workload": "decode GEMV C2 with x fp32 (the session API's activation type), out fp32",
                     "algorithmic_bytes": dbytes,
                     "frac": round(dbytes / (d_us * 1e-6) / 1e9 / hbm_peak, 4), "peak_kind": peak_kind}
            del g32
        except _lib.BybyCudaError as e:
            dec32 = {"error": str(e)}

    # ---- weight ingestion: a checkpoint mapping copied into HBM (residentUploadQ4Mapped's copy)
    ingest = None
    if world == 1 and not args.no_q4asym:
        import tempfile
        from bybylang_b200.mapped_file import openReadOnlyMapping, unmapReadOnlyFile
        path = None
        try:
            nbytes = 1 << 30
            fd, path = tempfile.mkstemp(prefix="bybyb200_ingest_", suffix=".bin")
            blk = np.random.default_rng(SEED).integers(0, 256, 64 << 20, dtype=np.uint8).tobytes()
            with os.fdopen(fd, "wb") as f:
                for _ in range(nbytes // len(blk)):
                    f.write(blk)
            dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            m = openReadOnlyMapping(path)
            try:
                rates = []
                for _ in range(3):
                    torch.cuda.synchronize()
                    t0 = time.perf_counter()
                    _lib.call("bybycu_upload_host_range", C.c_void_p(dst.data_ptr()), C.c_void_p(m.data), nbytes)
                    rates.append(nbytes / (time.perf_counter() - t0) / 1e9)
                ok = torch.equal(dst[:len(blk)], torch.from_numpy(np.frombuffer(blk, np.uint8).copy()).to(dev))
                with warnings.catch_warnings():   # a read-only mapping: torch only reads it here
                    warnings.simplefilter("ignore", UserWarning)
                    src = torch.from_numpy(m.view())   # pageable: the driver's own staging
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                dst.copy_(src)
                torch.cuda.synchronize()
                plain = nbytes / (time.perf_counter() - t0) / 1e9
            finally:
                unmapReadOnlyFile(m)
            ingest = {"value": round(max(rates), 2), "unit": "GB/s", "runs": [round(r, 2) for r in rates],
                      "workload": "1 GiB file mapping -> HBM through bybycu_upload_host_range (staged, "
                                  f"{os.cpu_count()} host threads), page cache warm, host clock",
                      "plain_pageable_copy_gbs": round(plain, 2), "bit_exact": bool(ok)}
            del dst
        except Exception as e:   # an I/O problem on the box must not cost the decode numbers
            ingest = {"error": str(e)}
        finally:
            if path and os.path.exists(path):
                os.unlink(path)

    if rank == 0:
        base = None
        if not args.no_cpu_baseline and world == 1:   # the host-core baseline: rank 0 at N = 1 only
            base = cpu_baseline(1, 5.0)
            base.pop("seconds_per_step", None)
        clocks = sampler.summary()
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": steps,
            "warmup": reps_w * copies, "ms_per_step": round(per_launch_ms, 6), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "decode GEMV C2: M=1 K=4096 N=11008 per GPU, Q4B32 (int4 + fp16 scale / 32), "
                                   "x bf16, out fp32",
                       "route": "gemv", "weight_copies": copies,
                       "l2": f"inputs larger than L2: {copies} rotating weight copies ({copies * W_BYTES >> 20} MiB)",
                       "parallelism": "none" if world == 1 else f"column-sharded x{world}, device all-gather",
                       "global_batch": M_DEC, "algorithmic_bytes_per_step": STEP_BYTES,
                       "timing": "CUDA graph replay, CUDA events on the launching stream"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "traffic": profiled_traffic("gemv_m1_decode_c2.md"),
                         "traffic_source": "ncu --set full, one launch: profiles/gemv_m1_decode_c2.md",
                         "algorithmic_bytes": STEP_BYTES, "peak_kind": peak_kind},
            "cpu_baseline": base, "e2e": e2e, "gpu_launches": steps * launches_per_step, "clocks": clocks,
            "prefill": prefill,
            "q4_asym_decode": q4asym,
            "q4_asym_prefill": q4asym_prefill,
            "f16_decode": f16dec,
            "decode_x_f32": dec32,
            "ingest": ingest,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        del graph
        bufs.close()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
