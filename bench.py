"""Benchmark of the Q4B32 tile-GEMM path on B200 (one JSON line on rank 0).

Headline workload (every N): BASELINE config C5, the LM-head vocab projection at decode -
x bf16 [1, 4096] ~N(0,1), Q4B32 weights [128256, 4096] (int4 uniform [-8, 7], one fp16 scale
|N(0, 0.02)| per 32-block), fp32 logits - column-sharded over the N GPUs by the reference's
partition rule (distributed.nim:109-135, 64-column blocks) with the fp32 logits all-gathered
over NVLink inside the same launch, in split phase (bybycu_tile_gemm_allgather_split: no launch
waits for the other ranks at its end; the next launch, or bybycu_allgather_wait at the end of
the timed region, does).  C5 is the configuration
BASELINE names for 1, 2, 4 and 8 GPUs, so the same workload gives one strong-scaling curve.
Algorithmic bytes per step: 295,501,824 weight + 8,192 x per rank + 513,024 logits per rank.

* value        whole-job GB/s with inputs resident in HBM: K steps (exactly --steps) replayed
               from one CUDA graph after exactly --warmup untimed steps, each step reading its
               weights from one of several rotating copies (together more than 4x the 126 MB
               L2), CUDA events on the launching stream, max over ranks.  A device-side hold
               kernel runs before the start event, so the graph is queued on the device before
               timing starts and the host's enqueue latency stays out of the timed region.
* check        after timing, the gathered logits of one step against the exact SIMT route
               (bit-identical to the reference CPU VM in tests/) on columns from every shard.
* e2e          the same metric through the C ABI with host buffers: pinned x in, the sharded
               GEMV with its gather, the whole [1, 128256] logits back to pinned host memory,
               stream sync - every step, on every rank.
* roofline     the rank's algorithmic bytes per launch / average launch duration vs the
               measured HBM copy bandwidth (MEASURED_PEAKS.json).
* cpu_baseline the reference's own CPU C (oracle/_ref: OP_TILE_GEMM through
               nimf_cpu_vm_run_slots, single-threaded as the reference is) on the same shape.
* decode_c2    config C2 (M=1, K=4096, N=11008), the single-GPU decode GEMV, timed the same way.
* lm_head_m64  config C5 at M=64 (tensor-core route + device all-gather), TFLOP/s, checked.
* c4_layer     config C4: the seven Llama-7B projections of one layer in sequence at
               M = 1, 16 and 128, each column-sharded and gathered over the N GPUs.
* prefill      config C3 (M=2048, K=N=4096) TFLOP/s on the tensor-core route with exact weights
               (AUTO's), and prefill_fp16w on the one-rounding form (N = 1).
* c1           config C1 (M=32, K=N=4096, x fp32) through the automatic route (N = 1).
* q4_asym_decode / q4_asym_prefill / f16_decode / decode_x_f32 / ingest   (N = 1): the
               asymmetric Q4 data of matmul_q4, format 1 (fp16 weights), fp32 activation rows,
               and a checkpoint mapping copied into HBM.

`--impl reference` times the reference's CPU implementation (oracle/_ref, column-sharded over
all host threads) on the headline workload and prints the same line with "impl": "reference".
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
K_DEC = 4096
N_HEAD = 128256          # C5
N_C2 = 11008             # C2
L2_BYTES = 126 * 1024 * 1024
SEED = 2463534242
SHARD_ALIGN = 64


def wbytes(N: int, K: int) -> int:
    """Algorithmic bytes of Q4B32 weights: 0.5 B of nibble + 2/32 B of scale per weight."""
    return N * (K // 2) + N * (K // 32) * 2


HEAD_W_BYTES = wbytes(N_HEAD, K_DEC)
HEAD_STEP_BYTES = HEAD_W_BYTES + K_DEC * 2 + N_HEAD * 4       # one GPU: W + x + logits


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def profiled_traffic(summary: str):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of a kernel, from
    its committed ncu summary under profiles/ (one `--set full` capture)."""
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
        self.windows = []

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
        self.windows.append((t0, t1))

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
            if len(p) >= 9:
                rows.append((t, p))
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        inside = [r for r in rows if any(a - 0.2 <= r[0] <= b + 0.2 for a, b in self.windows)]
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
                "window": "timed regions (+-0.2 s)" if inside else "whole run"}


# --------------------------------------------------------------------------------------
# The reference's CPU implementation (oracle/_ref) - the cpu_baseline leg and --impl reference
# --------------------------------------------------------------------------------------

def _reference_inputs(N: int):
    """The headline's shape through the reference VM's table form: Q4B32 weights whose scales
    come from a <= 256-entry palette (the VM's scale table), x bf16 widened to fp32."""
    import numpy as np
    from oracle import oracle as O
    p, s = O.gen_q4b32(N, K_DEC, seed=SEED)
    x = O.bf16_to_f32(O.gen_x_bf16(1, K_DEC, seed=SEED + 2))
    pal = s.ravel()[:256].copy()
    s = pal[(np.arange(s.size) * 7919) % 256].reshape(s.shape)
    blob, table = O.q4b32_to_fp4km(p, s, N, K_DEC)
    if O.ref_available():
        return "reference", (lambda th: O.ref_tile_gemm(x, blob, table, 1, K_DEC, N, threads=th)), \
            "OP_TILE_GEMM via nimf_cpu_vm_run_slots (oracle/_ref, reference C unchanged)"
    return "port", (lambda th: O.tile_gemm_q4b32(x, p, s, 1, K_DEC, N, threads=th)), \
        "q4_oracle.c restatement of cpu_vm.c:605-626"


def cpu_baseline(threads: int, min_seconds: float):
    """The reference's own CPU C on the headline workload (kind "reference"), else the port."""
    kind, fn, what = _reference_inputs(N_HEAD)
    fn(threads)
    reps, t0 = 0, time.perf_counter()
    while True:
        fn(threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    per = el / reps
    return {"value": round(HEAD_STEP_BYTES / per / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": f"{reps} full LM-head GEMVs (M=1, K=4096, N=128256) on {threads} thread(s), {what}; "
                      f"{per * 1e3:.1f} ms per GEMV"}


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    kind, fn, what = _reference_inputs(N_HEAD)
    for _ in range(args.warmup):
        fn(threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn(threads)
    el = time.perf_counter() - t0
    v = HEAD_STEP_BYTES * args.steps / el / 1e9
    line = {"metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": "C5 LM head: M=1 K=4096 N=128256 Q4B32 (x bf16 widened to fp32), fp32 logits",
                       "cpu_threads": threads},
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": threads, "kind": kind,
                             "sample": f"{args.steps} full LM-head GEMVs, column-sharded over {threads} host threads "
                                       f"(the distributed.nim split), {what}"},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------------
# GPU timing helpers
# --------------------------------------------------------------------------------------

class Timer:
    """Times device work queued on one stream: a hold kernel first (so everything after it is
    queued on the device before the start event fires), then CUDA events around the work,
    max over ranks."""

    def __init__(self, torch, dist, stream, world, sampler):
        self.torch, self.dist, self.stream, self.world, self.sampler = torch, dist, stream, world, sampler

    def _sync_all(self):
        self.stream.synchronize()
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def run(self, enqueue_warm, enqueue_timed, hold_cycles=20_000_000):
        """enqueue_warm() and enqueue_timed() queue work on the stream; returns the ms of the
        timed part (max over ranks)."""
        torch = self.torch
        self._sync_all()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0 = time.time()
        with torch.cuda.stream(self.stream):
            torch.cuda._sleep(hold_cycles)
            enqueue_warm()
            e0.record(self.stream)
            enqueue_timed()
            e1.record(self.stream)
        self.stream.synchronize()
        w1 = time.time()
        if self.sampler is not None:
            self.sampler.mark(w0, w1)
        ms = e0.elapsed_time(e1)
        if self.world > 1:
            t = torch.tensor([ms], device=torch.device("cuda", torch.cuda.current_device()))
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
            ms = float(t.item())
        self._sync_all()
        return ms


def capture(torch, stream, fn, n, start, tail=None):
    """A CUDA graph of fn(start), fn(start + 1), ... fn(start + n - 1) on `stream`, then tail()
    (the completion of a split-phase gather) when given."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(n):
            fn(start + i)
        if tail is not None:
            tail()
    return g


def upload_graph(graph, stream):
    """cudaGraphUpload of a captured graph: its first replay then starts without the one-time
    upload of the executable graph to the device (nothing runs)."""
    try:
        cudart = C.CDLL("libcudart.so.12")
        cudart.cudaGraphUpload.argtypes = [C.c_void_p, C.c_void_p]
        cudart.cudaGraphUpload.restype = C.c_int
        ex = graph.raw_cuda_graph_exec()
        ex = ex if isinstance(ex, int) else int(ex)
        return cudart.cudaGraphUpload(C.c_void_p(ex), C.c_void_p(stream.cuda_stream)) == 0
    except Exception:
        return False


def graph_steps(torch, timer, stream, fn, steps, warmup, tail=None):
    """Exactly `warmup` untimed then exactly `steps` timed calls of fn(i), each set replayed
    from its own CUDA graph (both uploaded before the hold) and ended by tail() when given;
    returns ms per step (max over ranks)."""
    gw = capture(torch, stream, fn, warmup, 0, tail) if warmup else None
    gt = capture(torch, stream, fn, steps, warmup, tail)
    for g in (gw, gt):
        if g is not None:
            upload_graph(g, stream)
    stream.synchronize()
    ms = timer.run(lambda: gw.replay() if gw else None, gt.replay)
    del gw, gt
    return ms / steps


def check_device(_lib):
    code = _lib.device_error()
    if code:
        raise RuntimeError(f"device error {code} recorded by a kernel (bounded wait or range check)")


def roofline(achieved, peak, unit, bound, peak_kind, traffic=None, source=None, **extra):
    r = {"bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
         "frac": round(achieved / peak, 4), "traffic": traffic, "peak_kind": peak_kind}
    if source:
        r["traffic_source"] = source
    r.update(extra)
    return r


# --------------------------------------------------------------------------------------
# Sharded Q4B32 projections (every N)
# --------------------------------------------------------------------------------------

class ShardedProjection:
    """One projection W [N, K], column-sharded: this rank's rotating weight copies (copy 0 is
    the shard of a full seeded matrix, kept for the check), a gathered output buffer, and the
    launch of one step."""

    def __init__(self, ctx, N, K, M, seed, min_copies=2, x_dtype=None):
        torch, gb = ctx.torch, ctx.gb
        from bybylang_b200.formats import synthetic_q4b32, synthetic_x
        from bybylang_b200.distributed import shard_range
        self.ctx, self.N, self.K, self.M = ctx, N, K, M
        self.n0, self.n1 = shard_range(N, ctx.world, ctx.rank, SHARD_ALIGN)
        self.cols = self.n1 - self.n0
        wb = wbytes(self.cols, K) if self.cols else 1
        self.copies = max(min_copies, -(-4 * L2_BYTES // wb))
        nib0, sc0 = synthetic_q4b32(N, K, seed=seed, device=ctx.dev)
        self.full0 = (nib0, sc0)                      # the whole matrix of copy 0, for the check
        self.w = [gb.Q4B32Weights(nib0[self.n0:self.n1], sc0[self.n0:self.n1], device=ctx.dev)]
        for c in range(1, self.copies):
            nib, sc = synthetic_q4b32(self.cols, K, seed=seed + 7919 * c + 101 * ctx.rank, device=ctx.dev)
            self.w.append(gb.Q4B32Weights(nib, sc, device=ctx.dev))
        self.x = synthetic_x(M, K, seed=seed + 2, device=ctx.dev, dtype=x_dtype)
        self.make_outputs(M)

    def make_outputs(self, M):
        """The gathered output: at N > 1 two buffer sets that split-phase steps alternate
        between (one signal array, the first set's), else one local buffer."""
        torch, ctx = self.ctx.torch, self.ctx
        if ctx.world > 1:
            from bybylang_b200.distributed import PeerBuffers
            self.bufs = [PeerBuffers(M, self.N, ctx.world, ctx.rank), PeerBuffers(M, self.N, ctx.world, ctx.rank)]
            self.out = self.bufs[0].out
        else:
            self.bufs = None
            self.out = torch.empty(M, self.N, dtype=torch.float32, device=ctx.dev)

    def bytes_per_rank(self):
        return wbytes(self.cols, self.K) + self.M * self.K * self.x.element_size() + self.M * self.cols * 4 * self.ctx.world

    def bytes_whole_job(self):
        return wbytes(self.N, self.K) + self.ctx.world * (self.M * self.K * self.x.element_size() + self.M * self.N * 4)

    def launch(self, i, x=None, route=None):
        """Step i: the rank's slice, gathered in split phase into buffer set i % 2 (N > 1)."""
        _lib, gb, ctx = self.ctx._lib, self.ctx.gb, self.ctx
        w = self.w[i % self.copies]
        x = self.x if x is None else x
        if ctx.world > 1:
            b = self.bufs[i % 2]
            _lib.check(ctx.lib.bybycu_tile_gemm_allgather_split(
                2, self.M, self.K, self.N, self.n0, self.n1, C.c_void_p(x.data_ptr()), gb._dtype_code(x),
                C.c_void_p(w.packed.data_ptr()), w.packed.numel(), w.scale_base, None, 0, 0,
                C.c_void_p(b.out.data_ptr()), b.peer_out, self.bufs[0].peer_sig, ctx.world, ctx.rank, 0,
                C.c_void_p(ctx.stream.cuda_stream)))
        else:
            gb.tile_gemm(2, x, w.packed, self.out, M=self.M, K=self.K, N=self.N, scale_base=w.scale_base,
                         route=_lib.ROUTE_AUTO if route is None else route, stream=ctx.stream)

    def finish(self):
        """Completes the last split-phase step (N > 1): every rank's slices have landed."""
        ctx = self.ctx
        if ctx.world > 1:
            ctx._lib.check(ctx.lib.bybycu_allgather_wait(self.bufs[0].peer_sig, ctx.world, ctx.rank, 0,
                                                         C.c_void_p(ctx.stream.cuda_stream)))

    def check(self, n_cols=1024):
        """Step with copy 0 into buffer set 0, completed, then its gathered output on `n_cols`
        columns spread over every shard against the exact SIMT route on the same columns of
        the full matrix."""
        torch, gb, _lib = self.ctx.torch, self.ctx.gb, self.ctx._lib
        with torch.cuda.stream(self.ctx.stream):
            self.launch(0)
            self.finish()
        self.ctx.stream.synchronize()
        idx = torch.linspace(0, self.N - 1, min(n_cols, self.N), device=self.ctx.dev).round().long().unique()
        nib, sc = self.full0
        ws = gb.Q4B32Weights(nib[idx].contiguous(), sc[idx].contiguous(), device=self.ctx.dev)
        ref = ws.matmul(self.x, route=_lib.ROUTE_SIMT)
        torch.cuda.synchronize()
        got = self.out[:, idx]
        d = (got - ref).abs()
        peak = max(1.0, float(ref.abs().max()))
        per_el = float((d / ref.abs().clamp(min=1.0)).max())
        return {"vs": "SIMT route (fmaf in the reference VM's order; bit-identical to the reference CPU VM in tests)",
                "columns": int(idx.numel()), "rows": self.M, "max_abs_err_over_peak": round(float(d.max()) / peak, 9),
                "max_elem_rel_err": round(per_el, 9), "finite": bool(torch.isfinite(self.out).all())}

    def close(self):
        if self.bufs is not None:
            for b in self.bufs:
                b.close()


class Ctx:
    pass


LINES = ("lm_head_m64", "c4_layer", "decode_c2", "c1", "prefill", "q4_asym", "f16_decode", "ingest")


def on(args, name):
    """Whether the secondary line `name` runs (--lines)."""
    return args.lines == "all" or name in args.lines.split(",")


# --------------------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="only the headline, its check and e2e")
    ap.add_argument("--lines", default="all",
                    help="comma-separated secondary lines to run (default all): " + ", ".join(LINES))
    args = ap.parse_args()
    if args.impl == "reference":
        return reference_arm(args)
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")

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
            from datetime import timedelta
            dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=120))
            dist.barrier()
        finally:
            os.dup2(saved, 1)
            os.close(saved)
    gb.ensureGpuInit(gb.GpuBackend.gbCuda, local)
    dev = torch.device("cuda", local)
    hbm_peak, tc_peak, peak_kind = peaks()
    stream = torch.cuda.Stream(device=dev)
    lib = _lib.load()
    sampler = ClockSampler(local)
    sampler.start()
    timer = Timer(torch, dist, stream, world, sampler)
    ctx = Ctx()
    ctx.torch, ctx.gb, ctx._lib, ctx.lib = torch, gb, _lib, lib
    ctx.world, ctx.rank, ctx.dev, ctx.stream = world, rank, dev, stream
    K, W = args.steps, args.warmup
    launches = 0

    # ---- headline: C5 LM head at M=1, column-sharded, gathered in the GEMV's own launch
    head = ShardedProjection(ctx, N_HEAD, K_DEC, 1, SEED)
    per_ms = graph_steps(torch, timer, stream, head.launch, K, W, tail=head.finish)
    launches += K
    check_device(_lib)
    value = head.bytes_whole_job() / (per_ms / 1e3) / 1e9
    achieved = head.bytes_per_rank() / (per_ms / 1e3) / 1e9
    check = head.check()
    check["pass"] = check["finite"] and check["max_abs_err_over_peak"] <= 1e-4 and check["max_elem_rel_err"] <= 1e-3

    # ---- e2e through the C ABI, host buffers, copies inside the timed region
    xh = head.x.cpu().pin_memory()
    oh = torch.empty(1, N_HEAD, dtype=torch.float32).pin_memory()
    xd = torch.empty_like(head.x)
    sp = C.c_void_p(stream.cuda_stream)
    x_bytes, o_bytes = K_DEC * 2, N_HEAD * 4
    if world > 1:
        def e2e_step(i):
            w, b = head.w[i % head.copies], head.bufs[i % 2]
            _lib.check(lib.bybycu_upload(C.c_void_p(xd.data_ptr()), C.c_void_p(xh.data_ptr()), x_bytes, sp))
            _lib.check(lib.bybycu_tile_gemm_allgather_split(
                2, 1, K_DEC, N_HEAD, head.n0, head.n1, C.c_void_p(xd.data_ptr()), _lib.DT_BF16,
                C.c_void_p(w.packed.data_ptr()), w.packed.numel(), w.scale_base, None, 0, 0,
                C.c_void_p(b.out.data_ptr()), b.peer_out, head.bufs[0].peer_sig, world, rank, 0, sp))
            _lib.check(lib.bybycu_allgather_wait(head.bufs[0].peer_sig, world, rank, 0, sp))
            _lib.check(lib.bybycu_download(C.c_void_p(oh.data_ptr()), C.c_void_p(b.out.data_ptr()), o_bytes, sp))
            _lib.check(lib.bybycu_synchronize(sp))
        api = "bybycu_upload + bybycu_tile_gemm_allgather_split + bybycu_allgather_wait + bybycu_download + " \
              "bybycu_synchronize (C ABI) on every rank, pinned host x and logits, max over ranks"
    else:
        od = torch.empty(1, N_HEAD, dtype=torch.float32, device=dev)

        def e2e_step(i):
            w = head.w[i % head.copies]
            _lib.check(lib.bybycu_tile_gemm_host(2, 1, K_DEC, N_HEAD, C.c_void_p(xh.data_ptr()), _lib.DT_BF16,
                                                 C.c_void_p(w.packed.data_ptr()), w.packed.numel(), w.scale_base,
                                                 None, 0, 0, C.c_void_p(oh.data_ptr()), _lib.DT_F32,
                                                 C.c_void_p(xd.data_ptr()), C.c_void_p(od.data_ptr()),
                                                 _lib.ROUTE_AUTO, sp))
        api = "bybycu_tile_gemm_host (C ABI): pinned host x in, logits out to pinned host memory, stream sync"
    for i in range(W):
        e2e_step(i)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(K):
        e2e_step(W + i)
    el = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([el], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        el = float(t.item())
    e2e = {"value": round(head.bytes_whole_job() * K / el / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": x_bytes * world, "d2h_bytes_per_step": o_bytes * world, "steps": K,
           "us_per_step": round(el / K * 1e6, 2), "api": api}

    extras = {}
    if not args.no_extras:
        # ---- C5 at M=64: the tensor-core route, then the device all-gather of the logits
        if on(args, "lm_head_m64"):
            try:
                x64 = synthetic_x(64, K_DEC, seed=SEED + 64, device=dev)
                h64 = ShardedProjection.__new__(ShardedProjection)
                h64.__dict__.update(head.__dict__)
                h64.M, h64.x = 64, x64
                h64.make_outputs(64)
                reps = min(K, 50)
                ms = graph_steps(torch, timer, stream, h64.launch, reps, W, tail=h64.finish)
                check_device(_lib)
                ck = h64.check(n_cols=512)
                ck["pass"] = ck["finite"] and ck["max_abs_err_over_peak"] <= 1e-3
                fl = 2.0 * 64 * N_HEAD * K_DEC
                tf = fl / (ms / 1e3) / 1e12
                extras["lm_head_m64"] = {
                    "value": round(tf, 2), "unit": "TFLOP/s", "us_per_step": round(ms * 1e3, 2), "steps": reps,
                    "gbs_whole_job": round(h64.bytes_whole_job() / (ms / 1e3) / 1e9, 2),
                    "workload": "C5 at M=64: x bf16 [64, 4096], Q4B32 [128256, 4096] column-sharded, fp32 logits "
                                "gathered on every rank",
                    "route": "tensor-core GEMM (staging pass + tcgen05) + device all-gather" if world > 1
                             else "tensor-core GEMM (staging pass + tcgen05)",
                    "roofline": roofline(tf / world, tc_peak, "TFLOP/s", "tensor", peak_kind, per="GPU"),
                    "check": ck}
                h64.close()
                del h64
            except _lib.BybyCudaError as e:
                extras["lm_head_m64"] = {"error": str(e)}

        # ---- C4: the seven projections of one Llama-7B layer, each sharded and gathered
        if on(args, "c4_layer"):
            try:
                shapes = [("q", 4096, 4096), ("k", 4096, 4096), ("v", 4096, 4096), ("o", 4096, 4096),
                          ("gate", 11008, 4096), ("up", 11008, 4096), ("down", 4096, 11008)]
                c4 = {}
                for M in (1, 16, 128):
                    projs = [ShardedProjection(ctx, n, k, M, SEED + 300 + 17 * j, min_copies=2)
                             for j, (_, n, k) in enumerate(shapes)]

                    def layer(i, projs=projs):
                        for p in projs:
                            p.launch(i)

                    def layer_done(projs=projs):
                        for p in projs:
                            p.finish()
                    reps = min(K, 50)
                    ms = graph_steps(torch, timer, stream, layer, reps, W, tail=layer_done)
                    check_device(_lib)
                    checks = [p.check(n_cols=256) for p in projs]
                    tol = 1e-4 if M <= 16 else 1e-3
                    ok = all(c["finite"] and c["max_abs_err_over_peak"] <= tol for c in checks)
                    byts = sum(p.bytes_whole_job() for p in projs)
                    fl = 2.0 * M * sum(n * k for _, n, k in shapes)
                    gbs, tf = byts / (ms / 1e3) / 1e9, fl / (ms / 1e3) / 1e12
                    t_roof = max(byts / world / (hbm_peak * 1e9), fl / world / (tc_peak * 1e12))
                    c4[f"M{M}"] = {"us_per_layer": round(ms * 1e3, 2), "gbs_whole_job": round(gbs, 2),
                                   "tflops_whole_job": round(tf, 3), "steps": reps,
                                   "roofline_frac": round(t_roof / (ms / 1e3), 4),
                                   "bound": "hbm" if byts / (hbm_peak * 1e9) >= fl / (tc_peak * 1e12) else "tensor",
                                   "check_pass": ok,
                                   "max_abs_err_over_peak": max(c["max_abs_err_over_peak"] for c in checks)}
                    for p in projs:
                        p.close()
                    del projs
                    torch.cuda.empty_cache()
                extras["c4_layer"] = dict(c4, workload="C4: Llama-7B layer projections q, k, v, o [4096x4096], gate, up "
                                                       "[11008x4096], down [4096x11008] in sequence, x bf16, each "
                                                       "column-sharded and gathered; roofline = max(bytes/HBM, flop/peak) "
                                                       "per GPU over the measured time")
            except _lib.BybyCudaError as e:
                extras["c4_layer"] = {"error": str(e)}

    if world == 1 and not args.no_extras:
        single_gpu_lines(args, ctx, timer, extras, hbm_peak, tc_peak, peak_kind)

    sampler.stop()
    if rank == 0:
        base = None
        if not args.no_cpu_baseline and world == 1:   # the host-core baseline: rank 0 at N = 1 only
            base = cpu_baseline(1, 8.0)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(per_ms, 6), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "C5 LM head: x bf16 [1, 4096], Q4B32 [128256, 4096] (int4 + fp16 scale / 32), "
                                   "fp32 logits, column-sharded over the GPUs with a device all-gather",
                       "global_batch": 1, "parallelism": "none" if world == 1 else
                       f"column-sharded x{world} (distributed.nim partition, 64-column blocks), NVLink all-gather "
                       "fused into the GEMV",
                       "shard_columns": head.cols, "weight_copies": head.copies,
                       "l2": f"inputs larger than L2: {head.copies} rotating weight copies per rank "
                             f"({head.copies * wbytes(head.cols, K_DEC) >> 20} MiB)",
                       "algorithmic_bytes_per_step": head.bytes_whole_job(),
                       "timing": "CUDA graph of exactly --steps launches after --warmup launches, behind a device "
                                 "hold kernel; CUDA events on the launching stream; max over ranks"},
            "roofline": roofline(achieved, hbm_peak, "GB/s", "hbm", peak_kind,
                                 profiled_traffic("gemv_m1_lm_head_c5.md") if world == 1 else None,
                                 "ncu --set full, one launch: profiles/gemv_m1_lm_head_c5.md" if world == 1 else None,
                                 algorithmic_bytes=head.bytes_per_rank(), per="GPU (this rank's shard)"),
            "cpu_baseline": base, "e2e": e2e, "gpu_launches": launches, "clocks": sampler.summary(),
            "check": check,
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    head.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def single_gpu_lines(args, ctx, timer, extras, hbm_peak, tc_peak, peak_kind):
    """The single-GPU configurations (C2, C3, C1) and the other formats' lines."""
    torch, gb, _lib, lib, dev, stream = ctx.torch, ctx.gb, ctx._lib, ctx.lib, ctx.dev, ctx.stream
    from bybylang_b200.formats import synthetic_q4b32, synthetic_x
    K, W = args.steps, args.warmup

    # ---- C2: the decode GEMV, resident inputs, exactly K graph-replayed steps
    if on(args, "decode_c2"):
        c2 = ShardedProjection(ctx, N_C2, K_DEC, 1, SEED + 11)
        c2_bytes = c2.bytes_per_rank()
        ms = graph_steps(torch, timer, stream, lambda i: c2.launch(i, route=_lib.ROUTE_GEMV), K, W)
        check_device(_lib)
        ck = c2.check()
        ck["pass"] = ck["finite"] and ck["max_abs_err_over_peak"] <= 1e-4 and ck["max_elem_rel_err"] <= 1e-3
        gbs = c2_bytes / (ms / 1e3) / 1e9
        x32 = c2.x.float().contiguous()
        ms32 = graph_steps(torch, timer, stream, lambda i: c2.launch(i, x=x32, route=_lib.ROUTE_GEMV), K, W)
        b32 = c2_bytes + K_DEC * 2
        extras["decode_c2"] = {
            "value": round(gbs, 2), "unit": "GB/s", "us_per_launch": round(ms * 1e3, 3), "steps": K, "warmup": W,
            "workload": "C2 decode GEMV: M=1 K=4096 N=11008 Q4B32, x bf16, out fp32 (GEMV route)",
            "algorithmic_bytes": c2_bytes,
            "roofline": roofline(gbs, hbm_peak, "GB/s", "hbm", peak_kind, profiled_traffic("gemv_m1_decode_c2.md"),
                                 "ncu --set full, one launch: profiles/gemv_m1_decode_c2.md"),
            "x_f32": {"value": round(b32 / (ms32 / 1e3) / 1e9, 2), "us_per_launch": round(ms32 * 1e3, 3),
                      "frac": round(b32 / (ms32 / 1e3) / 1e9 / hbm_peak, 4)},
            "l2": f"inputs larger than L2: {c2.copies} rotating weight copies", "check": ck}
        c2.close()
        del c2

    # ---- C1: M=32, K=N=4096, x fp32 through the automatic route
    if on(args, "c1"):
        try:
            c1 = ShardedProjection(ctx, 4096, 4096, 32, SEED + 21, x_dtype=torch.float32)
            ms = graph_steps(torch, timer, stream, c1.launch, K, W)
            check_device(_lib)
            ck = c1.check(n_cols=512)
            fl = 2.0 * 32 * 4096 * 4096
            byts = c1.bytes_per_rank()
            extras["c1"] = {"us_per_call": round(ms * 1e3, 3), "gbs": round(byts / (ms / 1e3) / 1e9, 2),
                            "tflops": round(fl / (ms / 1e3) / 1e12, 3),
                            "route": _lib.ROUTE_NAMES[gb.route_for(2, 32, 4096, 4096, _lib.DT_F32)],
                            "roofline": roofline(byts / (ms / 1e3) / 1e9, hbm_peak, "GB/s", "hbm", peak_kind),
                            "workload": "C1: M=32 K=N=4096 Q4B32, x fp32, out fp32", "check": ck}
            c1.close()
            del c1
        except _lib.BybyCudaError as e:
            extras["c1"] = {"error": str(e)}

    # ---- C3 prefill on the tensor-core route
    if on(args, "prefill"):
        if not args.no_prefill:
            Mp, Kp, Np = 2048, 4096, 4096
            try:
                per_set = wbytes(Np, Kp) + Mp * Kp * 2 + Mp * Np * 2
                n_sets = max(2, -(-4 * L2_BYTES // per_set))
                sets = []
                for c in range(n_sets):
                    nib, sc = synthetic_q4b32(Np, Kp, seed=SEED + 7 + c, device=dev)
                    sets.append((gb.Q4B32Weights(nib, sc, device=dev), synthetic_x(Mp, Kp, seed=SEED + 100 + c, device=dev),
                                 torch.empty(Mp, Np, dtype=torch.bfloat16, device=dev)))

                reps = max(K, 20)
                for key, route, what, prof in (
                        ("prefill", _lib.ROUTE_TC, "route TC (AUTO): every weight exact as two fp16 terms, twice the MMAs",
                         "tc_gemm_prefill_c3.md"),
                        ("prefill_fp16w", _lib.ROUTE_TC_FP16W,
                         "route TC_FP16W: each weight rounded once to fp16 (the reference's cooperative lowering)",
                         "tc_gemm_prefill_c3_fp16w.md")):
                    def pf(i, route=route):
                        wp, xp, op = sets[i % n_sets]
                        wp.matmul(xp, op, route=route, stream=stream)
                    ms = graph_steps(torch, timer, stream, pf, reps, W)
                    check_device(_lib)
                    tf = 2.0 * Mp * Np * Kp / (ms / 1e3) / 1e12
                    extras[key] = {
                        "value": round(tf, 2), "unit": "TFLOP/s", "workload": "C3 M=2048 K=N=4096 Q4B32, x bf16, bf16 out",
                        "route": what, "ms_per_call": round(ms, 5), "calls": reps,
                        "roofline": roofline(tf, tc_peak, "TFLOP/s", "tensor", peak_kind, profiled_traffic(prof),
                                             f"ncu --set full, one gemm_kernel launch: profiles/{prof}"),
                        "includes": "every launch of the call (staging pass + tcgen05 GEMM)",
                        "l2": f"inputs larger than L2: {n_sets} rotating (W, x, out) sets ({n_sets * per_set >> 20} MiB)"}
                del sets
            except _lib.BybyCudaError as e:
                extras["prefill"] = {"error": str(e)}

    # ---- asymmetric Q4 (matmul_q4's data): decode, the fused gate/up form, and prefill
    if on(args, "q4_asym"):
        try:
            G = K_DEC // 32
            wb = N_C2 * K_DEC // 2 + N_C2 * G * 8
            ab = wb + K_DEC * 4 + N_C2 * 4
            n_sets = max(2, -(-4 * L2_BYTES // wb))
            gen = torch.Generator(device=dev).manual_seed(SEED + 31)
            qsets = []
            for c in range(n_sets):
                wq = torch.randint(0, 256, (N_C2, K_DEC // 2), dtype=torch.uint8, device=dev, generator=gen)
                sc = torch.rand(N_C2, G, device=dev, generator=gen) * 0.02 + 1e-4
                zp = torch.rand(N_C2, G, device=dev, generator=gen) * 15
                qsets.append((gb.Q4AsymWeights(wq, sc, zp, K_DEC), torch.empty(1, N_C2, device=dev)))
            xa = torch.randn(1, K_DEC, device=dev, generator=gen)

            def qa(i):
                wqs, o = qsets[i % n_sets]
                wqs.matmul(xa, o, route=_lib.ROUTE_GEMV, stream=stream)
            ms = graph_steps(torch, timer, stream, qa, K, W)
            gbs = ab / (ms / 1e3) / 1e9
            q4 = {"value": round(gbs, 2), "unit": "GB/s", "us_per_launch": round(ms * 1e3, 3),
                  "workload": "asymmetric Q4 decode M=1 K=4096 N=11008 (nibbles, fp32 scales + zero points per "
                              "32-block, x fp32, out fp32)", "algorithmic_bytes": ab,
                  "roofline": roofline(gbs, hbm_peak, "GB/s", "hbm", peak_kind)}
            gamma = torch.rand(1, K_DEC, device=dev, generator=gen) + 0.5
            resid = torch.randn(1, N_C2, device=dev, generator=gen)
            pairs = [(qsets[2 * i][0], qsets[2 * i + 1][0], torch.empty(1, N_C2, device=dev),
                      torch.empty(1, N_C2, device=dev)) for i in range(n_sets // 2)]

            def fused(i):
                wg, wu, o0, o1 = pairs[i % len(pairs)]
                gb.matmul_q4_fused(1, xa, [wg, wu], [o0, o1], res=resid, gamma=gamma, eps=1e-5, stream=stream)
            ms = graph_steps(torch, timer, stream, fused, K, W)
            fb = 2 * wb + 2 * K_DEC * 4 + 2 * N_C2 * 4
            q4["fused_gate_up"] = {"value": round(fb / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
                                   "us_per_launch": round(ms * 1e3, 3),
                                   "workload": "fused decode GEMV mode 1: RMSNorm(x), silu(x.Wg) * (x.Wu) + residual, "
                                               "Wg, Wu 11008 x 4096 asymmetric Q4, one launch",
                                   "roofline": roofline(fb / (ms / 1e3) / 1e9, hbm_peak, "GB/s", "hbm", peak_kind)}
            check_device(_lib)
            extras["q4_asym_decode"] = q4
            del qsets, pairs
        except _lib.BybyCudaError as e:
            extras["q4_asym_decode"] = {"error": str(e)}

        if not args.no_prefill:
            try:
                Mp, Kp, Np = 2048, 4096, 4096
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

                def asym_call(i):
                    wq, sc, zp, xa_, oa = asets[i % n_sets]
                    _lib.check(lib.bybycu_matmul_q4(C.c_void_p(xa_.data_ptr()), C.c_void_p(wq.data_ptr()),
                                                    C.c_void_p(sc.data_ptr()), C.c_void_p(zp.data_ptr()),
                                                    C.c_void_p(oa.data_ptr()), Mp, Kp, Np, 32, Gp, _lib.ROUTE_TC,
                                                    C.c_void_p(stream.cuda_stream)))
                reps = max(K, 20)
                ms = graph_steps(torch, timer, stream, asym_call, reps, W)
                check_device(_lib)
                tf = 2.0 * Mp * Np * Kp / (ms / 1e3) / 1e12
                extras["q4_asym_prefill"] = {
                    "value": round(tf, 2), "unit": "TFLOP/s", "ms_per_call": round(ms, 5), "calls": reps,
                    "workload": "asymmetric Q4 prefill M=2048 K=N=4096 (group 32), x fp32, out fp32",
                    "roofline": roofline(tf, tc_peak, "TFLOP/s", "tensor", peak_kind),
                    "includes": "every launch of the call (staging pass + tcgen05 GEMM)"}
                del asets
            except _lib.BybyCudaError as e:
                extras["q4_asym_prefill"] = {"error": str(e)}

    # ---- format 1 (fp16 weights, 2 B per weight) decode at the C2 shape
    if on(args, "f16_decode"):
        try:
            fbytes = N_C2 * K_DEC * 2
            n_sets = max(2, -(-4 * L2_BYTES // fbytes))
            gen = torch.Generator(device=dev).manual_seed(SEED + 41)
            hsets = [((torch.randn(N_C2, K_DEC, device=dev, generator=gen) * 0.05).half().view(torch.uint8),
                      torch.empty(1, N_C2, device=dev)) for _ in range(n_sets)]
            xh = synthetic_x(1, K_DEC, seed=SEED + 2, device=dev)

            def f16(i):
                wh, o = hsets[i % n_sets]
                gb.tile_gemm(1, xh, wh, o, M=1, K=K_DEC, N=N_C2, route=_lib.ROUTE_GEMV, stream=stream)
            ms = graph_steps(torch, timer, stream, f16, K, W)
            check_device(_lib)
            hb = fbytes + K_DEC * 2 + N_C2 * 4
            extras["f16_decode"] = {"value": round(hb / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
                                    "us_per_launch": round(ms * 1e3, 3),
                                    "workload": "format 1 (fp16 weights) decode M=1 K=4096 N=11008, x bf16, out fp32",
                                    "roofline": roofline(hb / (ms / 1e3) / 1e9, hbm_peak, "GB/s", "hbm", peak_kind)}
            del hsets
        except _lib.BybyCudaError as e:
            extras["f16_decode"] = {"error": str(e)}

    # ---- weight ingestion: a checkpoint mapping copied into HBM (residentUploadQ4Mapped's copy)
    if on(args, "ingest"):
        import tempfile
        import numpy as np
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
            extras["ingest"] = {"value": round(max(rates), 2), "unit": "GB/s", "runs": [round(r, 2) for r in rates],
                                "workload": "1 GiB file mapping -> HBM through bybycu_upload_host_range (staged, "
                                            f"{os.cpu_count()} host threads), page cache warm, host clock",
                                "plain_pageable_copy_gbs": round(plain, 2), "bit_exact": bool(ok)}
            del dst
        except Exception as e:   # an I/O problem on the box must not cost the decode numbers
            extras["ingest"] = {"error": str(e)}
        finally:
            if path and os.path.exists(path):
                os.unlink(path)


if __name__ == "__main__":
    main()
