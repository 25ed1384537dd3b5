"""The autotuner and its plan cache on the GPU (bybycu_prepare_*_tuned, the CUDA side of
vulkanPrepareQ4Tuned, backends/vulkan/q4_autotune.nim:387-543, and of its JSON plan cache,
q4_autotune.nim:32-117).

What is checked:
* preparing a shape installs a plan that passed the tuner's parity gate, and ROUTE_AUTO calls
  of that shape then run it (the dispatch count rises) with results inside the tolerance of
  the route the plan names, as the routes' own parity tests require, with the reference
  test's metric max|diff| <= tol * max(1, max|ref|): 1e-4 for the GEMV routes, 1e-3 for the
  tensor-core route (weights rounded once to fp16);
* the prefill class of M: a plan tuned for M = 64 serves M = 40 (class 64) and not M = 200;
* a hand-installed SIMT plan makes ROUTE_AUTO bit-identical to the explicit SIMT route;
* the cache file: a second process reads the plan back ("cache hit") instead of tuning, and
  the file is the JSON the reference writes (version, signature, plans by key);
* BYBY_Q4_TUNED=0 and BYBY_GPU_AUTOTUNE=0 switch tuning off; format 0 has nothing to tune.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from bybylang_b200 import _lib  # noqa: E402
from bybylang_b200 import gpubackend as gb  # noqa: E402
from oracle import oracle as O  # noqa: E402

from gpu_helpers import DEV, peak_err  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(autouse=True)
def _fresh(tmp_path, monkeypatch):
    gb.ensureGpuInit(gb.GpuBackend.gbCuda, 0)
    monkeypatch.setenv("BYBY_CUDA_TUNE_DIR", str(tmp_path / "plans"))
    _lib.call("bybycu_plan_clear")
    yield
    _lib.call("bybycu_plan_clear")
    assert _lib.device_error() == 0


def q4b32_weights(N, K, seed=1):
    p, s = O.gen_q4b32(N, K, seed=seed)
    return p, s, gb.Q4B32Weights(torch.from_numpy(p), torch.from_numpy(s.view(np.float16)), device=DEV)


def test_q4b32_decode_plan_is_used_and_correct():
    K, N = 4096, 4096
    p, s, w = q4b32_weights(N, K)
    assert w.prepare(1)
    plan = gb.tunedPlan(_lib.OP_TILE_GEMM, fmt=_lib.FMT_Q4B32, M=1, K=K, N=N)
    assert plan is not None and plan.name and plan.ms > 0
    assert plan.route in (_lib.ROUTE_GEMV, _lib.ROUTE_TC, _lib.ROUTE_SIMT)
    # the decode GEMV streams 9 MB in microseconds; the exact tile loop cannot win
    assert plan.route == _lib.ROUTE_GEMV, plan
    n0, d0 = gb.q4TuningStats()
    assert n0 == 1
    xb = O.gen_x_bf16(1, K)
    want = O.tile_gemm_q4b32(O.bf16_to_f32(xb), p, s, 1, K, N)
    got = w.matmul(torch.from_numpy(xb).to(DEV).view(torch.bfloat16))
    torch.cuda.synchronize()
    assert peak_err(want, got.cpu().numpy()) <= 1e-4
    assert gb.q4TuningStats()[1] == d0 + 1
    # preparing again is a table hit, not a second tune
    assert w.prepare(1)
    assert gb.q4TuningStats()[0] == 1
    # fp32 rows have their own plan (the integer mode's two images, or the general kernel's
    # two bf16 terms)
    assert gb.tunedPlan(_lib.OP_TILE_GEMM, fmt=_lib.FMT_Q4B32, x_dtype=_lib.DT_F32, M=1, K=K, N=N) is None
    assert w.prepare(1, _lib.DT_F32)
    plan32 = gb.tunedPlan(_lib.OP_TILE_GEMM, fmt=_lib.FMT_Q4B32, x_dtype=_lib.DT_F32, M=1, K=K, N=N)
    assert plan32 is not None and plan32.route == _lib.ROUTE_GEMV, plan32
    xf = O.bf16_to_f32(xb)
    got = w.matmul(torch.from_numpy(xf).to(DEV))
    torch.cuda.synchronize()
    assert peak_err(want, got.cpu().numpy()) <= 1e-4


def test_q4b32_prefill_class():
    K, N = 4096, 2048
    p, s, w = q4b32_weights(N, K, seed=5)
    assert w.prepare(64)
    plan = gb.tunedPlan(_lib.OP_TILE_GEMM, fmt=_lib.FMT_Q4B32, M=40, K=K, N=N)
    assert plan is not None
    assert plan.route == _lib.ROUTE_TC, plan   # 64 rows: the tensor-core tile
    assert gb.tunedPlan(_lib.OP_TILE_GEMM, fmt=_lib.FMT_Q4B32, M=200, K=K, N=N) is None   # class 128
    assert gb.tunedPlan(_lib.OP_TILE_GEMM, fmt=_lib.FMT_Q4B32, M=1, K=K, N=N) is None
    M = 40
    xb = O.gen_x_bf16(M, K)
    want = O.tile_gemm_q4b32(O.bf16_to_f32(xb), p, s, M, K, N)
    d0 = gb.q4TuningStats()[1]
    got = w.matmul(torch.from_numpy(xb).to(DEV).view(torch.bfloat16))
    torch.cuda.synchronize()
    assert gb.q4TuningStats()[1] == d0 + 1
    assert peak_err(want, got.cpu().numpy()) <= 1e-3


def test_f16_decode_plan():
    K, N, M = 2048, 3000, 2
    rng = np.random.default_rng(3)
    halves = rng.normal(0, 0.05, size=(N, K)).astype(np.float16)
    packed = torch.from_numpy(halves.view(np.uint8).reshape(-1).copy()).to(DEV)
    assert gb.prepareTileGemmTuned(_lib.FMT_F16, packed, M=M, K=K, N=N, x_dtype=_lib.DT_F32)
    plan = gb.tunedPlan(_lib.OP_TILE_GEMM, fmt=_lib.FMT_F16, x_dtype=_lib.DT_F32, M=M, K=K, N=N)
    assert plan is not None and plan.route == _lib.ROUTE_GEMV and plan.name.startswith(b"f16gemv-cta"), plan
    x = O.gen_x_f32(M, K)
    want = O.tile_gemm_f16(x, halves.view(np.uint16), M, K, N)
    out = torch.empty(M, N, dtype=torch.float32, device=DEV)
    gb.tile_gemm(_lib.FMT_F16, torch.from_numpy(x).to(DEV), packed, out, M=M, K=K, N=N)
    torch.cuda.synchronize()
    assert peak_err(want, out.cpu().numpy()) <= 1e-4


def test_asym_decode_plan_through_resident_api():
    K, N = 4096, 4096
    rng = np.random.default_rng(7)
    groups = K // 32
    wq = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    scales = (np.abs(rng.normal(0, 0.02, size=(N, groups))) + 1e-4).astype(np.float32)
    zeros = rng.uniform(0, 15, size=(N, groups)).astype(np.float32)
    a = rng.normal(0, 1, size=(1, K)).astype(np.float32)
    be = gb.GpuBackend.gbCuda
    w = gb.residentUploadQ4(be, wq, scales, zeros, K, N, 32, groups)
    try:
        assert gb.residentPrepareQ4(w, 1)
        plan = gb.tunedPlan(_lib.OP_MATMUL_Q4, M=1, K=K, N=N, groupSize=32, nGroupsPerRow=groups)
        assert plan is not None and plan.route == _lib.ROUTE_GEMV, plan
        want = O.ref_matmul_q4(a, wq, scales, zeros, 1, K, N, 32)
        d0 = gb.q4TuningStats()[1]
        gb.sessionBegin(be)
        ah = gb.sessionUpload(be, a)
        c = gb.SessionHandle()
        gb.sessionMatmulQ4(be, ah, w, c, 1)
        gb.sessionEnd(be)
        got = gb.sessionRead(be, c, N)
        gb.sessionFree(be, ah)
        gb.sessionFree(be, c)
        assert gb.q4TuningStats()[1] == d0 + 1
        assert peak_err(want.reshape(-1), got) <= 1e-4
        # a prefill class: the tensor-core GEMM against the exact kernel
        assert gb.residentPrepareQ4(w, 16)
        plan16 = gb.tunedPlan(_lib.OP_MATMUL_Q4, M=9, K=K, N=N, groupSize=32, nGroupsPerRow=groups)
        assert plan16 is not None and plan16.route == _lib.ROUTE_TC, plan16
    finally:
        gb.residentFreeQ4(be, w)


def test_hand_installed_plan_and_removal():
    K, N, M = 1024, 512, 3
    p, s, w = q4b32_weights(N, K, seed=9)
    x = torch.from_numpy(O.gen_x_bf16(M, K)).to(DEV).view(torch.bfloat16)
    exact = w.matmul(x, route=_lib.ROUTE_SIMT)
    plan = _lib.Plan(route=_lib.ROUTE_SIMT, variant=-1, stages=0, ms=0.0, name=b"by-hand")
    _lib.call("bybycu_plan_set", _lib.OP_TILE_GEMM, _lib.FMT_Q4B32, _lib.DT_BF16, M, K, N, 0, 0, plan)
    assert gb.route_for(_lib.FMT_Q4B32, M, K, N) == _lib.ROUTE_SIMT
    auto = w.matmul(x)
    torch.cuda.synchronize()
    assert torch.equal(auto, exact)
    _lib.call("bybycu_plan_set", _lib.OP_TILE_GEMM, _lib.FMT_Q4B32, _lib.DT_BF16, M, K, N, 0, 0, None)
    assert gb.tunedPlan(_lib.OP_TILE_GEMM, fmt=_lib.FMT_Q4B32, M=M, K=K, N=N) is None
    assert gb.route_for(_lib.FMT_Q4B32, M, K, N) == _lib.ROUTE_GEMV


def test_fp32_decode_general_kernel_plan():
    """A plan with variant 0 (the bf16 operand mode, which has no fp32 form) sends fp32 decode
    rows to the general kernel's two bf16 terms; within 1e-3 per element of the oracle too."""
    K, N = 4096, 2048
    p, s, w = q4b32_weights(N, K, seed=5)
    xf = O.gen_x_f32(1, K, seed=6)
    want = O.tile_gemm_q4b32(xf, p, s, 1, K, N)
    x = torch.from_numpy(xf).to(DEV)
    plan = _lib.Plan(route=_lib.ROUTE_GEMV, variant=0, stages=0, ms=0.0, name=b"gemv-split")
    _lib.call("bybycu_plan_set", _lib.OP_TILE_GEMM, _lib.FMT_Q4B32, _lib.DT_F32, 1, K, N, 0, 0, plan)
    got = w.matmul(x).cpu().numpy().astype(np.float64)
    _lib.call("bybycu_plan_set", _lib.OP_TILE_GEMM, _lib.FMT_Q4B32, _lib.DT_F32, 1, K, N, 0, 0, None)
    d = np.abs(got - want) / np.maximum(1.0, np.abs(want))
    assert d.max() <= 1e-3, d.max()
    # the default (integer mode, two images) agrees with it to within both errors
    dflt = w.matmul(x).cpu().numpy().astype(np.float64)
    assert (np.abs(dflt - want) / np.maximum(1.0, np.abs(want))).max() <= 1e-4


def test_switches_and_untunable_format(monkeypatch):
    K, N = 1024, 1024
    _, _, w = q4b32_weights(N, K, seed=11)
    monkeypatch.setenv("BYBY_Q4_TUNED", "0")
    assert not w.prepare(1)
    monkeypatch.delenv("BYBY_Q4_TUNED")
    monkeypatch.setenv("BYBY_GPU_AUTOTUNE", "0")
    assert not w.prepare(1)
    monkeypatch.delenv("BYBY_GPU_AUTOTUNE")
    assert gb.q4TuningStats()[0] == 0
    fp4 = torch.zeros(N * K // 2 + N * K // 32, dtype=torch.uint8, device=DEV)
    assert not gb.prepareTileGemmTuned(_lib.FMT_FP4KM, fp4, M=1, K=K, N=N, scale_base=N * K // 2)


_CHILD = r"""
import sys
sys.path.insert(0, {root!r})
import numpy as np, torch
from bybylang_b200 import _lib, gpubackend as gb
from oracle import oracle as O
gb.ensureGpuInit(gb.GpuBackend.gbCuda, 0)
p, s = O.gen_q4b32(2048, 4096, seed=13)
w = gb.Q4B32Weights(torch.from_numpy(p), torch.from_numpy(s.view(np.float16)), device="cuda:0")
assert w.prepare(1)
plan = gb.tunedPlan(_lib.OP_TILE_GEMM, fmt=_lib.FMT_Q4B32, M=1, K=4096, N=2048)
print("PLAN", plan.name.decode(), plan.route, plan.variant, plan.stages)
print("PATH", gb.tuneCachePath())
"""


def test_plan_cache_file_round_trip(tmp_path):
    env = dict(os.environ, BYBY_CUDA_TUNE_DIR=str(tmp_path / "cache"))
    code = _CHILD.format(root=ROOT)
    r1 = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r1.returncode == 0, r1.stderr[-2000:]
    assert "[q4-tune:cuda] tile_gemm 4096x2048 M=1:" in r1.stderr and "cache hit" not in r1.stderr
    plan1 = [ln for ln in r1.stdout.splitlines() if ln.startswith("PLAN")][0]
    path = [ln for ln in r1.stdout.splitlines() if ln.startswith("PATH")][0].split(" ", 1)[1]
    assert path.startswith(str(tmp_path / "cache")) and os.path.basename(path).startswith("q4-plans-")
    doc = json.load(open(path))
    assert doc["version"] == 1 and doc["signature"].startswith("version=1;device=")
    entry = doc["plans"]["op=0;fmt=2;x=1;K=4096;N=2048;group=0;groups=0;M=1"]
    assert entry["name"] == plan1.split()[1] and entry["ms"] > 0
    r2 = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r2.returncode == 0, r2.stderr[-2000:]
    assert "cache hit " + entry["name"] in r2.stderr
    assert [ln for ln in r2.stdout.splitlines() if ln.startswith("PLAN")][0] == plan1
    # a damaged file counts as absent: the next process tunes again and rewrites it
    with open(path, "w") as f:
        f.write("{\"version\": 1, \"plans\": [")
    r3 = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r3.returncode == 0, r3.stderr[-2000:]
    assert "cache hit" not in r3.stderr
    assert json.load(open(path))["plans"]
