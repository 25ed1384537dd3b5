"""Generate the golden fixtures from the reference's own CPU C (oracle/_ref/libref_oracle.so).

Run where the reference tree exists (it builds oracle/_ref first):

    python tests/golden/make_golden.py

Fixtures written to tests/golden/:

* ``ref_tile_cases.npz`` - the reference test's cases (tests/t_fp4_tile_gemm.nim:147-148 and
  :207-208, xorshift32 seed 2463534242, drawn in the test's order): inputs and the reference
  CPU VM's outputs for OP_TILE_GEMM format 0 (dynamic and fixed rows), the legacy
  OP_FP4_COOP_GEMM blob, and format 1.
* ``ref_gate.npz`` - the exact-data parity gate of backends/vulkan/vulkan_driver.nim:2681-2762
  (M=37, K=128, N=80) for both formats, with the reference VM outputs.
* ``ref_q4b32.npz`` - Q4B32 (int4 + fp16 block scale) cases with palette-drawn scales, so the
  reference VM computes them through OP_TILE_GEMM format 0, plus nimf_cpu_matmul_q4 on the
  asymmetric repack of the same weights, and the legacy OP_Q4_GEMV / OP_Q4_COOP_GEMM blobs.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import oracle as O  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))

# Q4B32 shapes: the reference test's five, two with K % 256 == 0 and a decode-like one.
Q4_SHAPES = [(1, 64, 16), (5, 128, 96), (20, 64, 72), (37, 128, 130), (70, 96, 64),
             (3, 512, 144), (16, 1024, 80), (1, 4096, 48)]


def run_vm(code, M, N, packed, lut, x):
    rc, mem, err = O.ref_vm_run_slots(code, M * N, packed, lut, x)
    assert rc == 0, err
    return mem.reshape(M, N)


def fp4_blob(packed, table, K, N):
    """The legacy one-blob form: nibbles, scale bytes, word pad, then the 272-float table
    (t_fp4_tile_gemm.nim:92-99, session_vm.nim:447-450)."""
    lut_word = (N * (K // 2) + N * (K // 32) + 3) // 4
    blob = np.zeros(lut_word * 4 + 272 * 4, np.uint8)
    blob[:len(packed)] = packed
    blob[lut_word * 4:] = np.asarray(table, np.float32).view(np.uint8)
    return blob


def q4_asym_blob(wq, scales, zeros, K, N):
    """The OP_Q4_GEMV / OP_Q4_COOP_GEMM blob (cpu_vm.c:440-447): nibbles [N, K/2], then
    fp32 scales at float (N*K/2+3)/4, then the zeros."""
    sb = (N * (K // 2) + 3) // 4
    blob = np.zeros((sb + 2 * len(scales)) * 4, np.uint8)
    blob[:len(wq)] = wq
    f = blob.view(np.float32)
    f[sb:sb + len(scales)] = scales
    f[sb + len(scales):] = zeros
    return blob


def main():
    O.build()
    assert O.ref_available(), "oracle/_ref/libref_oracle.so did not build"
    fp4, f16 = O.reference_test_cases()

    d = {}
    for i, (M, K, N, x, packed, table) in enumerate(fp4):
        sb = N * (K // 2)
        d[f"fp4_{i}_shape"] = np.array([M, K, N])
        d[f"fp4_{i}_x"] = x
        d[f"fp4_{i}_packed"] = packed
        d[f"fp4_{i}_table"] = table
        d[f"fp4_{i}_dyn"] = run_vm(O.fp4_tile_program(0, K, N, sb), M, N, packed, table, x)
        d[f"fp4_{i}_fixed"] = run_vm(O.fp4_tile_program(M, K, N, sb), M, N, packed, table, x)
        if K % 64 == 0 and N >= 16:
            blob = fp4_blob(packed, table, K, N)
            code = np.array([O.OP_FP4_COOP_GEMM, M, K, N, 32, K // 32, O.OP_HALT], np.uint32)
            d[f"fp4_{i}_legacy"] = run_vm(code, M, N, blob, blob.view(np.float32), x)
    for i, (M, K, N, x, w, halves) in enumerate(f16):
        d[f"f16_{i}_shape"] = np.array([M, K, N])
        d[f"f16_{i}_x"] = x
        d[f"f16_{i}_halves"] = halves
        d[f"f16_{i}_dyn"] = run_vm(O.f16_tile_program(0, K, N), M, N, halves.view(np.uint8).ravel(),
                                   np.zeros(1, np.float32), x)
        # the test's own fp64 yardstick (t_fp4_tile_gemm.nim:221-227)
        d[f"f16_{i}_f64"] = (x.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)
    np.savez_compressed(os.path.join(OUT, "ref_tile_cases.npz"), **d)

    g = {}
    x, packed, table = O.gate_fp4()
    g["fp4_x"], g["fp4_packed"], g["fp4_table"] = x, packed, table
    g["fp4_vm"] = run_vm(O.fp4_tile_program(0, 128, 80, 80 * 64), 37, 80, packed, table, x)
    xh, w, halves = O.gate_f16()
    g["f16_x"], g["f16_halves"] = xh, halves
    g["f16_vm"] = run_vm(O.f16_tile_program(0, 128, 80), 37, 80, halves.view(np.uint8).ravel(),
                         np.zeros(1, np.float32), xh)
    g["f16_f64"] = (xh.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)
    np.savez_compressed(os.path.join(OUT, "ref_gate.npz"), **g)

    q = {}
    for i, (M, K, N) in enumerate(Q4_SHAPES):
        p, s = O.gen_q4b32(N, K, seed=O.Xorshift32.SEED + 17 * i)
        G = K // 32
        pal = s.ravel()[:256].copy()
        s = pal[(np.arange(N * G) * 7919) % len(pal)].reshape(N, G)
        xb = O.gen_x_bf16(M, K, seed=O.Xorshift32.SEED + 17 * i + 2)
        xf = O.bf16_to_f32(xb)
        conv = O.q4b32_to_fp4km(p, s, N, K)
        assert conv is not None
        blob, table = conv
        q[f"q4_{i}_shape"] = np.array([M, K, N])
        q[f"q4_{i}_packed"] = p
        q[f"q4_{i}_scales"] = s
        q[f"q4_{i}_x_bf16"] = xb
        q[f"q4_{i}_vm"] = run_vm(O.fp4_tile_program(0, K, N, N * (K // 2)), M, N, blob, table, xf)
        wq, sc, zp = O.q4b32_to_asym(p, s, N, K)
        q[f"q4_{i}_matmul_q4"] = O.ref_matmul_q4(xf, wq, sc, zp, M, K, N)
        ablob = q4_asym_blob(wq, sc, zp, K, N)
        code = np.array([O.OP_Q4_GEMV, M, K, N, 32, K // 32, O.OP_HALT], np.uint32)
        q[f"q4_{i}_q4gemv"] = run_vm(code, M, N, ablob, ablob.view(np.float32), xf)
    np.savez_compressed(os.path.join(OUT, "ref_q4b32.npz"), **q)
    for f in ("ref_tile_cases.npz", "ref_gate.npz", "ref_q4b32.npz"):
        print(f, os.path.getsize(os.path.join(OUT, f)), "bytes")


if __name__ == "__main__":
    main()
