"""Profiling build of the library: the fp16 GEMM (q8_gemm_sk_kernel) at benchmark config 4 (M = 512) and beyond.

    python -m vvllm_b200.gemm_trace build              # profiling copy of the library -> vvllm_b200/_trace/
    python -m vvllm_b200.gemm_trace phases [KxN ...]   # per-CTA phase times of one launch after an L2 flush
    python -m vvllm_b200.gemm_trace sweep              # per-call time back to back, every tile width / grid
    python -m vvllm_b200.gemm_trace roles KxN:M ...    # per-role wait / loop cycles per K-stage of one launch

The profiling copy is the same sources built with -DB200Q8_TRACE: the GEMM then stamps each CTA's
phases (%globaltimer at its start, SM cycles to each phase after it) into a device array that
b200q8_trace_gemm reads back, and its tile width / grid choice can be forced with the environment
variables B200Q8_TRACE_BN (16, 32, 64, 128, 256) and B200Q8_TRACE_GRID (1 = one CTA per tile,
2 = stream-K over all SMs, larger = that many CTAs).  Each GEMM CTA also counts the SM cycles its
roles spend waiting on their barriers and in their loops (b200q8_trace_gemm_roles, the `roles`
command).  The profiling build's int8 digit GEMV takes B200Q8_TRACE_PF_MB (L2 burst at the start,
MB over the grid), B200Q8_TRACE_EARLY (0: dependents launch at the epilogue's end) and
B200Q8_TRACE_EVICT (0: weights loaded with the default L2 policy).  The product library has none
of these.
"""
from __future__ import annotations

import concurrent.futures as cf
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys

from vvllm_b200 import build as b

OUT = os.path.join(b.HERE, "_trace")
LIB = os.path.join(OUT, "libb200q8.so")
SHAPES = [(896, 896), (896, 128), (896, 4864), (4864, 896)]  # (K, N), M = 512
M = 512
L2_BYTES = 126 << 20
SM_MHZ = 1965.0


def build_trace() -> str:
    os.makedirs(OUT, exist_ok=True)
    objs, jobs = [], []
    for src in b.SOURCES:
        o = os.path.join(OUT, src.replace(".cu", ".o"))
        objs.append(o)
        jobs.append([b.nvcc(), *b.NVCC_FLAGS, "-DB200Q8_TRACE", "-c", os.path.join(b.CSRC, src), "-o", o])
    with cf.ThreadPoolExecutor(8) as ex:
        for r in ex.map(lambda j: subprocess.run(j, capture_output=True, text=True), jobs):
            if r.returncode:
                raise RuntimeError(r.stderr)
    r = subprocess.run([b.nvcc(), *b.ARCH, "-shared", "-o", LIB, *objs, "-ldl", "-lpthread", "-lrt"],
                       capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(r.stderr)
    for o in objs:
        os.remove(o)
    return LIB


def _load():
    from vvllm_b200 import _lib

    if not os.path.exists(LIB):
        raise SystemExit(f"{LIB} missing: run `python -m vvllm_b200.gemm_trace build` first")
    _lib.LIB_PATH = LIB  # before the first call loads a library
    L = _lib.lib()
    L.b200q8_trace_gemm.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
    L.b200q8_trace_gemm.restype = ctypes.c_int
    import vvllm_b200

    return vvllm_b200, L


def phases(shapes) -> None:
    import numpy as np
    import torch

    v, L = _load()
    dev = torch.device("cuda", 0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for K, N in shapes:
        q = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev)
        s = torch.rand(N, device=dev) * 1e-3
        x = torch.randn(M, K, device=dev).half()
        out = torch.empty(M, N, device=dev, dtype=torch.float16)
        for _ in range(3):
            v.linear_q8(out, x, q, s)
        flush.zero_()
        L.b200q8_trace_gemm(None, 0)
        torch.cuda.synchronize()
        v.linear_q8(out, x, q, s)
        torch.cuda.synchronize()
        buf = np.zeros((1024, 8), dtype=np.uint64)
        L.b200q8_trace_gemm(buf.ctypes.data, buf.nbytes)
        n = int((buf[:, 0] > 0).sum())
        start = buf[:n, 0].astype(np.int64)
        rel = (start - start.min()) / 1e3
        cyc = buf[:n, 1:].astype(np.int64) / SM_MHZ  # µs since each CTA's start
        med = {name: round(float(np.median(cyc[:, i])), 2) for i, name in enumerate(
            ["past_pdl_wait", "tmem_ready", "first_mma", "last_mma_commit", "epilogue_first", "epilogue_done",
             "exit"])}
        print(f"K={K} N={N} M={M}", json.dumps(dict(ctas=n, start_spread_us=round(float(rel.max()), 2), **med,
                                                    grid_span_us=round(float((rel + cyc[:, 6]).max()), 2))),
              flush=True)


ROLE_SLOTS = ["mma_wait_stage", "mma_wait_a", "mma_wait_acc", "mma_loop", "mma_stages",
              "deq0_wait_stage", "deq0_wait_a_free", "deq0_loop", "deq1_wait_stage", "deq1_wait_a_free", "deq1_loop",
              "prod_wait_free", "prod_loop", "epi_wait_acc", "epi_loop"]


def roles(cases) -> None:
    """Median over the CTAs of one launch (after three warm-up calls) of each role's barrier
    waits and whole loop, in SM cycles per K-stage the CTA's MMA thread issued."""
    import numpy as np
    import torch

    v, L = _load()
    L.b200q8_trace_gemm_roles.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
    L.b200q8_trace_gemm_roles.restype = ctypes.c_int
    dev = torch.device("cuda", 0)
    for case in cases:
        shape, _, m = case.partition(":")
        K, N = (int(a) for a in shape.split("x"))
        Mt = int(m or M)
        q = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev)
        s = torch.rand(N, device=dev) * 1e-3
        x = torch.randn(Mt, K, device=dev).half()
        out = torch.empty(Mt, N, device=dev, dtype=torch.float16)
        for _ in range(3):
            v.linear_q8(out, x, q, s)
        torch.cuda.synchronize()
        buf = np.zeros((1024, 16), dtype=np.uint64)
        L.b200q8_trace_gemm_roles(None, 0)  # cleared: CTAs of earlier launches leave no counts
        torch.cuda.synchronize()
        v.linear_q8(out, x, q, s)
        torch.cuda.synchronize()
        L.b200q8_trace_gemm_roles(buf.ctypes.data, buf.nbytes)
        live = buf[:, 3] > 0
        st = np.maximum(buf[live, 4].astype(np.float64), 1.0)
        per = {name: round(float(np.median(buf[live, i] / st)), 1) for i, name in enumerate(ROLE_SLOTS) if i != 4}
        print(f"K={K} N={N} M={Mt}", json.dumps(dict(ctas=int(live.sum()), stages_median=float(np.median(st)),
                                                   loop_us=round(float(np.median(buf[live, 3])) / SM_MHZ, 2),
                                                   cycles_per_stage=per)), flush=True)


def sweep() -> None:
    import torch

    v, _ = _load()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)

    def make(K, N, copies):
        return [(torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev), torch.rand(N, device=dev) * 1e-3,
                 torch.randn(M, K, device=dev).half(), torch.empty(M, N, device=dev, dtype=torch.float16))
                for _ in range(copies)]

    def timed(calls, reps=7):
        for q, s, x, o in calls:
            v.linear_q8(o, x, q, s, stream=stream)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for q, s, x, o in calls:
                v.linear_q8(o, x, q, s, stream=stream)
        g.replay()
        torch.cuda.synchronize()
        ms = []
        for _ in range(reps):
            a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            g.replay()
            e.record(stream)
            e.synchronize()
            ms.append(a.elapsed_time(e))
        del g
        return statistics.median(ms) * 1e3 / len(calls)

    data = {}
    for K, N in SHAPES:
        per = N * K + 2 * M * K + 2 * M * N
        data[(K, N)] = make(K, N, max(8, math.ceil(2 * L2_BYTES / per)))
    for K, N in SHAPES:
        for bn in ("", "32", "64", "128", "256"):
            for grid in (("",) if not bn else ("1", "2")):
                os.environ.pop("B200Q8_TRACE_BN", None)
                os.environ.pop("B200Q8_TRACE_GRID", None)
                if bn:
                    os.environ["B200Q8_TRACE_BN"] = bn
                    os.environ["B200Q8_TRACE_GRID"] = grid
                us = timed(data[(K, N)])
                tf = 2.0 * M * N * K / (us * 1e-6) / 1e12
                print(f"K={K} N={N} BN={bn or 'auto'} grid={grid or 'auto'} us={us:.2f} TFLOP/s={tf:.1f}", flush=True)
    os.environ.pop("B200Q8_TRACE_BN", None)
    os.environ.pop("B200Q8_TRACE_GRID", None)
    n = min(len(data[k]) for k in SHAPES)
    us = timed([data[k][i] for i in range(n) for k in SHAPES]) * len(SHAPES)
    fl = sum(2.0 * M * N * K for K, N in SHAPES)
    print(f"set of four, back to back: {us:.2f} us, {fl / (us * 1e-6) / 1e12:.1f} TFLOP/s", flush=True)


if __name__ == "__main__":
    cmd = sys.argv[1] if len(sys.argv) > 1 else ""
    if cmd == "build":
        print(build_trace())
    elif cmd == "phases":
        phases([tuple(int(a) for a in s.split("x")) for s in sys.argv[2:]] or SHAPES + [(3584, 37888)])
    elif cmd == "sweep":
        sweep()
    elif cmd == "roles":
        roles(sys.argv[2:] or ["3584x152064:64", "3584x37888:64", "18944x3584:64", "896x896:512",
                              "4864x896:512", "896x4864:512", "3584x37888:512"])
    else:
        print(__doc__)
