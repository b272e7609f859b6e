"""Builds libb200q8.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m vvllm_b200.build            # incremental
    python -m vvllm_b200.build --force    # rebuild everything

Objects go to ``vvllm_b200/_build/`` (git-ignored); the shared library is
written next to this file so it travels with the source tree.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libb200q8.so")

SOURCES = ["b200q8_api.cu", "q8_gemv.cu", "q8_quantize.cu", "q8_gemm_tc.cu", "q8_gemv_tc.cu", "gather.cu", "prologue.cu", "q8st.cu"]
HEADERS = ["common.cuh", "kernels.h", "tc_utils.cuh", "sk_common.cuh", "tmap.cuh", "prologue.cuh", "p2p.cuh"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# No --use_fast_math / -ftz: the quantize kernel must keep denormals and IEEE division.
NVCC_FLAGS = ARCH + [
    "-O3", "-std=c++20", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include"), "-I" + CSRC,
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    cc = nvcc()
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "b200q8.h")]
    objs, jobs = [], []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            cmd = [cc, *NVCC_FLAGS, "-c", s, "-o", o]
            if ptxas_v:
                cmd[1:1] = ["-Xptxas", "-v"]
            jobs.append(cmd)
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        futs = {ex.submit(subprocess.run, j, capture_output=True, text=True): j for j in jobs}
        for f in cf.as_completed(futs):
            r = f.result()
            if verbose or ptxas_v:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
                raise RuntimeError("nvcc failed: " + " ".join(futs[f]))
    if force or jobs or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [cc, *ARCH, "-shared", "-o", tmp, *objs, "-ldl", "-lpthread", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register / smem usage")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_v=a.ptxas_v))
