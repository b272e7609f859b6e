"""CPU checkers for the quantized-linear path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
import this package.  It is never on the product path: ``vvllm_b200`` does not
import it and has no CPU fallback.

Two libraries are wrapped:

* ``liboracle.so`` -- ``q8_oracle.c``, a C restatement of
  ``src/quantize/quantize.cc:9-48`` and ``src/backend/backend_naive.cc:155-335``
  (hoobean1996/vvllm), bit-identical to the reference's x86 AVX2+FMA build.
* ``_ref/libvvllm_ref.so`` -- the reference's own ``backend_naive.cc`` and
  ``quantize.cc`` compiled in place by ``oracle/Makefile`` (present where the
  reference tree was available at build time; it travels as a built file).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libvvllm_ref.so")

_c_size = ctypes.c_size_t
_vp = ctypes.c_void_p


def build(ref: str | None = None) -> None:
    """Compile the checkers with oracle/Makefile (REF is the reference tree)."""
    cmd = ["make", "-s", "-C", HERE]
    if ref:
        cmd.append(f"REF={ref}")
    subprocess.run(cmd, check=True)


def _ptr(a: np.ndarray | None) -> int | None:
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


class _Lib:
    def __init__(self, path: str, prefix: str):
        self.path = path
        self.lib = ctypes.CDLL(path)
        p = prefix
        self._q = getattr(self.lib, f"{p}quantize_per_channel")
        self._l = getattr(self.lib, f"{p}linear_q8")
        self._la = getattr(self.lib, f"{p}linear_q8_add")
        self._lmt = getattr(self.lib, f"{p}linear_q8_mt")
        self._q.argtypes = [_vp, _c_size, _c_size, _vp, _vp]
        self._l.argtypes = [_vp, _vp, _vp, _vp, _vp, _c_size, _c_size, _c_size]
        self._la.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _c_size, _c_size, _c_size]
        self._lmt.argtypes = [_vp, _vp, _vp, _vp, _vp, _c_size, _c_size, _c_size, ctypes.c_int]
        for f in (self._q, self._l, self._la, self._lmt):
            f.restype = ctypes.c_int
        self._rn = getattr(self.lib, f"{p}rms_norm")
        self._sm = getattr(self.lib, f"{p}silu_mul")
        self._rn.argtypes = [_vp, _vp, _vp, _c_size, _c_size, ctypes.c_float]
        self._sm.argtypes = [_vp, _vp, _c_size, _c_size]

    # backend_naive.cc:67-75 per token (transformer.cc:40-50): [M, K] -> [M, K]
    def rms_norm(self, x, w, eps):
        x = np.ascontiguousarray(x, dtype=np.float32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        M, K = x.shape
        y = np.empty((M, K), dtype=np.float32)
        self._rn(_ptr(y), _ptr(x), _ptr(w), M, K, float(eps))
        return y

    # backend_naive.cc:293-300 per [gate | up] row (transformer.h:175-180): [M, 2K] -> [M, K]
    def silu_mul(self, gate_up):
        gu = np.ascontiguousarray(gate_up, dtype=np.float32)
        M, K2 = gu.shape
        y = np.empty((M, K2 // 2), dtype=np.float32)
        self._sm(_ptr(y), _ptr(gu), M, K2 // 2)
        return y

    # quantize.cc:9-48 -- returns (int8 [N,K], fp32 scales [N])
    def quantize_per_channel(self, w: np.ndarray):
        w = np.ascontiguousarray(w, dtype=np.float32)
        N, K = w.shape
        q = np.empty((N, K), dtype=np.int8)
        s = np.empty((N,), dtype=np.float32)
        self._q(_ptr(w), N, K, _ptr(q), _ptr(s))
        return q, s

    # backend_naive.cc:155-291
    def linear_q8(self, x, wq, scales, bias=None, out=None):
        x = np.ascontiguousarray(x, dtype=np.float32)
        M, K = x.shape
        N = wq.shape[0]
        y = np.empty((M, N), dtype=np.float32) if out is None else out
        self._l(_ptr(y), _ptr(x), _ptr(wq), _ptr(scales), _ptr(bias), M, N, K)
        return y

    # backend_naive.cc:322-335 (residual may be the output array itself)
    def linear_q8_add(self, x, wq, scales, bias, residual, out=None):
        x = np.ascontiguousarray(x, dtype=np.float32)
        M, K = x.shape
        N = wq.shape[0]
        y = np.empty((M, N), dtype=np.float32) if out is None else out
        self._la(_ptr(y), _ptr(x), _ptr(wq), _ptr(scales), _ptr(bias), _ptr(residual), M, N, K)
        return y

    def linear_q8_mt(self, x, wq, scales, bias=None, nthreads=None, out=None):
        x = np.ascontiguousarray(x, dtype=np.float32)
        M, K = x.shape
        N = wq.shape[0]
        y = np.empty((M, N), dtype=np.float32) if out is None else out
        n = nthreads or os.cpu_count() or 1
        self._lmt(_ptr(y), _ptr(x), _ptr(wq), _ptr(scales), _ptr(bias), M, N, K, n)
        return y


class Oracle(_Lib):
    """The C restatement (liboracle.so)."""

    def __init__(self):
        if not os.path.exists(ORACLE_SO):
            build()
        super().__init__(ORACLE_SO, "q8o_")
        self._rows = self.lib.q8o_linear_q8_gather
        self._rows.argtypes = [_vp, _vp, _vp, _vp, _vp, _c_size, _c_size, _vp, _c_size]
        self._rows.restype = None

    def linear_q8_rows(self, x, wq, scales, bias, rows):
        """Outputs for the listed output channels only: [M, len(rows)]."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows = np.ascontiguousarray(rows, dtype=np.int64)
        M, K = x.shape
        y = np.empty((M, rows.size), dtype=np.float32)
        self._rows(_ptr(y), _ptr(x), _ptr(wq), _ptr(scales), _ptr(bias), M, K, _ptr(rows), rows.size)
        return y


class Reference(_Lib):
    """The reference's own CPU code (oracle/_ref/libvvllm_ref.so)."""

    def __init__(self):
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(REF_SO)
        super().__init__(REF_SO, "vref_")


def have_reference() -> bool:
    return os.path.exists(REF_SO)
