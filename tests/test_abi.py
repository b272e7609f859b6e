"""The C-ABI library loads and exports what include/b200q8.h declares (no GPU calls)."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "b200q8.h")


def declared_symbols():
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"B200Q8_API\s+[\w\s\*]+?\b(b200q8_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "b200q8_linear_q8" in syms and "b200q8_quantize_per_channel" in syms
    assert len(syms) >= 19


def test_library_exports_every_declared_symbol():
    from vvllm_b200 import _lib

    lib = _lib.lib()
    for s in declared_symbols():
        assert hasattr(lib, s), s
    assert set(declared_symbols()) == set(_lib.EXPORTED)
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True)
    if out.returncode == 0:
        exported = set(re.findall(r"\bT (b200q8_\w+)", out.stdout))
        assert set(declared_symbols()) <= exported


def test_abi_version_and_no_launch_yet():
    import vvllm_b200

    assert vvllm_b200.lib().b200q8_abi_version() == 1
    assert vvllm_b200.launch_count() >= 0


def test_argument_errors_without_device():
    """Argument validation happens before any CUDA call, so it works on a CPU-only host."""
    from vvllm_b200 import _lib

    L = _lib.lib()
    # bad dtype
    assert L.b200q8_linear_q8(1 << 20, 7, 2 << 20, 0, 3 << 20, 4 << 20, None, 1, 4, 16, None) == -1
    assert b"dtype" in L.b200q8_last_error()
    # null weight
    assert L.b200q8_linear_q8(1 << 20, 0, 2 << 20, 0, None, 4 << 20, None, 1, 4, 16, None) == -1
    # empty problem is a no-op
    assert L.b200q8_linear_q8(None, 0, None, 0, None, None, None, 0, 4, 16, None) == 0
    # inp overlapping out
    assert L.b200q8_linear_q8(1 << 20, 0, (1 << 20) + 8, 0, 3 << 20, 4 << 20, None, 1, 4, 16, None) == -1
    assert b"overlap" in L.b200q8_last_error()
    # residual partially overlapping out
    assert L.b200q8_linear_q8_add(1 << 20, 0, 2 << 20, 0, 3 << 20, 4 << 20, None, (1 << 20) + 4,
                                  1, 4, 16, None) == -1
    # quantize null pointers
    assert L.b200q8_quantize_per_channel(None, 4, 4, None, None, None) == -1
    # shard_range bad rank
    a, b = ctypes.c_size_t(), ctypes.c_size_t()
    assert L.b200q8_shard_range(10, 2, 2, ctypes.byref(a), ctypes.byref(b)) == -1
    # comm with null handle
    assert L.b200q8_linear_q8_sharded(None, None, 0, None, 0, None, None, None, 1, 4, 4, None, None) == -1
    # grouped projections: count out of range, null arrays, outputs overlapping x or each other
    P = ctypes.c_void_p * 2
    ns = (ctypes.c_size_t * 2)(4, 4)
    w, s, o = P(3 << 20, 5 << 20), P(4 << 20, 6 << 20), P(1 << 20, 7 << 20)
    assert L.b200q8_linear_q8_group(0, o, 0, 2 << 20, 0, None, 0.0, w, s, None, ns, 1, 16, None) == -1
    assert L.b200q8_linear_q8_group(5, o, 0, 2 << 20, 0, None, 0.0, w, s, None, ns, 1, 16, None) == -1
    assert L.b200q8_linear_q8_group(2, None, 0, 2 << 20, 0, None, 0.0, w, s, None, ns, 1, 16, None) == -1
    assert L.b200q8_linear_q8_group(2, P((2 << 20) + 4, 7 << 20), 0, 2 << 20, 0, None, 0.0, w, s, None, ns, 1, 16,
                                    None) == -1
    assert b"overlap" in L.b200q8_last_error()
    assert L.b200q8_linear_q8_group(2, P(1 << 20, (1 << 20) + 8), 0, 2 << 20, 0, None, 0.0, w, s, None, ns, 1, 16,
                                    None) == -1
    assert b"overlap" in L.b200q8_last_error()


@pytest.mark.parametrize("N,G", [(152064, 8), (18944, 4), (3584, 2), (10, 4), (3, 4), (1, 1), (7, 3)])
def test_shard_range_partitions_rows(N, G):
    import vvllm_b200

    got = [vvllm_b200.shard_range(N, G, r) for r in range(G)]
    per = -(-N // G)
    nxt = 0
    for r0, n in got:
        assert r0 == min(nxt, N)
        assert 0 <= n <= per
        nxt = r0 + n
    assert nxt == N
    if N % G == 0:
        assert all(n == N // G for _, n in got)


def test_group_binding_checks_shapes_and_dtypes():
    """The Python group binding refuses mixed output dtypes and mis-shaped buffers before any call."""
    import torch

    import vvllm_b200 as v

    x = torch.zeros((2, 64))
    w = [torch.zeros((8, 64), dtype=torch.int8), torch.zeros((4, 64), dtype=torch.int8)]
    s = [torch.zeros(8), torch.zeros(4)]
    with pytest.raises(ValueError, match="dtype"):
        v.linear_q8_group([torch.zeros((2, 8)), torch.zeros((2, 4), dtype=torch.float16)], x, w, s)
    with pytest.raises(ValueError, match="projection 1"):
        v.linear_q8_group([torch.zeros((2, 8)), torch.zeros((2, 5))], x, w, s)
    with pytest.raises(ValueError, match="projection 0"):
        v.linear_q8_group([torch.zeros((2, 8)), torch.zeros((2, 4))], x,
                          [torch.zeros((8, 32), dtype=torch.int8), w[1]], s)
    with pytest.raises(ValueError, match="same length"):
        v.linear_q8_group([torch.zeros((2, 8))], x, w, s)
    outs = [torch.zeros((2, 8)), torch.zeros((2, 4))]
    with pytest.raises(ValueError, match="scales"):  # a short scales vector would be read past its end
        v.linear_q8_group(outs, x, w, [s[0], torch.zeros(3)])
    with pytest.raises(ValueError, match="bias"):
        v.linear_q8_group(outs, x, w, s, [torch.zeros(8), torch.zeros(2)])
    with pytest.raises(ValueError, match="x must be contiguous"):
        v.linear_q8_group(outs, torch.zeros((64, 2)).t(), w, s)
    with pytest.raises(ValueError, match="weights must be contiguous"):
        v.linear_q8_group(outs, x, [w[0], torch.zeros((64, 4), dtype=torch.int8).t()], s)


def test_diag_peer_wait_argument_errors():
    """The failure-test entry point validates its arguments before any CUDA call."""
    from vvllm_b200 import _lib

    L = _lib.lib()
    assert L.b200q8_diag_peer_wait(None, 1, 1, 0.1, 0, None, None, None, None, 0, 0, None) == -1
    assert L.b200q8_diag_peer_wait(1 << 20, 9, 1, 0.1, 0, None, None, None, None, 0, 0, None) == -1
    assert L.b200q8_diag_peer_wait(1 << 20, 1, 1, 0.1, 0, None, None, None, None, 0, 0, None) == -1
    assert L.b200q8_diag_peer_wait(1 << 20, 1, 0, 20.0, 0, None, None, None, None, 0, 0, None) == -1
    assert b"timeout" in L.b200q8_last_error()
    assert L.b200q8_diag_peer_wait(1 << 20, 1, 0, 0.1, 3, None, None, None, None, 0, 0, None) == -1
    assert L.b200q8_diag_peer_wait(1 << 20, 1, 0, 0.1, 1, None, None, None, None, 16, 16, None) == -1
    assert b"GEMV needs" in L.b200q8_last_error()
