"""Pins the CPU oracle (oracle/q8_oracle.c) to the reference's own results.

The expected values come from tests/golden/, produced by the reference's
quantize_per_channel and BackendCPU::linear_q8 (see gen_golden.py).  The
oracle must reproduce them bit for bit; the GPU parity tests then trust it.
"""
import hashlib
import json
import os

import numpy as np
import pytest

from tests._util import make_weight, make_x

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


def _hex(a):
    return [f"{v:08x}" for v in _bits(a).ravel().tolist()]


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def ka():
    with open(os.path.join(GOLD, "known_answers.json")) as f:
        return json.load(f)


def test_known_answer_quantize(oracle, ka):
    for name in ("roundtrip", "zero_row", "saturation"):
        case = ka[name]
        q, s = oracle.quantize_per_channel(np.array(case["w"], np.float32))
        assert q.tolist() == case["q"], name
        assert _hex(s) == case["scales_hex"], name
    # quantize_test.cc:57-79: scale == 128/127 and q[1] == -127
    sat = ka["saturation"]
    assert sat["scales_hex"][0] == sat["expect_scale_hex"]
    assert sat["q"][0][1] == sat["expect_q1"]
    # quantize_test.cc:44-55: zero row -> scale 0, q 0
    assert ka["zero_row"]["scales_hex"] == ["00000000"]
    # quantize_test.cc:13-42: |deq - orig| <= scale + 1e-6
    rt = ka["roundtrip"]
    w = np.array(rt["w"], np.float32)
    s = np.array([int(h, 16) for h in rt["scales_hex"]], np.uint32).view(np.float32)
    deq = np.array(rt["q"], np.float32) * s[:, None]
    assert np.all(np.abs(deq - w) <= s[:, None] + 1e-6)


def test_known_answer_large_matrix(oracle, ka):
    i = np.arange(64 * 128)
    w = ((i % 255).astype(np.float32) / np.float32(127.0) - np.float32(1.0)).astype(np.float32).reshape(64, 128)
    q, s = oracle.quantize_per_channel(w)
    assert _sha(q) == ka["large_matrix"]["q_sha256"]
    assert _hex(s) == ka["large_matrix"]["scales_hex"]
    assert np.all(s > 0)


def test_known_answer_linear(oracle, ka):
    c = ka["linear_with_bias"]
    s = np.array([int(h, 16) for h in c["scales_hex"]], np.uint32).view(np.float32)
    y = oracle.linear_q8(np.array(c["x"], np.float32), np.array(c["wq"], np.int8), s,
                         np.array(c["bias"], np.float32))
    assert _hex(y) == c["y_hex"]
    assert np.allclose(y.ravel(), c["expect"], atol=c["tol"])
    c = ka["linear_matches_fp32"]
    s = np.array([int(h, 16) for h in c["scales_hex"]], np.uint32).view(np.float32)
    y = oracle.linear_q8(np.array(c["x"], np.float32), np.array(c["wq"], np.int8), s, None)
    assert _hex(y) == c["y_hex"]
    assert np.all(np.abs(y.ravel() - np.array(c["y_fp32"])) <= np.array(c["tol"]))


def test_quantize_edges_bitexact(oracle):
    g = np.load(os.path.join(GOLD, "quantize_edge.npz"))
    for suffix in ("", "_ragged", "_long"):
        q, s = oracle.quantize_per_channel(g["w" + suffix])
        assert np.array_equal(q, g["q" + suffix]), suffix
        assert np.array_equal(_bits(s), _bits(g["s" + suffix])), suffix


def test_linear_small_bitexact(oracle):
    g = np.load(os.path.join(GOLD, "linear_small.npz"))
    idx = 0
    while f"c{idx}_q" in g:
        p = f"c{idx}_"
        b = g[p + "b"] if p + "b" in g else None
        if p + "r" in g:
            out = g[p + "r"].copy()  # in-place residual, as the model calls it
            oracle.linear_q8_add(g[p + "x"], g[p + "q"], g[p + "s"], b, out, out=out)
            y = out
        else:
            y = oracle.linear_q8(g[p + "x"], g[p + "q"], g[p + "s"], b)
        assert np.array_equal(_bits(y), _bits(g[p + "y"])), p
        idx += 1
    assert idx >= 8


@pytest.fixture(scope="module")
def digests():
    with open(os.path.join(GOLD, "digests.json")) as f:
        return json.load(f)


@pytest.mark.parametrize("name", ["config1_4864x896", "qwen05b_down_896x4864", "qwen05b_k_128x896",
                                  "smol_lm_head_49152x576"])
def test_full_size_digests(oracle, digests, name):
    if digests["numpy"] != np.__version__:
        pytest.skip(f"digests made with numpy {digests['numpy']}, have {np.__version__}")
    c = digests["cases"][name]
    w = make_weight(c["N"], c["K"], c["w_seed"])
    q, s = oracle.quantize_per_channel(w)
    assert _sha(q) == c["q_sha256"]
    assert _sha(s) == c["scales_sha256"]
    x = make_x(1, c["K"], c["x_seed"])
    y = oracle.linear_q8_mt(x, q, s, None)
    assert _sha(y) == c["y_sha256"]


def test_oracle_matches_compiled_reference_random():
    """Where the reference was compiled here, compare against it on fresh random cases."""
    from oracle import Oracle, Reference, have_reference

    if not have_reference():
        pytest.skip("oracle/_ref not built")
    o, r = Oracle(), Reference()
    rng = np.random.default_rng(123)
    for M, N, K in [(1, 300, 896), (3, 65, 100), (2, 7, 4864), (1, 1, 1), (4, 3, 31)]:
        w = rng.standard_normal((N, K), dtype=np.float32)
        x = rng.standard_normal((M, K), dtype=np.float32)
        b = rng.standard_normal(N, dtype=np.float32)
        q1, s1 = o.quantize_per_channel(w)
        q2, s2 = r.quantize_per_channel(w)
        assert np.array_equal(q1, q2) and np.array_equal(_bits(s1), _bits(s2))
        assert np.array_equal(_bits(o.linear_q8(x, q1, s1, b)), _bits(r.linear_q8(x, q1, s1, b)))


def test_oracle_rows_match_full(oracle):
    w = make_weight(97, 896, 9)
    q, s = oracle.quantize_per_channel(w)
    x = make_x(2, 896, 10)
    b = np.arange(97, dtype=np.float32)
    full = oracle.linear_q8(x, q, s, b)
    rows = np.array([0, 5, 96, 50], np.int64)
    part = oracle.linear_q8_rows(x, q, s, b, rows)
    assert np.array_equal(_bits(part), _bits(full[:, rows]))


def test_prologue_golden(oracle):
    """rms_norm / silu_mul restatements equal the reference's outputs bit for bit (NaN-aware)."""
    d = np.load(os.path.join(GOLD, "prologue_small.npz"))
    n_rn = len([k for k in d.files if k.startswith("rn") and k.endswith("_y")])
    n_sm = len([k for k in d.files if k.startswith("sm") and k.endswith("_y")])
    assert n_rn >= 5 and n_sm >= 3
    for i in range(n_rn):
        p = f"rn{i}_"
        y = oracle.rms_norm(d[p + "x"], d[p + "w"], float(d[p + "eps"]))
        assert np.array_equal(_bits(y), _bits(d[p + "y"])), p
    for i in range(n_sm):
        p = f"sm{i}_"
        y = oracle.silu_mul(d[p + "gu"])
        assert np.array_equal(_bits(y), _bits(d[p + "y"])), p
    # the reference tests' own expectations (backend_naive_test.cc:199-236)
    assert np.allclose(d["rn0_y"], 1.0, atol=1e-5)
    x1, w1 = d["rn1_x"][0], d["rn1_w"]
    rms = np.sqrt(np.float32(14.0) / np.float32(3.0) + np.float32(1e-6))
    assert np.allclose(d["rn1_y"][0], x1 / rms * w1, atol=1e-5)
    # edge rows: zero row stays zero, an overflowing sum of squares gives rms = inf -> zeros
    assert not d["rn4_y"][0].any() and not d["rn4_y"][1].any()
