"""Generates the golden fixtures in tests/golden/ from the reference's own code.

    make -C oracle REF=<vvllm checkout>     # builds oracle/_ref/libvvllm_ref.so
    python tests/golden/gen_golden.py

Every expected value below is produced by hoobean1996/vvllm's
``quantize_per_channel`` (src/quantize/quantize.cc:9-48) and
``BackendCPU::linear_q8`` / ``linear_q8_add`` (src/backend/backend_naive.cc:
155-291, 322-335), compiled unmodified where they lie (oracle/Makefile) and
called through oracle/ref_shim.cc.  Outputs:

* known_answers.json -- the reference unit tests' own cases
  (src/quantize/quantize_test.cc:13-100, src/backend/backend_naive_test.cc:
  355-425) with the reference's exact results (float bit patterns in hex);
* quantize_edge.npz  -- edge rows (zeros, NaN, +-Inf, subnormals, ties);
* linear_small.npz   -- seeded small linear_q8 / linear_q8_add cases;
* prologue_small.npz -- BackendCPU::rms_norm / silu_mul (backend_naive.cc:67-75, :293-300)
  applied per token, on the reference tests' two rms_norm cases
  (backend_naive_test.cc:199-236), seeded rows and edge rows;
* digests.json       -- SHA-256 of the reference's outputs at full benchmark
  sizes for inputs regenerated from numpy seeds (tests rebuild the inputs and
  compare digests, so megabytes of data need not be committed).
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import Reference  # noqa: E402
from tests._util import make_bias, make_weight, make_x  # noqa: E402


def hexbits(a: np.ndarray) -> list[str]:
    return [f"{v:08x}" for v in np.asarray(a, dtype=np.float32).view(np.uint32).ravel().tolist()]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def known_answers(ref: Reference) -> dict:
    out = {}
    # quantize_test.cc:13-42 RoundtripAccuracy
    w = np.array([[0.5, -0.3, 0.1, 0.9], [1.0, 0.0, -1.0, 0.5], [0.0, 0.2, 0.4, -0.8]], np.float32)
    q, s = ref.quantize_per_channel(w)
    out["roundtrip"] = {"w": w.tolist(), "q": q.tolist(), "scales_hex": hexbits(s)}
    # quantize_test.cc:44-55 ZeroRow
    w = np.zeros((1, 4), np.float32)
    q, s = ref.quantize_per_channel(w)
    out["zero_row"] = {"w": w.tolist(), "q": q.tolist(), "scales_hex": hexbits(s)}
    # quantize_test.cc:57-79 Saturation
    w = np.array([[127.0, -128.0, 0.0, 50.0]], np.float32)
    q, s = ref.quantize_per_channel(w)
    out["saturation"] = {"w": w.tolist(), "q": q.tolist(), "scales_hex": hexbits(s),
                         "expect_scale_hex": hexbits(np.float32(128.0) / np.float32(127.0))[0],
                         "expect_q1": -127}
    # quantize_test.cc:81-100 LargeMatrix: w[i] = (i % 255) / 127 - 1 over 64 x 128
    i = np.arange(64 * 128)
    w = ((i % 255).astype(np.float32) / np.float32(127.0) - np.float32(1.0)).astype(np.float32).reshape(64, 128)
    q, s = ref.quantize_per_channel(w)
    out["large_matrix"] = {"q_sha256": sha(q), "scales_hex": hexbits(s)}
    # backend_naive_test.cc:407-425 LinearQ8WithBias
    wq = np.array([[127, 0], [0, 127]], np.int8)
    sc = np.array([1.0 / 127.0, 1.0 / 127.0], np.float32)
    b = np.array([10.0, 20.0], np.float32)
    x = np.array([[3.0, 5.0]], np.float32)
    y = ref.linear_q8(x, wq, sc, b)
    out["linear_with_bias"] = {"wq": wq.tolist(), "scales_hex": hexbits(sc), "bias": b.tolist(),
                               "x": x.tolist(), "y_hex": hexbits(y), "expect": [13.0, 25.0], "tol": 1e-4}
    # backend_naive_test.cc:355-405 LinearQ8MatchesFp32 (its quantizer divides, :387)
    w = np.array([[0.5, -0.3, 0.1, 0.9], [1.0, 0.0, -1.0, 0.5], [0.0, 0.2, 0.4, -0.8]], np.float32)
    absmax = np.max(np.abs(w), axis=1)
    scl = (absmax / np.float32(127.0)).astype(np.float32)
    wq = np.clip(np.round(w / scl[:, None]), -128, 127).astype(np.int8)  # np.round ties-to-even: no ties here
    x = np.array([[1.0, 2.0, 3.0, 4.0]], np.float32)
    y = ref.linear_q8(x, wq, scl, None)
    y32 = (x.astype(np.float64) @ w.T.astype(np.float64)).astype(np.float32)
    out["linear_matches_fp32"] = {"wq": wq.tolist(), "scales_hex": hexbits(scl), "x": x.tolist(),
                                  "y_hex": hexbits(y), "y_fp32": y32.ravel().tolist(),
                                  "tol": (scl * np.float32(4 * 0.5) + np.float32(1e-5)).tolist()}
    return out


def quantize_edges(ref: Reference) -> dict:
    rows = [
        [0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0],
        [1e-40, -2e-40, 0.0, -0.0, 1e-41, 3e-40, -1e-45, 0.0],        # subnormal absmax -> inv = +inf
        [np.nan, 1.0, 2.0, 3.0, -4.0, 0.5, np.nan, 0.0],                 # NaN skipped by absmax, maps to 127
        [np.inf, 1.0, -np.inf, 0.0, 5.0, -5.0, 2.0, 1.0],                # scale = inf
        [np.nan] * 8,                                                   # all NaN -> scale 0
        [127.0, -128.0, 0.0, 50.0, 1.0, -1.0, 63.5, -63.5],              # saturation, ties
        [1.0, 0.5, -0.5, 1.5 / 127, -2.5 / 127, 0.25, -0.75, 0.0],       # half-way cases
        [3.4e38, -3.4e38, 1.0, -1.0, 1e30, 0.0, 2e38, -1e38],            # near FLT_MAX
        [1e-30, -1e-30, 5e-31, 0.0, 2e-31, -7e-31, 1e-31, 3e-31],        # small normal
        [-0.0, -0.0, -0.0, -0.0, -0.0, -0.0, -0.0, -0.0],                # negative zeros
    ]
    w = np.array(rows, np.float32)
    # plus ragged K (not a multiple of 4 or 16) and a long row
    rng = np.random.default_rng(5)
    w_ragged = (rng.standard_normal((7, 37), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    w_long = (rng.standard_normal((3, 20000), dtype=np.float32)).astype(np.float32)
    q, s = ref.quantize_per_channel(w)
    qr, sr = ref.quantize_per_channel(w_ragged)
    ql, sl = ref.quantize_per_channel(w_long)
    return dict(w=w, q=q, s=s, w_ragged=w_ragged, q_ragged=qr, s_ragged=sr, w_long=w_long, q_long=ql,
                s_long=sl)


LINEAR_CASES = [
    # (M, N, K, seed, bias, residual)
    (1, 17, 32, 1, True, False),
    (1, 128, 576, 2, False, False),
    (2, 64, 896, 3, True, True),
    (3, 33, 48, 4, True, False),    # K % 32 != 0: reference's scalar tail
    (4, 40, 1536, 5, False, True),
    (1, 8, 17, 6, True, True),      # K % 16 != 0
    (5, 24, 64, 7, True, False),
    (1, 48, 4864, 8, False, True),
]


def linear_small(ref: Reference) -> dict:
    data = {}
    for idx, (M, N, K, seed, has_b, has_r) in enumerate(LINEAR_CASES):
        w = make_weight(N, K, 100 + seed)
        q, s = ref.quantize_per_channel(w)
        x = make_x(M, K, 200 + seed)
        b = make_bias(N, 300 + seed) if has_b else None
        if has_r:
            r = make_x(M, N, 400 + seed)
            y = ref.linear_q8_add(x, q, s, b, r)
        else:
            r = None
            y = ref.linear_q8(x, q, s, b)
        p = f"c{idx}_"
        data[p + "q"], data[p + "s"], data[p + "x"], data[p + "y"] = q, s, x, y
        if b is not None:
            data[p + "b"] = b
        if r is not None:
            data[p + "r"] = r
    return data


# Full-size configs (benchmark configs 1, 3, 5 shapes); seeds as documented in tests.
DIGEST_CASES = [
    # name, N, K, weight seed, x seed
    ("config1_4864x896", 4864, 896, 1000, 42),
    ("qwen05b_gate_4864x896", 4864, 896, 1004, 42),
    ("qwen05b_down_896x4864", 896, 4864, 1006, 43),
    ("qwen05b_k_128x896", 128, 896, 1001, 44),
    ("smol_lm_head_49152x576", 49152, 576, 1015, 45),
    ("qwen05b_lm_head_151936x896", 151936, 896, 1015, 46),
    ("qwen7b_down_3584x18944", 3584, 18944, 1006, 47),
]


def digests(ref: Reference) -> dict:
    out = {"numpy": np.__version__, "cases": {}}
    for name, N, K, ws, xs in DIGEST_CASES:
        w = make_weight(N, K, ws)
        q, s = ref.quantize_per_channel(w)
        x = make_x(1, K, xs)
        y = ref.linear_q8_mt(x, q, s, None)
        out["cases"][name] = {"N": N, "K": K, "w_seed": ws, "x_seed": xs, "q_sha256": sha(q),
                              "scales_sha256": sha(s), "y_sha256": sha(y)}
        print(name, "done", flush=True)
    return out


def prologue_small(ref: Reference) -> dict:
    data = {}
    rng = np.random.default_rng(77)
    # rms_norm: (x [M, K], w [K], eps)
    rn = [
        (np.full((1, 4), 2.0, np.float32), np.ones(4, np.float32), 1e-6),             # RmsNormUniform
        (np.array([[1, 2, 3]], np.float32), np.array([0.5, 1, 2], np.float32), 1e-6),  # RmsNormWithWeight
        (make_x(3, 896, 501), (1 + 0.1 * rng.standard_normal(896)).astype(np.float32), 1e-6),
        (make_x(2, 3584, 502) * np.float32(40), rng.standard_normal(3584).astype(np.float32), 1e-5),
    ]
    edge = make_x(3, 64, 503)
    edge[0] = 0.0                 # zero row: rms = sqrt(eps)
    edge[1, 5] = np.float32(1e20)  # x^2 overflows: rms = inf
    edge[2, ::7] = -edge[2, ::7]
    rn.append((edge, rng.standard_normal(64).astype(np.float32), 1e-6))
    for i, (x, w, eps) in enumerate(rn):
        p = f"rn{i}_"
        data[p + "x"], data[p + "w"], data[p + "eps"] = x, w, np.float32(eps)
        data[p + "y"] = ref.rms_norm(x, w, eps)
    # silu_mul: gate_up [M, 2K]
    sm = [make_x(2, 2 * 896, 511) * np.float32(3), make_x(1, 2 * 4864, 512) * np.float32(8)]
    g = np.array([-100, -88, -20, -1, -0.0, 0, 1e-30, 0.5, 1, 20, 88, 100, -87.5, 87.5, -3, 3], np.float32)
    sm.append(np.concatenate([g, rng.standard_normal(16).astype(np.float32)])[None, :])
    for i, gu in enumerate(sm):
        p = f"sm{i}_"
        data[p + "gu"] = gu
        data[p + "y"] = ref.silu_mul(gu)
    return data


def main():
    ref = Reference()
    if sys.argv[1:] == ["prologue"]:  # only the prologue fixtures
        np.savez_compressed(os.path.join(HERE, "prologue_small.npz"), **prologue_small(ref))
        return
    with open(os.path.join(HERE, "known_answers.json"), "w") as f:
        json.dump(known_answers(ref), f, indent=1)
    np.savez_compressed(os.path.join(HERE, "quantize_edge.npz"), **quantize_edges(ref))
    np.savez_compressed(os.path.join(HERE, "linear_small.npz"), **linear_small(ref))
    np.savez_compressed(os.path.join(HERE, "prologue_small.npz"), **prologue_small(ref))
    with open(os.path.join(HERE, "digests.json"), "w") as f:
        json.dump(digests(ref), f, indent=1)


if __name__ == "__main__":
    main()
