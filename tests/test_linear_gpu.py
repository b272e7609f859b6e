"""GPU parity of b200q8_linear_q8 / _add (through the C ABI) against the CPU oracle.

Tolerances (normwise over each token row, max|y - y_ref| / max|y_ref|):
  fp32 activations: 1e-5      fp16 activations: 2e-3 (after the kernel's fp16 rounding)
The fp16 oracle runs on the exact fp32 widening of the same fp16 inputs.
"""
import os
import zlib

import numpy as np
import pytest

from tests._util import (TOL_F16, TOL_F32, make_bias, make_weight, make_x, rowwise_normwise_err,
                         sample_rows)

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _t(a, dev, dtype=None):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


def run_gpu(cuda, x, q, s, b=None, res=None, in16=False, out16=False, inplace=False, algo=None):
    """Runs the kernel; returns (y as fp32 numpy, oracle inputs x_eff, res_eff).
    algo=None goes through b200q8_linear_q8 / _add (automatic kernel choice);
    otherwise b200q8_linear_q8_ex with that kernel."""
    import torch

    import vvllm_b200 as v

    xt = _t(x, cuda, torch.float16 if in16 else torch.float32)
    qt, st = _t(q, cuda), _t(s, cuda)
    bt = _t(b, cuda) if b is not None else None
    odt = torch.float16 if out16 else torch.float32
    M, N = x.shape[0], q.shape[0]
    rt = None
    if res is not None:
        rt = _t(res, cuda, odt)
        res_eff = rt.float().cpu().numpy()
        out = rt if inplace else torch.empty((M, N), dtype=odt, device=cuda)
    else:
        res_eff = None
        out = torch.empty((M, N), dtype=odt, device=cuda)
    if algo is not None:
        v.linear_q8_ex(out, xt, qt, st, bt, rt, algo=algo)
    elif rt is not None:
        v.linear_q8_add(out, xt, qt, st, bt, rt)
    else:
        v.linear_q8(out, xt, qt, st, bt)
    torch.cuda.synchronize()
    assert v.kernel_error() == 0
    x_eff = xt.float().cpu().numpy()
    return out.float().cpu().numpy(), x_eff, res_eff


def oracle_ref(oracle, x_eff, q, s, b, res_eff):
    if res_eff is not None:
        return oracle.linear_q8_add(x_eff, q, s, b, res_eff)
    return oracle.linear_q8(x_eff, q, s, b)


def test_golden_cases_fp32(cuda):
    """The reference's own outputs (tests/golden/linear_small.npz) at 1e-5."""
    g = np.load(os.path.join(GOLD, "linear_small.npz"))
    idx = 0
    while f"c{idx}_q" in g:
        p = f"c{idx}_"
        b = g[p + "b"] if p + "b" in g else None
        r = g[p + "r"] if p + "r" in g else None
        y, _, _ = run_gpu(cuda, g[p + "x"], g[p + "q"], g[p + "s"], b, r, inplace=r is not None)
        err = rowwise_normwise_err(y, g[p + "y"])
        assert err <= TOL_F32, (p, err)
        idx += 1


SHAPES = [
    # name, M, N, K
    ("config1", 1, 4864, 896),
    ("smol_q", 1, 576, 576), ("smol_kv", 1, 192, 576), ("smol_up", 1, 1536, 576),
    ("smol_down", 1, 576, 1536),
    ("qwen_q", 1, 896, 896), ("qwen_kv", 1, 128, 896), ("qwen_gate_up", 1, 9728, 896),
    ("qwen_down", 1, 896, 4864),
    ("q7b_down_shard8", 1, 448, 18944), ("q7b_up_shard8", 1, 4736, 3584),
    ("m2", 2, 1000, 896), ("m3", 3, 333, 1536), ("m4", 4, 4864, 896), ("m5", 5, 300, 576),
    ("m8", 8, 512, 896), ("m17", 17, 100, 3584),
]


@pytest.mark.parametrize("in16,out16", [(False, False), (True, True), (True, False), (False, True)])
@pytest.mark.parametrize("name,M,N,K", SHAPES)
def test_linear_shapes(cuda, oracle, name, M, N, K, in16, out16):
    w = make_weight(N, K, zlib.crc32(name.encode()) % 1000 + 1)
    q, s = oracle.quantize_per_channel(w)
    x = make_x(M, K, 42)
    b = make_bias(N, 7) if name.startswith("qwen_q") or name.startswith("qwen_kv") or M > 1 else None
    y, xe, _ = run_gpu(cuda, x, q, s, b, in16=in16, out16=out16)
    ref = oracle_ref(oracle, xe, q, s, b, None)
    tol = TOL_F16 if (in16 or out16) else TOL_F32
    err = rowwise_normwise_err(y, ref)
    assert err <= tol, err


TC_SHAPES = [
    # name, M, N, K -- the tensor-core kernel across token tiles (BN 16..256) and ragged edges
    ("tc_m1", 1, 4864, 896), ("tc_m1_k3584", 1, 1000, 3584), ("tc_m3", 3, 640, 576),
    ("tc_m16", 16, 384, 1536), ("tc_m17", 17, 300, 896), ("tc_m32", 32, 256, 4864),
    ("tc_m40", 40, 130, 896), ("tc_m64", 64, 512, 3584), ("tc_m100", 100, 200, 1536),
    ("tc_m128", 128, 256, 896), ("tc_m200", 200, 129, 576), ("tc_m300", 300, 384, 896),
    ("tc_k_tail", 8, 256, 16 * 37), ("tc_n1", 5, 1, 896), ("tc_n127", 2, 127, 128),
    ("tc_n448_k18944", 1, 448, 18944),  # few rows on a long K: the 7B down shard at 8 GPUs
]


@pytest.mark.parametrize("out16", [True, False])
@pytest.mark.parametrize("algo_name", ["simt", "tc", "tc_i8"])
@pytest.mark.parametrize("name,M,N,K", TC_SHAPES)
def test_fp16_paths_explicit(cuda, oracle, name, M, N, K, algo_name, out16):
    """Every kernel on the fp16-activation path, called explicitly, against the oracle."""
    import vvllm_b200 as v

    if algo_name == "simt" and M > 40:
        pytest.skip("SIMT path streams W once per 4 tokens: covered at small M")
    algo = {"simt": v.ALGO_SIMT, "tc": v.ALGO_TC, "tc_i8": v.ALGO_TC_I8}[algo_name]
    w = make_weight(N, K, zlib.crc32(name.encode()) % 1000 + 3)
    q, s = oracle.quantize_per_channel(w)
    x = make_x(M, K, 77)
    b = make_bias(N, 78)
    res = make_x(M, N, 79) if M % 2 else None
    y, xe, re = run_gpu(cuda, x, q, s, b, res, in16=True, out16=out16, inplace=res is not None, algo=algo)
    ref = oracle_ref(oracle, xe, q, s, b, re)
    assert rowwise_normwise_err(y, ref) <= TOL_F16


I8_FP32_SHAPES = [
    # fp32 activations on the int8 tensor-core kernel: exact digits must hold the 1e-5 bar
    ("i8_m1", 1, 4864, 896), ("i8_m1_k4864", 1, 896, 4864), ("i8_m2", 2, 300, 576), ("i8_m4", 4, 1536, 576),
    ("i8_m5", 5, 200, 1536), ("i8_m8", 8, 384, 1536), ("i8_m16", 16, 640, 896), ("i8_m33", 33, 256, 3584), ("i8_m64", 64, 130, 896),
    ("i8_m100", 100, 128, 576), ("i8_k16", 3, 50, 16), ("i8_k18944", 1, 448, 18944),
]


@pytest.mark.parametrize("name,M,N,K", I8_FP32_SHAPES)
def test_i8_digits_fp32(cuda, oracle, name, M, N, K):
    import vvllm_b200 as v

    w = make_weight(N, K, zlib.crc32(name.encode()) % 1000 + 5)
    q, s = oracle.quantize_per_channel(w)
    x = make_x(M, K, 81) * np.float32(3.0)
    b = make_bias(N, 82)
    res = make_x(M, N, 83) if M % 2 else None
    y, xe, re = run_gpu(cuda, x, q, s, b, res, inplace=res is not None, algo=v.ALGO_TC_I8)
    assert rowwise_normwise_err(y, oracle_ref(oracle, xe, q, s, b, re)) <= TOL_F32


def test_i8_digits_wide_dynamic_range(cuda, oracle):
    """Activations spanning many binades (tiny, huge, zero rows) keep the fp32 tolerance."""
    import vvllm_b200 as v

    N, K, M = 384, 1536, 4
    q, s = oracle.quantize_per_channel(make_weight(N, K, 91))
    x = make_x(M, K, 92)
    x[0] *= np.float32(1e-30)
    x[1] *= np.float32(1e30)
    x[2] = 0.0
    x[3, ::7] *= np.float32(1e4)
    y, xe, _ = run_gpu(cuda, x, q, s, None, None, algo=v.ALGO_TC_I8)
    ref = oracle_ref(oracle, xe, q, s, None, None)
    assert np.all(y[2] == 0.0)
    for i in (0, 1, 3):
        assert rowwise_normwise_err(y[i], ref[i]) <= TOL_F32, i


def test_i8_nonfinite_rows_give_nan(cuda, oracle):
    """A token row holding Inf/NaN yields NaN outputs on the digit kernel; other rows are exact."""
    import vvllm_b200 as v

    N, K = 256, 896
    q, s = oracle.quantize_per_channel(make_weight(N, K, 93))
    x = make_x(3, K, 94)
    x[1, 5] = np.inf
    y, xe, _ = run_gpu(cuda, x, q, s, None, None, algo=v.ALGO_TC_I8)
    assert np.all(np.isnan(y[1]))
    ref = oracle_ref(oracle, xe, q, s, None, None)
    for i in (0, 2):
        assert rowwise_normwise_err(y[i], ref[i]) <= TOL_F32


# (M, N, K, position of the bad value): fp16 rows scanned in-kernel for one token up to 20480
# wide and for up to 4 tokens up to 4096 wide; from the prep kernel's words otherwise
FP16_BAD = [
    (1, 256, 896, -3),
    (1, 512, 18944, -1),     # 7B down width, one token: in-kernel, by the epilogue warps alone
    (1, 384, 24576, 0),      # wider: prep kernel, folded by the epilogue warps alone
    (2, 256, 896, 100),
    (3, 320, 8192, -5),      # several tokens on long rows: prep kernel
    (8, 256, 896, 7),        # five tokens or more: the prep kernel's digit tiles
    (6, 300, 3584, -2),
]


@pytest.mark.parametrize("M,N,K,pos", FP16_BAD)
@pytest.mark.parametrize("val", [np.inf, np.nan])
def test_i8_fp16_nonfinite_rows_give_nan(cuda, oracle, M, N, K, pos, val):
    """fp16 digits use the fixed exponent; only the epilogue warps look for Inf/NaN. The token
    holding one gets NaN outputs, wherever in the row it sits, and the others match the oracle."""
    import vvllm_b200 as v

    q, s = oracle.quantize_per_channel(make_weight(N, K, 130 + K % 97))
    x = make_x(M, K, 131 + M)
    bad = M // 2
    x[bad, pos] = val
    y, xe, _ = run_gpu(cuda, x, q, s, None, None, in16=True, algo=v.ALGO_TC_I8)
    assert np.all(np.isnan(y[bad]))
    ref = oracle_ref(oracle, xe, q, s, None, None)
    for i in range(M):
        if i != bad:
            assert rowwise_normwise_err(y[i], ref[i]) <= TOL_F16, i


def test_i8_prep_kernel_scratch_across_token_counts(cuda, oracle):
    """Rows longer than 4096 take the prep kernel, several CTAs per token combining through
    zero-at-rest words in the per-stream scratch.  Calls with different token counts in a row
    (fp32: exponents differ per token; an Inf row in between) must each be right: no call may
    leave those words dirty for the next, whatever its M."""
    import vvllm_b200 as v

    N, K = 320, 8192
    q, s = oracle.quantize_per_channel(make_weight(N, K, 95))
    for M, seed in ((7, 96), (1, 97), (3, 98), (5, 99), (1, 100), (7, 101)):
        x = make_x(M, K, seed) * np.float32(10.0 ** (seed % 5 - 2))
        if M == 5:
            x[2, 11] = np.inf
        y, xe, _ = run_gpu(cuda, x, q, s, None, None, algo=v.ALGO_TC_I8)
        ref = oracle_ref(oracle, xe, q, s, None, None)
        for i in range(M):
            if M == 5 and i == 2:
                assert np.all(np.isnan(y[i]))
            else:
                assert rowwise_normwise_err(y[i], ref[i]) <= TOL_F32, (M, i)


def _exact_i8_f16(xh, q, s, b, res):
    """The digit kernel's fp16-activation result, emulated bit for bit: the exact dot product of
    the int8 row and the fp16 activations (float64 is exact here: every product is a multiple of
    2^-24 below 2^34 of them, every partial sum below 2^53 of them), rounded once to fp32, then
    * scale (+ bias) (+ res) in fp32 and rounded to the output type."""
    acc = (xh.astype(np.float64) @ q.astype(np.float64).T).astype(np.float32)
    y = acc * s[None, :]
    if b is not None:
        y = y + b[None, :]
    if res is not None:
        y = y + res
    return y


# (M, N, K, fp16 outputs): one to four tokens digitize in-kernel; from five tokens on (and for
# several tokens on long rows of large weights) the prep kernel makes each stage's digit tile once
EXACT_F16 = [
    (1, 300, 896, True), (2, 257, 3584, False), (4, 130, 1536, True), (5, 300, 896, True),
    (8, 256, 3584, True), (8, 129, 16 * 37, False), (16, 384, 1536, True), (33, 200, 896, False),
    (42, 130, 4864, True), (2, 3000, 12288, True), (6, 300, 3584, True), (7, 131, 896, False),
]


@pytest.mark.parametrize("M,N,K,out16", EXACT_F16)
def test_i8_fp16_exact_rounding(cuda, oracle, M, N, K, out16):
    """With fp16 activations the digit kernel's outputs are the correctly rounded dot products:
    bit-identical to an exact emulation, on both the in-kernel digits and the prep kernel's
    digit tiles (stage tails, zero digit rows past 6M, ragged N)."""
    import vvllm_b200 as v

    q, s = oracle.quantize_per_channel(make_weight(N, K, 140 + M))
    x = make_x(M, K, 141 + M)
    b = make_bias(N, 142)
    res = make_x(M, N, 143) if M % 2 else None
    y, xe, re = run_gpu(cuda, x, q, s, b, res, in16=True, out16=out16, algo=v.ALGO_TC_I8)
    want = _exact_i8_f16(xe, q, s, b, re)
    if out16:
        want = want.astype(np.float16).astype(np.float32)
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32)), float(np.max(np.abs(y - want)))


def test_i8_fp16_digit_tiles_across_token_counts(cuda, oracle):
    """The prep kernel's digit tiles live in per-stream scratch: calls with different token
    counts (and digit-tile widths) in a row, one with an Inf, must each be exact."""
    import vvllm_b200 as v

    N, K = 320, 3584
    q, s = oracle.quantize_per_channel(make_weight(N, K, 150))
    for M, seed in ((16, 151), (5, 152), (42, 153), (8, 154), (6, 155), (16, 156)):
        x = make_x(M, K, seed)
        if M == 6:
            x[3, 1000] = np.inf
        y, xe, _ = run_gpu(cuda, x, q, s, None, None, in16=True, algo=v.ALGO_TC_I8)
        want = _exact_i8_f16(xe, q, s, None, None)
        for i in range(M):
            if M == 6 and i == 3:
                assert np.all(np.isnan(y[i]))
            else:
                assert np.array_equal(y[i].view(np.uint32), want[i].view(np.uint32)), (M, i)


# 33-64 tokens: 64-token tiles with two MMA-issuing threads taking alternate K-stages into two
# accumulators; stream-K segments of one stage (second accumulator unused), odd and even lengths
TWO_ISSUERS = [
    (64, 19000, 896),   # 149 row tiles of 7 stages on 148 CTAs: split segments of every length
    (48, 20000, 1152),  # 9 stages per tile
    (36, 4000, 3584),   # 28 stages per tile, few tiles
    (64, 512, 3584),    # 4 tiles: one-stage segments
]


@pytest.mark.parametrize("M,N,K", TWO_ISSUERS)
def test_gemm_two_issuers(cuda, oracle, M, N, K):
    import vvllm_b200 as v

    q, s = oracle.quantize_per_channel(make_weight(N, K, 160 + M))
    x = make_x(M, K, 161)
    b = make_bias(N, 162)
    res = make_x(M, N, 163) if M % 2 else None
    for out16 in (True, False):
        y, xe, re = run_gpu(cuda, x, q, s, b, res, in16=True, out16=out16, algo=v.ALGO_TC)
        assert rowwise_normwise_err(y, oracle_ref(oracle, xe, q, s, b, re)) <= TOL_F16, out16


# Few row tiles on a long K: the GEMM splits every tile into the same number of pieces (28 tiles
# x 5 pieces = 140 CTAs) and the digit GEMV picks its own grid (28 x 4); both against the oracle.
FEW_TILES = [(8, 3584, 9472, "tc"), (64, 3584, 4096, "tc"), (1, 3584, 9472, "tc_i8"), (2, 3584, 9472, "tc_i8")]


@pytest.mark.parametrize("M,N,K,algo_name", FEW_TILES)
def test_few_row_tiles_split_grids(cuda, oracle, M, N, K, algo_name):
    import vvllm_b200 as v

    algo = {"tc": v.ALGO_TC, "tc_i8": v.ALGO_TC_I8}[algo_name]
    q, s = oracle.quantize_per_channel(make_weight(N, K, 170 + M))
    x = make_x(M, K, 171)
    b = make_bias(N, 172)
    y, xe, _ = run_gpu(cuda, x, q, s, b, None, in16=True, out16=True, algo=algo)
    assert rowwise_normwise_err(y, oracle_ref(oracle, xe, q, s, b, None)) <= TOL_F16


PREFILL = [(896, 896), (896, 128), (896, 4864), (4864, 896)]  # benchmark config 4 (K, N) pairs


@pytest.mark.parametrize("K,N", PREFILL)
def test_prefill_config4(cuda, oracle, K, N):
    """M = 512 tokens, fp16 in / fp16 out, int8 per-row weights (config 4); sampled rows checked."""
    import torch

    import vvllm_b200 as v

    M = 512
    w = make_weight(N, K, 500 + N)
    q, s = oracle.quantize_per_channel(w)
    x = make_x(M, K, 501)
    xt = torch.from_numpy(x).to(cuda).half()
    out = torch.empty((M, N), dtype=torch.float16, device=cuda)
    v.linear_q8(out, xt, torch.from_numpy(q).to(cuda), torch.from_numpy(s).to(cuda))
    torch.cuda.synchronize()
    assert v.kernel_error() == 0
    rows = sample_rows(N, 256)
    ref = oracle.linear_q8(xt.float().cpu().numpy(), q[rows], s[rows], None)
    y = out.float().cpu().numpy()[:, rows]
    assert rowwise_normwise_err(y, ref) <= TOL_F16


@pytest.mark.parametrize("in16", [False, True])
@pytest.mark.parametrize("M,N,K", [(1, 896, 896), (1, 896, 4864), (3, 576, 1536), (6, 200, 896)])
def test_linear_add_inplace_and_separate(cuda, oracle, M, N, K, in16):
    w = make_weight(N, K, 11)
    q, s = oracle.quantize_per_channel(w)
    x = make_x(M, K, 12)
    res = make_x(M, N, 13)
    tol = TOL_F16 if in16 else TOL_F32
    for inplace in (True, False):
        y, xe, re = run_gpu(cuda, x, q, s, None, res, in16=in16, out16=in16, inplace=inplace)
        ref = oracle_ref(oracle, xe, q, s, None, re)
        assert rowwise_normwise_err(y, ref) <= tol


@pytest.mark.parametrize("M,N,K", [(1, 7, 17), (2, 5, 33), (1, 1, 1), (3, 64, 100), (1, 31, 48)])
def test_ragged_k_generic_path(cuda, oracle, M, N, K):
    w = make_weight(N, K, 21)
    q, s = oracle.quantize_per_channel(w)
    x = make_x(M, K, 22)
    b = make_bias(N, 23)
    y, xe, _ = run_gpu(cuda, x, q, s, b)
    assert rowwise_normwise_err(y, oracle_ref(oracle, xe, q, s, b, None)) <= TOL_F32


def test_misaligned_pointers(cuda, oracle):
    """Activation/weight views at odd offsets take the generic kernel and stay correct."""
    import torch

    import vvllm_b200 as v

    N, K = 300, 896
    w = make_weight(N, K, 31)
    q, s = oracle.quantize_per_channel(w)
    x = make_x(1, K, 32)
    xb = torch.zeros(K + 3, device=cuda)
    xb[3:] = torch.from_numpy(x[0]).to(cuda)
    qb = torch.zeros(N * K + 5, dtype=torch.int8, device=cuda)
    qb[5:] = torch.from_numpy(q.ravel()).to(cuda)
    out = torch.empty((1, N), device=cuda)
    L = v.lib()
    st = L.b200q8_linear_q8(out.data_ptr(), 0, xb[3:].data_ptr(), 0, qb[5:].data_ptr(),
                            torch.from_numpy(s).to(cuda).data_ptr(), None, 1, N, K, None)
    assert st == 0
    torch.cuda.synchronize()
    ref = oracle.linear_q8(x, q, s, None)
    assert rowwise_normwise_err(out.cpu().numpy(), ref) <= TOL_F32


def test_deterministic(cuda, oracle):
    import torch

    import vvllm_b200 as v

    N, K = 4864, 896
    q, s = oracle.quantize_per_channel(make_weight(N, K, 41))
    xt = torch.from_numpy(make_x(1, K, 42)).to(cuda)
    qt, st = torch.from_numpy(q).to(cuda), torch.from_numpy(s).to(cuda)
    outs = []
    for _ in range(3):
        o = torch.empty((1, N), device=cuda)
        v.linear_q8(o, xt, qt, st)
        outs.append(o)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


def test_empty_and_streams(cuda, oracle):
    import torch

    import vvllm_b200 as v

    q, s = oracle.quantize_per_channel(make_weight(64, 64, 51))
    qt, st = torch.from_numpy(q).to(cuda), torch.from_numpy(s).to(cuda)
    x = torch.randn(0, 64, device=cuda)
    out = torch.empty(0, 64, device=cuda)
    v.linear_q8(out, x, qt, st)  # M = 0: no-op
    side = torch.cuda.Stream()
    x1 = torch.from_numpy(make_x(1, 64, 52)).to(cuda)
    o1 = torch.empty(1, 64, device=cuda)
    side.wait_stream(torch.cuda.current_stream())
    v.linear_q8(o1, x1, qt, st, stream=side)
    side.synchronize()
    ref = oracle.linear_q8(x1.cpu().numpy(), q, s, None)
    assert rowwise_normwise_err(o1.cpu().numpy(), ref) <= TOL_F32


LARGE = [
    # name, N, K, M  -- benchmark config 3 lm_head and config 5 (7B) shapes at full size
    ("qwen05b_lm_head", 151936, 896, 1),
    ("q7b_gate_up", 37888, 3584, 1),
    ("q7b_down", 3584, 18944, 1),
    ("q7b_lm_head", 152064, 3584, 1),
    ("q7b_gate_up_m8", 37888, 3584, 8),
    ("q7b_down_m64", 3584, 18944, 64),
]


@pytest.mark.parametrize("name,N,K,M", LARGE)
def test_full_size_sampled_rows(cuda, oracle, name, N, K, M):
    """Full-size weights made and quantized on the GPU; a row sample is checked on the CPU:
    the GPU quantization of those rows bit-exactly, the fp16 outputs within 2e-3."""
    import torch

    import vvllm_b200 as v

    g = torch.Generator(device=cuda)
    g.manual_seed(zlib.crc32(name.encode()) % 10000)
    w = torch.randn((N, K), generator=g, device=cuda, dtype=torch.float32) * 0.02
    q = torch.empty((N, K), dtype=torch.int8, device=cuda)
    s = torch.empty((N,), dtype=torch.float32, device=cuda)
    v.quantize_per_channel(w, q, s)
    x = torch.randn((M, K), generator=g, device=cuda).half()
    out = torch.empty((M, N), dtype=torch.float16, device=cuda)
    v.linear_q8(out, x, q, s)
    torch.cuda.synchronize()
    rows = torch.from_numpy(sample_rows(N, 384)).to(cuda)
    w_rows = w[rows].cpu().numpy()
    q_rows, s_rows = q[rows].cpu().numpy(), s[rows].cpu().numpy()
    del w
    oq, os_ = oracle.quantize_per_channel(w_rows)
    assert np.array_equal(oq, q_rows)
    assert np.array_equal(os_.view(np.uint32), s_rows.view(np.uint32))
    ref = oracle.linear_q8(x.float().cpu().numpy(), q_rows, s_rows, None)
    y = out[:, rows].float().cpu().numpy()
    assert rowwise_normwise_err(y, ref) <= TOL_F16


@pytest.mark.parametrize("M", [1, 3, 6])
def test_i8_fp16_x_8byte_aligned(cuda, oracle, M):
    """fp16 activations only 8-byte aligned (a view 4 halves into a buffer) on the digit GEMV,
    with the in-kernel exponents (M <= 4) and with the prep kernel (M > 4)."""
    import torch

    import vvllm_b200 as v

    N, K = 640, 896
    q, s = oracle.quantize_per_channel(make_weight(N, K, 61))
    x = make_x(M, K, 62)
    xb = torch.zeros(M * K + 8, dtype=torch.float16, device=cuda)
    xv = xb[4:4 + M * K].view(M, K)
    xv.copy_(torch.from_numpy(x).to(cuda).half())
    assert xv.data_ptr() % 16 == 8
    out = torch.empty((M, N), dtype=torch.float16, device=cuda)
    v.linear_q8_ex(out, xv, torch.from_numpy(q).to(cuda), torch.from_numpy(s).to(cuda), algo=v.ALGO_TC_I8)
    torch.cuda.synchronize()
    assert v.kernel_error() == 0
    ref = oracle.linear_q8(xv.float().cpu().numpy(), q, s, None)
    assert rowwise_normwise_err(out.float().cpu().numpy(), ref) <= TOL_F16
