"""Quantized lm_head with the greedy argmax fused into the int8 GEMV (b200q8_linear_q8_argmax).

The argmax follows the reference CPU sampler (SamplerCPU::sample, temperature 0:
std::max_element over the logits, src/sampler/sampler.cc:20-24): first maximum wins, NaNs are
skipped unless the first logit is NaN.  It is checked exactly against that rule applied to the
kernel's own logits (as stored), with and without writing the logits, across decode and
stream-K split-tile shapes, ties and NaN rows; the logits themselves are checked against the
CPU oracle like every linear_q8 output.
"""
import numpy as np
import pytest

from tests._util import TOL_F16, TOL_F32, make_weight, make_x, rowwise_normwise_err

pytestmark = pytest.mark.gpu


def max_element(row):
    """std::max_element's index: largest <, first wins; a NaN never replaces the current best."""
    best = 0
    for i in range(1, row.shape[0]):
        if row[best] < row[i]:
            best = i
    return best


def first_max(row):
    """Vectorised max_element for rows whose first entry is not NaN."""
    finite = np.where(np.isnan(row), -np.inf, row)
    return int(np.argmax(finite)) if not np.isnan(row[0]) else 0


@pytest.mark.parametrize("M,N,K,in16,out16", [
    (1, 151936, 896, True, True),     # Qwen2.5-0.5B tied lm_head shape, decode
    (1, 49152, 576, False, False),    # SmolLM lm_head, fp32 activations
    (3, 20000, 896, True, False),     # several tokens
    (1, 300, 18944, True, True),      # long K: every tile split over many stream-K pieces
    (8, 30000, 3584, True, True),     # eight fp16 tokens: digit tiles made by the prep kernel
])
def test_argmax_matches_logits(cuda, oracle, M, N, K, in16, out16):
    import torch

    import vvllm_b200 as v

    q, s = oracle.quantize_per_channel(make_weight(N, K, 1000 + N % 997))
    x = make_x(M, K, 1001)
    xt = torch.from_numpy(x).to(cuda)
    xt = xt.half() if in16 else xt
    qt, st = torch.from_numpy(q).to(cuda), torch.from_numpy(s).to(cuda)
    odt = torch.float16 if out16 else torch.float32
    out = torch.empty((M, N), dtype=odt, device=cuda)
    am = torch.full((M,), -1, dtype=torch.int32, device=cuda)
    am2 = torch.full((M,), -1, dtype=torch.int32, device=cuda)
    for _ in range(2):  # the scratch must be left clean for the next call
        v.linear_q8_argmax(out, xt, qt, st, None, am)
        v.linear_q8_argmax(None, xt, qt, st, None, am2, out_dtype=v.F16 if out16 else v.F32)
    torch.cuda.synchronize()
    assert v.kernel_error() == 0
    y = out.float().cpu().numpy()
    for m in range(M):
        assert int(am[m]) == first_max(y[m]), m
        assert int(am2[m]) == int(am[m]), m
    ref = oracle.linear_q8(xt.float().cpu().numpy(), q, s, None)
    assert rowwise_normwise_err(y, ref) <= (TOL_F16 if (in16 or out16) else TOL_F32)


def test_argmax_ties_and_nan(cuda, oracle):
    import torch

    import vvllm_b200 as v

    N, K = 4096, 896
    q, s = oracle.quantize_per_channel(make_weight(N, K, 77))
    x = make_x(2, K, 78)
    # rows 3000 and 1234 identical to row 3500: equal logits; whichever is largest, the smallest
    # index of a tie must win
    for j in (1234, 3000):
        q[j] = q[3500]
        s[j] = s[3500]
    x[1, 17] = np.nan  # token 1: every logit NaN -> max_element keeps index 0
    qt, st = torch.from_numpy(q).to(cuda), torch.from_numpy(s).to(cuda)
    xt = torch.from_numpy(x).to(cuda)
    out = torch.empty((2, N), device=cuda)
    am = torch.full((2,), -1, dtype=torch.int32, device=cuda)
    v.linear_q8_argmax(out, xt, qt, st, None, am)
    torch.cuda.synchronize()
    assert v.kernel_error() == 0
    y = out.cpu().numpy()
    assert int(am[0]) == max_element(y[0])
    assert np.isnan(y[1]).all() and int(am[1]) == 0
    # force the tie to be the maximum: scale the tied rows up
    s2 = s.copy()
    for j in (1234, 3000, 3500):
        s2[j] = s[3500] * 50.0
    st2 = torch.from_numpy(s2).to(cuda)
    xt0 = xt[:1].contiguous()
    out0 = torch.empty((1, N), device=cuda)
    am0 = torch.full((1,), -1, dtype=torch.int32, device=cuda)
    v.linear_q8_argmax(out0, xt0, qt, st2, None, am0)
    torch.cuda.synchronize()
    y0 = out0.cpu().numpy()[0]
    if y0[1234] == y0.max():
        assert int(am0[0]) == 1234
    assert int(am0[0]) == max_element(y0)
