"""Grouped projections of one activation: b200q8_linear_q8_group.

vvllm's attention block normalizes x once and runs q, k and v on the result
(include/vvllm/model/transformer.h:134-144).  The group call does that in one launch for few
tokens (x staged and normalized once per CTA, the projections' row groups numbered one matrix
after another), and one projection at a time otherwise.  Checked here:

* every output against the CPU oracle chain (oracle rms_norm -> oracle linear_q8) within the
  path's tolerance, on Qwen2.5-0.5B and -7B q/k/v shapes, with and without the norm and bias;
* every output against the single-projection call on the same inputs (same tolerance: the
  group launch may split K differently, so the summation order can differ);
* the one-at-a-time route (more tokens, K % 16 != 0, weights over 48 MiB), skipped projections
  (N = 0) and argument errors.
"""
import numpy as np
import pytest

from tests._util import TOL_F16, TOL_F32, make_bias, make_weight, make_x, rowwise_normwise_err

pytestmark = pytest.mark.gpu

EPS = 1e-6


def _h(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def _setup(cuda, oracle, Ns, K, seed, with_bias):
    import torch

    qs, ss, bs, ws = [], [], [], []
    for i, N in enumerate(Ns):
        q, s = oracle.quantize_per_channel(make_weight(max(N, 1), K, seed + i))
        q, s = q[:N], s[:N]
        b = make_bias(N, seed + 10 + i) if (with_bias and i != 1) else None  # projection 1 without bias
        ws.append((q, s, b))
        qs.append(torch.from_numpy(np.ascontiguousarray(q)).to(cuda))
        ss.append(torch.from_numpy(np.ascontiguousarray(s)).to(cuda))
        bs.append(torch.from_numpy(b).to(cuda) if b is not None else None)
    return ws, qs, ss, bs


# (M, Ns, K, in16, out16, norm, bias)
CASES = [
    (1, (896, 128, 128), 896, False, False, True, True),      # Qwen2.5-0.5B q/k/v
    (1, (896, 128, 128), 896, True, True, True, True),
    (2, (896, 128, 128), 896, True, False, False, True),
    (3, (3584, 512, 512), 3584, False, True, True, True),     # Qwen2.5-7B q/k/v
    (4, (3584, 512, 512), 3584, True, True, True, False),
    (1, (3584, 512, 512), 3584, True, True, True, True),
    (1, (4864, 4864), 896, True, True, True, False),          # gate / up as two matrices
    (1, (100, 36, 7, 1), 256, False, False, True, True),      # ragged row counts, four matrices
    (8, (896, 128, 128), 896, True, True, True, True),        # more tokens: one at a time
    (20, (896, 128, 128), 896, False, False, True, True),
    (1, (896, 128), 200, False, False, False, True),          # K % 16 != 0: one at a time
    (1, (256, 0, 128), 512, False, False, True, True),        # a skipped projection
]


@pytest.mark.parametrize("M,Ns,K,in16,out16,norm,bias", CASES)
def test_group(cuda, oracle, M, Ns, K, in16, out16, norm, bias):
    import torch

    import vvllm_b200 as v

    ws, qs, ss, bs = _setup(cuda, oracle, Ns, K, 900 + M + K, bias)
    idt = torch.float16 if in16 else torch.float32
    odt = torch.float16 if out16 else torch.float32
    x = make_x(M, K, 950 + M) * np.float32(3)
    xt = torch.from_numpy(x).to(cuda).to(idt)
    g = (1 + 0.2 * make_x(1, K, 951)[0]).astype(np.float32)
    gt = torch.from_numpy(g).to(cuda) if norm else None
    outs = [torch.full((M, N), float("nan"), dtype=odt, device=cuda) for N in Ns]
    v.linear_q8_group(outs, xt, qs, ss, bs if bias else None, gt, EPS)
    singles = []
    for i, N in enumerate(Ns):
        o = torch.empty((M, N), dtype=odt, device=cuda)
        if N:
            if norm:
                v.rms_norm_linear_q8(o, xt, gt, EPS, qs[i], ss[i], bs[i] if bias else None)
            else:
                v.linear_q8(o, xt, qs[i], ss[i], bs[i] if bias else None)
        singles.append(o)
    torch.cuda.synchronize()
    assert v.kernel_error() == 0
    xf = xt.float().cpu().numpy()
    if norm:
        act = oracle.rms_norm(xf, _h(g) if in16 else g, EPS)
        if in16:
            act = _h(act)
    else:
        act = xf
    tol = TOL_F16 if (in16 or out16) else TOL_F32
    for i, N in enumerate(Ns):
        if N == 0:
            continue
        q, s, b = ws[i]
        ref = oracle.linear_q8(act, q, s, b if bias else None)
        got = outs[i].float().cpu().numpy()
        assert np.isfinite(got).all(), f"projection {i}: rows left unwritten"
        assert rowwise_normwise_err(got, ref) <= tol, f"projection {i}"
        assert rowwise_normwise_err(got, singles[i].float().cpu().numpy()) <= tol, f"projection {i} vs single"


def test_group_large_weights_one_at_a_time(cuda, oracle):
    """More than 48 MiB of weights with one token: each projection through the ordinary dispatch."""
    import torch

    import vvllm_b200 as v

    K, Ns = 3584, (9472, 9472)  # 2 x 34 MB
    ws, qs, ss, _ = _setup(cuda, oracle, Ns, K, 990, False)
    xt = torch.from_numpy(make_x(1, K, 991)).to(cuda).half()
    outs = [torch.empty((1, N), dtype=torch.float16, device=cuda) for N in Ns]
    v.linear_q8_group(outs, xt, qs, ss)
    torch.cuda.synchronize()
    assert v.kernel_error() == 0
    for i in range(2):
        ref = oracle.linear_q8(xt.float().cpu().numpy(), ws[i][0], ws[i][1], None)
        assert rowwise_normwise_err(outs[i].float().cpu().numpy(), ref) <= TOL_F16


def test_group_errors(cuda, oracle):
    import torch

    import vvllm_b200 as v

    K = 256
    _, qs, ss, _ = _setup(cuda, oracle, (64, 64, 64, 64, 64), K, 995, False)
    xt = torch.zeros((1, K), device=cuda)
    outs = [torch.empty((1, 64), device=cuda) for _ in range(5)]
    with pytest.raises(v.B200Q8Error) as e:  # more than B200Q8_MAX_GROUP projections
        v.linear_q8_group(outs, xt, qs, ss)
    assert e.value.status == -1
    with pytest.raises(v.B200Q8Error) as e:  # two outputs in the same memory
        v.linear_q8_group([outs[0], outs[0]], xt, qs[:2], ss[:2])
    assert e.value.status == -1
    with pytest.raises(v.B200Q8Error) as e:  # misaligned norm weight
        g = torch.ones(K + 1, device=cuda)
        v.linear_q8_group(outs[:2], xt, qs[:2], ss[:2], None, g[1:], EPS)
    assert e.value.status == -3
