"""Projections with the elementwise op before them fused in (rms_norm -> linear_q8,
silu_mul -> linear_q8_add) and the standalone ops.

vvllm runs rms_norm per token before q/k/v and gate_up (include/vvllm/model/transformer.h:
135-144, :167-169) and silu_mul before down (:171-188).  Checked here:

* the fused call equals the standalone op followed by the plain projection bit for bit, on
  every path the dispatcher takes (the SIMT GEMV applying it while staging x; the digit GEMV's
  prep kernel, also in 42-token groups; the standalone kernel + fp16 GEMM for prefill);
* the standalone ops against the CPU oracle's restatement of BackendCPU::rms_norm / silu_mul
  (pinned bit for bit to the reference by tests/test_oracle.py);
* the fused call against the oracle chain (oracle op -> oracle linear_q8) within the path's
  tolerance, fp16 mode following the reference fp16 backend (norm weight and result rounded
  to fp16, src/backend/backend_cuda.cc:135-145, cuda_kernels.cu:876-910).
"""
import numpy as np
import pytest

from tests._util import TOL_F16, TOL_F32, make_bias, make_weight, make_x, rowwise_normwise_err

pytestmark = pytest.mark.gpu

EPS = 1e-6


def _h(a):
    """Round to fp16 and back (fp16 mode semantics on the host)."""
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def _same(a, b):
    a = a.float().cpu().numpy() if hasattr(a, "cpu") else a
    b = b.float().cpu().numpy() if hasattr(b, "cpu") else b
    return np.array_equal(a.view(np.uint32), b.view(np.uint32)) or np.array_equal(a, b, equal_nan=True)


# (M, N, K, in16, out16): few tokens on small weights (SIMT), on weights over 48 MiB or more
# tokens (digit GEMV + prep kernel), fp32 42-token groups, fp16 prefill on the GEMM
RN_CASES = [
    (1, 4864, 896, True, True),
    (1, 896, 896, False, False),
    (1, 16384, 3584, True, True),   # weights > 48 MiB: the prep kernel writes the activations
    (4, 1152, 3584, False, True),
    (5, 640, 896, False, False),
    (9, 4864, 896, True, True),
    (50, 384, 896, False, False),
    (20, 1024, 896, True, True),
    (128, 4864, 896, True, False),
]


@pytest.mark.parametrize("M,N,K,in16,out16", RN_CASES)
def test_rms_norm_linear(cuda, oracle, M, N, K, in16, out16):
    import torch

    import vvllm_b200 as v

    q, s = oracle.quantize_per_channel(make_weight(N, K, 700 + M))
    b = make_bias(N, 701)
    x = make_x(M, K, 702 + M) * np.float32(4)
    g = (1 + 0.2 * make_x(1, K, 703)[0]).astype(np.float32)
    idt = torch.float16 if in16 else torch.float32
    odt = torch.float16 if out16 else torch.float32
    xt = torch.from_numpy(x).to(cuda).to(idt)
    qt, st, bt, gt = (torch.from_numpy(a).to(cuda) for a in (q, s, b, g))
    fused = torch.empty((M, N), dtype=odt, device=cuda)
    v.rms_norm_linear_q8(fused, xt, gt, EPS, qt, st, bt)
    normed = torch.empty((M, K), dtype=idt, device=cuda)
    v.rms_norm(normed, xt, gt, EPS)
    plain = torch.empty((M, N), dtype=odt, device=cuda)
    v.linear_q8(plain, normed, qt, st, bt)
    torch.cuda.synchronize()
    assert v.kernel_error() == 0
    assert _same(fused, plain)
    # standalone op vs the oracle
    xf = xt.float().cpu().numpy()
    ref_n = oracle.rms_norm(xf, _h(g) if in16 else g, EPS)
    if in16:
        ref_n = _h(ref_n)
    assert rowwise_normwise_err(normed.float().cpu().numpy(), ref_n) <= (TOL_F16 if in16 else 2e-6)
    # fused vs the oracle chain
    ref = oracle.linear_q8(ref_n, q, s, b)
    tol = TOL_F16 if (in16 or out16) else TOL_F32
    assert rowwise_normwise_err(fused.float().cpu().numpy(), ref) <= tol


# (M, N, K, in16, out16, inplace): K = 4864 / 18944 are down-projection widths (> 4096: prep kernel)
SM_CASES = [
    (1, 896, 4864, True, True, True),
    (1, 3584, 18944, False, False, True),
    (3, 896, 1024, False, False, False),
    (1, 14336, 4096, True, False, False),   # weights > 48 MiB with few tokens: prep kernel path
    (2, 512, 4096, True, False, False),
    (45, 256, 1024, False, False, True),
    (64, 896, 4864, True, True, True),
]


@pytest.mark.parametrize("M,N,K,in16,out16,inplace", SM_CASES)
def test_silu_mul_linear_add(cuda, oracle, M, N, K, in16, out16, inplace):
    import torch

    import vvllm_b200 as v

    q, s = oracle.quantize_per_channel(make_weight(N, K, 800 + M))
    gu = make_x(M, 2 * K, 801 + M) * np.float32(2)
    r = make_x(M, N, 802 + M)
    idt = torch.float16 if in16 else torch.float32
    odt = torch.float16 if out16 else torch.float32
    gut = torch.from_numpy(gu).to(cuda).to(idt)
    qt, st = torch.from_numpy(q).to(cuda), torch.from_numpy(s).to(cuda)
    rt = torch.from_numpy(r).to(cuda).to(odt)
    fused = rt.clone() if inplace else torch.empty((M, N), dtype=odt, device=cuda)
    v.silu_mul_linear_q8_add(fused, gut, qt, st, None, fused if inplace else rt)
    h = torch.empty((M, K), dtype=idt, device=cuda)
    v.silu_mul(h, gut)
    plain = torch.empty((M, N), dtype=odt, device=cuda)
    v.linear_q8_add(plain, h, qt, st, None, rt)
    torch.cuda.synchronize()
    assert v.kernel_error() == 0
    assert _same(fused, plain)
    guf = gut.float().cpu().numpy()
    ref_h = oracle.silu_mul(guf)
    if in16:
        ref_h = _h(ref_h)
    assert rowwise_normwise_err(h.float().cpu().numpy(), ref_h) <= (TOL_F16 if in16 else 2e-6)
    ref = oracle.linear_q8_add(ref_h, q, s, None, rt.float().cpu().numpy())
    tol = TOL_F16 if (in16 or out16) else TOL_F32
    assert rowwise_normwise_err(fused.float().cpu().numpy(), ref) <= tol


def test_silu_mul_no_residual(cuda, oracle):
    import torch

    import vvllm_b200 as v

    M, N, K = 1, 640, 896
    q, s = oracle.quantize_per_channel(make_weight(N, K, 901))
    gu = make_x(M, 2 * K, 902)
    gut = torch.from_numpy(gu).to(cuda)
    qt, st = torch.from_numpy(q).to(cuda), torch.from_numpy(s).to(cuda)
    out = torch.empty((M, N), device=cuda)
    v.silu_mul_linear_q8_add(out, gut, qt, st)
    torch.cuda.synchronize()
    ref = oracle.linear_q8(oracle.silu_mul(gu), q, s, None)
    assert rowwise_normwise_err(out.cpu().numpy(), ref) <= TOL_F32


@pytest.mark.parametrize("in16", [False, True])
def test_prologue_edge_rows(cuda, oracle, in16):
    """Zero row (rms = sqrt(eps)), a NaN row and an overflowing row give the same results fused and
    unfused; a NaN / Inf activation row yields non-finite outputs for its token."""
    import torch

    import vvllm_b200 as v

    M, N, K = 4, 512, 896
    q, s = oracle.quantize_per_channel(make_weight(N, K, 911))
    x = make_x(M, K, 912)
    x[0] = 0.0
    x[1, 3] = np.nan
    x[3, 10] = 6e4 if in16 else 1e30
    g = np.ones(K, np.float32)
    idt = torch.float16 if in16 else torch.float32
    xt = torch.from_numpy(x).to(cuda).to(idt)
    qt, st, gt = (torch.from_numpy(a).to(cuda) for a in (q, s, g))
    fused = torch.empty((M, N), device=cuda)
    v.rms_norm_linear_q8(fused, xt, gt, EPS, qt, st)
    normed = torch.empty((M, K), dtype=idt, device=cuda)
    v.rms_norm(normed, xt, gt, EPS)
    plain = torch.empty((M, N), device=cuda)
    v.linear_q8(plain, normed, qt, st)
    torch.cuda.synchronize()
    assert v.kernel_error() == 0
    assert _same(fused, plain)
    y = fused.cpu().numpy()
    assert not y[0].any()                  # zero row -> zero activations -> zero outputs
    assert np.isnan(y[1]).all()            # NaN row
    assert np.isfinite(y[2]).all() and np.isfinite(y[3]).all()
    # silu_mul: gate values that overflow exp and an fp16 product that overflows to Inf
    gu = make_x(2, 2 * K, 913)
    gu[0, :4] = [-100.0, 100.0, -88.0, 88.0]
    if in16:
        gu[1, 7], gu[1, K + 7] = 300.0, 300.0   # 300 * 300 > 65504: fp16 Inf -> NaN row
    gut = torch.from_numpy(gu).to(cuda).to(idt)
    fused2 = torch.empty((2, N), device=cuda)
    v.silu_mul_linear_q8_add(fused2, gut, qt, st)
    h = torch.empty((2, K), dtype=idt, device=cuda)
    v.silu_mul(h, gut)
    plain2 = torch.empty((2, N), device=cuda)
    v.linear_q8(plain2, h, qt, st)
    torch.cuda.synchronize()
    assert _same(fused2, plain2)
    y2 = fused2.cpu().numpy()
    assert np.isfinite(y2[0]).all()
    # an Inf activation makes every output of its token non-finite: NaN on the digit GEMV,
    # +-Inf (NaN where it meets a zero weight) on the SIMT GEMV, which takes this small shape
    assert (~np.isfinite(y2[1])).all() == in16


def test_prologue_rejects_bad_shapes(cuda):
    import torch

    import vvllm_b200 as v

    x = torch.zeros((1, 18), device=cuda)
    g = torch.ones(18, device=cuda)
    w = torch.zeros((8, 18), dtype=torch.int8, device=cuda)
    s = torch.ones(8, device=cuda)
    out = torch.empty((1, 8), device=cuda)
    with pytest.raises(v.B200Q8Error):
        v.rms_norm_linear_q8(out, x, g, EPS, w, s)  # K % 4 != 0
    with pytest.raises(ValueError):
        v.silu_mul_linear_q8_add(out, torch.zeros((1, 20), device=cuda), w, s)  # gate_up not [M, 2K]
