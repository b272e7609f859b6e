"""b200q8_linear_q8_noalloc: the allocation-free entry point.

Some callers may not call cudaMalloc -- their device memory belongs to a pool
or budget nothing may bypass, or their decode loop cannot take the device-wide
synchronisation cudaMalloc/cudaFree may cause.  For them the library offers one
entry point whose scratch is a fixed device array.  This file checks, through
the C ABI, that it gives the same results as the regular entry point
(b200q8_linear_q8_ex) and as the CPU oracle (the reference's linear_q8 /
linear_q8_add on the same inputs), within the tolerances every other test
uses, on two calls in a row (the second call reuses the array the first one
left behind), and that shapes beyond the array's limits are refused.

It is named to be collected last, so a run that stops at the first failure has
run every other test before this one; it also passes alone in a fresh process.
"""
import numpy as np
import pytest

from tests._util import TOL_F16, TOL_F32, make_bias, make_weight, make_x, rowwise_normwise_err

pytestmark = pytest.mark.gpu


def _noalloc(out, x, w, s, b, res, stream):
    from vvllm_b200 import _lib

    M, K = x.shape
    N = w.shape[0]
    return _lib.lib().b200q8_linear_q8_noalloc(
        out.data_ptr(), _lib._dtype_code(out), x.data_ptr(), _lib._dtype_code(x), w.data_ptr(), s.data_ptr(),
        None if b is None else b.data_ptr(), None if res is None else res.data_ptr(), M, N, K, stream)


CASES = [
    # M, N, K, fp16 activations, bias, residual
    (1, 4864, 896, True, True, False),     # benchmark config 1 shape, decode
    (1, 448, 18944, True, False, True),    # 7B down-proj shard: every tile split (stream-K fixup)
    (2, 1000, 3584, False, True, True),    # fp32 activations, two tokens
    (1, 152064, 896, True, False, False),  # Qwen-0.5B lm_head width
]


@pytest.mark.parametrize("M,N,K,in16,has_b,has_r", CASES)
def test_noalloc_matches_regular_entry_two_calls(cuda, oracle, M, N, K, in16, has_b, has_r):
    import torch

    import vvllm_b200 as v

    act = torch.float16 if in16 else torch.float32
    tol = TOL_F16 if in16 else TOL_F32
    q, s = oracle.quantize_per_channel(make_weight(N, K, 700 + N % 97))
    qt, st = torch.from_numpy(q).to(cuda), torch.from_numpy(s).to(cuda)
    bt = torch.from_numpy(make_bias(N, 701)).to(cuda) if has_b else None
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # two calls in a row on the shared array
        x = torch.from_numpy(make_x(M, K, 710 + call)).to(cuda).to(act)
        res = torch.from_numpy(make_x(M, N, 720 + call)).to(cuda).to(act) if has_r else None
        got = torch.full((M, N), float("nan"), dtype=act, device=cuda)
        want = torch.empty((M, N), dtype=act, device=cuda)
        assert _noalloc(got, x, qt, st, bt, res, stream) == 0, v.lib().b200q8_last_error()
        v.linear_q8_ex(want, x, qt, st, bt, res)
        torch.cuda.synchronize()
        assert v.kernel_error() == 0
        y = got.float().cpu().numpy()
        err = rowwise_normwise_err(y, want.float().cpu().numpy())
        assert err <= tol, (call, err)
        # and against the oracle on the same (widened) inputs
        xf = x.float().cpu().numpy()
        b = bt.cpu().numpy() if has_b else None
        if has_r:
            ref = oracle.linear_q8_add(xf, q, s, b, np.ascontiguousarray(res.float().cpu().numpy()))
        else:
            ref = oracle.linear_q8(xf, q, s, b)
        err = rowwise_normwise_err(y, ref)
        assert err <= tol, (call, "oracle", err)


def test_noalloc_rejects_shapes_beyond_its_array(cuda):
    import torch

    import vvllm_b200 as v

    K = 896
    w = torch.zeros((8, K), dtype=torch.int8, device=cuda)
    s = torch.ones(8, device=cuda)
    x = torch.zeros((3, K), dtype=torch.float16, device=cuda)  # 3 tokens: over the 2-token limit
    out = torch.zeros((3, 8), dtype=torch.float16, device=cuda)
    st = _noalloc(out, x, w, s, None, None, None)
    assert st == -3  # B200Q8_ERR_UNSUPPORTED
    assert b"tokens" in v.lib().b200q8_last_error()
    x1 = torch.zeros((1, 24), dtype=torch.float16, device=cuda)  # K % 16 != 0
    w1 = torch.zeros((8, 24), dtype=torch.int8, device=cuda)
    out1 = torch.zeros((1, 8), dtype=torch.float16, device=cuda)
    assert _noalloc(out1, x1, w1, s, None, None, None) == -3
