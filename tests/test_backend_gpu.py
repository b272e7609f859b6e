"""The Backend-shaped layer (host weight pointers cached on the device) on the GPU.

Mirrors how vvllm's transformer_forward calls Backend::linear_q8 / linear_q8_add
(include/vvllm/model/transformer.h:139-188): device activations, host int8
weights and scales owned by the model, o_proj/down_proj in place (out ==
residual), fp16 activations behind float* when the backend is in fp16 mode.
"""
import numpy as np
import pytest

from tests._util import TOL_F16, TOL_F32, make_bias, make_weight, make_x, rowwise_normwise_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fp16", [False, True])
def test_backend_layer_sequence(cuda, oracle, fp16):
    import torch

    import vvllm_b200 as v

    H, I, M = 896, 4864, 2
    act = torch.float16 if fp16 else torch.float32
    tol = TOL_F16 if fp16 else TOL_F32
    be = v.Backend(0, fp16=fp16)
    qkv_w = make_weight(H, H, 1)
    q_q, q_s = oracle.quantize_per_channel(qkv_w)
    q_b = make_bias(H, 2)
    down_q, down_s = oracle.quantize_per_channel(make_weight(H, I, 3))

    x = torch.from_numpy(make_x(M, H, 4)).to(cuda).to(act)
    out = torch.empty((M, H), dtype=act, device=cuda)
    be.linear_q8(out, x, q_q, q_s, q_b, M, H, H)
    torch.cuda.synchronize()
    ref = oracle.linear_q8(x.float().cpu().numpy(), q_q, q_s, q_b)
    assert rowwise_normwise_err(out.float().cpu().numpy(), ref) <= tol
    cached = be.cached_bytes()
    assert cached == H * H + 4 * H + 4 * H

    # second call with the same host pointers: no new upload
    be.linear_q8(out, x, q_q, q_s, q_b, M, H, H)
    assert be.cached_bytes() == cached

    # down_proj in place: x_res = x_res + down(gate)
    gate = torch.from_numpy(make_x(M, I, 5)).to(cuda).to(act)
    resid = torch.from_numpy(make_x(M, H, 6)).to(cuda).to(act)
    res_before = resid.float().cpu().numpy()
    be.linear_q8_add(resid, gate, down_q, down_s, None, resid, M, H, I)
    torch.cuda.synchronize()
    ref = oracle.linear_q8_add(gate.float().cpu().numpy(), down_q, down_s, None, res_before)
    assert rowwise_normwise_err(resid.float().cpu().numpy(), ref) <= tol
    be.close()


def test_backend_quantize_host_io(cuda, oracle):
    import vvllm_b200 as v

    be = v.Backend(0)
    w = make_weight(257, 896, 9)
    w[3] = 0.0
    q, s = be.quantize_per_channel(w)
    oq, os_ = oracle.quantize_per_channel(w)
    assert np.array_equal(q, oq)
    assert np.array_equal(s.view(np.uint32), os_.view(np.uint32))
    be.close()


def test_backend_rejects_bad_args(cuda):
    import vvllm_b200 as v

    be = v.Backend(0)
    w = np.zeros((4, 16), np.int8)
    s = np.ones(4, np.float32)
    with pytest.raises(v.B200Q8Error):
        be.linear_q8_add(0, 0, w, s, None, None, 1, 4, 16)  # null residual
    be.close()
