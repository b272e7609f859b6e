"""GPU quantize_per_channel is bit-identical to the reference's.

Bit-exact means: int8 arrays equal, and fp32 scales equal as bit patterns.
Expected values come from the reference itself (tests/golden/, made by
gen_golden.py from src/quantize/quantize.cc compiled unmodified) or from the
oracle that tests/test_oracle.py pins to it.
"""
import hashlib
import json
import os

import numpy as np
import pytest

from tests._util import make_weight

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def gpu_quantize(cuda, w_np, offset_floats=0):
    import torch

    import vvllm_b200 as v

    N, K = w_np.shape
    buf = torch.zeros(N * K + offset_floats, dtype=torch.float32, device=cuda)
    buf[offset_floats:] = torch.from_numpy(np.ascontiguousarray(w_np).ravel()).to(cuda)
    w = buf[offset_floats:].view(N, K)
    q = torch.full((N, K), 99, dtype=torch.int8, device=cuda)
    s = torch.full((N,), -1.0, dtype=torch.float32, device=cuda)
    v.quantize_per_channel(w, q, s)
    torch.cuda.synchronize()
    return q.cpu().numpy(), s.cpu().numpy()


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_golden_edges(cuda):
    g = np.load(os.path.join(GOLD, "quantize_edge.npz"))
    for suffix in ("", "_ragged", "_long"):
        q, s = gpu_quantize(cuda, g["w" + suffix])
        assert np.array_equal(q, g["q" + suffix]), suffix
        assert np.array_equal(_bits(s), _bits(g["s" + suffix])), suffix


def test_known_answers(cuda):
    with open(os.path.join(GOLD, "known_answers.json")) as f:
        ka = json.load(f)
    for name in ("roundtrip", "zero_row", "saturation"):
        q, s = gpu_quantize(cuda, np.array(ka[name]["w"], np.float32))
        assert q.tolist() == ka[name]["q"]
        assert [f"{v:08x}" for v in _bits(s).tolist()] == ka[name]["scales_hex"]


@pytest.mark.parametrize("N,K", [(64, 576), (33, 896), (17, 1536), (9, 3584), (8, 4864),
                                 (5, 18944), (3, 20480), (2, 20484), (13, 37), (4, 1), (1, 4096)])
@pytest.mark.parametrize("offset", [0, 1])
def test_random_bitexact(cuda, oracle, N, K, offset):
    w = make_weight(N, K, N * 7 + K)
    w[0, 0] = 0.0
    if N > 2:
        w[1, :] = 0.0           # zero row
        w[2, K // 2] = np.float32(-3.0)  # dominant negative
    q, s = gpu_quantize(cuda, w, offset)
    oq, os_ = oracle.quantize_per_channel(w)
    assert np.array_equal(q, oq)
    assert np.array_equal(_bits(s), _bits(os_))


@pytest.mark.parametrize("name", ["config1_4864x896", "qwen05b_gate_4864x896", "qwen05b_down_896x4864",
                                  "qwen05b_k_128x896", "smol_lm_head_49152x576",
                                  "qwen05b_lm_head_151936x896", "qwen7b_down_3584x18944"])
def test_full_size_reference_digests(cuda, name):
    """Full benchmark-size matrices: SHA-256 of the GPU output equals that of the reference's."""
    with open(os.path.join(GOLD, "digests.json")) as f:
        d = json.load(f)
    if d["numpy"] != np.__version__:
        pytest.skip(f"digests made with numpy {d['numpy']}, have {np.__version__}")
    c = d["cases"][name]
    w = make_weight(c["N"], c["K"], c["w_seed"])
    q, s = gpu_quantize(cuda, w)
    assert hashlib.sha256(q.tobytes()).hexdigest() == c["q_sha256"]
    assert hashlib.sha256(s.tobytes()).hexdigest() == c["scales_sha256"]
