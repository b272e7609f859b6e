"""Load-time quantization: the bf16 quantize kernel and the quantized safetensors converter.

vvllm widens BF16 checkpoint tensors to fp32 on the host (SafeTensorsLoader::bf16_to_f32,
src/safetensors/safetensors.cc:131-137) and quantizes every projection at load
(src/model/qwen2/model.cc:27-38).  Checked here, bit for bit against the CPU oracle (itself
pinned to the reference's quantize_per_channel): the GPU quantize straight from bf16 bits, and
every quantized pair b200q8_st_quantize writes; all other tensors must come through byte for
byte, and the file must parse with an independent reader."""
import numpy as np
import pytest

from tests import st_util
from tests._util import make_weight

pytestmark = pytest.mark.gpu


def _edge_rows(K, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((8, K)) * 0.02).astype(np.float32)
    w[1] = 0.0                                   # zero row: scale 0, all q 0
    w[2, 3] = np.nan                             # NaN never wins the absmax
    w[3, 5] = np.inf                             # Inf absmax: scale inf, inv 0
    w[4] = np.float32(1e-39) * (1 + np.arange(K) % 5)   # subnormals (exact in bf16's range)
    w[5, :8] = [127.0, -63.5, 0.5, -0.5, 1.5, 2.5, -127.0, 64.0]  # ties under round-half-away
    w[6, 7] = -0.0
    return w


@pytest.mark.parametrize("N,K", [(64, 896), (37, 4864), (5, 18944), (3, 20484), (7, 17), (130, 1000)])
def test_quantize_bf16_bit_exact(cuda, oracle, N, K):
    import torch

    import vvllm_b200 as v

    w = make_weight(N, K, 300 + K % 97)
    if N >= 8:
        w[:8] = _edge_rows(K, 301)
    bits = st_util.bf16_bits(w)
    ref_q, ref_s = oracle.quantize_per_channel(st_util.bf16_widen(bits))
    wt = torch.from_numpy(bits.view(np.int16)).to(cuda)
    q = torch.empty((N, K), dtype=torch.int8, device=cuda)
    s = torch.empty(N, dtype=torch.float32, device=cuda)
    v.quantize_per_channel_bf16(wt, q, s)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), ref_q)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), ref_s.view(np.uint32))


def test_quantize_bf16_misaligned_takes_generic_path(cuda, oracle):
    import torch

    import vvllm_b200 as v

    N, K = 9, 896
    bits = st_util.bf16_bits(make_weight(N, K, 310))
    buf = torch.zeros(N * K + 1, dtype=torch.int16, device=cuda)
    buf[1:] = torch.from_numpy(bits.view(np.int16).ravel()).to(cuda)
    wt = buf[1:].view(N, K)  # 2-byte aligned only
    q = torch.empty((N, K), dtype=torch.int8, device=cuda)
    s = torch.empty(N, dtype=torch.float32, device=cuda)
    v.quantize_per_channel_bf16(wt, q, s)
    torch.cuda.synchronize()
    ref_q, ref_s = oracle.quantize_per_channel(st_util.bf16_widen(bits))
    assert np.array_equal(q.cpu().numpy(), ref_q) and np.array_equal(s.cpu().numpy(), ref_s)


def _checkpoint(dtype: str, tied: bool, seed: int = 5):
    """A two-layer Qwen2-shaped checkpoint (hidden 128, 4 heads, 2 kv heads, intermediate 384,
    vocab 1000), tensor names as vvllm's loader expects them (model.cc:17-80)."""
    H, I, KV, V = 128, 384, 64, 1000
    rng = np.random.default_rng(seed)

    def w(n, k):
        a = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        return ("BF16", st_util.bf16_bits(a)) if dtype == "BF16" else ("F32", a)

    t = {"model.embed_tokens.weight": w(V, H), "model.norm.weight": ("F32", np.ones(H, np.float32))}
    for i in range(2):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"] = ("F32", (1 + 0.1 * rng.standard_normal(H)).astype(np.float32))
        t[p + "post_attention_layernorm.weight"] = ("F32", np.ones(H, np.float32))
        t[p + "self_attn.q_proj.weight"] = w(H, H)
        t[p + "self_attn.q_proj.bias"] = ("F32", rng.standard_normal(H).astype(np.float32))
        t[p + "self_attn.k_proj.weight"] = w(KV, H)
        t[p + "self_attn.k_proj.bias"] = ("F32", rng.standard_normal(KV).astype(np.float32))
        t[p + "self_attn.v_proj.weight"] = w(KV, H)
        t[p + "self_attn.v_proj.bias"] = ("F32", rng.standard_normal(KV).astype(np.float32))
        t[p + "self_attn.o_proj.weight"] = w(H, H)
        t[p + "mlp.gate_proj.weight"] = w(I, H)
        t[p + "mlp.up_proj.weight"] = w(I, H)
        t[p + "mlp.down_proj.weight"] = w(H, I)
    if not tied:
        t["lm_head.weight"] = w(V, H)
    t["model.layers.1.mlp.down_proj.weight"][1][3, :] = 0.0  # a zero row survives the round trip
    return t


def _as_f32(dt, arr):
    return st_util.bf16_widen(arr) if dt == "BF16" else arr


@pytest.mark.parametrize("dtype", ["BF16", "F32"])
@pytest.mark.parametrize("tied,lm_head", [(True, False), (True, True), (False, True)])
def test_st_quantize_checkpoint(cuda, oracle, tmp_path, dtype, tied, lm_head):
    import vvllm_b200 as v

    src = _checkpoint(dtype, tied)
    sp, dp = str(tmp_path / "src.safetensors"), str(tmp_path / "q8.safetensors")
    st_util.write(sp, src, {"format": "pt", "note": "synthetic"})
    v.st_quantize(sp, dp, device=0, lm_head=lm_head)
    meta, out = st_util.read(dp)  # an independent reader
    assert meta["format"] == "pt" and meta["note"] == "synthetic" and "b200q8" in meta
    head = "lm_head.weight" if not tied else "model.embed_tokens.weight"
    expect_q = {n for n in src if n.endswith("_proj.weight")} | ({head} if lm_head else set())
    for name, (dt, arr) in src.items():
        replaced = name.endswith("_proj.weight") or (lm_head and name == "lm_head.weight")
        assert (name in out) != replaced, name
        if name in out:  # copied byte for byte
            assert out[name][0] == dt and out[name][1] == arr.shape and out[name][2] == arr.tobytes(), name
        if name in expect_q:
            ref_q, ref_s = oracle.quantize_per_channel(_as_f32(dt, arr))
            q, s = st_util.array(out[name + ".q8"]), st_util.array(out[name + ".q8_scales"])
            assert np.array_equal(q, ref_q), name
            assert np.array_equal(s.view(np.uint32), ref_s.view(np.uint32)), name
        else:
            assert name + ".q8" not in out
    # the library's own reader gives the same pairs as views into the map
    with v.SafeTensors(dp) as f:
        for name in expect_q:
            q, s = f.quantized(name)
            assert q.tobytes() == out[name + ".q8"][2] and s.tobytes() == out[name + ".q8_scales"][2]
        # gate and up stay separate: per-row quantization of their concatenation (model.cc:66-76)
        # equals the concatenation of their quantized rows and scales
        g = src["model.layers.0.mlp.gate_proj.weight"]
        u = src["model.layers.0.mlp.up_proj.weight"]
        cq, cs = oracle.quantize_per_channel(np.concatenate([_as_f32(*g), _as_f32(*u)]))
        gq, gs = f.quantized("model.layers.0.mlp.gate_proj.weight")
        uq, us = f.quantized("model.layers.0.mlp.up_proj.weight")
        assert np.array_equal(np.concatenate([gq, uq]), cq) and np.array_equal(np.concatenate([gs, us]), cs)


def test_st_quantize_errors(cuda, tmp_path):
    import vvllm_b200 as v

    with pytest.raises(v.B200Q8Error) as e:
        v.st_quantize(str(tmp_path / "missing.safetensors"), str(tmp_path / "o.safetensors"))
    assert e.value.status == -7
    sp = str(tmp_path / "s.safetensors")
    st_util.write(sp, {"a_proj.weight": ("F32", np.ones((2, 4), np.float32)),
                       "a_proj.weight.q8": ("I8", np.ones((2, 4), np.int8))})
    with pytest.raises(v.B200Q8Error) as e:  # the output name is taken already
        v.st_quantize(sp, str(tmp_path / "o.safetensors"))
    assert e.value.status == -1
    ok = str(tmp_path / "ok.safetensors")
    st_util.write(ok, {"a_proj.weight": ("F32", np.ones((2, 4), np.float32))})
    with pytest.raises(v.B200Q8Error) as e:  # unwritable destination
        v.st_quantize(ok, str(tmp_path / "no_such_dir" / "o.safetensors"))
    assert e.value.status == -7
