"""ctypes binding of libb200q8.so (include/b200q8.h).

Device buffers are passed as raw addresses (``int``) or torch CUDA tensors;
streams as ``cudaStream_t`` addresses (``torch.cuda.Stream.cuda_stream``).
Every wrapper checks the returned status and raises ``B200Q8Error`` with the
library's message.  Nothing here computes: the shared library does.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libb200q8.so")

F32 = 0
F16 = 1

_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_int = ctypes.c_int


class B200Q8Error(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"b200q8 status {status}: {msg}")
        self.status = status


_SIGS = {
    "b200q8_abi_version": ([], _int),
    "b200q8_last_error": ([], ctypes.c_char_p),
    "b200q8_launch_count": ([], ctypes.c_uint64),
    "b200q8_quantize_per_channel": ([_vp, _sz, _sz, _vp, _vp, _vp], _int),
    "b200q8_linear_q8": ([_vp, _int, _vp, _int, _vp, _vp, _vp, _sz, _sz, _sz, _vp], _int),
    "b200q8_linear_q8_add": ([_vp, _int, _vp, _int, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _vp], _int),
    "b200q8_linear_q8_ex": ([_vp, _int, _vp, _int, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _int, _vp], _int),
    "b200q8_kernel_error": ([ctypes.POINTER(_int), _int], _int),
    "b200q8_diag_peer_wait": ([_vp, _int, _int, ctypes.c_double, _int, _vp, _vp, _vp, _vp, _sz, _sz, _vp],
                              _int),
    "b200q8_linear_q8_noalloc": ([_vp, _int, _vp, _int, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _vp], _int),
    "b200q8_backend_create": ([_int, _int, ctypes.POINTER(_vp)], _int),
    "b200q8_backend_destroy": ([_vp], _int),
    "b200q8_backend_set_stream": ([_vp, _vp], _int),
    "b200q8_backend_cached_bytes": ([_vp, ctypes.POINTER(_sz)], _int),
    "b200q8_backend_linear_q8": ([_vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz], _int),
    "b200q8_backend_linear_q8_add": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz], _int),
    "b200q8_backend_quantize_per_channel": ([_vp, _vp, _sz, _sz, _vp, _vp], _int),
    "b200q8_shard_range": ([_sz, _int, _int, ctypes.POINTER(_sz), ctypes.POINTER(_sz)], _int),
    "b200q8_comm_unique_id": ([ctypes.c_char_p], _int),
    "b200q8_comm_init": ([_int, _int, _int, ctypes.c_char_p, ctypes.c_double, ctypes.POINTER(_vp)], _int),
    "b200q8_comm_destroy": ([_vp], _int),
    "b200q8_comm_abort": ([_vp], _int),
    "b200q8_comm_allgather": ([_vp, _vp, _sz, _int, _vp], _int),
    "b200q8_linear_q8_sharded": (
        [_vp, _vp, _int, _vp, _int, _vp, _vp, _vp, _sz, _sz, _sz, _vp, _vp], _int),
    "b200q8_comm_sym_alloc": ([_vp, _sz, ctypes.POINTER(_vp)], _int),
    "b200q8_comm_sym_free": ([_vp, _vp], _int),
    "b200q8_linear_q8_sharded_p2p": (
        [_vp, _vp, _int, _vp, _int, _vp, _vp, _vp, _sz, _sz, _sz, _vp], _int),
    "b200q8_linear_q8_sharded_p2p_ex": (
        [_vp, _vp, _int, _vp, _int, _vp, _vp, _vp, _sz, _sz, _sz, ctypes.c_uint, _vp], _int),
    "b200q8_comm_wait": ([_vp, _vp], _int),
    "b200q8_linear_q8_argmax": ([_vp, _int, _vp, _int, _vp, _vp, _vp, _sz, _sz, _sz, _vp, _vp], _int),
    "b200q8_rms_norm_linear_q8": (
        [_vp, _int, _vp, _int, _vp, ctypes.c_float, _vp, _vp, _vp, _sz, _sz, _sz, _vp], _int),
    "b200q8_silu_mul_linear_q8_add": ([_vp, _int, _vp, _int, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _vp], _int),
    "b200q8_rms_norm": ([_vp, _vp, _int, _vp, ctypes.c_float, _sz, _sz, _vp], _int),
    "b200q8_silu_mul": ([_vp, _vp, _int, _sz, _sz, _vp], _int),
    "b200q8_quantize_per_channel_bf16": ([_vp, _sz, _sz, _vp, _vp, _vp], _int),
    "b200q8_linear_q8_group": ([_int, _vp, _int, _vp, _int, _vp, ctypes.c_float, _vp, _vp, _vp, _vp, _sz, _sz, _vp],
                               _int),
    "b200q8_st_open": ([ctypes.c_char_p, ctypes.POINTER(_vp)], _int),
    "b200q8_st_close": ([_vp], _int),
    "b200q8_st_count": ([_vp, ctypes.POINTER(_sz)], _int),
    "b200q8_st_info": ([_vp, _sz, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_int), ctypes.POINTER(_sz),
                        ctypes.POINTER(ctypes.POINTER(_sz)), ctypes.POINTER(_vp), ctypes.POINTER(_sz)], _int),
    "b200q8_st_find": ([_vp, ctypes.c_char_p, ctypes.POINTER(_sz)], _int),
    "b200q8_st_quantized": ([_vp, ctypes.c_char_p, ctypes.POINTER(_sz), ctypes.POINTER(_sz), ctypes.POINTER(_vp),
                             ctypes.POINTER(_vp)], _int),
    "b200q8_st_quantize": ([ctypes.c_char_p, ctypes.c_char_p, _int, ctypes.c_uint], _int),
}

# Symbols include/b200q8.h declares (kept in sync by tests/test_abi.py).
EXPORTED = tuple(_SIGS)

_lib = None


def lib():
    """Load libb200q8.so once; raise if it is absent (there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise B200Q8Error(-3, f"{LIB_PATH} not built (run `python -m vvllm_b200.build`)")
        L = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
        for name, (args, res) in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def _check(status: int) -> None:
    if status != 0:
        msg = lib().b200q8_last_error().decode(errors="replace")
        raise B200Q8Error(status, msg)


def _addr(t) -> int | None:
    """Device address of a torch tensor / int / None."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream(s) -> int | None:
    if s is None:
        return None
    if isinstance(s, int):
        return s
    return s.cuda_stream


def _dtype_code(t) -> int:
    import torch

    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.float16:
        return F16
    raise TypeError(f"unsupported activation dtype {t.dtype}")


def launch_count() -> int:
    return int(lib().b200q8_launch_count())


def quantize_per_channel(w, q, scales, stream=None) -> None:
    """q[N,K] int8, scales[N] fp32 = per-row absmax quantization of w[N,K] fp32 (device)."""
    N, K = w.shape
    _check(lib().b200q8_quantize_per_channel(_addr(w), N, K, _addr(q), _addr(scales), _stream(stream)))


def linear_q8(out, x, w, scales, bias=None, stream=None) -> None:
    """out[M,N] = (x[M,K] . W^T) * scales + bias, x/out fp32 or fp16 torch CUDA tensors."""
    M, K = x.shape
    N = w.shape[0]
    _check(lib().b200q8_linear_q8(_addr(out), _dtype_code(out), _addr(x), _dtype_code(x), _addr(w),
                                  _addr(scales), _addr(bias), M, N, K, _stream(stream)))


def linear_q8_add(out, x, w, scales, bias, residual, stream=None) -> None:
    M, K = x.shape
    N = w.shape[0]
    _check(lib().b200q8_linear_q8_add(_addr(out), _dtype_code(out), _addr(x), _dtype_code(x),
                                      _addr(w), _addr(scales), _addr(bias), _addr(residual), M, N,
                                      K, _stream(stream)))


def linear_q8_argmax(out, x, w, scales, bias, argmax, out_dtype=None, stream=None) -> None:
    """argmax[m] (int32 device tensor) = greedy argmax of out[m, :] = linear_q8(x, w); out may be
    None (logits not written; then out_dtype picks the comparison precision, default fp32)."""
    M, K = x.shape
    N = w.shape[0]
    odt = _dtype_code(out) if out is not None else (F32 if out_dtype is None else out_dtype)
    _check(lib().b200q8_linear_q8_argmax(_addr(out), odt, _addr(x), _dtype_code(x), _addr(w), _addr(scales),
                                         _addr(bias), M, N, K, _addr(argmax), _stream(stream)))


def rms_norm_linear_q8(out, x, norm_weight, eps, w, scales, bias=None, stream=None) -> None:
    """out[M,N] = linear_q8(rms_norm(x[M,K], norm_weight[K], eps)) with the norm fused into the GEMV."""
    M, K = x.shape
    N = w.shape[0]
    _check(lib().b200q8_rms_norm_linear_q8(_addr(out), _dtype_code(out), _addr(x), _dtype_code(x),
                                           _addr(norm_weight), float(eps), _addr(w), _addr(scales), _addr(bias),
                                           M, N, K, _stream(stream)))


def silu_mul_linear_q8_add(out, gate_up, w, scales, bias=None, residual=None, stream=None) -> None:
    """out[M,N] = linear_q8(silu(gate_up[:, :K]) * gate_up[:, K:]) (+ residual), K = w.shape[1]."""
    M = gate_up.shape[0]
    N, K = w.shape
    if gate_up.shape[1] != 2 * K:
        raise ValueError(f"gate_up must be [M, 2K] = [{M}, {2 * K}], got {tuple(gate_up.shape)}")
    _check(lib().b200q8_silu_mul_linear_q8_add(_addr(out), _dtype_code(out), _addr(gate_up), _dtype_code(gate_up),
                                               _addr(w), _addr(scales), _addr(bias), _addr(residual), M, N, K,
                                               _stream(stream)))


def linear_q8_group(outs, x, weights, scales, biases=None, norm_weight=None, eps=1e-6, stream=None) -> None:
    """outs[i][M,N_i] = linear_q8(rms_norm(x) if norm_weight is not None else x, weights[i], scales[i],
    biases[i]) for up to 4 projections of the same x (one launch for few tokens)."""
    n = len(weights)
    if not (len(outs) == len(scales) == n) or (biases is not None and len(biases) != n):
        raise ValueError("outs, weights, scales (and biases) must have the same length")
    M, K = x.shape
    if not x.is_contiguous():
        raise ValueError("x must be contiguous [M, K]")
    for i, (o, w) in enumerate(zip(outs, weights)):
        if o.dtype != outs[0].dtype:
            raise ValueError(f"outs[{i}] is {o.dtype}, outs[0] is {outs[0].dtype}: one output dtype per group")
        if tuple(w.shape) != (w.shape[0], K) or tuple(o.shape) != (M, w.shape[0]) or not o.is_contiguous():
            raise ValueError(f"projection {i}: weights must be [N, {K}] and outs [{M}, N] contiguous")
        if not w.is_contiguous():
            raise ValueError(f"projection {i}: weights must be contiguous")
        if scales[i].numel() != w.shape[0] or not scales[i].is_contiguous():
            raise ValueError(f"projection {i}: scales must hold N = {w.shape[0]} contiguous values")
        if biases is not None and biases[i] is not None and (biases[i].numel() != w.shape[0]
                                                              or not biases[i].is_contiguous()):
            raise ValueError(f"projection {i}: bias must hold N = {w.shape[0]} contiguous values")
    arr_p = ctypes.c_void_p * n
    outs_a = arr_p(*[_addr(o) for o in outs])
    w_a = arr_p(*[_addr(w) for w in weights])
    s_a = arr_p(*[_addr(s) for s in scales])
    b_a = arr_p(*[_addr(b) for b in biases]) if biases is not None else None
    ns = (ctypes.c_size_t * n)(*[w.shape[0] for w in weights])
    odt = _dtype_code(outs[0])
    _check(lib().b200q8_linear_q8_group(n, outs_a, odt, _addr(x), _dtype_code(x), _addr(norm_weight), float(eps),
                                        w_a, s_a, b_a, ns, M, K, _stream(stream)))


def rms_norm(out, x, norm_weight, eps, stream=None) -> None:
    """out[M,K] = rms_norm(x[M,K]) per token (same arithmetic as the fused prologue)."""
    M, K = x.shape
    _check(lib().b200q8_rms_norm(_addr(out), _addr(x), _dtype_code(x), _addr(norm_weight), float(eps), M, K,
                                 _stream(stream)))


def silu_mul(out, gate_up, stream=None) -> None:
    """out[M,K] = silu(gate_up[:, :K]) * gate_up[:, K:]."""
    M, K2 = gate_up.shape
    _check(lib().b200q8_silu_mul(_addr(out), _addr(gate_up), _dtype_code(gate_up), M, K2 // 2, _stream(stream)))


def quantize_per_channel_bf16(w_bits, q, scales, stream=None) -> None:
    """q[N,K] int8, scales[N] fp32 from bfloat16 bits w_bits[N,K] (int16/uint16 device tensor)."""
    N, K = w_bits.shape
    _check(lib().b200q8_quantize_per_channel_bf16(_addr(w_bits), N, K, _addr(q), _addr(scales), _stream(stream)))


ST_F32, ST_F16, ST_BF16, ST_I8, ST_OTHER = 0, 1, 2, 3, 4
ST_LM_HEAD = 1
_ST_NP = {ST_F32: "float32", ST_F16: "float16", ST_BF16: "uint16", ST_I8: "int8"}


class SafeTensors:
    """A safetensors file opened through b200q8_st_open: tensor data stays in the read-only map
    (numpy views, valid until close())."""

    def __init__(self, path: str):
        h = _vp()
        _check(lib().b200q8_st_open(os.fsencode(path), ctypes.byref(h)))
        self._h = h

    def close(self) -> None:
        if self._h:
            lib().b200q8_st_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __len__(self) -> int:
        n = _sz()
        _check(lib().b200q8_st_count(self._h, ctypes.byref(n)))
        return n.value

    def info(self, i: int):
        """(name, dtype code, shape tuple, data address, nbytes) of tensor i (file-data order)."""
        name, dt, nd, shp, data, nb = ctypes.c_char_p(), _int(), _sz(), ctypes.POINTER(_sz)(), _vp(), _sz()
        _check(lib().b200q8_st_info(self._h, i, ctypes.byref(name), ctypes.byref(dt), ctypes.byref(nd),
                                    ctypes.byref(shp), ctypes.byref(data), ctypes.byref(nb)))
        return name.value.decode(), dt.value, tuple(shp[j] for j in range(nd.value)), data.value or 0, nb.value

    def names(self) -> list[str]:
        return [self.info(i)[0] for i in range(len(self))]

    def find(self, name: str) -> int:
        i = _sz()
        _check(lib().b200q8_st_find(self._h, name.encode(), ctypes.byref(i)))
        return i.value

    @staticmethod
    def _view(addr: int, nbytes: int, dtype: str, shape):
        import numpy as np

        if nbytes == 0:
            return np.zeros(shape, dtype=dtype)
        buf = (ctypes.c_char * nbytes).from_address(addr)
        return np.frombuffer(buf, dtype=dtype).reshape(shape)

    def tensor(self, name: str):
        """numpy view of a F32 / F16 / BF16 (as uint16 bits) / I8 tensor; raw uint8 bytes otherwise."""
        _, dt, shape, addr, nb = self.info(self.find(name))
        if dt in _ST_NP:
            return self._view(addr, nb, _ST_NP[dt], shape)
        return self._view(addr, nb, "uint8", (nb,))

    def quantized(self, name: str):
        """(q int8 [N, K], scales fp32 [N]) of projection `name`, as quantize_per_channel returns them."""
        N, K, q, sc = _sz(), _sz(), _vp(), _vp()
        _check(lib().b200q8_st_quantized(self._h, name.encode(), ctypes.byref(N), ctypes.byref(K), ctypes.byref(q),
                                         ctypes.byref(sc)))
        return (self._view(q.value or 0, N.value * K.value, "int8", (N.value, K.value)),
                self._view(sc.value or 0, N.value * 4, "float32", (N.value,)))


def st_quantize(src: str, dst: str, device: int = 0, lm_head: bool = False) -> None:
    """Write dst = src with every projection quantized on GPU `device` (b200q8_st_quantize)."""
    _check(lib().b200q8_st_quantize(os.fsencode(src), os.fsencode(dst), device, ST_LM_HEAD if lm_head else 0))


ALGO_AUTO, ALGO_SIMT, ALGO_TC, ALGO_TC_I8 = 0, 1, 2, 3


def linear_q8_ex(out, x, w, scales, bias=None, residual=None, algo=ALGO_AUTO, stream=None) -> None:
    """linear_q8 / linear_q8_add with an explicit kernel choice (ALGO_SIMT / ALGO_TC)."""
    M, K = x.shape
    N = w.shape[0]
    _check(lib().b200q8_linear_q8_ex(_addr(out), _dtype_code(out), _addr(x), _dtype_code(x), _addr(w),
                                     _addr(scales), _addr(bias), _addr(residual), M, N, K, algo,
                                     _stream(stream)))


def kernel_error(clear: bool = True) -> int:
    """Device error word (bit 0: a bounded wait in the tensor-core kernel gave up)."""
    c = _int()
    _check(lib().b200q8_kernel_error(ctypes.byref(c), int(clear)))
    return c.value


def diag_peer_wait(counts, self_index: int, timeout_s: float, where: int = 0, out=None, x=None, w=None, scales=None,
                   stream=None) -> None:
    """The gathered calls' bounded peer wait on `counts` (uint64 / int64 device tensor of n
    completion counts, 2^20 per finished call): it holds until every count holds as many whole
    calls as counts[self_index].  where 0 = the standalone wait kernel, 1 = inside the digit GEMV,
    2 = inside its prep kernel (1 and 2 run out[1, N] = linear_q8(x[1, K] fp16, w, scales) behind
    the wait).  A wait that runs out is reported by kernel_error() (bit 1), not by this call."""
    N, K = (w.shape[0], w.shape[1]) if w is not None else (0, 0)
    _check(lib().b200q8_diag_peer_wait(_addr(counts), counts.numel(), self_index, float(timeout_s), where, _addr(out),
                                       _addr(x), _addr(w), _addr(scales), N, K, _stream(stream)))


def shard_range(N: int, nranks: int, rank: int) -> tuple[int, int]:
    r0, n = _sz(), _sz()
    _check(lib().b200q8_shard_range(N, nranks, rank, ctypes.byref(r0), ctypes.byref(n)))
    return r0.value, n.value


class Backend:
    """vvllm::Backend-shaped handle: host weight pointers (numpy), device activations."""

    def __init__(self, device: int = 0, fp16: bool = False):
        h = _vp()
        _check(lib().b200q8_backend_create(device, int(fp16), ctypes.byref(h)))
        self.h = h
        self.fp16 = fp16

    def close(self):
        if self.h:
            lib().b200q8_backend_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream) -> None:
        _check(lib().b200q8_backend_set_stream(self.h, _stream(stream)))

    def cached_bytes(self) -> int:
        n = _sz()
        _check(lib().b200q8_backend_cached_bytes(self.h, ctypes.byref(n)))
        return n.value

    def linear_q8(self, out, inp, weight, scales, bias, M, N, K) -> None:
        """out/inp: device tensors; weight/scales/bias: host numpy arrays (cache keys)."""
        _check(lib().b200q8_backend_linear_q8(
            self.h, _addr(out), _addr(inp), weight.ctypes.data, scales.ctypes.data,
            None if bias is None else bias.ctypes.data, M, N, K))

    def linear_q8_add(self, out, inp, weight, scales, bias, residual, M, N, K) -> None:
        _check(lib().b200q8_backend_linear_q8_add(
            self.h, _addr(out), _addr(inp), weight.ctypes.data, scales.ctypes.data,
            None if bias is None else bias.ctypes.data, _addr(residual), M, N, K))

    def quantize_per_channel(self, w):
        """Host fp32 [N,K] -> (host int8 [N,K], host fp32 [N]), computed on the GPU."""
        import numpy as np

        w = np.ascontiguousarray(w, dtype=np.float32)
        N, K = w.shape
        q = np.empty((N, K), dtype=np.int8)
        s = np.empty((N,), dtype=np.float32)
        _check(lib().b200q8_backend_quantize_per_channel(self.h, w.ctypes.data, N, K, q.ctypes.data,
                                                         s.ctypes.data))
        return q, s


class Comm:
    """NCCL communicator over the ranks of one node (non-blocking init with a deadline)."""

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        _check(lib().b200q8_comm_unique_id(buf))
        return buf.raw

    def __init__(self, device: int, nranks: int, rank: int, uid: bytes, timeout_s: float = 60.0):
        assert len(uid) == 128
        h = _vp()
        _check(lib().b200q8_comm_init(device, nranks, rank, uid, timeout_s, ctypes.byref(h)))
        self.h = h
        self.nranks, self.rank = nranks, rank

    def destroy(self) -> None:
        """Collective.  Symmetric buffers die with the communicator: drop their tensors first."""
        if self.h:
            h, self.h = self.h, None
            _check(lib().b200q8_comm_destroy(h))

    def allgather(self, buf, count: int, dtype: int, stream=None) -> None:
        """In place: rank r's slice is buf[r*count:(r+1)*count]."""
        _check(lib().b200q8_comm_allgather(self.h, _addr(buf), count, dtype, _stream(stream)))

    def sym_alloc(self, nbytes: int):
        """Collective: a uint8 CUDA tensor of `nbytes` zeroed bytes that every peer has mapped.

        The tensor does not own the memory; it stays valid until sym_free or destroy."""
        import torch

        p = _vp()
        _check(lib().b200q8_comm_sym_alloc(self.h, nbytes, ctypes.byref(p)))

        class _Raw:
            __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (p.value, False),
                                        "version": 3, "strides": None}

        return torch.as_tensor(_Raw(), device="cuda")

    def sym_free(self, t) -> None:
        _check(lib().b200q8_comm_sym_free(self.h, _addr(t)))

    def wait(self, stream=None) -> None:
        """Enqueue the completion wait a deferred gathered call still owes (no-op if none)."""
        _check(lib().b200q8_comm_wait(self.h, _stream(stream)))

    def abort(self) -> None:
        if self.h:
            h, self.h = self.h, None
            lib().b200q8_comm_abort(h)


def linear_q8_sharded(comm: Comm, out, x, w_shard, scales_shard, bias_shard, N: int, gather=None,
                      stream=None) -> None:
    """out[M,N] (all ranks) = linear_q8 over the column-sharded weight, NCCL all-gathered."""
    M, K = x.shape
    _check(lib().b200q8_linear_q8_sharded(comm.h, _addr(out), _dtype_code(out), _addr(x),
                                          _dtype_code(x), _addr(w_shard), _addr(scales_shard),
                                          _addr(bias_shard), M, N, K, _addr(gather),
                                          _stream(stream)))


P2P_DEFER_WAIT = 1


def linear_q8_sharded_p2p(comm: Comm, out, x, w_shard, scales_shard, bias_shard, N: int,
                          stream=None, defer_wait: bool = False) -> None:
    """out[M,N] (all ranks) = linear_q8 over the column-sharded weight; the GEMV stores every
    rank's slice into every rank's `out` over NVLink.  `out` lies in a Comm.sym_alloc tensor.
    defer_wait: leave the completion wait to the next gathered call or Comm.wait()."""
    M, K = x.shape
    _check(lib().b200q8_linear_q8_sharded_p2p_ex(comm.h, _addr(out), _dtype_code(out), _addr(x),
                                                 _dtype_code(x), _addr(w_shard), _addr(scales_shard),
                                                 _addr(bias_shard), M, N, K,
                                                 P2P_DEFER_WAIT if defer_wait else 0, _stream(stream)))
