"""vvllm_b200 -- B200 (sm_100a) quantized-linear hot path of vvllm.

The product is ``libb200q8.so`` (CUDA kernels + the C ABI in
``include/b200q8.h``).  This package only binds that library with ctypes so
the tests and ``bench.py`` call exactly what a C/C++ caller would; it contains
no compute of its own and no CPU fallback.  If the library is missing or a
call fails, an exception is raised.
"""
from ._lib import (  # noqa: F401
    B200Q8Error,
    F16,
    F32,
    Backend,
    Comm,
    lib,
    launch_count,
    linear_q8,
    linear_q8_add,
    linear_q8_argmax,
    linear_q8_ex,
    kernel_error,
    diag_peer_wait,
    ALGO_AUTO,
    ALGO_SIMT,
    ALGO_TC,
    ALGO_TC_I8,
    linear_q8_sharded,
    linear_q8_sharded_p2p,
    quantize_per_channel,
    quantize_per_channel_bf16,
    SafeTensors,
    st_quantize,
    ST_BF16,
    ST_F16,
    ST_F32,
    ST_I8,
    ST_OTHER,
    rms_norm,
    rms_norm_linear_q8,
    linear_q8_group,
    shard_range,
    silu_mul,
    silu_mul_linear_q8_add,
)
