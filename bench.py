"""Benchmark of the B200 quantized-linear hot path (vvllm Backend::linear_q8).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (benchmark config 5, M = 1 decode): the Qwen2.5-7B-shaped int8
projections -- fused gate/up 3584 -> 37888, down 18944 -> 3584 and lm_head
3584 -> 152064 -- with fp16 activations, fp32 accumulation and fp16 outputs.
Weights are synthetic N(0, 0.02), quantized per row by absmax on the GPU;
activations N(0, 1).  With N GPUs every projection is column-sharded by output
channel (rank r owns rows [r*N/G, (r+1)*N/G)) and each rank's GEMV stores its
slice into every rank's output over NVLink (the gather fused into the kernel;
the GEMV-then-NCCL-allgather alternative is reported beside it), so the total
work is fixed as N grows ("strong" scaling).

One step = the three projections once.  `value` is the whole-job algorithmic
HBM bytes moved per second (int8 weights + fp32 scales + activations in +
outputs out, summed over ranks), timed on the device with CUDA events over K
steps, max over ranks.  Weight sets rotate so one cycle per rank exceeds 2x
the 126 MB L2 (inputs larger than L2).  Output: one JSON line on rank 0.

Beside the headline, the line carries: a parity verdict (N = 1: the reference's
own CPU linear_q8 on a row sample of every projection; N > 1: every rank's
gathered outputs against the unsharded digit GEMV of each rank's rows, bit for
bit); benchmark configs 1-4 and config 5 at M = 8 and 64 (rank 0, N = 1); the
GPU quantize against the reference's single-threaded quantize_per_channel; and
the reference's CPU linear_q8 on working sets larger than twice the host's LLC.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HIDDEN, INTER, VOCAB = 3584, 18944, 152064
PROJ = [  # name, N (output channels), K (input features)
    ("gate_up", 2 * INTER, HIDDEN),
    ("down", HIDDEN, INTER),
    ("lm_head", VOCAB, HIDDEN),
]
METRIC = "linear_q8 GEMV HBM GB/s (% peak) + prefill GEMM TFLOP/s at Qwen-0.5B/7B shapes"
WORKLOAD = "qwen2.5-7b-shaped decode projections (gate_up 3584->37888, down 18944->3584, lm_head 3584->152064), M=1"
L2_BYTES = 126 * 1024 * 1024


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def algo_bytes(N: int, K: int, M: int = 1, a: int = 2, o: int = 2) -> int:
    """int8 weights + fp32 scales + activations in + outputs out (weights read once)."""
    return N * K + 4 * N + M * K * a + M * N * o


def profiled_traffic(kernel: str):
    """DRAM bytes per launch of the dominant kernel (dram__bytes_read.sum + dram__bytes_write.sum
    of one ncu capture), from profiles/roofline_traffic.json, if recorded."""
    try:
        with open(os.path.join(ROOT, "profiles", "roofline_traffic.json")) as f:
            return int(json.load(f)[kernel]["dram_bytes_per_launch"])
    except (OSError, KeyError, ValueError, TypeError):
        return None


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.samples, self.reasons = [], 0  # samples: (time, SM MHz, reason bits)
        self.period = period_s
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # pragma: no cover - no NVML here
            self.err = str(e)
            self.max_mhz = None

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((time.monotonic(), mhz, r))
                self.reasons |= r
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.ok:
            self.t.join()

    def _names(self, bits):
        return [n for bit, n in self.REASONS.items() if bits & bit and n != "gpu_idle"]

    def summary(self, window=None):
        """Median SM clock and the clock-event reasons seen, over the whole sampled run and over
        `window` = (t0, t1) (time.monotonic()), the timed region."""
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        out = {"sm_mhz": statistics.median(m for _, m, _ in self.samples) if self.samples else None,
               "sm_max_mhz": self.max_mhz, "reasons": self._names(self.reasons), "samples": len(self.samples),
               "period_ms": self.period * 1e3, "covers": "warm-up through the last GPU leg of the run"}
        if window is not None:
            inside = [(m, r) for t, m, r in self.samples if window[0] <= t <= window[1]]
            bits = 0
            for _, r in inside:
                bits |= r
            out["timed_region"] = {"sm_mhz": statistics.median(m for m, _ in inside) if inside else None,
                                   "samples": len(inside), "reasons": self._names(bits)}
        return out


def cpu_info():
    name = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    name = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return name, os.cpu_count() or 1


def cpu_reference_lib():
    """The reference's own CPU linear_q8 (oracle/_ref) if it was built, else the C restatement."""
    from oracle import Oracle, Reference, have_reference

    if have_reference():
        return Reference(), "reference"
    return Oracle(), "port"


def llc_bytes() -> int:
    """Size of the host's largest CPU cache level (sysfs), 0 if unknown."""
    best = 0
    base = "/sys/devices/system/cpu/cpu0/cache"
    try:
        names = os.listdir(base)
    except OSError:
        return 0
    for d in names:
        if not d.startswith("index"):
            continue
        try:
            with open(os.path.join(base, d, "size")) as f:
                txt = f.read().strip()
            mult = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}.get(txt[-1:], 1)
            best = max(best, int(txt.rstrip("KMG")) * mult)
        except (OSError, ValueError):
            continue
    return best


def cpu_sample_bytes(requested_mb: float) -> int:
    """int8 weight bytes the CPU legs stream per pass: as requested, else twice the host's LLC
    (at least 64 MB), so the reference reads its weights from DRAM as in the real workload."""
    if requested_mb > 0:
        return int(requested_mb * 1e6)
    return max(2 * llc_bytes(), 64 << 20)


def time_cpu_linear(lib, shapes, threads: int, budget_s: float, min_iters: int = 1):
    """Times lib.linear_q8_mt over `shapes` (list of (x, q, s)); returns (GB/s, seconds/iter, iters)."""
    total_bytes = sum(algo_bytes(q.shape[0], q.shape[1], 1, 4, 4) for _, q, _ in shapes)
    for x, q, s in shapes:  # warm the pages
        lib.linear_q8_mt(x, q, s, None, nthreads=threads)
    iters, t0 = 0, time.perf_counter()
    while True:
        for x, q, s in shapes:
            lib.linear_q8_mt(x, q, s, None, nthreads=threads)
        iters += 1
        el = time.perf_counter() - t0
        if el >= budget_s and iters >= min_iters:
            break
    return total_bytes * iters / el / 1e9, el / iters, iters


def host_sample_weights(min_bytes: int, seed: int = 0):
    """Host int8 weights for the same fraction of every projection's rows, at least `min_bytes` in
    all (values do not change the CPU's timing: random bytes repeated from an 8 MB block).
    Returns (list of (x, q, s), fraction of the rows)."""
    total = sum(N * K for _, N, K in PROJ)
    frac = min(1.0, max(min_bytes / total, 1e-3))
    rng = np.random.default_rng(seed)
    block = rng.integers(-127, 128, size=1 << 23, dtype=np.int8)
    out = []
    for name, N, K in PROJ:
        n = max(1, int(math.ceil(N * frac)))
        q = np.resize(block, n * K).reshape(n, K)
        s = (rng.random(n, dtype=np.float32) * np.float32(1e-3)).astype(np.float32)
        x = rng.standard_normal((1, K), dtype=np.float32).astype(np.float16).astype(np.float32)
        out.append((x, q, s))
    return out, frac


def run_reference(args):
    """--impl reference: the reference's CPU linear_q8 on all host threads, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    lib, kind = cpu_reference_lib()
    model, cores = cpu_info()
    shapes, frac = host_sample_weights(cpu_sample_bytes(args.cpu_sample_mb))
    sample_bytes = sum(algo_bytes(q.shape[0], q.shape[1], 1, 4, 4) for _, q, _ in shapes)
    for _ in range(args.warmup):
        for x, q, s in shapes:
            lib.linear_q8_mt(x, q, s, None, nthreads=cores)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for x, q, s in shapes:
            lib.linear_q8_mt(x, q, s, None, nthreads=cores)
        times.append(time.perf_counter() - t0)
    el = sum(times)
    gbs = sample_bytes * args.steps / el / 1e9
    sample = (f"{frac:.3f} of the rows of each projection ({sample_bytes / 1e6:.1f} MB algorithmic per step, "
              f"> 2x the host's {llc_bytes() / 2**20:.0f} MiB LLC), fp32 activations widened from fp16, "
              f"{cores} threads on disjoint output-channel slices; CPU: {model}")
    ref_gpu = reference_gpu(args)
    line = {
        "metric": METRIC, "impl": "reference", "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * el / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8 weights x f32 activations, f32 accumulate",
        "data": "synthetic", "config": {"workload": WORKLOAD, "M": 1, "parallelism": "cpu threads"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if ref_gpu is not None:
        line["reference_gpu"] = ref_gpu
    print(json.dumps(line), flush=True)
    return 0


def reference_gpu(args):
    """The reference's own GPU linear_q8 (vvllm::BackendCUDA, fp16 mode: cuBLAS GemmEx on the fp16
    dequantized copy of each int8 weight, src/backend/backend_cuda.cc:188-213), built from the
    reference sources for sm_100a into oracle/_ref/libvvllm_refgpu.so, on the same 7B decode step
    (gate_up, down, lm_head, one fp16 token) on GPU 0; None without a GPU or that library.  Timed
    with CUDA events on the legacy default stream the reference launches on, over the K steps
    after W warm-up steps (the first call of each weight uploads and dequantizes it).  `value`
    uses this bench's algorithmic bytes (int8 weights), so it compares with the B200 arm's value
    directly; `fp16_weight_gbs` counts the 2 bytes per weight cuBLAS actually streams."""
    import ctypes

    path = os.path.join(ROOT, "oracle", "_ref", "libvvllm_refgpu.so")
    try:
        import torch

        if not torch.cuda.is_available() or not os.path.exists(path):
            return None
    except ImportError:
        return None
    import vvllm_b200

    vvllm_b200.lib()  # the reference GPU library links the in-tree libb200q8.so (its adapter)
    L = ctypes.CDLL(path)
    L.vref_gpu_create.restype = ctypes.c_void_p
    L.vref_gpu_create.argtypes = [ctypes.c_int]
    L.vref_gpu_linear_q8.restype = ctypes.c_int
    L.vref_gpu_linear_q8.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_size_t] * 3
    L.vref_gpu_destroy.argtypes = [ctypes.c_void_p]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rng = np.random.default_rng(9)
    block = rng.integers(-127, 128, size=1 << 23, dtype=np.int8)
    host = []
    for name, N, K in PROJ:
        q = np.resize(block, N * K).reshape(N, K)
        s = (rng.random(N, dtype=np.float32) * np.float32(1e-3)).astype(np.float32)
        x = torch.randn(1, K, device=dev).half()
        out = torch.empty(1, N, device=dev, dtype=torch.float16)
        host.append((q, s, x, out, N, K))
    be = L.vref_gpu_create(1)
    stream = torch.cuda.default_stream(dev)

    def step():
        for q, s, x, out, N, K in host:
            if L.vref_gpu_linear_q8(be, out.data_ptr(), x.data_ptr(), q.ctypes.data, s.ctypes.data, None, 1, N, K):
                raise RuntimeError("reference BackendCUDA::linear_q8 failed")

    try:
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                step()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(args.steps):
                step()
            b.record(stream)
            torch.cuda.synchronize()
        ms = a.elapsed_time(b) / args.steps
    finally:
        L.vref_gpu_destroy(be)
    nb = sum(algo_bytes(N, K) for _, N, K in PROJ)
    nb16 = sum(2 * N * K + 2 * K + 2 * N for _, N, K in PROJ)
    return {"value": round(nb / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 5),
            "fp16_weight_gbs": round(nb16 / (ms * 1e-3) / 1e9, 2), "steps": args.steps,
            "path": "vvllm::BackendCUDA::linear_q8, fp16 mode (cuBLAS GemmEx on fp16 dequantized weights), "
                    "reference sources built for sm_100a, one GPU, direct calls on the legacy default stream"}


def cpu_quantize(lib, min_bytes: int, budget_s: float):
    """The reference's quantize_per_channel, one thread (as the reference runs it at model load),
    on a [R, 3584] fp32 matrix of at least `min_bytes`; bytes = 4NK read + NK + 4N written."""
    K = HIDDEN
    R = max(1024, int(math.ceil(min_bytes / (4 * K))))
    rng = np.random.default_rng(5)
    block = (rng.standard_normal(1 << 22, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    w = np.resize(block, R * K).reshape(R, K)
    lib.quantize_per_channel(w[:256])  # warm the code
    iters, t0 = 0, time.perf_counter()
    while True:
        lib.quantize_per_channel(w)
        iters += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    nbytes = 5 * R * K + 4 * R
    return {"value": round(nbytes * iters / el / 1e9, 3), "unit": "GB/s", "cores": 1,
            "sample": f"[{R}, {K}] fp32 ({4 * R * K / 1e6:.0f} MB in), {iters} pass(es) in {el:.1f} s"}


PREFILL = [(896, 896), (896, 128), (896, 4864), (4864, 896)]  # benchmark config 4 (K, N), M = 512


def prefill_tflops(v, dev, stream, warmup: int, iters: int, tc_peak: float):
    """Config 4: the four prefill GEMMs (M = 512, fp16 in/out), each timed as a CUDA graph of
    back-to-back calls over rotating copies of its weights, activations and outputs (together more
    than 2x L2, so every call reads HBM, as consecutive projections of a prefill pass do); the set
    of four the same way, set after set.  Also a Qwen2.5-7B-shaped prefill projection (gate/up,
    3584 -> 37888, M = 512) as the large-shape reference point.  Per-call time = median replay
    time / calls in the graph."""
    import torch

    M = 512
    torch.manual_seed(1)
    stream = torch.cuda.Stream(device=dev)  # graphs are captured on a non-default stream
    stream.wait_stream(torch.cuda.current_stream(dev))

    def make(K, N):
        q = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev)
        s = torch.rand(N, device=dev) * 1e-3
        x = torch.randn(M, K, device=dev).half()
        out = torch.empty(M, N, device=dev, dtype=torch.float16)
        return (K, N, q, s, x, out)

    def copies_for(shapes):
        per = sum(N * K + 2 * M * K + 2 * M * N for K, N in shapes)
        return max(2, math.ceil(2 * L2_BYTES / per))

    def timed(calls):
        """Median device time (ms) of one graph replay of `calls` in order."""
        for _ in range(warmup):
            for K, N, q, s, x, out in calls:
                v.linear_q8(out, x, q, s, stream=stream)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for K, N, q, s, x, out in calls:
                v.linear_q8(out, x, q, s, stream=stream)
        ms = []
        with torch.cuda.stream(stream):
            for _ in range(iters):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                g.replay()
                b.record(stream)
                b.synchronize()
                ms.append(a.elapsed_time(b))
        del g
        return statistics.median(ms)

    n = copies_for(PREFILL)
    sets = [[make(K, N) for K, N in PREFILL] for _ in range(n)]
    per = {}
    for j, (K, N) in enumerate(PREFILL):
        t = timed([sets[c][j] for c in range(n)]) / n
        per[f"{K}x{N}"] = {"TFLOP/s": round(2.0 * M * N * K / (t * 1e-3) / 1e12, 1), "us": round(t * 1e3, 2)}
    total_flop = sum(2.0 * M * N * K for K, N in PREFILL)
    t_set = timed([c for st in sets for c in st]) / n
    value = total_flop / (t_set * 1e-3) / 1e12
    del sets
    big = [make(HIDDEN, 2 * INTER) for _ in range(2)]
    t_big = timed(big) / len(big)
    v_big = 2.0 * M * big[0][1] * big[0][0] / (t_big * 1e-3) / 1e12
    return {"value": round(value, 1), "unit": "TFLOP/s", "frac": round(value / tc_peak, 4),
            "peak": tc_peak, "M": M, "per_shape": per, "set_us": round(t_set * 1e3, 2), "copies": n,
            "gate_up_7b_M512": {"TFLOP/s": round(v_big, 1), "frac": round(v_big / tc_peak, 4),
                                "us": round(t_big * 1e3, 2)},
            "timing": "median CUDA-graph replay of back-to-back calls over rotating copies (> 2x L2) / calls"}


def decode_stacks(v, dev, warmup: int, iters: int, hbm_peak: float):
    """benchmark configs 2 and 3 as whole decode stacks at M = 1, each step one CUDA-graph replay
    of every projection of every layer in order (the library's ctypes host call costs more than
    the small projections take on the device):
      SmolLM-135M-shaped, fp32 activations: 30 x {q 576, k/v 576->192, o 576 (+residual),
        gate|up 576->3072 (fused as the reference model fuses them), down 1536->576 (+residual)},
        lm_head 576->49152; 136.7 MB of weights, two copies alternated so a cycle exceeds 2x L2;
      Qwen2.5-0.5B-shaped, fp16 activations: 24 x {q 896 (+bias), k/v 896->128 (+bias),
        o 896 (+residual), gate|up 896->9728, down 4864->896 (+residual)}, tied lm_head
        896->151936; 494 MB of weights (> 2x L2).
    value = algorithmic bytes of the step (weights, scales, biases, activations, outputs and the
    residual reads) / median device time of one replay.  "qkv_grouped": the same step with each
    layer's q/k/v as one linear_q8_group call on one x (same byte count)."""
    import torch

    torch.manual_seed(2)
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))

    def stack(layers, hidden, kv, inter, vocab, bias_qkv, in16, copies):
        adt = torch.float16 if in16 else torch.float32
        a = 2 if in16 else 4
        shapes = []  # (N, K, has_bias, residual)
        for _ in range(layers):
            shapes += [(hidden, hidden, bias_qkv, False), (kv, hidden, bias_qkv, False), (kv, hidden, bias_qkv, False),
                       (hidden, hidden, False, True), (2 * inter, hidden, False, False), (hidden, inter, False, True)]
        shapes.append((vocab, hidden, False, False))
        sets = []
        for _ in range(copies):
            calls = []
            for N, K, hb, res in shapes:
                q = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev)
                sc = torch.rand(N, device=dev) * 1e-3
                b = torch.randn(N, device=dev) * 0.1 if hb else None
                x = torch.randn(1, K, device=dev).to(adt)
                out = torch.randn(1, N, device=dev).to(adt)
                calls.append((q, sc, b, x, out, res))
            sets.append(calls)
        nbytes = sum(algo_bytes(N, K, 1, a, a) + (4 * N if hb else 0) + (a * N if res else 0)
                     for N, K, hb, res in shapes)

        def run(calls, grouped):
            i = 0
            while i < len(calls):
                q, sc, b, x, out, res = calls[i]
                if grouped and i % 6 == 0 and i + 3 <= len(calls) - 1:  # q, k, v of one layer
                    grp = calls[i:i + 3]
                    v.linear_q8_group([c[4] for c in grp], x, [c[0] for c in grp], [c[1] for c in grp],
                                      [c[2] for c in grp] if bias_qkv else None, stream=stream)
                    i += 3
                    continue
                if res:
                    v.linear_q8_add(out, x, q, sc, b, out, stream=stream)
                else:
                    v.linear_q8(out, x, q, sc, b, stream=stream)
                i += 1

        def timed(grouped):
            graphs = []
            for calls in sets:
                for _ in range(warmup):
                    run(calls, grouped)
                stream.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    run(calls, grouped)
                graphs.append(g)
            ms = []
            with torch.cuda.stream(stream):
                for i in range(iters * copies):
                    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a0.record(stream)
                    graphs[i % copies].replay()
                    a1.record(stream)
                    a1.synchronize()
                    ms.append(a0.elapsed_time(a1))
            del graphs
            return statistics.median(ms)

        t = timed(False)
        gbs = nbytes / (t * 1e-3) / 1e9
        tg = timed(True)
        return {"value": round(gbs, 1), "unit": "GB/s", "frac": round(gbs / hbm_peak, 4), "us": round(t * 1e3, 2),
                "calls": len(shapes), "bytes": nbytes, "weight_copies": copies,
                "qkv_grouped": {"value": round(nbytes / (tg * 1e-3) / 1e9, 1), "us": round(tg * 1e3, 2),
                                "calls": len(shapes) - 2 * layers}}

    return {"smollm135m_fp32": stack(30, 576, 192, 1536, 49152, False, False, 2),
            "qwen05b_fp16": stack(24, 896, 128, 4864, 151936, True, True, 1),
            "timing": "median CUDA-graph replay of one whole step (device time), weights cycled beyond L2"}


def config1_gemv(v, dev, warmup: int, iters: int, hbm_peak: float):
    """benchmark config 1: one fp32 decode GEMV, x [1, 896] -> y [1, 4864] (4.4 MB of int8 weights).
    One CUDA graph runs the call once on each of enough weight copies to exceed 2x L2, so every
    call streams its weights from HBM; per-call time = median replay time / copies."""
    import torch

    N, K = 4864, 896
    torch.manual_seed(3)
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    copies = int(math.ceil(2 * L2_BYTES / (N * K)))
    ws = [(torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev), torch.rand(N, device=dev) * 1e-3)
          for _ in range(copies)]
    x = torch.randn(1, K, device=dev)
    out = torch.empty(1, N, device=dev)
    for _ in range(warmup):
        for q, s in ws:
            v.linear_q8(out, x, q, s, stream=stream)
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for q, s in ws:
            v.linear_q8(out, x, q, s, stream=stream)
    ms = []
    with torch.cuda.stream(stream):
        for _ in range(iters):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            g.replay()
            b.record(stream)
            b.synchronize()
            ms.append(a.elapsed_time(b))
    del g
    t_call = statistics.median(ms) / copies
    gbs = algo_bytes(N, K, 1, 4, 4) / (t_call * 1e-3) / 1e9
    return {"value": round(gbs, 1), "unit": "GB/s", "frac": round(gbs / hbm_peak, 4), "us_per_call": round(t_call * 1e3, 3),
            "shape": "x fp32 [1, 896] -> y fp32 [1, 4864]", "weight_copies": copies,
            "timing": "median CUDA-graph replay of one call per weight copy (copies > 2x L2), divided by copies"}


def gpu_quantize(v, dev, iters: int, hbm_peak: float):
    """The GPU quantize_per_channel on a [32768, 3584] fp32 matrix (470 MB in, > L2), median of
    `iters` launches timed with events; bytes = 4NK read + NK + 4N written."""
    import torch

    R, K = 32768, HIDDEN
    w = torch.randn(R, K, device=dev) * 0.02
    q = torch.empty(R, K, dtype=torch.int8, device=dev)
    s = torch.empty(R, device=dev)
    stream = torch.cuda.current_stream(dev)
    v.quantize_per_channel(w, q, s, stream=stream)
    ms = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        v.quantize_per_channel(w, q, s, stream=stream)
        b.record(stream)
        b.synchronize()
        ms.append(a.elapsed_time(b))
    t = statistics.median(ms)
    nbytes = 5 * R * K + 4 * R
    gbs = nbytes / (t * 1e-3) / 1e9
    del w, q, s
    return {"value": round(gbs, 1), "unit": "GB/s", "frac": round(gbs / hbm_peak, 4), "us": round(t * 1e3, 2),
            "shape": f"[{R}, {K}] fp32 -> int8 + fp32 scales"}


def profile_case(args):
    """Small single-projection run for ncu: warmup + 1 launches of one linear_q8 on one GPU.
    Weights are random int8 made with one torch launch (values do not change the memory traffic)."""
    import torch

    import vvllm_b200 as v

    name, _, m = args.profile_case.partition(":")
    M = int(m) if m else 1
    if "x" in name:  # explicit N x K (e.g. "4864x896:512", a prefill GEMM of benchmark config 4)
        N, K = (int(v) for v in name.split("x"))
    else:
        N, K = {n: (N, K) for n, N, K in PROJ}[name]
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    q = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev)
    s = torch.rand(N, device=dev) * 1e-3
    x = torch.randn(M, K, device=dev).half()
    out = torch.empty(M, N, device=dev, dtype=torch.float16)
    for _ in range(args.warmup + 1):
        v.linear_q8(out, x, q, s)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": name, "M": M, "N": N, "K": K,
                      "algorithmic_bytes": algo_bytes(N, K, M), "launches": args.warmup + 1}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--cpu-sample-mb", type=float, default=0.0,
                    help="int8 weight MB the CPU legs stream per pass (default: 2x the host's LLC, >= 64 MB)")
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU baseline timing")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-case", default=None,
                    help="run one projection (gate_up|down|lm_head, optional :M) warmup+1 times for ncu")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.profile_case:
        return profile_case(args)

    import torch
    import torch.distributed as dist

    import vvllm_b200 as v

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        args.gpus = world
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    hbm_peak, tc_peak, peak_kind = peaks()

    # ---- weights (per rank shard), made and quantized on the device -------------------------
    gen = torch.Generator(device=dev)
    shards = []
    for pi, (name, N, K) in enumerate(PROJ):
        r0, rows = v.shard_range(N, world, rank)
        q = torch.empty((rows, K), dtype=torch.int8, device=dev)
        s = torch.empty((rows,), dtype=torch.float32, device=dev)
        step = 8192
        for a in range(0, rows, step):  # quantize in slabs to bound the fp32 staging memory
            b = min(rows, a + step)
            gen.manual_seed(1000 + 16 * 28 + pi * 1000003 + r0 + a)
            w = torch.randn((b - a, K), generator=gen, device=dev) * 0.02
            v.quantize_per_channel(w, q[a:b], s[a:b])
        shards.append((name, N, K, r0, rows, q, s))
    torch.cuda.synchronize()
    per_rank_bytes = sum(algo_bytes(rows, K) for _, _, K, _, rows, _, _ in shards)
    copies = max(1, math.ceil(2 * L2_BYTES / per_rank_bytes))
    sets = [[(q, s) for (_, _, _, _, _, q, s) in shards]]
    for _ in range(copies - 1):
        sets.append([(q.clone(), s.clone()) for (_, _, _, _, _, q, s) in shards])
    xs = [torch.randn((1, K), generator=gen, device=dev).half() for (_, _, K, _, _, _, _) in shards]
    per = [-(-N // world) for (_, N, _, _, _, _, _) in shards]
    outs = [torch.empty((1, p * world), dtype=torch.float16, device=dev) for p in per]

    comm = None
    sym = None
    if world > 1:
        uid = [v.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = v.Comm(local, world, rank, uid[0], timeout_s=120.0)
        # Outputs of the fused gather: [1, N] fp16 each, in one symmetric allocation that
        # every peer has mapped (256-byte aligned slots); two sets of slots, one per step parity
        # of the end-to-end leg (the timed loop uses set 0).
        offs, o = [], 0
        for (_, N, _, _, _, _, _) in shards:
            offs.append(o)
            o += -(-N * 2 // 256) * 256
        sym = comm.sym_alloc(2 * o)
        sym_sets = [[sym[h * o + a:h * o + a + 2 * N].view(torch.float16).view(1, N)
                     for a, (_, N, _, _, _, _, _) in zip(offs, shards)] for h in range(2)]
        sym_src = [sym[h * o:(h + 1) * o].view(torch.float16) for h in range(2)]
        p2p_outs = sym_sets[0]

    # Every leg runs on one dedicated stream (a CUDA graph cannot be captured on the legacy
    # default stream, and the library keeps its scratch per stream).
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    torch.cuda.set_stream(stream)
    lm_idx = [n for n, *_ in PROJ].index("lm_head")

    def step(it, ev=None, mode="p2p"):
        """mode: "p2p" = gather fused into the GEMV (the product path for N > 1);
        "nccl" = GEMV then NCCL all-gather; "local" = GEMV only (no gather)."""
        ws = sets[it % copies]
        for i, (name, N, K, r0, rows, _, _) in enumerate(shards):
            q, s = ws[i]
            if ev is not None and i == lm_idx:
                ev[0].record(stream)
            if comm is not None and mode == "p2p":
                # each call's completion wait is paid by the next gathered call (inside its GEMV
                # when it can) or by the Comm.wait() that ends the timed region
                v.linear_q8_sharded_p2p(comm, p2p_outs[i], xs[i], q, s, None, N, stream=stream,
                                        defer_wait=True)
            else:
                slot = outs[i][:, rank * per[i]: rank * per[i] + rows]
                v.linear_q8(slot, xs[i], q, s, None, stream=stream)
            if ev is not None and i == lm_idx:
                ev[1].record(stream)
            if comm is not None and mode == "nccl":
                comm.allgather(outs[i], per[i], v.F16, stream=stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # SM clocks are sampled from the first warm-up step to the end of the last GPU leg.
    sampler = ClockSampler(local)
    sampler.__enter__()
    for it in range(args.warmup):
        step(it)
    if comm is not None:
        comm.wait(stream)
    barrier()

    # The K timed steps are one CUDA graph, captured once and replayed once inside the timed
    # region: a serving loop replays its decode step the same way, and the host's per-call
    # launch cost (Python + ctypes + the library, measured below as host_us_per_step) no longer
    # leaves the GPU idle between the small per-rank projections at N > 1.  The gathered calls
    # carry no host-side state into the kernels (relative completion counts), so the replay runs
    # the same protocol as direct calls.  Nothing else is in the timed region.
    def capture(mode, n):
        g = torch.cuda.CUDAGraph()
        l0 = v.launch_count()
        with torch.cuda.graph(g, stream=stream):
            for it in range(n):
                step(it, mode=mode)
            if comm is not None and mode == "p2p":
                comm.wait(stream)
        return g, v.launch_count() - l0

    graph, n_launch = capture("p2p", args.steps)
    graph.replay()  # warm the graph's first launch
    barrier()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    win0 = time.monotonic()
    t_start.record(stream)
    graph.replay()
    t_end.record(stream)
    barrier()
    win1 = time.monotonic()
    ms = t_start.elapsed_time(t_end)
    del graph
    # The host's cost of issuing one step by direct calls (no graph): wall time of the enqueue loop.
    h0 = time.perf_counter()
    for it in range(args.steps):
        step(it)
    if comm is not None:
        comm.wait(stream)
    host_us = (time.perf_counter() - h0) / args.steps * 1e6
    barrier()
    # The lm_head roofline: the same K steps again, events around each lm_head launch (live, on
    # the launching stream; these events cost the steps their overlap, not the lm_head launch).
    lm_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                 for _ in range(args.steps)]
    barrier()
    for it in range(args.steps):
        step(it, lm_events[it])
    if comm is not None:
        comm.wait(stream)
    barrier()
    lm_ms = statistics.mean(a.elapsed_time(b) for a, b in lm_events)

    # ---- N > 1 parity: every rank's gathered outputs (the last step's, in the symmetric buffers)
    # ---- against each rank's rows computed locally by the same digit GEMV, gathered by NCCL ------
    parity = None
    if comm is not None:
        same = 1
        for i, (name, N, K, r0, rows, _, _) in enumerate(shards):
            q, s = sets[0][i]
            loc = torch.empty((1, per[i] * world), dtype=torch.float16, device=dev)
            mine = loc[:, rank * per[i]:rank * per[i] + per[i]]
            v.linear_q8(mine[:, :rows], xs[i], q, s, stream=stream)
            full = torch.empty((1, per[i] * world), dtype=torch.float16, device=dev)
            dist.all_gather_into_tensor(full, mine.contiguous())
            same &= int(torch.equal(full[:, :N], p2p_outs[i]))
        flag = torch.tensor([same], device=dev, dtype=torch.int32)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        parity = {"ok": bool(flag.item()), "ranks": world,
                  "check": "every rank's gathered [1, N] outputs of the last timed step equal, bit for bit, "
                           "each rank's rows computed by the local dispatch (the kernel the gathered call runs "
                           "per shard) and all-gathered by NCCL; those kernels are checked against the "
                           "reference in tests/"}
    if world > 1:
        t = torch.tensor([ms, lm_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, lm_ms = t.tolist()
    ms_step = ms / args.steps
    total_bytes = sum(algo_bytes(N, K) for _, N, K in PROJ)  # whole job, all ranks
    value = total_bytes / (ms_step * 1e-3) / 1e9
    lm_rows = shards[lm_idx][4]
    lm_bytes = algo_bytes(lm_rows, HIDDEN)
    lm_gbs = lm_bytes / (lm_ms * 1e-3) / 1e9

    # ---- N > 1: the same steps without any gather (compute share of the step) and with the
    # ---- GEMV followed by a separate NCCL all-gather (the unfused alternative) ---------------
    compute_only = nccl_leg = None
    if comm is not None:
        def leg(mode):
            for it in range(args.warmup):
                step(it, mode=mode)
            barrier()
            g, _ = capture(mode, args.steps)
            g.replay()
            barrier()
            c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            c0.record(stream)
            g.replay()
            c1.record(stream)
            barrier()
            del g  # a graph holding NCCL calls is released before the process group
            t = torch.tensor([c0.elapsed_time(c1)], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            c_ms = t.item()
            return {"value": round(total_bytes / (c_ms / args.steps * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(c_ms / args.steps, 5)}

        compute_only = leg("local")
        nccl_leg = leg("nccl")

    # ---- end to end through the C ABI with host buffers -------------------------------------
    # Each step copies its activations in (one pinned host -> device copy of all three inputs)
    # and its outputs out (one device -> pinned host copy of all three outputs).  The copies run
    # on their own streams, double-buffered and ordered by events, so step i's copies overlap its
    # neighbours' projections, as a serving loop would run them.  Input and output copies take
    # separate streams: on one stream the next step's input copy would queue behind this step's
    # wait for its projections, and the copies would serialise with them again.  At N > 1 the
    # outputs are two sets of symmetric slots that the peers write: a peer runs at most one
    # gathered call ahead of this rank (each call waits for every rank's part of the previous
    # one), so holding this rank's last call of step i + 1 until step i's outputs are in host
    # memory keeps every peer off that set until then.
    Ks = [K for (_, _, K, _, _, _, _) in shards]
    nbuf = 2
    h_in = torch.empty((sum(Ks),), dtype=torch.float16).pin_memory()
    o = 0
    for K, x in zip(Ks, xs):
        h_in[o:o + K].copy_(x.view(-1).cpu())
        o += K
    d_in_all = [torch.empty((sum(Ks),), dtype=torch.float16, device=dev) for _ in range(nbuf)]
    d_in = [[d_in_all[b][o0:o0 + K].view(1, K) for o0, K in zip([sum(Ks[:i]) for i in range(len(Ks))], Ks)]
            for b in range(nbuf)]
    if comm is None:
        Ns = [N for (_, N, _, _, _, _, _) in shards]
        out_src = [torch.empty((sum(Ns),), dtype=torch.float16, device=dev) for _ in range(nbuf)]
        d_outs = [[out_src[b][o0:o0 + N].view(1, N) for o0, N in zip([sum(Ns[:i]) for i in range(len(Ns))], Ns)]
                  for b in range(nbuf)]
    else:
        out_src = sym_src
        d_outs = sym_sets
    h_out = [torch.empty(out_src[0].shape, dtype=torch.float16).pin_memory() for _ in range(nbuf)]
    h2d = h_in.numel() * 2
    d2h = h_out[0].numel() * 2
    in_stream = torch.cuda.Stream(device=dev)
    out_stream = torch.cuda.Stream(device=dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_ready = [ev() for _ in range(nbuf)]   # input copy b landed
    out_done = [ev() for _ in range(nbuf)]   # output copy b read out (buffers b free again)
    comp_done = [ev() for _ in range(nbuf)]  # projections of buffer b finished

    def e2e_step(it):
        ws = sets[it % copies]
        b = it % nbuf
        if it >= nbuf:
            in_stream.wait_event(out_done[b])  # buffer b's previous step is fully done
        with torch.cuda.stream(in_stream):
            d_in_all[b].copy_(h_in, non_blocking=True)
        in_ready[b].record(in_stream)
        stream.wait_event(in_ready[b])
        for i, (name, N, K, r0, rows, _, _) in enumerate(shards):
            q, s = ws[i]
            if comm is None:
                v.linear_q8(d_outs[b][i], d_in[b][i], q, s, None, stream=stream)
            else:
                if i == len(shards) - 1 and it >= 1:
                    # the other set's outputs (step it - 1) are in host memory before this call
                    # lets any peer start step it + 1 into that set
                    stream.wait_event(out_done[(it - 1) % nbuf])
                v.linear_q8_sharded_p2p(comm, d_outs[b][i], d_in[b][i], q, s, None, N, stream=stream,
                                        defer_wait=True)
        if comm is not None:
            comm.wait(stream)  # every gathered output complete before the copy out
        comp_done[b].record(stream)
        out_stream.wait_event(comp_done[b])
        with torch.cuda.stream(out_stream):
            h_out[b].copy_(out_src[b], non_blocking=True)
        out_done[b].record(out_stream)

    def e2e_drain():
        for b in range(nbuf):
            stream.wait_event(out_done[b])  # the last outputs are in host memory

    for it in range(args.warmup):
        e2e_step(it)
    e2e_drain()
    barrier()
    # The K steps (copies, projections, events between the three streams) are captured as one
    # CUDA graph, like the device-only leg; the copy streams fork from the capture stream, so no
    # copy of the replay starts before the timed region begins.
    eg = torch.cuda.CUDAGraph()
    with torch.cuda.graph(eg, stream=stream):
        in_stream.wait_stream(stream)
        out_stream.wait_stream(stream)
        for it in range(args.steps):
            e2e_step(it)
        e2e_drain()
    eg.replay()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    eg.replay()
    e1.record(stream)
    barrier()
    del eg
    e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = t.item()
    e2e_value = total_bytes / (e_ms / args.steps * 1e-3) / 1e9

    # ---- benchmark config 5 at M = 8 and 64 tokens, configs 1-4, and the GPU quantize (rank 0, N = 1) ----
    prefill = stacks = cfg1 = quant = None
    tokens = {}
    if world == 1:
        for M in (8, 64):
            xm = [torch.randn((M, K), generator=gen, device=dev).half() for (_, _, K, _, _, _, _) in shards]
            om = [torch.empty((M, rows), dtype=torch.float16, device=dev) for (_, _, _, _, rows, _, _) in shards]

            def tok_step(it, xm=xm, om=om):
                ws = sets[it % copies]
                for i in range(len(shards)):
                    q, s = ws[i]
                    v.linear_q8(om[i], xm[i], q, s, None, stream=stream)

            nsteps = max(20, args.steps // 4)
            for it in range(args.warmup):
                tok_step(it)
            barrier()
            g = torch.cuda.CUDAGraph()  # the steps as one graph, like the headline
            with torch.cuda.graph(g, stream=stream):
                for it in range(nsteps):
                    tok_step(it)
            g.replay()
            barrier()
            c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            c0.record(stream)
            g.replay()
            c1.record(stream)
            barrier()
            del g
            t_step = c0.elapsed_time(c1) / nsteps
            nb = sum(algo_bytes(N, K, M) for _, N, K in PROJ)
            gbs = nb / (t_step * 1e-3) / 1e9
            tokens[f"M{M}"] = {"value": round(gbs, 1), "unit": "GB/s", "frac": round(gbs / hbm_peak, 4),
                               "us_per_step": round(t_step * 1e3, 2),
                               "TFLOP/s": round(sum(2.0 * M * N * K for _, N, K in PROJ) / (t_step * 1e-3) / 1e12, 1),
                               "timing": "one CUDA-graph replay of the steps",
                               # the library's automatic choice (b200q8.h, B200Q8_ALGO_AUTO)
                               "kernels": {n: ("q8_gemv_dig_kernel (int8 tensor cores)"
                                               if M <= 4 or (M <= 8 and N >= 16384)
                                               else "q8_gemm_sk_kernel (fp16 tensor cores)") for n, N, _ in PROJ}}
            del xm, om
        cfg1 = config1_gemv(v, dev, args.warmup, max(20, args.steps // 4), hbm_peak)
        prefill = prefill_tflops(v, dev, stream, args.warmup, max(5, args.steps // 10), tc_peak)
        stacks = decode_stacks(v, dev, args.warmup, max(10, args.steps // 10), hbm_peak)
        quant = gpu_quantize(v, dev, max(5, args.steps // 20), hbm_peak)
    sampler.__exit__(None, None, None)

    # ---- CPU baseline: the reference's linear_q8 on the host cores (rank 0, N = 1), and the
    # ---- parity check of this run's outputs against it on a row sample of every projection ------
    cpu_baseline = None
    if world == 1 and not args.no_cpu_baseline:
        lib, kind = cpu_reference_lib()
        model, cores = cpu_info()
        want = cpu_sample_bytes(args.cpu_sample_mb)
        shapes, frac = host_sample_weights(want)
        gbs, sec, iters = time_cpu_linear(lib, shapes, cores, args.cpu_budget)
        sb = sum(algo_bytes(q.shape[0], q.shape[1], 1, 4, 4) for _, q, _ in shapes)
        # the reference runs single-threaded: time that too, on the same working set
        gbs1, sec1, iters1 = time_cpu_linear(lib, shapes, 1, args.cpu_budget / 2)
        del shapes
        cq = cpu_quantize(lib, want, args.cpu_budget / 2)
        if quant is not None:
            quant["cpu_reference_single_thread"] = cq
        llc = llc_bytes()
        cpu_baseline = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind,
                        "sample": f"{frac:.3f} of each projection's rows ({sb / 1e6:.1f} MB algorithmic, "
                                  f"host LLC {llc / 2**20:.0f} MiB), {iters} passes in {sec * iters:.1f} s, "
                                  f"{cores} threads (disjoint output-row slices); CPU: {model}",
                        "single_thread": {"value": round(gbs1, 3), "unit": "GB/s", "cores": 1,
                                          "sample": f"the same rows, {iters1} passes in {sec1 * iters1:.1f} s"}}
        # parity: 64 sampled output channels of every projection (first, middle and last included),
        # this run's GPU outputs of the last timed step against the reference's linear_q8 on the
        # same int8 rows, scales and (fp16-widened) activations
        worst = 0.0
        for i, (name, N, K, r0, rows, q, s) in enumerate(shards):
            pick = sorted(set(np.random.default_rng(11 + i).choice(N, size=61, replace=False).tolist())
                          | {0, N // 2, N - 1})
            idx = torch.tensor(pick, device=dev)
            qh = q.index_select(0, idx).cpu().numpy()
            sh = s.index_select(0, idx).cpu().numpy()
            xh = xs[i].float().cpu().numpy()
            ref = lib.linear_q8(xh, np.ascontiguousarray(qh), np.ascontiguousarray(sh), None)[0]
            got = outs[i][0].index_select(0, idx).float().cpu().numpy()
            den = float(np.max(np.abs(ref)))
            worst = max(worst, float(np.max(np.abs(got - ref))) / den if den > 0 else float(np.max(np.abs(got))))
        parity = {"ok": worst <= 2e-3, "max_normwise_err": worst, "tol": 2e-3,
                  "check": f"64 output channels of each projection, this run's fp16 outputs against the {kind} "
                           f"CPU linear_q8 on the same int8 rows and fp16-widened activations"}

    if rank == 0:
        traffic = profiled_traffic("q8_gemv_dig_lm_head_7b") if world == 1 else None
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8 weights x f16 activations, f32 accumulate", "data": "synthetic",
            "config": {"workload": WORKLOAD, "M": 1, "activations": "fp16", "parallelism": f"column-shard x{world}",
                       "collective": "gather fused into the GEMV (peer stores over NVLink)" if world > 1
                       else "none",
                       "l2": f"{copies} rotating weight set(s), {copies * per_rank_bytes / 1e6:.0f} MB per rank per cycle (> L2)"},
            "roofline": {"bound": "hbm", "kernel": "q8_gemv_dig_kernel (lm_head shard)", "achieved": round(lm_gbs, 2),
                         "peak": hbm_peak, "unit": "GB/s", "frac": round(lm_gbs / hbm_peak, 4),
                         "peak_kind": peak_kind, "traffic": traffic,
                         "algorithmic_bytes_per_launch": lm_bytes, "launch_ms": round(lm_ms, 5)},
            "pct_of_hbm_peak": round(100 * value / (hbm_peak * world), 2),
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e_ms / args.steps, 5)},
            "gpu_launches": int(n_launch),
            "timing": "the K steps captured as one CUDA graph and replayed once between CUDA events "
                      "(barrier + synchronize on both sides, max over ranks)",
            "host_us_per_step": round(host_us, 2),
            "clocks": sampler.summary((win0, win1)),
            "parity": parity,
        }
        if compute_only is not None:
            line["compute_only"] = compute_only
        if nccl_leg is not None:
            line["gemv_then_nccl_allgather"] = nccl_leg
        if tokens:
            line["tokens"] = tokens
        if cfg1 is not None:
            line["config1_gemv_fp32"] = cfg1
        if quant is not None:
            line["quantize"] = quant
        if prefill is not None:
            line["prefill"] = prefill
        if stacks is not None:
            line["decode_stacks"] = stacks
        if cpu_baseline is not None:
            line["cpu_baseline"] = cpu_baseline
        print(json.dumps(line), flush=True)

    if comm is not None:
        torch.cuda.synchronize()
        del p2p_outs, sym_sets, sym_src, sym, d_outs, out_src
        comm.destroy()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
