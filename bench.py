#!/usr/bin/env python
"""Benchmark of the four-op hot path on B200; prints ONE JSON line (rank 0).

Headline workload (N=1): swiglu at the Llama-3-8B MLP shape, x [4096, 4096], w1/w3
[4096, 14336] fp16 (seed 1), metric TFLOP/s = 4*M*N*K / time. With N GPUs (torchrun, one
process per GPU) the same problem is column-sharded over N (each rank computes
out[:, N/g slice]); the GEMM epilogue stores each tile once through an NVLink multicast
address, so the NVSwitch writes it into every rank's [M, N] output (torch symmetric memory;
without multicast: into each rank's output over NVLink, CUDA IPC peer buffers), and
synchronises with the peers inside the kernel, or with --comm nccl the slices are
all-gathered (strong scaling). At N>1 every rank checks 256
sampled rows of its gathered output bit for bit against the single-GPU operator.

Also on the line:
* "ops" (N=1): the other three operators at their configurations (rmsnorm_rope,
  flash_attention causal/non-causal, paged_attention decode) and the extensions, each with a
  roofline; the four reference operators also with a CPU baseline (the oracle on the host
  cores, sampled and extrapolated where the full problem is too large) and an end-to-end
  figure through the public operator with pinned host inputs and result copied every step.
* "sharded_cfg5" (every N): the Llama-3-70B-shaped sharded workloads -- swiglu
  x [8192, 8192], w [8192, 28672] column-sharded with the output gathered; causal
  flash_attention [8, 64, 8192, 128] head-sharded; paged decode B256 H64 D128 bs32, lens
  U[1024, 32768], batch-sharded over a token-balanced partition -- whole-job throughput from
  the max-over-ranks device time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the CPU oracle (a numpy restatement of the reference's
python/triton_llm/reference/swiglu.py) on the host cores on a bounded row sample of the same
workload; under torchrun only rank 0 runs it.
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
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# Measured peer-copy rate per direction per GPU over NVLink on this pool (nominal 900 GB/s).
NVLINK_GBS = 770.0
SWIGLU_SHAPE = (4096, 4096, 14336)  # M, K, N
CFG5_SWIGLU = (8192, 8192, 28672)  # M, K, N
CFG5_FLASH = (8, 64, 8192, 128)  # B, H, S, D (causal)
CFG5_PAGED = (256, 64, 128, 32, 1024, 32768)  # B, H, D, block_size, min len, max len
L2_FLUSH_BYTES = 256 << 20
PARITY_ROWS = (1920, 2176)  # sampled row block of the headline output


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-ops", action="store_true", help="skip the per-operator extras")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline legs")
    ap.add_argument("--no-cfg5", action="store_true", help="skip the 70B-shaped sharded workloads")
    ap.add_argument("--chunks", type=int, default=1,
                    help="N>1 with --comm nccl: row chunks whose all-gather overlaps the next GEMM")
    ap.add_argument("--e2e-chunks", type=int, default=8,
                    help="column blocks of the 1-GPU end-to-end host pipeline")
    ap.add_argument("--comm", choices=["auto", "multicast", "peers", "nccl"], default="peers",
                    help="N>1: multicast = the GEMM epilogue stores each tile once through an "
                         "NVLink multicast address (NVSwitch writes every rank's output); peers "
                         "= it stores into every rank's output over NVLink; nccl = "
                         "all_gather_into_tensor + permute; auto = multicast where the devices "
                         "offer it, else peers")
    ap.add_argument("--op", choices=sorted(OP_CASES), default=None,
                    help="run only this operator case (steps+warmup launches) and print its timing")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {k: float(p[k]) for k in FALLBACK_PEAKS}, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(name: str):
    """Bytes per launch recorded in a committed ncu summary (line 'traffic_bytes_per_launch: N')."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(path):
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples the SM clock and clock-event (throttle) reasons while the timed region runs.

    NVML is read from a background thread every millisecond (a timed region of a few tens
    of milliseconds would fall between nvidia-smi's 200 ms samples); nvidia-smi is the
    fallback when NVML is unavailable. Only samples taken while the GPU reports activity
    (not the GpuIdle reason) count.
    """

    NAMES = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
             "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
             "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
             "sw_power_cap": "nvmlClocksEventReasonSwPowerCap",
             "hw_power_brake": "nvmlClocksEventReasonHwPowerBrakeSlowdown"}

    def __init__(self, index: int):
        self.index = index
        self.samples = []  # (sm_mhz, reasons bitmask)
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)

            def loop():
                while not self._stop.is_set():
                    try:
                        mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((mhz, rs))
                    except Exception:
                        pass
                    time.sleep(0.001)

            self._thread = threading.Thread(target=loop, daemon=True)
            self._thread.start()
        except Exception:
            self._nvml = None
        time.sleep(0.01)
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self):
        if self._nvml is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        pm = self._nvml
        idle = getattr(pm, "nvmlClocksEventReasonGpuIdle", 1)
        busy = [(m, r) for m, r in self.samples if not (r & idle)] or self.samples
        reasons = sorted(n for n, attr in self.NAMES.items()
                         if any(r & getattr(pm, attr, 0) for _, r in busy))
        return {"sm_mhz": statistics.median(m for m, _ in busy), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(busy), "source": "NVML, 1 ms"}


# ------------------------------------------------------------------------------------------
def _events_time(torch, fn, steps, warmup, flush=None):
    """Runs fn() warmup+steps times; returns per-step device milliseconds (CUDA events on the
    current stream), flushing L2 between timed steps when `flush` is given."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    st = torch.cuda.current_stream()
    for _ in range(steps):
        if flush is not None:
            flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(st)
        fn()
        b.record(st)
        times.append((a, b))
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in times]


# ------------------------------------------------------------------------------------------
# CPU baselines: the oracle (a numpy restatement of the reference's own *_ref functions) on
# the host cores, on seeded inputs of the workload's shapes and distributions.
def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def _blas_threads(n: int):
    """Context setting the BLAS pool to n threads (torchrun starts ranks with one)."""
    try:
        from threadpoolctl import threadpool_limits

        return threadpool_limits(limits=n, user_api="blas")
    except Exception:
        import contextlib

        return contextlib.nullcontext()


def _normal_f16(rng, shape, scale=1.0, reservoir=1 << 22):
    """fp16-representable float32 array of N(0, scale^2) values. Large arrays repeat a seeded
    reservoir (values only feed timing samples there)."""
    import numpy as np

    from oracle import ops_oracle as O

    n = int(np.prod(shape))
    if n <= reservoir:
        return O.round_to(rng.standard_normal(shape, dtype=np.float32) * np.float32(scale), "fp16")
    base = O.round_to(rng.standard_normal(reservoir, dtype=np.float32) * np.float32(scale), "fp16")
    return np.resize(base, shape)


def _parallel(items, fn, threads):
    """fn over items on `threads` Python threads (numpy releases the GIL in BLAS and ufuncs),
    BLAS limited to one thread each; returns the wall time."""
    from concurrent.futures import ThreadPoolExecutor

    with _blas_threads(1):
        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(fn, items))
        return time.perf_counter() - t0


def cpu_swiglu_inputs(rows=512, shape=SWIGLU_SHAPE, cols=None, seed=1):
    """A row (and optionally column) sample of a swiglu workload for the CPU oracle."""
    import numpy as np

    M, K, N = shape
    n = N if cols is None else cols
    rng = np.random.default_rng(seed)
    x = _normal_f16(rng, (rows, K))
    w1 = _normal_f16(rng, (K, n), 1.0 / math.sqrt(K))
    w3 = _normal_f16(rng, (K, n), 1.0 / math.sqrt(K))
    return x, w1, w3


def cpu_swiglu_baseline(inputs=None, min_seconds=5.0, rows=512, shape=SWIGLU_SHAPE):
    """Times the numpy oracle on a bounded sample of a swiglu workload (BLAS on all cores)."""
    from oracle import ops_oracle as O

    M, K, N = shape
    x, w1, w3 = inputs if inputs is not None else cpu_swiglu_inputs(rows, shape)
    x = x[:rows]
    cores = cpu_cores()
    with _blas_threads(cores):
        O.swiglu(x[:16], w1, w3)  # warm the BLAS thread pool
        reps, t0 = 0, time.perf_counter()
        while True:
            O.swiglu(x, w1, w3)
            reps += 1
            el = time.perf_counter() - t0
            if (el >= min_seconds and reps >= 2) or reps >= 50:
                break
    flops = 4.0 * x.shape[0] * K * w1.shape[1] * reps
    return {"value": flops / el / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{reps} x numpy-oracle swiglu on {x.shape[0]} of {M} rows and "
                      f"{w1.shape[1]} of {N} columns (K={K}), {el:.1f} s; rate extrapolated "
                      f"to the full workload",
            "seconds_per_rep": el / reps}


def cpu_rmsnorm_baseline(shape=(2, 128, 8, 64), min_seconds=2.0):
    """The rmsnorm_rope oracle on the full (small) configuration; numpy elementwise work runs
    on one core."""
    import numpy as np

    from oracle import ops_oracle as O

    b, s, h, d = shape
    rng = np.random.default_rng(0)
    x = _normal_f16(rng, shape)
    w = O.round_to(1 + 0.1 * rng.standard_normal(d, dtype=np.float32), "fp16")
    pos = np.arange(s, dtype=np.float32)
    inv = 1.0 / (10000 ** (np.arange(0, d, 2, dtype=np.float32) / d))
    emb = np.concatenate([np.outer(pos, inv)] * 2, axis=-1)
    cos, sin = O.round_to(np.cos(emb), "fp16"), O.round_to(np.sin(emb), "fp16")
    nbytes = 2 * (b * s * h * d * 2) + d * 2 + 2 * (s * d * 2)
    reps, t0 = 0, time.perf_counter()
    while True:
        O.rmsnorm_rope(x, w, cos, sin)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds and reps >= 3:
            break
    return {"value": nbytes * reps / el / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"full configuration {list(shape)}, {reps} calls in {el:.1f} s "
                      f"(numpy elementwise: one core)"}


def cpu_flash_baseline(b, h, s, d, causal, heads, threads=None):
    """The flash_attention oracle on `heads` of the b*h heads (one head per thread at a time),
    rate extrapolated to the whole problem."""
    import numpy as np

    from oracle import ops_oracle as O

    threads = threads or cpu_cores()
    heads = max(heads, min(threads, b * h))
    rng = np.random.default_rng(2)
    qkv = [tuple(_normal_f16(rng, (1, 1, s, d)) for _ in range(3)) for _ in range(heads)]
    el, reps = 0.0, 0
    while el < 2.0 and reps < 20:
        el += _parallel(qkv, lambda t: O.flash_attention(*t, causal=causal), min(threads, heads))
        reps += 1
    flops_head = 4.0 * s * s * d * (0.5 if causal else 1.0)
    return {"value": flops_head * heads * reps / el / 1e12, "unit": "TFLOP/s",
            "cores": min(threads, heads), "kind": "port",
            "sample": f"{reps} x {heads} of {b * h} heads [S={s}, D={d}{', causal' if causal else ''}] "
                      f"in {el:.1f} s, one head per thread; extrapolated to the full problem"}


def cpu_paged_baseline(lens, h, d, bs, threads=None):
    """The paged_attention oracle on the sequences of `lens` (one sequence per thread at a
    time), each with its own block pool; GB/s of the algorithmic bytes."""
    import numpy as np

    from oracle import ops_oracle as O

    threads = threads or cpu_cores()
    rng = np.random.default_rng(3)
    cases = []
    nbytes = 0
    for n in lens:
        nb = (n + bs - 1) // bs
        kc = _normal_f16(rng, (nb, bs, h, d)).astype(np.float16)
        vc = _normal_f16(rng, (nb, bs, h, d)).astype(np.float16)
        q = _normal_f16(rng, (1, h, 1, d))
        bt = np.arange(nb, dtype=np.int32)[None]
        cases.append((q, kc, vc, bt, np.array([n], np.int32)))
        nbytes += n * h * d * 2 * 2 + 2 * h * d * 2 + nb * 4 + 4
    el, reps = 0.0, 0
    while el < 2.0 and reps < 20:
        el += _parallel(cases, lambda c: O.paged_attention(*c, block_size=bs), min(threads, len(lens)))
        reps += 1
    return {"value": nbytes * reps / el / 1e9, "unit": "GB/s", "cores": min(threads, len(lens)),
            "kind": "port",
            "sample": f"{reps} x {len(lens)} sequences (lengths {min(lens)}..{max(lens)}, H={h}, "
                      f"D={d}, block {bs}) in {el:.1f} s, one sequence per thread; extrapolated"}


# Single-operator cases (used to profile one kernel at a time from committed code).
OP_CASES = {
    "swiglu": "swiglu M4096 K4096 N14336 fp16",
    "flash_causal": "flash_attention causal [4,32,4096,128] fp16",
    "flash_full": "flash_attention non-causal [4,32,1024,128] fp16",
    "paged": "paged_attention decode B64 H32 D128 bs16 lens U[512,8192] fp16",
    "paged_small": "paged_attention decode B16 H32 D128 bs16 lens U[512,8192] fp16",
    "rmsnorm": "rmsnorm_rope [2,128,8,64] fp16",
    "rmsnorm_bw": "rmsnorm_rope [16,4096,32,128] fp16",
    "gqa_decode": "paged_attention_prefill GQA decode B64 Hq32 Hkv8 Sq1 D128 bs16 lens U[512,8192] fp16",
    "gqa_spec4": "paged_attention_prefill GQA 4-token decode B64 Hq32 Hkv8 Sq4 D128 bs16 lens U[512,8192] fp16",
    "gqa_chunk": "paged_attention_prefill causal chunk B8 Hq32 Hkv8 Sq512 ctx4096 D128 bs16 fp16",
    "kv_append_rope": "paged_kv_append_rope B16 T2048 H8 D128 bs16 fp16",
    "flash_varlen": "flash_attention_varlen causal 16 sequences U[256,4096] H32 D128 fp16",
    "flash_bwd": "flash_attention_backward causal [4,32,4096,128] fp16",
    "swiglu_fp8": "swiglu_fp8 e4m3 M4096 K4096 N14336, fp16 out",
    "flash_fp8_causal": "flash_attention_fp8 e4m3 causal [4,32,4096,128], fp16 out",
    "qkv_norm_rope": "qkv_norm_rope M4096 K4096 Hq32 Hkv8 D128 fp16 (Llama-3-8B QKV)",
    "swiglu_colshard8_local": "column-sharded swiglu kernel of one of 8 ranks (M4096 K4096 N/8=1792), "
                              "its 8 destination slices all on this GPU (no peer handshake)",
}


def _paged_inputs(torch, batch, seed=3):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(512, 8193, (batch,), dtype=torch.int32, generator=g)
    nb = [(int(n) + 15) // 16 for n in lens]
    pool = sum(nb)
    perm = torch.randperm(pool, generator=g)
    bt = torch.zeros(batch, max(nb), dtype=torch.int32)
    pos = 0
    for i, n in enumerate(nb):
        bt[i, :n] = perm[pos:pos + n].to(torch.int32)
        pos += n
    gd = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn((pool, 16, 32, 128), generator=gd, device="cuda").half()
    vc = torch.randn((pool, 16, 32, 128), generator=gd, device="cuda").half()
    q = torch.randn((batch, 32, 1, 128), generator=gd, device="cuda").half()
    nbytes = int(lens.sum()) * 32 * 128 * 2 * 2 + 2 * batch * 32 * 128 * 2 + sum(nb) * 4 + batch * 4
    return q, kc, vc, bt.cuda(), lens.cuda(), nbytes


def _gqa_inputs(torch, batch, hq, hkv, sq, lens=None, seed=3):
    """Paged GQA case: lens U[512,8192] (seed 3, as the decode case) unless given."""
    g = torch.Generator().manual_seed(seed)
    if lens is None:
        lens = torch.randint(512, 8193, (batch,), dtype=torch.int32, generator=g)
    nb = [(int(n) + 15) // 16 for n in lens]
    pool = sum(nb)
    perm = torch.randperm(pool, generator=g)
    bt = torch.zeros(batch, max(nb), dtype=torch.int32)
    pos = 0
    for i, n in enumerate(nb):
        bt[i, :n] = perm[pos:pos + n].to(torch.int32)
        pos += n
    gd = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn((pool, 16, hkv, 128), generator=gd, device="cuda").half()
    vc = torch.randn((pool, 16, hkv, 128), generator=gd, device="cuda").half()
    q = torch.randn((batch, hq, sq, 128), generator=gd, device="cuda").half()
    kv_bytes = int(lens.sum()) * hkv * 128 * 2 * 2
    nbytes = kv_bytes + 2 * batch * hq * sq * 128 * 2 + sum(nb) * 4 + batch * 4
    # causal FLOPs: query s of a sequence of length n sees n - sq + s + 1 keys
    keys = sum(sq * int(n) - sq * (sq - 1) // 2 for n in lens)
    flops = 4.0 * hq * 128 * keys
    return q, kc, vc, bt.cuda(), lens.cuda(), nbytes, flops


def _append_inputs(torch, b=16, t=2048, h=8, d=128, seed=5):
    gd = torch.Generator(device="cuda").manual_seed(seed)
    kn = torch.randn((b, t, h, d), generator=gd, device="cuda").half()
    vn = torch.randn((b, t, h, d), generator=gd, device="cuda").half()
    nblk = (t + 15) // 16
    pool = b * nblk
    perm = torch.randperm(pool, generator=torch.Generator().manual_seed(seed))
    bt = perm.to(torch.int32).view(b, nblk).cuda()
    kc = torch.empty((pool, 16, h, d), device="cuda", dtype=torch.float16)
    vc = torch.empty_like(kc)
    start = torch.zeros(b, dtype=torch.int32, device="cuda")
    w = (1 + 0.1 * torch.randn(d, generator=gd, device="cuda")).half()
    pos = torch.arange(t, device="cuda", dtype=torch.float32)
    inv = 1.0 / (10000 ** (torch.arange(0, d, 2, device="cuda").float() / d))
    emb = torch.cat([torch.outer(pos, inv)] * 2, dim=-1)
    nbytes = 4 * b * t * h * d * 2 + d * 2 + 2 * t * d * 2 + pool * 4 + b * 4
    return kn, vn, kc, vc, bt, start, w, emb.cos().half(), emb.sin().half(), nbytes


def _varlen_inputs(torch, n=16, h=32, d=128, seed=6):
    """Packed prefill batch: n sequences with lengths U[256, 4096] (seed 6)."""
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(256, 4097, (n,), generator=g)
    cu = torch.zeros(n + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0)
    total = int(cu[-1])
    gd = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = (torch.randn((total, h, d), generator=gd, device="cuda").half() for _ in range(3))
    flops = sum(4.0 * h * d * int(x) * int(x) * 0.5 for x in lens)
    return q, k, v, cu.cuda(), int(lens.max()), flops


def _qkv_inputs(torch, rn, m=4096, k=4096, hq=32, hkv=8):
    n = (hq + 2 * hkv) * 128
    x, w = rn((m, k)), rn((k, n), k ** -0.5)
    wq = (1 + 0.1 * torch.randn(128, device="cuda")).half()
    wk = (1 + 0.1 * torch.randn(128, device="cuda")).half()
    pos = torch.arange(8192, device="cuda", dtype=torch.float32)
    inv = 1.0 / (10000 ** (torch.arange(0, 128, 2, device="cuda").float() / 128))
    emb = torch.cat([torch.outer(pos, inv)] * 2, dim=-1)
    positions = torch.arange(m, device="cuda", dtype=torch.int32)
    return x, w, wq, wk, emb.cos().half(), emb.sin().half(), positions


def run_op(args):
    """Runs one operator case warmup+steps times; prints {"op", "ms", "value", "unit"}."""
    import torch

    import tritonllmcompiler_b200 as T

    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    gd = torch.Generator(device="cuda").manual_seed(1)

    def rn(shape, scale=1.0):
        return (torch.randn(shape, generator=gd, device="cuda") * scale).half()

    op = args.op
    if op == "swiglu":
        M, K, N = SWIGLU_SHAPE
        x, w1, w3 = rn((M, K)), rn((K, N), K ** -0.5), rn((K, N), K ** -0.5)
        fn, work, unit = (lambda: T.swiglu(x, w1, w3)), 4.0 * M * K * N, "TFLOP/s"
    elif op in ("flash_causal", "flash_full"):
        causal = op == "flash_causal"
        s = 4096 if causal else 1024
        q, k, v = rn((4, 32, s, 128)), rn((4, 32, s, 128)), rn((4, 32, s, 128))
        fn = lambda: T.flash_attention(q, k, v, causal=causal)  # noqa: E731
        work, unit = 4.0 * 4 * 32 * s * s * 128 * (0.5 if causal else 1.0), "TFLOP/s"
    elif op in ("paged", "paged_small"):
        q, kc, vc, bt, cl, work = _paged_inputs(torch, 64 if op == "paged" else 16)
        fn, unit = (lambda: T.paged_attention(q, kc, vc, bt, cl, block_size=16)), "GB/s"
    elif op in ("gqa_decode", "gqa_spec4", "gqa_chunk"):
        from tritonllmcompiler_b200.ops.paged_kv import paged_attention_prefill
        if op == "gqa_chunk":
            q, kc, vc, bt, cl, _, work = _gqa_inputs(
                torch, 8, 32, 8, 512, lens=torch.full((8,), 4096, dtype=torch.int32))
            unit = "TFLOP/s"
        else:
            q, kc, vc, bt, cl, work, _ = _gqa_inputs(torch, 64, 32, 8, 1 if op == "gqa_decode" else 4)
            unit = "GB/s"
        fn = lambda: paged_attention_prefill(q, kc, vc, bt, cl, block_size=16)  # noqa: E731
    elif op == "flash_varlen":
        from tritonllmcompiler_b200.ops.flash_varlen import flash_attention_varlen
        q, k, v, cu, mx, work = _varlen_inputs(torch)
        fn = lambda: flash_attention_varlen(q, k, v, cu, cu, mx, mx, causal=True)  # noqa: E731
        unit = "TFLOP/s"
    elif op == "qkv_norm_rope":
        from tritonllmcompiler_b200.ops.qkv_norm_rope import qkv_norm_rope
        args_ = _qkv_inputs(torch, rn)
        fn = lambda: qkv_norm_rope(*args_, num_q_heads=32, num_kv_heads=8)  # noqa: E731
        work, unit = 2.0 * 4096 * 4096 * 6144, "TFLOP/s"
    elif op == "swiglu_fp8":
        from tritonllmcompiler_b200.ops.swiglu_fp8 import quantize_e4m3, swiglu_fp8
        M, K, N = SWIGLU_SHAPE
        x8, sx = quantize_e4m3(rn((M, K)))
        w18, s1 = quantize_e4m3(rn((N, K), K ** -0.5))
        w38, s3 = quantize_e4m3(rn((N, K), K ** -0.5))
        fn = lambda: swiglu_fp8(x8, w18, w38, sx, s1, s3)  # noqa: E731
        work, unit = 4.0 * M * K * N, "TFLOP/s"
    elif op == "flash_fp8_causal":
        from tritonllmcompiler_b200.ops.flash_fp8 import flash_attention_fp8, quantize_qkv_e4m3
        q8, k8, vt8, s1, s2, s3 = quantize_qkv_e4m3(*(rn((4, 32, 4096, 128)) for _ in range(3)))
        fn = lambda: flash_attention_fp8(q8, k8, vt8, s1, s2, s3, causal=True)  # noqa: E731
        work, unit = 4.0 * 4 * 32 * 4096 * 4096 * 128 * 0.5, "TFLOP/s"
    elif op == "flash_bwd":
        from tritonllmcompiler_b200.ops.flash_backward import flash_attention_backward, flash_attention_fwd_lse
        q, k, v, do = rn((4, 32, 4096, 128)), rn((4, 32, 4096, 128)), rn((4, 32, 4096, 128)), rn((4, 32, 4096, 128))
        o, lse = flash_attention_fwd_lse(q, k, v, causal=True)
        fn = lambda: flash_attention_backward(q, k, v, o, lse, do, causal=True)  # noqa: E731
        work, unit = 2.5 * 4.0 * 4 * 32 * 4096 * 4096 * 128 * 0.5, "TFLOP/s"
    elif op == "swiglu_colshard8_local":
        # The column-sharded CTA-pair kernel exactly as one rank of 8 runs it, with the 8
        # destinations (this rank's and 7 peers' [M, N] outputs) all allocated on this GPU, so
        # the kernel can be profiled alone; HBM stands in for NVLink.
        import ctypes

        from tritonllmcompiler_b200 import _lib
        M, K, N = SWIGLU_SHAPE
        g8, n_loc = 8, N // 8
        x, w1, w3 = rn((M, K)), rn((K, n_loc), K ** -0.5), rn((K, n_loc), K ** -0.5)
        dsts = [torch.empty((M, N), dtype=torch.float16, device="cuda") for _ in range(g8)]
        arr = (ctypes.c_void_p * g8)(*[d.data_ptr() for d in dsts])
        lib = _lib.load()
        fn = lambda: _lib.check(lib.tllm_swiglu_colshard(  # noqa: E731
            x.data_ptr(), w1.data_ptr(), w3.data_ptr(), arr, g8, 3 * n_loc, M, n_loc, K, K, n_loc,
            n_loc, N, 0, torch.cuda.current_stream().cuda_stream))
        work, unit = 4.0 * M * K * n_loc, "TFLOP/s"
    elif op == "kv_append_rope":
        from tritonllmcompiler_b200.ops.paged_kv import paged_kv_append_rope
        kn, vn, kc, vc, bt, start, w, cos, sin, work = _append_inputs(torch)
        fn = lambda: paged_kv_append_rope(kn, vn, w, cos, sin, kc, vc, bt, start, block_size=16)  # noqa: E731
        unit = "GB/s"
    else:
        b, s, h, d = (2, 128, 8, 64) if op == "rmsnorm" else (16, 4096, 32, 128)
        x = rn((b, s, h, d))
        w = (1 + 0.1 * torch.randn(d, device="cuda")).half()
        pos = torch.arange(s, device="cuda", dtype=torch.float32)
        inv = 1.0 / (10000 ** (torch.arange(0, d, 2, device="cuda").float() / d))
        emb = torch.cat([torch.outer(pos, inv)] * 2, dim=-1)
        cos, sin = emb.cos().half(), emb.sin().half()
        fn = lambda: T.rmsnorm_rope(x, w, cos, sin)  # noqa: E731
        work, unit = 2 * (b * s * h * d * 2) + d * 2 + 2 * (s * d * 2), "GB/s"
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    ts = _events_time(torch, fn, args.steps, args.warmup, flush)
    ms = statistics.median(ts)
    scale = 1e12 if unit == "TFLOP/s" else 1e9
    print(json.dumps({"op": op, "case": OP_CASES[op], "ms": ms, "value": work / (ms * 1e-3) / scale,
                      "unit": unit, "launches": args.steps + args.warmup}), flush=True)


def resolve_comm(comm: str) -> str:
    """'auto' -> 'multicast' where this GPU offers NVLink multicast, else 'peers'."""
    if comm != "auto":
        return comm
    try:
        import torch
        from torch._C._distributed_c10d import _SymmetricMemory

        if torch.cuda.is_available() and _SymmetricMemory.has_multicast_support(
                torch._C._autograd.DeviceType.CUDA, int(os.environ.get("LOCAL_RANK", "0"))):
            return "multicast"
    except Exception:  # no symmetric-memory support in this build: plain peer stores
        pass
    return "peers"


def headline_config(world: int, comm: str, chunks: int) -> dict:
    """The headline workload's config, shared by both arms so the driver sees one config."""
    M, K, N = SWIGLU_SHAPE
    return {"workload": f"swiglu M{M} K{K} N{N} fp16 (Llama-3-8B MLP)",
            "parallelism": "single GPU" if world == 1 else (
                f"column-shard N over {world} ranks; GEMM epilogue stores every tile once "
                f"through an NVLink multicast address (NVSwitch writes all ranks' [M, N] "
                f"outputs), peer handshake inside the kernel"
                if comm == "multicast" else
                f"column-shard N over {world} ranks; GEMM epilogue stores every tile into all "
                f"ranks' [M, N] outputs over NVLink (CUDA IPC), peer handshake inside the kernel"
                if comm == "peers" else
                f"column-shard N over {world} ranks + NCCL all_gather_into_tensor + permute "
                f"into [M, N] ({chunks} row chunk(s))"),
            "l2": "256 MiB buffer written between timed steps; inputs 267 MB > L2"}


def run_reference(args):
    """CPU arm: the oracle port of the reference's swiglu_ref on the host cores, each step a
    256-row sample of the headline workload (rate reported; per-step time measured)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    M, K, N = SWIGLU_SHAPE
    rows = 256
    inputs = cpu_swiglu_inputs(rows)
    vals, secs, cores = [], [], cpu_cores()
    for i in range(args.warmup + args.steps):
        b = cpu_swiglu_baseline(inputs, min_seconds=0.0, rows=rows)
        if i >= args.warmup:
            vals.append(b["value"])
            secs.append(b["seconds_per_rep"])
    v = statistics.median(vals)
    ms = statistics.median(secs) * 1e3
    line = {
        "impl": "reference", "metric": "swiglu TFLOP/s", "value": v, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (seeded normal, x~N(0,1), w~N(0,1/K))",
        "config": headline_config(world, args.comm, args.chunks),
        "note": (f"CPU oracle (numpy restatement of reference/swiglu.py) on {cores} host threads; "
                 f"each step is one {rows}-row sample of the workload ({ms:.0f} ms measured); value "
                 f"is the sample's rate; the full workload would take "
                 f"{4.0 * M * K * N / (v * 1e12) * 1e3:.0f} ms per step at that rate"),
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": f"{rows}-row samples of the swiglu workload, one per step"},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------
def _median_ms(torch, fn, steps, warmup, flush=None):
    return statistics.median(_events_time(torch, fn, steps, warmup, flush))


def _e2e(torch, pairs, run, out_host, steps=3, warmup=2, note=""):
    """End to end through the public operator: each step copies every (pinned host, device)
    input pair host -> device, runs the operator and copies its result into the pinned host
    buffer, all on the current stream; CUDA events around the whole step."""
    def step():
        for h, d in pairs:
            d.copy_(h, non_blocking=True)
        out_host.copy_(run(), non_blocking=True)

    ms = _median_ms(torch, step, steps, warmup)
    h2d = sum(h.numel() * h.element_size() for h, _ in pairs)
    d2h = out_host.numel() * out_host.element_size()
    return {"ms": ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "path": note or "H2D copies from pinned host memory, the public operator, D2H copy; one stream"}


def _pinned_like(torch, t):
    h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    h.copy_(t)
    return h


def _roofline(achieved, peak, unit, bound, peak_src, traffic=None, kernel=None, note=None):
    r = {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
         "frac": achieved / peak, "traffic": traffic, "peak_source": peak_src}
    if kernel:
        r["kernel"] = kernel
    if note:
        r["note"] = note
    return r


def _paged_meta(batch, seed=3, lo=512, hi=8192, h=32, d=128, bs=16):
    """Lengths and algorithmic bytes of the seeded paged decode case (no device memory)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(lo, hi + 1, (batch,), dtype=torch.int32, generator=g)
    nb = [(int(n) + bs - 1) // bs for n in lens]
    nbytes = int(lens.sum()) * h * d * 2 * 2 + 2 * batch * h * d * 2 + sum(nb) * 4 + batch * 4
    return [int(n) for n in lens], nbytes


# ------------------------------------------------------------------------------------------
def extra_ops(torch, T, peaks, peak_src, with_cpu=True):
    """The other three operators at their configurations and the extensions (N=1, rank 0)."""
    res = {}
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    hbm = peaks["hbm_gbs"]
    tc = peaks["bf16_tflops"]
    hbm_src = f"{peak_src} hbm_gbs (copy)"
    tc_src = f"{peak_src} bf16_tflops (dense, burst)"

    def gen(shape, seed, scale=1.0):
        g = torch.Generator(device="cuda").manual_seed(seed)
        return (torch.randn(shape, generator=g, device="cuda") * scale).half()

    def rope_tables(s, d):
        pos = torch.arange(s, device="cuda", dtype=torch.float32)
        inv = 1.0 / (10000 ** (torch.arange(0, d, 2, device="cuda").float() / d))
        emb = torch.cat([torch.outer(pos, inv)] * 2, dim=-1)
        return emb.cos().half(), emb.sin().half()

    # rmsnorm_rope: config [2,128,8,64] and a bandwidth-scale variant [16,4096,32,128].
    for name, (b, s, h, d) in [("rmsnorm_rope_cfg_2x128x8x64", (2, 128, 8, 64)),
                               ("rmsnorm_rope_bw_16x4096x32x128", (16, 4096, 32, 128))]:
        x = gen((b, s, h, d), 0)
        w = (1 + 0.1 * torch.randn(d, device="cuda")).half()
        cos, sin = rope_tables(s, d)
        nbytes = 2 * (b * s * h * d * 2) + d * 2 + 2 * (s * d * 2)
        fn = lambda: T.rmsnorm_rope(x, w, cos, sin)  # noqa: E731
        with ClockSampler(torch.cuda.current_device()) as clk:
            t = _median_ms(torch, fn, 20, 5, flush)
        gbs = nbytes / (t * 1e-3) / 1e9
        cfg = b == 2
        traffic = None if cfg else profile_traffic("rmsnorm_rope_vec_kernel_16x4096x32x128_fp16.md")
        ent = {"value": gbs, "unit": "GB/s", "ms": t, "bytes": nbytes, "roofline_frac": gbs / hbm,
               "bound": "hbm", "l2": "flushed", "sm_mhz": clk.summary().get("sm_mhz"),
               "roofline": _roofline(gbs, hbm, "GB/s", "hbm", hbm_src, traffic,
                                     "rmsnorm_rope_vec_kernel")}
        if cfg:
            # 557 KB is below launch latency: the same operator on one row, timed the same way,
            # gives the floor of a single timed launch.
            x1 = x[:1, :1, :1].contiguous()
            c1, s1 = cos[:1].contiguous(), sin[:1].contiguous()
            ent["one_row_launch_ms"] = _median_ms(torch, lambda: T.rmsnorm_rope(x1, w, c1, s1), 20, 5, flush)
            hx, hw, hc, hs = (_pinned_like(torch, t_) for t_ in (x, w, cos, sin))
            hout = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
            dx, dw, dc, ds = (torch.empty_like(t_) for t_ in (x, w, cos, sin))
            e = _e2e(torch, [(hx, dx), (hw, dw), (hc, dc), (hs, ds)],
                     lambda: T.rmsnorm_rope(dx, dw, dc, ds), hout, steps=20, warmup=5)
            e.update(value=nbytes / (e["ms"] * 1e-3) / 1e9, unit="GB/s")
            ent["e2e"] = e
            if with_cpu:
                ent["cpu_baseline"] = cpu_rmsnorm_baseline((b, s, h, d))
        res[name] = ent
        del x
    # flash_attention: causal [4,32,4096,128] and non-causal [4,32,1024,128].
    for name, (b, h, s, d), causal, cpu_heads in [
            ("flash_causal_4x32x4096x128", (4, 32, 4096, 128), True, 8),
            ("flash_full_4x32x1024x128", (4, 32, 1024, 128), False, 32)]:
        q, k, v = gen((b, h, s, d), 2), gen((b, h, s, d), 3), gen((b, h, s, d), 4)
        flops = 4.0 * b * h * s * s * d * (0.5 if causal else 1.0)
        with ClockSampler(torch.cuda.current_device()) as clk:
            t = _median_ms(torch, lambda: T.flash_attention(q, k, v, causal=causal), 10, 3, flush)
        tf = flops / (t * 1e-3) / 1e12
        traffic = profile_traffic("flash_pp_kernel_causal_b4_h32_s4096_d128_fp16.md") if causal else None
        ent = {"value": tf, "unit": "TFLOP/s", "ms": t, "flops": flops, "roofline_frac": tf / tc,
               "bound": "tensor", "sm_mhz": clk.summary().get("sm_mhz"),
               "roofline": _roofline(tf, tc, "TFLOP/s", "tensor", tc_src, traffic, "flash_pp_kernel")}
        hq, hk, hv = (_pinned_like(torch, t_) for t_ in (q, k, v))
        hout = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
        dq, dk, dv = (torch.empty_like(t_) for t_ in (q, k, v))
        e = _e2e(torch, [(hq, dq), (hk, dk), (hv, dv)],
                 lambda: T.flash_attention(dq, dk, dv, causal=causal), hout)
        e.update(value=flops / (e["ms"] * 1e-3) / 1e12, unit="TFLOP/s")
        ent["e2e"] = e
        if with_cpu:
            ent["cpu_baseline"] = cpu_flash_baseline(b, h, s, d, causal, cpu_heads)
        res[name] = ent
        del q, k, v, dq, dk, dv, hq, hk, hv, hout
    # paged_attention decode: B64 H32 D128 bs16, lens U[512,8192] (seed 3).
    qd, kc, vc, btd, cl, nbytes = _paged_inputs(torch, 64)
    fn = lambda: T.paged_attention(qd, kc, vc, btd, cl, block_size=16)  # noqa: E731
    with ClockSampler(torch.cuda.current_device()) as clk:
        t = _median_ms(torch, fn, 20, 5, flush)
    gbs = nbytes / (t * 1e-3) / 1e9
    tr16 = profile_traffic("paged_split_kernel_b16_h32_d128_bs16_fp16.md")
    traffic = tr16 * nbytes / _paged_meta(16)[1] if tr16 else None
    ent = {"value": gbs, "unit": "GB/s", "ms": t, "bytes": nbytes, "roofline_frac": gbs / hbm,
           "bound": "hbm", "kv_tokens": int(cl.sum().item()), "sm_mhz": clk.summary().get("sm_mhz"),
           "roofline": _roofline(gbs, hbm, "GB/s", "hbm", hbm_src, traffic, "paged_split_kernel",
                                 "traffic: the B16 capture scaled to B64 by algorithmic bytes")}
    hq, hk, hv, hb, hl = (_pinned_like(torch, t_) for t_ in (qd, kc, vc, btd, cl))
    hout = torch.empty(qd.shape, dtype=qd.dtype, pin_memory=True)
    dq, dk, dv, db, dl = (torch.empty_like(t_) for t_ in (qd, kc, vc, btd, cl))
    e = _e2e(torch, [(hq, dq), (hk, dk), (hv, dv), (hb, db), (hl, dl)],
             lambda: T.paged_attention(dq, dk, dv, db, dl, block_size=16), hout,
             note="every input (the 4.3 GB KV cache included) copied from pinned host memory, "
                  "the operator, the result copied back; one stream")
    e.update(value=nbytes / (e["ms"] * 1e-3) / 1e9, unit="GB/s")
    del dk, dv
    er = _e2e(torch, [(hq, dq), (hb, db), (hl, dl)],
              lambda: T.paged_attention(dq, kc, vc, db, dl, block_size=16), hout, steps=10,
              note="KV cache resident in HBM (as a serving engine holds it); q, block tables and "
                   "lengths copied in and the result out every step")
    er.update(value=nbytes / (er["ms"] * 1e-3) / 1e9, unit="GB/s")
    e["cache_resident"] = er
    ent["e2e"] = e
    if with_cpu:
        lens64, _ = _paged_meta(64)
        ent["cpu_baseline"] = cpu_paged_baseline(lens64[:16], 32, 128, 16)
    res["paged_decode_b64_h32_d128_bs16"] = ent
    del kc, vc, hk, hv
    torch.cuda.empty_cache()
    # Operators either side of decode (extensions of the reference's set): GQA decode with 1
    # and 4 new tokens per sequence and a causal prefill chunk through the paged cache, and
    # the fused K-RoPE cache append.
    from tritonllmcompiler_b200.ops.paged_kv import paged_attention_prefill, paged_kv_append_rope
    for name, sq in [("gqa_decode_b64_hq32_hkv8_sq1", 1), ("gqa_decode_b64_hq32_hkv8_sq4", 4)]:
        q, kc, vc, bt, cl, nbytes, _ = _gqa_inputs(torch, 64, 32, 8, sq)
        with ClockSampler(torch.cuda.current_device()) as clk:
            ts = _events_time(torch, lambda: paged_attention_prefill(q, kc, vc, bt, cl, block_size=16),
                              20, 5, flush)
        t = statistics.median(ts)
        gbs = nbytes / (t * 1e-3) / 1e9
        res[name] = {"value": gbs, "unit": "GB/s", "ms": t, "bytes": nbytes,
                     "roofline_frac": gbs / hbm, "bound": "hbm", "kv_tokens": int(cl.sum().item()),
                     "sm_mhz": clk.summary().get("sm_mhz")}
        del kc, vc
    q, kc, vc, bt, cl, nbytes, flops = _gqa_inputs(torch, 8, 32, 8, 512,
                                                   lens=torch.full((8,), 4096, dtype=torch.int32))
    with ClockSampler(torch.cuda.current_device()) as clk:
        ts = _events_time(torch, lambda: paged_attention_prefill(q, kc, vc, bt, cl, block_size=16),
                          10, 3, flush)
    t = statistics.median(ts)
    tf = flops / (t * 1e-3) / 1e12
    res["gqa_prefill_chunk_b8_hq32_hkv8_sq512_ctx4096"] = {
        "value": tf, "unit": "TFLOP/s", "ms": t, "flops": flops, "roofline_frac": tf / tc,
        "bound": "tensor", "sm_mhz": clk.summary().get("sm_mhz")}
    del kc, vc
    # QKV projection with RMSNorm + RoPE in the epilogue (Llama-3-8B: K 4096, 32 q and 8 kv heads).
    from tritonllmcompiler_b200.ops.qkv_norm_rope import qkv_norm_rope
    qa = _qkv_inputs(torch, lambda shape, scale=1.0: gen(shape, 11, scale))
    flops = 2.0 * 4096 * 4096 * 6144
    with ClockSampler(torch.cuda.current_device()) as clk:
        ts = _events_time(torch, lambda: qkv_norm_rope(*qa, num_q_heads=32, num_kv_heads=8), 20, 5, flush)
    t = statistics.median(ts)
    tf = flops / (t * 1e-3) / 1e12
    res["qkv_norm_rope_m4096_k4096_hq32_hkv8"] = {"value": tf, "unit": "TFLOP/s", "ms": t, "flops": flops,
                                                  "roofline_frac": tf / tc, "bound": "tensor",
                                                  "sm_mhz": clk.summary().get("sm_mhz")}
    del qa
    # FP8 (e4m3) swiglu at the headline shape (an extension: not the fp16 headline metric).
    from tritonllmcompiler_b200.ops.swiglu_fp8 import quantize_e4m3, swiglu_fp8
    M, K, N = SWIGLU_SHAPE
    x8, sx = quantize_e4m3(gen((M, K), 7))
    w18, s1 = quantize_e4m3(gen((N, K), 8, K ** -0.5))
    w38, s3 = quantize_e4m3(gen((N, K), 9, K ** -0.5))
    flops = 4.0 * M * K * N
    with ClockSampler(torch.cuda.current_device()) as clk:
        ts = _events_time(torch, lambda: swiglu_fp8(x8, w18, w38, sx, s1, s3), 20, 5, flush)
    t = statistics.median(ts)
    tf = flops / (t * 1e-3) / 1e12
    res["swiglu_fp8_m4096_k4096_n14336"] = {"value": tf, "unit": "TFLOP/s", "ms": t, "flops": flops,
                                            "roofline_frac_of_bf16_peak": tf / tc, "bound": "tensor",
                                            "sm_mhz": clk.summary().get("sm_mhz")}
    del x8, w18, w38
    # FP8 (e4m3) flash attention forward, causal [4,32,4096,128] (an extension).
    from tritonllmcompiler_b200.ops.flash_fp8 import flash_attention_fp8, quantize_qkv_e4m3
    q8, k8, vt8, s1, s2, s3 = quantize_qkv_e4m3(*(gen((4, 32, 4096, 128), s_) for s_ in (2, 3, 4)))
    flops = 4.0 * 4 * 32 * 4096 * 4096 * 128 * 0.5
    with ClockSampler(torch.cuda.current_device()) as clk:
        ts = _events_time(torch, lambda: flash_attention_fp8(q8, k8, vt8, s1, s2, s3, causal=True),
                          10, 3, flush)
    t = statistics.median(ts)
    tf = flops / (t * 1e-3) / 1e12
    res["flash_fp8_causal_4x32x4096x128"] = {"value": tf, "unit": "TFLOP/s", "ms": t, "flops": flops,
                                             "roofline_frac_of_bf16_peak": tf / tc, "bound": "tensor",
                                             "sm_mhz": clk.summary().get("sm_mhz")}
    del q8, k8, vt8
    # FlashAttention backward, causal [4,32,4096,128]: 2.5x the forward's FLOPs (five GEMMs
    # against two), the FlashAttention convention.
    from tritonllmcompiler_b200.ops.flash_backward import flash_attention_backward, flash_attention_fwd_lse
    q, k, v, do = (gen((4, 32, 4096, 128), s_) for s_ in (2, 3, 4, 5))
    o, lse = flash_attention_fwd_lse(q, k, v, causal=True)
    flops = 2.5 * 4.0 * 4 * 32 * 4096 * 4096 * 128 * 0.5
    with ClockSampler(torch.cuda.current_device()) as clk:
        ts = _events_time(torch, lambda: flash_attention_backward(q, k, v, o, lse, do, causal=True), 5, 3, flush)
    t = statistics.median(ts)
    tf = flops / (t * 1e-3) / 1e12
    res["flash_bwd_causal_4x32x4096x128"] = {"value": tf, "unit": "TFLOP/s", "ms": t, "flops": flops,
                                             "roofline_frac": tf / tc, "bound": "tensor",
                                             "sm_mhz": clk.summary().get("sm_mhz")}
    del q, k, v, do, o, lse
    torch.cuda.empty_cache()
    from tritonllmcompiler_b200.ops.flash_varlen import flash_attention_varlen
    q, k, v, cu, mx, flops = _varlen_inputs(torch)
    with ClockSampler(torch.cuda.current_device()) as clk:
        ts = _events_time(torch, lambda: flash_attention_varlen(q, k, v, cu, cu, mx, mx, causal=True),
                          10, 3, flush)
    t = statistics.median(ts)
    tf = flops / (t * 1e-3) / 1e12
    res["flash_varlen_causal_16seq_u256_4096_h32_d128"] = {
        "value": tf, "unit": "TFLOP/s", "ms": t, "flops": flops, "roofline_frac": tf / tc,
        "bound": "tensor", "sm_mhz": clk.summary().get("sm_mhz")}
    del q, k, v
    kn, vn, kc, vc, bt, start, w, cos, sin, nbytes = _append_inputs(torch)
    with ClockSampler(torch.cuda.current_device()) as clk:
        ts = _events_time(torch, lambda: paged_kv_append_rope(kn, vn, w, cos, sin, kc, vc, bt, start,
                                                              block_size=16), 20, 5, flush)
    t = statistics.median(ts)
    gbs = nbytes / (t * 1e-3) / 1e9
    res["kv_append_rope_b16_t2048_h8_d128"] = {"value": gbs, "unit": "GB/s", "ms": t, "bytes": nbytes,
                                               "roofline_frac": gbs / hbm, "bound": "hbm",
                                               "sm_mhz": clk.summary().get("sm_mhz")}
    del kn, vn, kc, vc
    torch.cuda.empty_cache()
    return res


# ------------------------------------------------------------------------------------------
def _max_over_ranks(torch, dist, world, v):
    if world == 1:
        return v
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(torch, dist, world, v: int) -> int:
    if world == 1:
        return int(v)
    t = torch.tensor([int(v)], device="cuda", dtype=torch.int64)
    dist.all_reduce(t)
    return int(t.item())


def _all_ok(torch, dist, world, ok: bool) -> bool:
    if world == 1:
        return bool(ok)
    t = torch.tensor([1 if ok else 0], device="cuda", dtype=torch.int32)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def _bits_checksum(torch, t) -> int:
    """Exact checksum of a 16-bit tensor: the sum of its bit patterns (order-independent)."""
    flat = t.reshape(-1).view(torch.int16)
    total = 0
    step = 1 << 26
    for i in range(0, flat.numel(), step):
        total += int(flat[i:i + step].to(torch.int64).sum().item())
    return total


def _timed_ranks(torch, dist, world, fn, steps, warmup, flush=None):
    """Median per-step device time of fn on this rank, then the max over ranks."""
    fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = _median_ms(torch, fn, steps, warmup, flush)
    return _max_over_ranks(torch, dist, world, ms)


def sharded_cfg5(torch, dist, T, S, world, rank, local, peaks, peak_src, with_cpu,
                 multicast=False):
    """The Llama-3-70B-shaped sharded workloads at this world size (every rank)."""
    res = {}
    # These kernels run for milliseconds back to back: the sustained (power-capped) peak.
    tc = peaks["bf16_tflops_sustained"]
    hbm = peaks["hbm_gbs"]
    dev = torch.device("cuda", local)

    # swiglu: x [8192, 8192], w1/w3 [8192, 28672] column-sharded, output gathered on every rank.
    M, K, N = CFG5_SWIGLU
    n_loc = N // world
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn(M, K, generator=g, device="cuda").half()
    w1 = (torch.randn(K, N, generator=g, device="cuda") / math.sqrt(K)).half()
    w3 = (torch.randn(K, N, generator=g, device="cuda") / math.sqrt(K)).half()
    r0, r1 = 4096, 4352
    ref_rows = T.swiglu(x[r0:r1].contiguous(), w1, w3)
    w1l = w1[:, rank * n_loc:(rank + 1) * n_loc].contiguous()
    w3l = w3[:, rank * n_loc:(rank + 1) * n_loc].contiguous()
    del w1, w3
    torch.cuda.empty_cache()
    peers = None
    if world > 1:
        peers = S.PeerBuffers((M, N), torch.float16, dev, multicast=multicast)
        step = lambda: S.swiglu_column_sharded(x, w1l, w3l, peers=peers)  # noqa: E731
    else:
        step = lambda: T.swiglu(x, w1l, w3l)  # noqa: E731
    ms = _timed_ranks(torch, dist, world, step, 5, 2)
    out = step()
    torch.cuda.synchronize()
    ok = _all_ok(torch, dist, world, bool(torch.equal(out[r0:r1], ref_rows)))
    flops = 4.0 * M * K * N
    tf = flops / (ms * 1e-3) / 1e12
    t_tc = 4.0 * M * K * n_loc / (tc * 1e12)
    # bytes a rank sends: its slice once through the multicast address, else once per peer
    sent = (1 if multicast else world - 1) * M * n_loc * 2 if world > 1 else 0
    t_link = sent / (NVLINK_GBS * 1e9)
    ent = {"value": tf, "unit": "TFLOP/s", "ms": ms, "flops": flops,
           "per_rank": f"x [{M}, {K}] and w1/w3 column slices [{K}, {n_loc}]; every rank ends "
                       f"with the whole [{M}, {N}] output",
           "parity": {"ok": ok, "check": f"rows {r0}:{r1} of every rank's gathered output equal "
                                         f"bit for bit the single-GPU swiglu of those rows"},
           "roofline": {"bound": "tensor" if t_tc >= t_link else "nvlink",
                        "target_ms": max(t_tc, t_link) * 1e3, "tensor_ms": t_tc * 1e3,
                        "nvlink_ms": t_link * 1e3, "frac": max(t_tc, t_link) * 1e3 / ms,
                        "note": f"slower of local FLOPs / {peak_src} sustained bf16 peak {tc:.0f} TFLOP/s and "
                                f"bytes sent per rank / {NVLINK_GBS:.0f} GB/s peer-copy rate"}}
    if world > 1:
        ent["nvlink_gbs_per_rank"] = sent / (ms * 1e-3) / 1e9
    if with_cpu:
        ent["cpu_baseline"] = cpu_swiglu_baseline(cpu_swiglu_inputs(256, CFG5_SWIGLU, cols=4096, seed=4),
                                                  min_seconds=3.0, rows=256, shape=CFG5_SWIGLU)
    res["swiglu_m8192_k8192_n28672"] = ent
    if peers is not None:
        torch.cuda.synchronize()
        dist.barrier()
        peers.close()
    del x, w1l, w3l, ref_rows, out, peers
    torch.cuda.empty_cache()

    # flash_attention causal [8, 64, 8192, 128], heads sharded.
    B, H, Sq, D = CFG5_FLASH
    h0, h1 = S.head_range(H, rank, world)
    g = torch.Generator(device="cuda").manual_seed(4)
    loc = []
    for _ in range(3):
        full = torch.randn(B, H, Sq, D, generator=g, device="cuda").half()
        loc.append(full[:, h0:h1].contiguous())
        del full
        torch.cuda.empty_cache()
    q, k, v = loc
    fn = lambda: S.flash_attention_head_sharded(q, k, v, causal=True)  # noqa: E731
    ms = _timed_ranks(torch, dist, world, fn, 5, 2)
    out = fn()
    torch.cuda.synchronize()
    chk = _sum_over_ranks(torch, dist, world, _bits_checksum(torch, out))
    flops = 4.0 * B * H * Sq * Sq * D * 0.5
    tf = flops / (ms * 1e-3) / 1e12
    ent = {"value": tf, "unit": "TFLOP/s", "ms": ms, "flops": flops,
           "per_rank": f"heads [{h0}, {h1}) of q/k/v/o, no communication",
           "checksum_fp16_bits": chk,
           "roofline": _roofline(tf / world, tc, "TFLOP/s", "tensor", f"{peak_src} bf16_tflops_sustained",
                                 kernel="flash_pp_kernel", note="achieved per GPU")}
    if with_cpu:
        ent["cpu_baseline"] = cpu_flash_baseline(B, H, Sq, D, True, 4, threads=4)
    res["flash_causal_b8_h64_s8192_d128"] = ent
    del q, k, v, out, loc
    torch.cuda.empty_cache()

    # paged decode B256 H64 D128 bs32, lens U[1024, 32768], sequences balanced by tokens.
    Bp, Hp, Dp, bs, lo, hi = CFG5_PAGED
    gc = torch.Generator().manual_seed(4)
    lens = torch.randint(lo, hi + 1, (Bp,), dtype=torch.int32, generator=gc)
    nb = [(int(n) + bs - 1) // bs for n in lens]
    pool = sum(nb)
    perm = torch.randperm(pool, generator=gc)
    bt = torch.zeros(Bp, max(nb), dtype=torch.int32)
    pos = 0
    for i, n in enumerate(nb):
        bt[i, :n] = perm[pos:pos + n].to(torch.int32)
        pos += n
    parts = S.partition_sequences(lens.tolist(), world, "tokens")
    counts = S.partition_sequences(lens.tolist(), world, "count")
    toks = [sum(int(lens[i]) for i in p) for p in parts]
    toks_c = [sum(int(lens[i]) for i in p) for p in counts]
    seqs = parts[rank]
    ids, lbt, llen = S.localize_blocks(bt, lens, seqs, bs)
    # Physical block p of the global pool holds reservoir block p % R (seeded, identical on
    # every rank), so each rank builds only its own blocks and the values do not depend on
    # the world size.
    R = 2053
    gd = torch.Generator(device="cuda").manual_seed(4)
    res_k = torch.randn(R, bs, Hp, Dp, generator=gd, device="cuda").half()
    res_v = torch.randn(R, bs, Hp, Dp, generator=gd, device="cuda").half()
    q_all = torch.randn(Bp, Hp, 1, Dp, generator=gd, device="cuda").half()
    sel = (ids % R).cuda()
    kc = res_k.index_select(0, sel)
    vc = res_v.index_select(0, sel)
    del res_k, res_v, sel
    torch.cuda.empty_cache()
    qs = q_all[torch.tensor(seqs, dtype=torch.int64, device="cuda")].contiguous()
    lbt_d, llen_d = lbt.cuda(), llen.cuda()
    fn = lambda: T.paged_attention(qs, kc, vc, lbt_d, llen_d, block_size=bs)  # noqa: E731
    ms = _timed_ranks(torch, dist, world, fn, 5, 2)
    out = fn()
    torch.cuda.synchronize()
    chk = _sum_over_ranks(torch, dist, world, _bits_checksum(torch, out))
    nbytes = int(lens.sum()) * Hp * Dp * 2 * 2 + 2 * Bp * Hp * Dp * 2 + pool * 4 + Bp * 4
    gbs = nbytes / (ms * 1e-3) / 1e9
    mean = sum(toks) / world
    ent = {"value": gbs, "unit": "GB/s", "ms": ms, "bytes": nbytes, "kv_tokens": int(lens.sum()),
           "per_rank": f"{len(seqs)} whole sequences ({toks[rank]} tokens), their block-table rows "
                       f"and a rank-local pool of their {len(ids)} blocks; no communication",
           "balance": {"tokens_scheme_max_over_mean": max(toks) / mean,
                       "count_scheme_max_over_mean": max(toks_c) / mean},
           "checksum_fp16_bits": chk,
           "roofline": _roofline(gbs / world, hbm, "GB/s", "hbm", f"{peak_src} hbm_gbs",
                                 kernel="paged_split_kernel + paged_merge_kernel",
                                 note="achieved per GPU")}
    if with_cpu:
        ent["cpu_baseline"] = cpu_paged_baseline([int(n) for n in lens[:2]], Hp, Dp, bs, threads=2)
    res["paged_decode_b256_h64_d128_bs32"] = ent
    del kc, vc, q_all, qs, out
    torch.cuda.empty_cache()
    return res


def run_ours(args):
    import torch
    import torch.distributed as dist

    import tritonllmcompiler_b200 as T
    from tritonllmcompiler_b200 import sharded as S

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    peaks, peak_src = load_peaks()
    M, K, N = SWIGLU_SHAPE
    assert N % world == 0 and (N // world) % 8 == 0
    n_loc = N // world
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(M, K, generator=g, device="cuda").half()
    w1 = (torch.randn(K, N, generator=g, device="cuda") / math.sqrt(K)).half()
    w3 = (torch.randn(K, N, generator=g, device="cuda") / math.sqrt(K)).half()
    r0, r1 = PARITY_ROWS
    ref_rows = T.swiglu(x[r0:r1].contiguous(), w1, w3)  # parity reference: the rows alone
    w1l = w1[:, rank * n_loc:(rank + 1) * n_loc].contiguous()
    w3l = w3[:, rank * n_loc:(rank + 1) * n_loc].contiguous()
    del w1, w3
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")

    out_full = None
    peers = None
    if world > 1:
        if args.comm in ("peers", "multicast"):
            peers = S.PeerBuffers((M, N), torch.float16, torch.device("cuda", local),
                                  multicast=args.comm == "multicast")
        else:
            out_full = torch.empty((M, N), dtype=torch.float16, device="cuda")

    def step():
        if world == 1:
            return T.swiglu(x, w1l, w3l)
        if peers is not None:
            return S.swiglu_column_sharded(x, w1l, w3l, peers=peers)
        return S.swiglu_column_sharded(x, w1l, w3l, chunks=args.chunks, out=out_full)

    flops = 4.0 * M * K * N
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # The clock sampler starts (NVML set-up, its thread) before the barrier, so that every rank
    # enters the timed region together: at N > 1 a step waits inside the kernel for the ranks
    # that start it late.
    with ClockSampler(local) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        times = _events_time(torch, step, args.steps, 0, flush)
    torch.cuda.synchronize()
    t_step = _max_over_ranks(torch, dist, world, sum(times) / len(times))
    step_spread = {"median_ms": _max_over_ranks(torch, dist, world, statistics.median(times)),
                   "max_ms": _max_over_ranks(torch, dist, world, max(times)),
                   "min_ms": _max_over_ranks(torch, dist, world, min(times)),
                   "note": "per-step CUDA-event times, each the max over ranks; ms_per_step is the mean"}
    if world > 1:
        dist.barrier()
    value = flops / (t_step * 1e-3) / 1e12

    # Parity: the sampled rows of the (gathered) output against the rows computed alone.
    out = step()
    torch.cuda.synchronize()
    parity_ok = _all_ok(torch, dist, world, bool(torch.equal(out[r0:r1], ref_rows)))
    del out

    # Roofline of the kernel that runs in the step. One GPU (or the NCCL path): the swiglu
    # kernel alone on the local shard. Peer stores: the step is that one kernel.
    peak = peaks["bf16_tflops"]
    if world == 1 or peers is None:
        k_ms = _max_over_ranks(torch, dist, world,
                               _median_ms(torch, lambda: T.swiglu(x, w1l, w3l), max(5, args.steps // 2), 2, flush))
        achieved = 4.0 * M * K * n_loc / (k_ms * 1e-3) / 1e12
        roofline = _roofline(achieved, peak, "TFLOP/s", "tensor", f"{peak_src} bf16_tflops (dense, burst)",
                             profile_traffic("swiglu_pair_kernel_m4096_k4096_n14336_fp16.md") if world == 1 else None,
                             "swiglu_pair_kernel" + ("" if world == 1 else " (local shard, local output)"))
        roofline["kernel_ms"] = k_ms
    else:
        k_ms = t_step
        t_tc = 4.0 * M * K * n_loc / (peak * 1e12)
        mc = args.comm == "multicast"
        # bytes this rank sends over NVLink per step: its slice once (multicast) or per peer
        sent = (1 if mc else world - 1) * M * n_loc * 2
        t_link = sent / (NVLINK_GBS * 1e9)
        kname = ("swiglu_pair_kernel<peers> (GEMM + output stored once through an NVLink multicast "
                 "address)" if mc else
                 "swiglu_pair_kernel<peers> (GEMM + output all-gather over NVLink)")
        if t_tc >= t_link:
            roofline = _roofline(4.0 * M * K * n_loc / (k_ms * 1e-3) / 1e12, peak, "TFLOP/s", "tensor",
                                 f"{peak_src} bf16_tflops (dense, burst)", None, kname)
        else:
            roofline = _roofline(sent / (k_ms * 1e-3) / 1e9, NVLINK_GBS, "GB/s", "nvlink",
                                 "measured NVLink peer-copy rate per direction on this pool", None,
                                 kname)
        roofline.update(kernel_ms=k_ms, tensor_ms=t_tc * 1e3, nvlink_ms=t_link * 1e3,
                        bytes_sent_per_rank=sent,
                        local_tflops=4.0 * M * K * n_loc / (k_ms * 1e-3) / 1e12,
                        note="the step is this one kernel; its target is the slower of local FLOPs / "
                             "bf16 peak and bytes sent per rank / NVLink rate")
        traffic = profile_traffic(f"swiglu_pair_kernel_peers_m4096_k4096_n14336_g{world}.md")
        roofline["traffic"] = traffic
        if not mc:
            # The one-CTA column-sharded kernel (128 x 128 tiles, half a CTA pair's tile time, so
            # the first stores leave earlier) on the same step, for comparison.
            ms1 = _max_over_ranks(torch, dist, world, _median_ms(
                torch, lambda: S.swiglu_column_sharded(x, w1l, w3l, peers=peers, variant=1),
                max(5, args.steps // 2), 2, flush))
            roofline["one_cta_kernel_ms"] = ms1

    # End to end through the public API with pinned host buffers (H2D inputs, D2H result).
    hx = x.cpu().pin_memory()
    h1 = w1l.cpu().pin_memory()
    h3 = w3l.cpu().pin_memory()
    dx, d1, d3 = torch.empty_like(x), torch.empty_like(w1l), torch.empty_like(w3l)
    if world > 1:
        hout = torch.empty((M, N), dtype=torch.float16).pin_memory()
    else:
        # One GPU: the public host-memory entry, which pipelines the weight upload, the kernel
        # and the result download over column blocks on three streams.
        from tritonllmcompiler_b200.ops.host_pipeline import SwigluHostPipeline
        hout = torch.empty((M, n_loc), dtype=torch.float16).pin_memory()
        host_pipe = SwigluHostPipeline(M, n_loc, K, torch.float16, torch.device("cuda", local),
                                       chunks=args.e2e_chunks)

    def e2e_step():
        if world == 1:
            host_pipe(hx, h1, h3, hout)
            return
        dx.copy_(hx, non_blocking=True)
        d1.copy_(h1, non_blocking=True)
        d3.copy_(h3, non_blocking=True)
        if peers is not None:
            out = S.swiglu_column_sharded(dx, d1, d3, peers=peers)
        else:
            out = S.swiglu_column_sharded(dx, d1, d3, chunks=args.chunks, out=out_full)
        hout.copy_(out, non_blocking=True)

    e_ms = _max_over_ranks(torch, dist, world,
                           sum(_events_time(torch, e2e_step, max(3, args.steps // 4), 2)) / max(3, args.steps // 4))
    e2e = {"value": flops / (e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
           "h2d_bytes_per_step": (hx.numel() + h1.numel() + h3.numel()) * 2,
           "d2h_bytes_per_step": hout.numel() * 2, "ms_per_step": e_ms,
           "path": (f"ops.host_pipeline.SwigluHostPipeline, {len(host_pipe.blocks)} column blocks: "
                    f"upload, kernel and download overlapped on three streams") if world == 1 else
                   "per rank: H2D copies of x and its weight slices, sharded swiglu, D2H copy of the "
                   "whole [M, N] output; one stream"}
    del dx, d1, d3, hx, h1, h3, hout, x, w1l, w3l, flush
    if world == 1:
        del host_pipe
    if peers is not None:
        torch.cuda.synchronize()
        dist.barrier()
        peers.close()
        peers = None
    out_full = None
    torch.cuda.empty_cache()

    ops = None
    cpu = None
    if rank == 0 and world == 1:
        if not args.no_ops:
            ops = extra_ops(torch, T, peaks, peak_src, with_cpu=not args.no_cpu)
        if not args.no_cpu:
            cpu = cpu_swiglu_baseline()
    cfg5 = None
    if not args.no_cfg5:
        cfg5 = sharded_cfg5(torch, dist, T, S, world, rank, local, peaks, peak_src,
                            with_cpu=(rank == 0 and world == 1 and not args.no_cpu),
                            multicast=args.comm == "multicast")

    if rank == 0:
        line = {
            "metric": "swiglu TFLOP/s", "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_step,
            "step_spread": step_spread,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic (seeded normal, x~N(0,1), w~N(0,1/K))",
            "config": headline_config(world, args.comm, args.chunks),
            "parity": {"ok": parity_ok,
                       "check": f"rows {r0}:{r1} of the step's [M, N] output on every rank equal, bit "
                                f"for bit, swiglu of those rows computed alone on one GPU"},
            "roofline": roofline,
            "e2e": e2e,
            "gpu_launches": args.steps,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
        if ops is not None:
            line["ops"] = ops
        if cfg5 is not None:
            line["sharded_cfg5"] = cfg5
            line["sharded_cfg5_note"] = (
                "Llama-3-70B-shaped workloads sharded over the ranks of this run; value is the "
                "whole-job rate from the max-over-ranks device time (median of 5 steps after 2 "
                "warm-up); inputs larger than L2; the checksums are exact sums of the output's "
                "fp16 bit patterns, equal at every world size when the sharded result matches "
                "the single-GPU one")
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    args.comm = resolve_comm(args.comm)
    if args.op is not None:
        run_op(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
