"""Benchmark: causal bf16 GQA attention forward+backward.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one forward (with saved log-sum-exp) plus one backward of
``flash_attention`` on q [4, 32, 4096, 128], k/v [4, 8, 4096, 128], dO like q,
bf16, causal -- the configuration BASELINE.json's headline metric is quoted on.
Work per step uses the FlashAttention convention: forward 4*B*H*S^2*D / 2
(causal half) = 5.50e11 FLOP, backward 2.5x forward; 1.924e12 FLOP per step.
Inputs (320 MiB) exceed the 126 MB L2, so no flush is needed between steps.

``e2e`` is the same metric through the public API from pinned host buffers,
with every step's H2D of q/k/v/dO and D2H of dq/dk/dv inside the timed region:
double-buffered on two copy streams (step i+1's inputs and step i's gradients
move while step i computes), with the serial form reported beside it.

With N > 1 (torchrun, one process per GPU, NCCL) the step is PARTITIONED: the
32 (batch, kv-head) units of config 2 are split over the ranks
(``sharding.unit_slices``; a rank's units are re-batched as [units, 4, S, D]
queries over [units, 1, S, D] keys, which is the same work item set), with no
data-path collective.  ``value`` is the whole problem's FLOP / the max over
ranks of the device time (strong scaling); ``e2e`` copies only the rank's
slice.  Each rank also checks its gradients against the same units computed
inside the full single-call problem.

The secondary workloads run at every N, partitioned the same way: config 3
(64 units), config 4 paged decode (sequences greedy-balanced by length, each
rank with its own page pool and remapped tables), the config-4 fixed cache
(batch split), and config 5 (prompts split, tokens gathered with one NCCL
all_gather inside the timed region).  At N = 1 rank 0 also times the oracle's
numpy restatement of the reference beside each of them (``cpu_baseline``
objects: bounded samples scaled by work, core count stated).

``--impl reference`` times that CPU restatement of config 2 alone, one query
head of one (batch, kv-head group) unit per step (at most one untimed warm-up
head; timed steps stop after 150 s, so any K ends within minutes); its
``ms_per_step`` is the measured time of the sample, and the full-step time it
extrapolates to is reported beside it.  The reference is JAX on TPU; JAX is not
installed, so its own CPU path cannot run here.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "tpu-native-pallas-flashattention_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

B, H, HKV, S, D = 4, 32, 8, 4096, 128
FWD_FLOP = 4.0 * B * H * S * S * D / 2
BWD_FLOP = 2.5 * FWD_FLOP
STEP_FLOP = FWD_FLOP + BWD_FLOP
UNITS = B * HKV  # independent (batch, kv-head group) units of the step
LAUNCHES_PER_STEP = 4  # forward, delta preprocess, dK/dV (+ dS spill), dQ GEMM


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d["bf16_tflops_sustained"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled every 5 ms during the timed region.

    Reads NVML (read-only queries; nothing is set).  Records nothing if NVML is
    unavailable.
    """

    def __init__(self, index: int, period_s: float = 0.005):
        self.index, self.period = index, period_s
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thread = None

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            self.h = nv.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM))
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception:  # noqa: BLE001 - no NVML: no samples
            self._thread = None
        return self

    def _run(self):
        nv = self.nv
        names = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                 "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                 "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                 "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap,
                 "hw_power_brake_slowdown": nv.nvmlClocksEventReasonHwPowerBrakeSlowdown,
                 "applications_clocks_setting": nv.nvmlClocksEventReasonApplicationsClocksSetting,
                 "sync_boost": nv.nvmlClocksEventReasonSyncBoost,
                 "gpu_idle": nv.nvmlClocksEventReasonGpuIdle}
        while not self._stop.is_set():
            try:
                self.samples.append(float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)))
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for n, b in names.items():
                    if bits & b:
                        self.reasons.add(n)
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "sm_mhz_min_max": [float(min(self.samples)), float(max(self.samples))],
                "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "NVML, 5 ms period"}


# --------------------------------------------------------------------------- CPU side
def cpu_sample_step(q, k, v, do):
    """One unit of config 2 through the oracle (naive fwd + closed-form VJP, fp32 numpy)."""
    from oracle import attention_oracle as orc

    out = orc.reference_attention(q, k, v, causal=True, dtype=np.float32)
    orc.attention_vjp(q, k, v, do, causal=True, dtype=np.float32)
    return out


def cpu_baseline(steps: int = 1, warmup: int = 0, budget_s: float = 150.0):
    """The oracle's fp32 numpy restatement of the reference's XLA-CPU path on a bounded
    sample: each step is one query head of one (batch, kv-head group) unit of config 2
    (1/128 of the step's work, ~3 s on 16 host threads), scaled by FLOP.  Timed steps
    stop early once `budget_s` has elapsed, so any --steps keeps the run to minutes."""
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 1, S, D), dtype=np.float32)
    k = rng.standard_normal((1, 1, S, D), dtype=np.float32)
    v = rng.standard_normal((1, 1, S, D), dtype=np.float32)
    do = rng.standard_normal((1, 1, S, D), dtype=np.float32)
    # All host threads for the BLAS the oracle's numpy matmuls run on (torchrun
    # sets OMP_NUM_THREADS=1, which would otherwise pin it to one core).
    from threadpoolctl import threadpool_info, threadpool_limits
    with threadpool_limits(limits=os.cpu_count() or 1, user_api="blas"):
        cores = max([i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"] or [1])
        for _ in range(max(0, warmup)):
            cpu_sample_step(q, k, v, do)
        t0 = time.perf_counter()
        done = 0
        for _ in range(max(1, steps)):
            cpu_sample_step(q, k, v, do)
            done += 1
            if time.perf_counter() - t0 > budget_s:
                break
        dt = (time.perf_counter() - t0) / done
    head_flop = STEP_FLOP / (B * H)
    return {"value": head_flop / dt / 1e12, "unit": "TFLOP/s", "cores": cores,
            "kind": "port", "sample_ms": dt * 1e3,
            "sample": f"1 query head of 1 of {UNITS} (batch, kv-head group) units of config 2 (4096 x 128, "
                      f"causal), numpy fp32 naive fwd + closed-form VJP, {dt:.2f} s per head, scaled by FLOP; "
                      f"{done} timed step(s)"}


# --------------------------------------------------------------------------- GPU side
def make_inputs(dev, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn((B, H, S, D), device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn((B, HKV, S, D), device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn((B, HKV, S, D), device=dev, generator=g).to(torch.bfloat16)
    do = torch.randn((B, H, S, D), device=dev, generator=g).to(torch.bfloat16)
    return q, k, v, do


def step_device(pf, q, k, v, do):
    qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
    out = pf.flash_attention(qq, kk, vv, causal=True)
    out.backward(do)
    return qq.grad, kk.grad, vv.grad


def time_kernels(pf, q, k, v, do, iters=5):
    """Per-kernel-family device time (CUDA events on the launching stream)."""
    from pallas_flash.flash_attention import _fwd, _bwd

    scale = 1.0 / math.sqrt(D)
    s = torch.cuda.current_stream()
    out, lse = _fwd(q, k, v, True, scale, S, True)
    _bwd(q, k, v, out, lse, do, True, scale, S)
    torch.cuda.synchronize()
    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    fwd_ms = bwd_ms = 0.0
    for _ in range(iters):
        e[0].record(s)
        out, lse = _fwd(q, k, v, True, scale, S, True)
        e[1].record(s)
        _bwd(q, k, v, out, lse, do, True, scale, S)
        e[2].record(s)
        torch.cuda.synchronize()
        fwd_ms += e[0].elapsed_time(e[1])
        bwd_ms += e[1].elapsed_time(e[2])
    return fwd_ms / iters, bwd_ms / iters


def time_bwd_recompute(pf, q, k, v, do, iters=5):
    """Device ms of the backward without the dS spill (workspace holding only delta: the dQ
    kernel recomputes S and dP), for the record beside the default path."""
    from pallas_flash import _lib
    from pallas_flash.flash_attention import _fwd

    b, h, sq, d = q.shape
    hkv, sk = k.shape[1], k.shape[2]
    scale = 1.0 / math.sqrt(d)
    out, lse = _fwd(q, k, v, True, scale, sk, True)
    L = _lib.lib()
    ws = torch.empty(b * h * sq * 4, dtype=torch.uint8, device=q.device)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)

    def run():
        _lib.check(L.pf_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), do.data_ptr(), lse.data_ptr(),
                            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), _lib.dtype_code(q.dtype), b, h, hkv, sq, sk,
                            d, 1, scale, sk, ws.data_ptr(), ws.numel(), _lib.stream_of(q)))

    run()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(iters):
        run()
    e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


# --------------------------------------------------------------------------- partitioning
def take_units(x, units, n_kv):
    """Rows of ``x`` [B, n_kv * g, S, D] for the (batch, kv head) ``units``, re-batched as
    [len(units), g, S, D] (a copy): every unit is an independent problem."""
    b, hx, s_, d = x.shape
    g = hx // n_kv
    bi = torch.tensor([u[0] for u in units], device=x.device)
    hi = torch.tensor([u[1] for u in units], device=x.device)
    return x.view(b, n_kv, g, s_, d)[bi, hi].contiguous()


def max_over_ranks(dev, *vals):
    if not torch.distributed.is_initialized():
        return vals if len(vals) > 1 else vals[0]
    t = torch.tensor([float(v) for v in vals], device=dev, dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    out = tuple(float(x) for x in t.tolist())
    return out if len(out) > 1 else out[0]


def barrier():
    if torch.distributed.is_initialized():
        torch.distributed.barrier()


def timed(fn, iters, dev):
    """Device ms per call of ``fn`` (CUDA events on the current stream), max over ranks."""
    s = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(s)
    for _ in range(iters):
        fn()
    e1.record(s)
    torch.cuda.synchronize()
    return max_over_ranks(dev, e0.elapsed_time(e1) / iters)


def host_threads(fn):
    """Runs ``fn`` with all host threads for numpy's BLAS (torchrun sets OMP_NUM_THREADS=1);
    returns (result, threads used)."""
    from threadpoolctl import threadpool_info, threadpool_limits
    with threadpool_limits(limits=os.cpu_count() or 1, user_api="blas"):
        cores = max([i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"] or [1])
        return fn(), cores


# --------------------------------------------------------------------------- config 4: paged decode
def paged_problem(n_seqs=256, seed=0):
    """Config 4 lengths and block table (seeded numpy): kv_len ~ U[512, 32768], page 16,
    pool = ceil(1.1 * live pages), table = seeded permutation of the pool sliced per sequence."""
    rng = np.random.default_rng(seed)
    ps = 16
    lens = rng.integers(512, 32769, size=n_seqs)
    npages = [(int(x) + ps - 1) // ps for x in lens]
    pool = int(math.ceil(1.1 * sum(npages)))
    perm = rng.permutation(pool)
    table = np.zeros((n_seqs, max(npages)), np.int32)
    off = 0
    for b, n in enumerate(npages):
        table[b, :n] = perm[off:off + n]
        off += n
    return lens, npages, pool, table


def paged_bytes(lens, npages, n_seqs, hq=32, hkv=8, d=128):
    return int(sum(lens)) * hkv * d * 2 * 2 + 2 * n_seqs * hq * d * 2 + 4 * sum(npages)


def paged_decode_bench(pf, dev, iters=10, n_seqs=256, warmup=3, world=1, rank=0):
    """Config 4: paged decode HBM GB/s (bytes = 4096 B per live token + q/out + table).
    With N ranks the sequences are greedy-balanced by length; each rank decodes its own
    pool (``sharding.local_paged_problem``) and GB/s counts the whole workload's bytes."""
    from pallas_flash import sharding

    hq, hkv, ps, d = 32, 8, 16, 128
    lens, npages, pool, table = paged_problem(n_seqs)
    g = torch.Generator(device=dev).manual_seed(0)
    kp = torch.empty((pool, hkv, ps, d), device=dev, dtype=torch.bfloat16).normal_(generator=g)
    vp = torch.empty((pool, hkv, ps, d), device=dev, dtype=torch.bfloat16).normal_(generator=g)
    q = torch.randn((n_seqs, hq, 1, d), device=dev, generator=g).to(torch.bfloat16)
    tt = torch.from_numpy(table).to(dev)
    ll = torch.from_numpy(lens.astype(np.int32)).to(dev)
    mine = list(range(n_seqs))
    if world > 1:
        mine = sharding.greedy_balance(lens.tolist(), world)[rank]
        q, kp, vp, tt, ll = sharding.local_paged_problem(q, kp, vp, tt, ll, mine)
        torch.cuda.empty_cache()
    mx = int(lens[mine].max())
    run = lambda: pf.paged_flash_attention(q, kp, vp, tt, ll, max_context_len=mx)  # noqa: E731
    for _ in range(warmup):
        run()
    ms = timed(run, iters, dev)
    nbytes = paged_bytes(lens, npages, n_seqs)
    my_bytes = paged_bytes(lens[mine], [npages[i] for i in mine], len(mine))
    del kp, vp
    torch.cuda.empty_cache()
    return {"workload": f"config 4: {n_seqs} seqs, kv_len U[512,32768] (seed 0), page 16, H32/Hkv8/D128, bf16",
            "tokens": int(lens.sum()), "bytes": nbytes, "ms": ms, "GB/s": nbytes / ms / 1e6,
            "partition": f"{len(mine)} of {n_seqs} sequences on this rank ({my_bytes / nbytes:.3f} of the bytes), "
                         "greedy by length" if world > 1 else "single GPU"}


def fixed_decode_bench(pf, dev, iters=5, world=1, rank=0):
    """Config 4 fixed-cache variant: cache [256, 8, 32768, 128] bf16, cache_len 32768 (HBM GB/s);
    with N ranks each decodes its batch slice (256 / N sequences)."""
    from pallas_flash import sharding

    nb, hq, hkv, c, d = 256, 32, 8, 32768, 128
    sl = sharding.split_batch(nb, world, rank)
    mb = sl.stop - sl.start
    g = torch.Generator(device=dev).manual_seed(1 + rank)
    kc = torch.empty((mb, hkv, c, d), device=dev, dtype=torch.bfloat16).normal_(generator=g)
    vc = torch.empty((mb, hkv, c, d), device=dev, dtype=torch.bfloat16).normal_(generator=g)
    q = torch.randn((mb, hq, 1, d), device=dev, generator=g).to(torch.bfloat16)
    run = lambda: pf.flash_attention_decode(q, kc, vc, c)  # noqa: E731
    for _ in range(2):
        run()
    ms = timed(run, iters, dev)
    nbytes = nb * hkv * c * d * 2 * 2 + 2 * nb * hq * d * 2
    del kc, vc
    torch.cuda.empty_cache()
    return {"workload": "config 4 fixed cache: [256, 8, 32768, 128] bf16, cache_len 32768",
            "bytes": nbytes, "ms": ms, "GB/s": nbytes / ms / 1e6,
            "partition": f"{mb} of {nb} sequences on this rank" if world > 1 else "single GPU"}


# --------------------------------------------------------------------------- config 3: fused-RoPE prefill
def rope_prefill_bench(pf, dev, iters=5, world=1, rank=0):
    """Config 3: fused-RoPE prefill B8 H32 Hkv8 S8192 D128 causal bf16 (TFLOP/s, 4.398e12 FLOP),
    the 64 (batch, kv-head) units split over the ranks."""
    from pallas_flash import sharding

    b, h, hkv, s_, d = 8, 32, 8, 8192, 128
    units = sharding.unit_slices(b, hkv, world, rank)
    g = torch.Generator(device=dev).manual_seed(2)
    q = torch.randn((b, h, s_, d), device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn((b, hkv, s_, d), device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn((b, hkv, s_, d), device=dev, generator=g).to(torch.bfloat16)
    if world > 1:
        q, k, v = (take_units(t, units, hkv) for t in (q, k, v))
        torch.cuda.empty_cache()
    cos, sin = pf.precompute_rope(s_, d, 10000.0, device=dev)
    run = lambda: pf.flash_attention_rope(q, k, v, cos, sin, causal=True)  # noqa: E731
    for _ in range(2):
        run()
    ms = timed(run, iters, dev)
    flop = 4.0 * b * h * s_ * s_ * d / 2
    return {"workload": "config 3: fused-RoPE prefill B8 H32 Hkv8 S8192 D128 causal bf16 (theta 1e4)",
            "flop": flop, "ms": ms, "TFLOP/s": flop / ms / 1e9,
            "partition": f"{len(units)} of {b * hkv} (batch, kv-head) units on this rank" if world > 1
            else "single GPU"}


def c1_forward_bench(pf, dev, iters=50):
    """Config 1: fp32 forward [1, 8, 512, 128] causal (latency-dominated; 5.37e8 FLOP), with the
    oracle's numpy fp32 forward on the same inputs timed beside it on the host."""
    from oracle import attention_oracle as orc

    shape = (1, 8, 512, 128)
    g = torch.Generator(device=dev).manual_seed(1)
    q, k, v = (torch.randn(shape, device=dev, generator=g) for _ in range(3))
    for _ in range(3):
        pf.flash_attention(q, k, v, causal=True)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(iters):
        pf.flash_attention(q, k, v, causal=True)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    # The same call replayed from a CUDA graph: the device time without the
    # per-call host work of an eager loop.
    side = torch.cuda.Stream(dev)
    side.wait_stream(st)
    with torch.cuda.stream(side):
        pf.flash_attention(q, k, v, causal=True)
    st.wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(10):
            pf.flash_attention(q, k, v, causal=True)
    graph.replay()
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(iters // 10):
        graph.replay()
    e1.record(st)
    torch.cuda.synchronize()
    graph_ms = e0.elapsed_time(e1) / (10 * (iters // 10))
    qh, kh, vh = (t.cpu().numpy() for t in (q, k, v))
    t0 = time.perf_counter()
    orc.reference_attention(qh, kh, vh, causal=True, dtype=np.float32)
    cpu_ms = (time.perf_counter() - t0) * 1e3
    flop = 4.0 * 1 * 8 * 512 * 512 * 128 / 2
    return {"workload": "config 1: fp32 forward [1,8,512,128] causal", "flop": flop,
            "api_ms": ms, "graph_ms": graph_ms, "TFLOP/s": flop / graph_ms / 1e9,
            "timing": "api_ms: eager public-API calls; graph_ms: the same call replayed from a CUDA graph "
                      "(device time without per-call host work)",
            "kernel": pf._lib.forward_kernel_kind(torch.float32, 128), "cpu_oracle_ms": cpu_ms}


def paged_prefill_bench(pf, dev, iters=5):
    """Chunked prefill over a page pool: 16 sequences, contexts U[2048, 8192] (seed 0), 512-query
    chunks at the end of each context, H32/Hkv8/D128 bf16, page 16.  FLOP = 4*H*D * visible keys
    summed over the chunk rows (causal within the chunk)."""
    n, L, h, hkv, d, ps = 16, 512, 32, 8, 128, 16
    rng = np.random.default_rng(0)
    lens = rng.integers(2048, 8193, size=n)
    pps = int((lens.max() + ps - 1) // ps)
    num_pages = n * pps
    tables = torch.from_numpy(rng.permutation(num_pages).reshape(n, pps).astype(np.int32))
    g = torch.Generator(device=dev).manual_seed(3)
    q = torch.randn((n, h, L, d), device=dev, generator=g).to(torch.bfloat16)
    kp = torch.randn((num_pages, hkv, ps, d), device=dev, generator=g).to(torch.bfloat16)
    vp = torch.randn((num_pages, hkv, ps, d), device=dev, generator=g).to(torch.bfloat16)
    ctx = torch.from_numpy(lens.astype(np.int32))
    mx = int(lens.max())
    for _ in range(2):
        pf.paged_prefill_attention(q, kp, vp, tables, ctx, max_context_len=mx)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(iters):
        pf.paged_prefill_attention(q, kp, vp, tables, ctx, max_context_len=mx)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    flop = float(sum(4.0 * h * d * (L * (c - L) + L * (L + 1) / 2) for c in lens.tolist()))
    return {"workload": "paged chunked prefill: 16 seqs, ctx U[2048,8192], chunk 512, H32/Hkv8/D128 bf16, page 16",
            "flop": flop, "ms": ms, "TFLOP/s": flop / ms / 1e9,
            "note": "includes the context gather into contiguous rows (one pass over the live pages)"}


C5_CFG = dict(vocab_size=32000, dim=512, n_layers=8, n_heads=8, n_kv_heads=2, head_dim=64,
              ffn_hidden=1408, rope_theta=10000.0, rms_norm_eps=1e-5)


def generation_bench(pf, dev, world=1, rank=0):
    """Config 5: tiny-LLaMA greedy generation tokens/s (generate_cached, then ring streaming).
    With N ranks the 16 prompts are split and the tokens gathered with one NCCL all_gather
    (``sharding.generate_data_parallel``) inside the timed region."""
    from pallas_flash import sharding

    cfg = pf.ModelConfig(**C5_CFG)
    params = pf.init_params(0, cfg, dtype=torch.bfloat16, device=dev)
    g = torch.Generator(device=dev).manual_seed(0)
    prompts = torch.randint(0, 32000, (16, 128), device=dev, generator=g)

    def cached(n):
        return sharding.generate_data_parallel(
            lambda p: pf.generate_cached(params, p, n, cfg, cache_size=512), prompts, world, rank)

    def streaming(n):
        return sharding.generate_data_parallel(
            lambda p: pf.generate_streaming(params, p, n, cfg, window=512), prompts, world, rank)

    cached(256)  # warm-up at the timed size (graph capture, workspaces, library heuristics)
    streaming(8)
    cached(256)  # the first cached run after a streaming one still pays one-time costs

    def wall(fn):
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = fn()
        torch.cuda.synchronize()
        return max_over_ranks(dev, time.perf_counter() - t0), out

    tc, toks = wall(lambda: cached(256))
    ts, _ = wall(lambda: streaming(4096))
    return {"workload": "config 5: tiny LLaMA (dim 512, 8 layers, 8/2 heads, head_dim 64, bf16), batch 16, prompt 128",
            "cached_tokens_per_s": 16 * 256 / tc, "cached_s": tc,
            "streaming_tokens_per_s": 16 * 4096 / ts, "streaming_s": ts,
            "tokens_shape": list(toks.shape),
            "timing": "wall clock around the host loop, synchronised before and after, max over ranks",
            "partition": f"{sharding.split_batch(16, world, rank).stop - sharding.split_batch(16, world, rank).start}"
                         " of 16 prompts on this rank, tokens all_gathered (NCCL)" if world > 1 else "single GPU"}


# --------------------------------------------------------------------------- CPU baselines (oracle port)
def cpu_rope_prefill_baseline():
    """Config 3 on the host: one query head of one (batch, kv-head) unit (S 8192, D 128,
    causal), RoPE on q and k then the naive fp32 attention forward, scaled by FLOP."""
    from oracle import attention_oracle as orc

    s_, d = 8192, 128
    rng = np.random.default_rng(3)
    q, k, v = (rng.standard_normal((1, 1, s_, d), dtype=np.float32) for _ in range(3))
    cos, sin = orc.precompute_rope(s_, d, 10000.0)

    def run():
        t0 = time.perf_counter()
        orc.reference_attention(orc.apply_rope(q, cos, sin), orc.apply_rope(k, cos, sin), v, causal=True,
                                dtype=np.float32)
        return time.perf_counter() - t0

    dt, cores = host_threads(run)
    flop = 4.0 * s_ * s_ * d / 2
    return {"value": flop / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"1 query head of 1 of 64 (batch, kv-head) units of config 3, numpy fp32 RoPE + naive "
                      f"causal forward, {dt:.2f} s, scaled by FLOP"}


def cpu_paged_decode_baseline(n_sample=8):
    """Config 4 on the host: the first 8 sequences of the config-4 workload (same lengths),
    oracle paged decode (block-table gather + naive attention, fp32) over a float32 pool of
    their pages; GB/s counts the workload's bf16 bytes of those sequences."""
    from oracle import attention_oracle as orc

    lens, npages, _, _ = paged_problem()
    lens, npages = lens[:n_sample], npages[:n_sample]
    rng = np.random.default_rng(4)
    pool = sum(npages)
    kp = rng.standard_normal((pool, 8, 16, 128), dtype=np.float32)
    vp = rng.standard_normal((pool, 8, 16, 128), dtype=np.float32)
    perm = rng.permutation(pool)
    table = np.zeros((n_sample, max(npages)), np.int32)
    off = 0
    for b, n in enumerate(npages):
        table[b, :n] = perm[off:off + n]
        off += n
    q = rng.standard_normal((n_sample, 32, 1, 128), dtype=np.float32)

    def run():
        t0 = time.perf_counter()
        orc.paged_attention(q, kp, vp, table, lens, dtype=np.float32)
        return time.perf_counter() - t0

    dt, cores = host_threads(run)
    nbytes = paged_bytes(lens, npages, n_sample)
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"first {n_sample} of 256 config-4 sequences ({int(lens.sum())} tokens), numpy fp32 "
                      f"gather + naive decode, {dt:.2f} s; GB/s counts bf16 bytes (4096 B/token)"}


def cpu_fixed_decode_baseline(n_sample=2):
    """Config 4 fixed cache on the host: 2 of the 256 sequences at cache_len 32768 (fp32 naive)."""
    from oracle import attention_oracle as orc

    rng = np.random.default_rng(5)
    kc = rng.standard_normal((n_sample, 8, 32768, 128), dtype=np.float32)
    vc = rng.standard_normal((n_sample, 8, 32768, 128), dtype=np.float32)
    q = rng.standard_normal((n_sample, 32, 1, 128), dtype=np.float32)

    def run():
        t0 = time.perf_counter()
        orc.reference_attention(q, kc, vc, dtype=np.float32)
        return time.perf_counter() - t0

    dt, cores = host_threads(run)
    nbytes = n_sample * 8 * 32768 * 128 * 2 * 2 + 2 * n_sample * 32 * 128 * 2
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{n_sample} of 256 sequences at cache_len 32768, numpy fp32 naive decode, {dt:.2f} s; "
                      "GB/s counts bf16 bytes"}


def cpu_generation_baseline(pf, n_new=8):
    """Config 5 on the host: the oracle's cached greedy loop (numpy fp32) on the config-5 model
    and all 16 prompts, 8 new tokens (prefill included); tokens/s = 16 * 8 / time."""
    from oracle import attention_oracle as orc

    cfg = pf.ModelConfig(**C5_CFG)
    params = pf.init_params(0, cfg, dtype=torch.bfloat16, device="cpu")
    npp = {k: ([{a: b.float().numpy() for a, b in lay.items()} for lay in v] if k == "layers"
               else v.float().numpy()) for k, v in params.items()}
    prompts = np.random.default_rng(0).integers(0, 32000, size=(16, 128))

    def run():
        t0 = time.perf_counter()
        orc.tiny_llama_generate(npp, prompts, n_new, cfg)
        return time.perf_counter() - t0

    dt, cores = host_threads(run)
    return {"value": 16 * n_new / dt, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"16 prompts x 128 tokens, {n_new} new tokens each with a fixed KV cache "
                      f"(prefill included), numpy fp32, {dt:.2f} s"}


def e2e_step(pf, host_in, host_out, dev):
    """Public-API step from pinned host buffers: H2D inputs, fwd+bwd, D2H gradients."""
    q, k, v, do = (h.to(dev, non_blocking=True) for h in host_in)
    dq, dk, dv = step_device(pf, q, k, v, do)
    for h, t in zip(host_out, (dq, dk, dv)):
        h.copy_(t, non_blocking=True)


def e2e_pipelined(pf, host_in, host_out, dev, steps: int) -> float:
    """Public-API steps from pinned host buffers, double-buffered as a training
    loop would run them: step i+1's inputs are copied host->device on one copy
    stream while step i computes, and step i's gradients are read back on a
    second copy stream while step i+1 computes.  Every step's H2D and D2H copies
    are inside the timed region; returns ms per step (fill and drain included)."""
    comp = torch.cuda.current_stream(dev)
    cs_in, cs_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    bufs = [[torch.empty(h.shape, dtype=h.dtype, device=dev) for h in host_in] for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    free[0].record(comp)
    free[1].record(comp)

    def load(i):
        b = i % 2
        with torch.cuda.stream(cs_in):
            cs_in.wait_event(free[b])  # step i-2 has finished reading this buffer
            for d, h in zip(bufs[b], host_in):
                d.copy_(h, non_blocking=True)
            ready[b].record(cs_in)

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    load(0)
    for i in range(steps):
        b = i % 2
        comp.wait_event(ready[b])
        if i + 1 < steps:
            load(i + 1)
        grads = step_device(pf, *bufs[b])
        free[b].record(comp)
        done = torch.cuda.Event()
        done.record(comp)
        with torch.cuda.stream(cs_out):
            cs_out.wait_event(done)
            for h, t in zip(host_out, grads):
                h.copy_(t, non_blocking=True)
                t.record_stream(cs_out)
    tail = torch.cuda.Event()
    tail.record(cs_out)
    comp.wait_event(tail)
    e1.record(comp)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-extras", action="store_true", help="skip the secondary workloads and CPU baselines")
    ap.add_argument("--mode", choices=["bench", "profile-c2", "profile-bwd", "profile-decode", "profile-decode-f32",
                                       "profile-gen", "profile-rope", "profile-fixed"], default="bench",
                    help="profile-*: only launch the kernels of one workload (for ncu captures)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    config = {"workload": "config 2: causal GQA attention fwd+bwd", "batch": B, "heads": H, "kv_heads": HKV,
              "seq_len": S, "head_dim": D, "causal": True, "l2": "inputs 320 MiB > L2, no flush",
              "parallelism": (f"batch x kv-head partition: {UNITS // world if UNITS % world == 0 else '~' + str(UNITS // world)}"
                              f" of {UNITS} units per GPU over {world} GPU(s), no collective")}

    if args.impl == "reference":
        if rank != 0:
            return
        t0 = time.perf_counter()
        cb = cpu_baseline(steps=args.steps, warmup=min(1, max(0, args.warmup)))
        print(json.dumps({
            "impl": "reference", "metric": "fwd+bwd attention TFLOP/s", "value": cb["value"], "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": cb["sample_ms"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1))", "config": config,
            "cpu_baseline": cb, "wall_s": time.perf_counter() - t0,
            "extrapolated_full_step_ms": STEP_FLOP / (cb["value"] * 1e12) * 1e3,
            "e2e": {"value": cb["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "oracle port (numpy fp32) of the reference's XLA-CPU path; each step is a bounded sample "
                    "(one query head of one unit, ms_per_step is its measured time) and value scales it by "
                    "FLOP; JAX is absent so the reference itself and its Pallas interpret mode cannot run"}))
        return

    import pallas_flash as pf
    from pallas_flash import _lib, sharding

    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    dev = torch.device("cuda", local_rank if world > 1 else 0)
    torch.cuda.set_device(dev)
    _lib.load_library()

    if args.mode == "profile-decode":
        # config-4 shape on 32 sequences (~2.4 GB of KV): warmup + steps decode calls
        paged_decode_bench(pf, dev, iters=args.steps, n_seqs=32, warmup=args.warmup)
        print(json.dumps({"mode": args.mode, "ok": True}))
        return
    if args.mode == "profile-decode-f32":
        # the config-4 shape on 8 sequences in fp32 (the bulk-copy split-KV kernel; ~1.2 GB of KV)
        lens, npages, _, table = paged_problem(8)
        pool = sum(npages)
        g = torch.Generator(device=dev).manual_seed(0)
        kp = torch.randn((pool, 8, 16, 128), device=dev, generator=g)
        vp = torch.randn((pool, 8, 16, 128), device=dev, generator=g)
        q = torch.randn((8, 32, 1, 128), device=dev, generator=g)
        tt = torch.from_numpy(np.ascontiguousarray(table % pool)).to(dev)
        ll = torch.from_numpy(lens.astype(np.int32)).to(dev)
        for _ in range(args.warmup + args.steps):
            pf.paged_flash_attention(q, kp, vp, tt, ll, max_context_len=32768)
        torch.cuda.synchronize()
        print(json.dumps({"mode": args.mode, "ok": True}))
        return
    if args.mode == "profile-bwd":
        # one batch of config 2 (B1 H32 Hkv8 S4096 D128 causal): warmup + steps backward passes
        from pallas_flash.flash_attention import _fwd, _bwd
        g = torch.Generator(device=dev).manual_seed(0)
        q = torch.randn((1, H, S, D), device=dev, generator=g).to(torch.bfloat16)
        k = torch.randn((1, HKV, S, D), device=dev, generator=g).to(torch.bfloat16)
        v = torch.randn((1, HKV, S, D), device=dev, generator=g).to(torch.bfloat16)
        do = torch.randn((1, H, S, D), device=dev, generator=g).to(torch.bfloat16)
        out, lse = _fwd(q, k, v, True, 1.0 / math.sqrt(D), S, True)
        for _ in range(args.warmup + args.steps):
            _bwd(q, k, v, out, lse, do, True, 1.0 / math.sqrt(D), S)
        torch.cuda.synchronize()
        print(json.dumps({"mode": args.mode, "ok": True}))
        return
    if args.mode == "profile-fixed":
        # fixed-cache decode on 16 sequences at capacity 32768 (2.1 GB of KV)
        g = torch.Generator(device=dev).manual_seed(1)
        kc = torch.empty((16, 8, 32768, 128), device=dev, dtype=torch.bfloat16).normal_(generator=g)
        vc = torch.empty_like(kc).normal_(generator=g)
        q = torch.randn((16, 32, 1, 128), device=dev, generator=g).to(torch.bfloat16)
        for _ in range(args.warmup + args.steps):
            pf.flash_attention_decode(q, kc, vc, 32768)
        torch.cuda.synchronize()
        print(json.dumps({"mode": args.mode, "ok": True}))
        return
    if args.mode == "profile-rope":
        # config-3 shape on one batch (B1 H32 Hkv8 S8192 D128, 96 MB of q/k/v)
        g = torch.Generator(device=dev).manual_seed(2)
        q = torch.randn((1, 32, 8192, 128), device=dev, generator=g).to(torch.bfloat16)
        k = torch.randn((1, 8, 8192, 128), device=dev, generator=g).to(torch.bfloat16)
        v = torch.randn((1, 8, 8192, 128), device=dev, generator=g).to(torch.bfloat16)
        cos, sin = pf.precompute_rope(8192, 128, 10000.0, device=dev)
        for _ in range(args.warmup + args.steps):
            pf.flash_attention_rope(q, k, v, cos, sin, causal=True)
        torch.cuda.synchronize()
        print(json.dumps({"mode": args.mode, "ok": True}))
        return
    if args.mode == "profile-gen":
        # config-5 model: ring-streaming generation of `steps` tokens after a short warm-up run
        cfg = pf.ModelConfig(**C5_CFG)
        params = pf.init_params(0, cfg, dtype=torch.bfloat16, device=dev)
        g = torch.Generator(device=dev).manual_seed(0)
        prompts = torch.randint(0, 32000, (16, 128), device=dev, generator=g)
        pf.generate_streaming(params, prompts, max(2, args.warmup), cfg, window=512)
        pf.generate_streaming(params, prompts, args.steps, cfg, window=512)
        torch.cuda.synchronize()
        print(json.dumps({"mode": args.mode, "ok": True}))
        return

    # This rank's share of config 2: its (batch, kv-head) units, re-batched.
    units = sharding.unit_slices(B, HKV, world, rank)
    qf, kf, vf, dof = make_inputs(dev, seed=0)  # the whole problem (same on every rank)
    if world > 1:
        q, do = take_units(qf, units, HKV), take_units(dof, units, HKV)
        k, v = take_units(kf, units, HKV), take_units(vf, units, HKV)
    else:
        q, k, v, do = qf, kf, vf, dof
    if args.mode == "profile-c2":
        # warmup + steps fwd+bwd steps of config 2 and nothing else
        for _ in range(args.warmup + args.steps):
            step_device(pf, q, k, v, do)
        torch.cuda.synchronize()
        print(json.dumps({"mode": args.mode, "ok": True}))
        return
    partition_check = None
    if world > 1:
        # The rank's gradients against the same units inside the full single-call problem.
        full = step_device(pf, qf, kf, vf, dof)
        mine = step_device(pf, q, k, v, do)
        ref = (take_units(full[0], units, HKV), take_units(full[1], units, HKV), take_units(full[2], units, HKV))
        diffs = [float((a.float() - b.float()).abs().max()) for a, b in zip(mine, ref)]
        partition_check = {"max_abs_diff_dq_dk_dv": diffs, "bitwise_equal": all(d == 0.0 for d in diffs)}
        del full, mine, ref
    del qf, kf, vf, dof
    torch.cuda.empty_cache()
    for _ in range(max(3, args.warmup)):
        step_device(pf, q, k, v, do)
    torch.cuda.synchronize()

    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        barrier()
        torch.cuda.synchronize()
        e0.record(s)
        for _ in range(args.steps):
            step_device(pf, q, k, v, do)
        e1.record(s)
        torch.cuda.synchronize()
        barrier()
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = max_over_ranks(dev, ms)
    value = STEP_FLOP / (ms_max * 1e-3) / 1e12  # the whole problem's work / the slowest rank

    # end to end through the public API with pinned host buffers (this rank's slice)
    host_in = [t.cpu().pin_memory() for t in (q, k, v, do)]
    host_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in (q, k, v)]
    for _ in range(2):
        e2e_step(pf, host_in, host_out, dev)
    torch.cuda.synchronize()
    barrier()
    e0.record(s)
    e2e_steps = max(1, min(args.steps, 5))
    for _ in range(e2e_steps):
        e2e_step(pf, host_in, host_out, dev)
    e1.record(s)
    torch.cuda.synchronize()
    e2e_serial_ms = e0.elapsed_time(e1) / e2e_steps
    e2e_pipelined(pf, host_in, host_out, dev, 2)  # warm the copy streams
    barrier()
    e2e_ms = e2e_pipelined(pf, host_in, host_out, dev, max(2, min(args.steps, 16)))
    e2e_ms, e2e_serial_ms = max_over_ranks(dev, e2e_ms, e2e_serial_ms)
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = sum(t.numel() * t.element_size() for t in host_out)

    share = len(units) / UNITS
    fwd_ms, bwd_ms = time_kernels(pf, q, k, v, do)
    bwd_recompute_ms = time_bwd_recompute(pf, q, k, v, do)
    hbm, tf_burst, tf_sust, src = peaks()
    dom = (("backward (delta + dK/dV with dS spill + dQ GEMM)", bwd_ms, BWD_FLOP * share) if bwd_ms >= fwd_ms
           else ("forward", fwd_ms, FWD_FLOP * share))
    achieved = dom[2] / (dom[1] * 1e-3) / 1e12
    traffic = None
    tp = ROOT / "profiles" / "traffic.json"
    if tp.exists() and world == 1:
        traffic = json.loads(tp.read_text()).get("fwd_bwd_c2", {}).get("bwd" if dom[0].startswith("back") else "fwd")

    line = {
        "metric": "fwd+bwd attention TFLOP/s", "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1))",
        "config": config,
        "roofline": {"bound": "tensor", "kernel": dom[0], "achieved": achieved, "peak": tf_burst,
                     "unit": "TFLOP/s", "frac": achieved / tf_burst, "peak_source": f"{src} bf16 burst",
                     "traffic": traffic, "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
                     "fwd_tflops": FWD_FLOP * share / fwd_ms / 1e9, "bwd_tflops": BWD_FLOP * share / bwd_ms / 1e9,
                     "fwd_frac": FWD_FLOP * share / fwd_ms / 1e9 / tf_burst,
                     "bwd_ms_without_ds_spill": bwd_recompute_ms,
                     "per_rank": "rank 0's kernels on its share of the units" if world > 1 else "whole problem"},
        "e2e": {"value": STEP_FLOP / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "pipelining": "double-buffered: H2D of step i+1 and D2H of step i on two copy streams "
                              "overlap step i's kernels; fill and drain inside the timed region",
                "serial_value": STEP_FLOP / (e2e_serial_ms * 1e-3) / 1e12,
                "serial_ms_per_step": e2e_serial_ms,
                "bytes": "per rank (its slice of the units)" if world > 1 else "whole problem"},
        "gpu_launches": LAUNCHES_PER_STEP * args.steps,
        "clocks": clk.summary(),
    }
    if partition_check is not None:
        line["partition_check"] = partition_check
    if not args.no_extras:
        pd = paged_decode_bench(pf, dev, world=world, rank=rank)
        pd["frac_of_hbm"] = pd["GB/s"] / (hbm * world)
        pd["hbm_peak_gbs"] = hbm * world
        line["paged_decode"] = pd
        fd = fixed_decode_bench(pf, dev, world=world, rank=rank)
        fd["frac_of_hbm"] = fd["GB/s"] / (hbm * world)
        line["fixed_decode"] = fd
        rp = rope_prefill_bench(pf, dev, world=world, rank=rank)
        rp["frac_of_bf16_peak"] = rp["TFLOP/s"] / (tf_burst * world)
        line["rope_prefill"] = rp
        line["generation"] = generation_bench(pf, dev, world=world, rank=rank)
        if world == 1:
            line["c1_forward"] = c1_forward_bench(pf, dev)
            line["paged_prefill"] = paged_prefill_bench(pf, dev)
            if rank == 0:
                line["cpu_baseline"] = cpu_baseline(steps=4)  # ~10-15 s of host work
                pd["cpu_baseline"] = cpu_paged_decode_baseline()
                fd["cpu_baseline"] = cpu_fixed_decode_baseline()
                rp["cpu_baseline"] = cpu_rope_prefill_baseline()
                line["generation"]["cpu_baseline"] = cpu_generation_baseline(pf)
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
