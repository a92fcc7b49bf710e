#!/usr/bin/env python3
"""Benchmark of the quantized linear hot path on B200.

Workload (the config the headline metric is quoted on):
the FP8 e4m3 linear set of one Wan2.1-1.3B 3-latent-frame chunk, M = 4680
tokens, dim 1536:
    QKV   1536 -> 4608
    out   1536 -> 1536
    FFN1  1536 -> 8960, GELU-tanh
    FFN2  8960 -> 1536, + gated residual into h (dit.rs:748-760)
Weights N(0, 0.02) quantized with the reference's FP8 quantizer (group-128
scales along K), activations bf16 N(0, 1), all seeded (lightx2v-core Rng).
One step = those four linears. Every product is bf16 x bf16 -> f32 on
tcgen05 tensor cores, on weights decoded exactly (the reference's arithmetic)
and rounded to bf16.

value  TFLOP/s with inputs resident in HBM, device-timed with CUDA events per
       step on the library's stream; L2 is flushed (256 MB write) before every
       timed step, outside the timed region.
e2e    the same TFLOP/s through the C ABI with host buffers: every step uploads
       x and h from pinned f32 host memory and downloads h (f32) back.
Multi-GPU (torchrun, one process per GPU): the chunk's 4680 token rows are
split over the ranks with the weights replicated and no collective in the
data path (strong scaling; time = max over ranks). The same line carries
`weak` (every rank a whole chunk of its own) and `tp_ffn` (the chunk's FFN
tensor-parallel over the ranks, with its rel-L2 against the unsplit FFN).
On one GPU the line also carries `configs`: C1 (Q8 1560 x 1536 -> 8960) and
the C3 Q4 sweep at M in {1, 16, 4680} with the few-token chain.

--impl reference times the reference's CPU implementation of the path
(CpuBackend::linear, restated in C under oracle/ because the Rust reference
cannot be built here) on this host's cores, same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "lightx2v-rs_b200"))

M_TOKENS = 4680
DIM = 1536
FFN = 8960
LINEARS = [  # name, N, K, act, seed
    ("qkv", 3 * DIM, DIM, 0, 101),
    ("out", DIM, DIM, 0, 102),
    ("ffn1", FFN, DIM, 1, 103),
    ("ffn2", DIM, FFN, 0, 104),
]
GATE_FFN = 5
WORKLOAD = "fp8_linear_set_wan1.3b_chunk_m4680"


def step_flops(m: int) -> float:
    return float(sum(2.0 * m * n * k for _, n, k, _, _ in LINEARS))


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


def profile_traffic():
    """DRAM bytes per launch of the GEMM kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "gemm_fp8_linear_set.json")
    if os.path.exists(p):
        try:
            return json.load(open(p)).get("dram_bytes_per_launch")
        except Exception:
            return None
    return None


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled during the timed
    region: NVML polled every ~2 ms from a thread (the region is tens of
    milliseconds, shorter than nvidia-smi's sampling period); nvidia-smi is
    the fallback when NVML is unavailable."""

    # NVML clocks-event reason bits
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown"}

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.samples = []          # (time, sm_mhz, reasons_mask)
        self.max_mhz = None
        self.region = (None, None)
        self._stop = threading.Event()
        self._nvml = None
        self._smi = None

    def _handle(self, nv):
        try:
            import torch
            props = torch.cuda.get_device_properties(self.cuda_index)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.cuda_index)

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = self._handle(nv)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self._nvml = (nv, h)
            self._t = threading.Thread(target=self._poll_nvml, daemon=True)
            self._t.start()
        except Exception:
            self._nvml = None
            q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap")
            try:
                self._smi = subprocess.Popen(
                    ["nvidia-smi", "-i", str(self.cuda_index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                     "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self._t = threading.Thread(target=self._read_smi, daemon=True)
                self._t.start()
            except Exception:
                self._smi = None
        return self

    def _poll_nvml(self):
        nv, h = self._nvml
        while not self._stop.is_set():
            try:
                mhz = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                try:
                    mask = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                except AttributeError:
                    mask = int(nv.nvmlDeviceGetCurrentClocksThrottleReasons(h))
                self.samples.append((time.perf_counter(), mhz, mask))
            except Exception:
                return
            time.sleep(0.002)

    def _read_smi(self):
        bits = [0x8, 0x40, 0x20, 0x4]
        for line in self._smi.stdout:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 6:
                continue
            try:
                mhz, self.max_mhz = float(f[0]), float(f[1])
            except ValueError:
                continue
            mask = sum(b for b, v in zip(bits, f[2:6]) if v.lower().startswith("active"))
            self.samples.append((time.perf_counter(), mhz, mask))

    def start_region(self):
        self.region = (time.perf_counter(), None)

    def end_region(self):
        self.region = (self.region[0], time.perf_counter())

    def __exit__(self, *a):
        self._stop.set()
        if self._smi:
            self._smi.terminate()
            try:
                self._smi.wait(timeout=5)
            except Exception:
                self._smi.kill()
        if self._nvml:
            self._t.join(timeout=1)

    def summary(self):
        t0, t1 = self.region
        inside = [s for s in self.samples if t0 is not None and t1 is not None and t0 <= s[0] <= t1]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "source": "nvml" if self._nvml else "nvidia-smi"}
        reasons = sorted({name for _, _, m in inside for bit, name in self.REASONS.items() if m & bit})
        return {"sm_mhz": float(np.median([s[1] for s in inside])), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(inside), "source": "nvml" if self._nvml else "nvidia-smi"}


def make_inputs(m: int, seed_offset: int = 0):
    """Seeded host inputs: FP8-quantized weights, biases, x, h, mods."""
    from lightx2v_cuda import quant, rng
    ws = {}
    for name, n, k, act, seed in LINEARS:
        w = rng.normal(seed, n * k, 0.02)
        ws[name] = (quant.Fp8E4M3.quantize(w, n, k), rng.normal(seed + 1000, n, 0.01))
    x = rng.normal(11 + seed_offset, m * DIM)
    hid0 = None
    h = rng.normal(12 + seed_offset, m * DIM)
    mods = rng.normal(13, 6 * DIM, 0.01)
    return ws, x, h, mods, hid0


# ---------------------------------------------------------------------------------------------
def cpu_sample_rows(total_rows: int, n: int):
    return np.linspace(0, total_rows - 1, n).astype(int)


def run_cpu_linear_set(ws, x, rows_idx, threads: int) -> float:
    """The reference CPU linear (oracle port) on a sample of token rows for all
    four linears; returns seconds."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    deq = {name: (q.dequantize(), b) for name, (q, b) in ws.items()}
    xs = np.ascontiguousarray(x.reshape(-1, DIM)[rows_idx])
    r = len(rows_idx)
    t0 = time.perf_counter()
    qkv = oracle.linear(xs, r, deq["qkv"][0], 3 * DIM, DIM, bias=deq["qkv"][1], threads=threads)
    out = oracle.linear(xs, r, deq["out"][0], DIM, DIM, bias=deq["out"][1], threads=threads)
    hid = oracle.linear(xs, r, deq["ffn1"][0], FFN, DIM, bias=deq["ffn1"][1], act=1, threads=threads)
    y = oracle.linear(hid, r, deq["ffn2"][0], DIM, FFN, bias=deq["ffn2"][1], threads=threads)
    dt = time.perf_counter() - t0
    del qkv, out, y
    return dt


def reference_arm(args, rank: int, world: int):
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.build()
    threads = oracle.openmp_threads()
    ws, x, h, mods, _ = make_inputs(M_TOKENS)
    rows_per_step = max(8, 4 * threads)
    if args.warmup > 0:
        run_cpu_linear_set(ws, x, cpu_sample_rows(M_TOKENS, min(rows_per_step, 8)), threads)
    times = []
    for s in range(args.steps):
        idx = (cpu_sample_rows(M_TOKENS, rows_per_step) + s) % M_TOKENS
        times.append(run_cpu_linear_set(ws, x, idx, threads))
    flops = step_flops(rows_per_step) * args.steps
    tflops = flops / sum(times) / 1e12
    ms_sample_step = sum(times) / args.steps * 1e3
    ms_full_step = ms_sample_step * (M_TOKENS / rows_per_step)
    threading_note = (f"not the reference's threading: CpuBackend::linear is single-threaded; this arm runs "
                      f"the same scalar loop (restated in C) with token rows spread over {threads} OpenMP "
                      f"threads, all this host offers")
    line = {
        "impl": "reference", "metric": "fp8_linear_set_tflops", "value": tflops, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_sample_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "tokens": M_TOKENS, "dim": DIM, "ffn": FFN,
                   "sampled_rows_per_step": rows_per_step},
        "ms_per_full_chunk_extrapolated": ms_full_step,
        "threads": threads,
        "threading": threading_note,
        "cpu_baseline": {"value": tflops, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"each step is {rows_per_step} of {M_TOKENS} token rows through all four "
                                   f"linears (ms_per_step is that sample's measured time; the full chunk, "
                                   f"extrapolated by row count, is ms_per_full_chunk_extrapolated); "
                                   f"{threading_note}"},
        "e2e": {"value": tflops, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
# ---------------------------------------------------------------------------------------------
def ev():
    import torch
    return torch.cuda.Event(enable_timing=True)


def chunk_rows(total: int, rank: int, world: int):
    """Rank r's token rows [r0, r1) of a chunk split over `world` ranks."""
    return total * rank // world, total * (rank + 1) // world


class LinearSet:
    """The chunk's four FP8 linears on rows [0, m) of device buffers."""

    def __init__(self, be, dw, m, x_host, h_host, mods):
        from lightx2v_cuda import F32
        self.be, self.dw, self.m = be, dw, m
        self.xb = be.upload(x_host)           # bf16 activations (the CUDA backend's precision)
        self.hb = be.upload(h_host, F32)      # f32 residual stream
        self.mb = be.upload(mods)
        self.qkv = be.alloc(m * 3 * DIM)
        self.tmp = be.alloc(m * DIM)
        self.hid = be.alloc(m * FFN)

    def linear(self, name, hb=None):
        be, dw, m = self.be, self.dw, self.m
        if name == "qkv":
            be.linear(self.xb, 0, m, dw["qkv"][0], dw["qkv"][1], 0, self.qkv, 0)
        elif name == "out":
            be.linear(self.xb, 0, m, dw["out"][0], dw["out"][1], 0, self.tmp, 0)
        elif name == "ffn1":
            be.linear(self.xb, 0, m, dw["ffn1"][0], dw["ffn1"][1], 1, self.hid, 0)
        else:
            be.linear_gate_residual(self.hid, 0, m, dw["ffn2"][0], dw["ffn2"][1], 0,
                                    self.hb if hb is None else hb, 0, self.mb, GATE_FFN)

    def step(self):
        for name, *_ in LINEARS:
            self.linear(name)


def timed_steps(be, ext, flush, fn, steps, cushion=1):
    """CUDA-event time (ms) of each of `steps` calls of fn on the library's
    stream, L2 flushed (256 MB write) before each, outside the event pair.
    `cushion` > 1 repeats the flush so that the GPU is still busy with it when
    the host has queued the call: for calls of a few microseconds the event
    pair then brackets the kernel, not the host's submission time."""
    import torch
    pairs = []
    for _ in range(steps):
        with torch.cuda.stream(ext):
            for _ in range(cushion):
                flush.zero_()
        a, b = ev(), ev()
        a.record(ext)
        fn()
        b.record(ext)
        pairs.append((a, b))
    be.sync()
    return [a.elapsed_time(b) for a, b in pairs]


def bind_host_to_gpu(local_rank: int):
    """Run this process on the host cores that NVML reports as local to the
    GPU (read with nvmlDeviceGetCpuAffinity; nothing about the GPU is changed),
    so that the end-to-end leg's pinned buffers are first touched, and so
    placed, in that socket's memory and its copies cross no socket link.
    Returns the cores, or None when NVML or the affinity call is unavailable."""
    try:
        import pynvml
        import torch
        props = torch.cuda.get_device_properties(local_rank)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            mask = pynvml.nvmlDeviceGetCpuAffinity(handle, ((os.cpu_count() or 64) + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = {w * 64 + b for w, m in enumerate(mask) for b in range(64) if (m >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return sorted(cpus)
    except Exception:
        return None


def cuda_arm(args, rank: int, world: int, local_rank: int):
    """The headline: the C2 chunk (M = 4680 token rows) through the four FP8
    linears. With N ranks the chunk's rows are split (rank r takes rows
    [r M / N, (r + 1) M / N), weights replicated, no collective in the data
    path: strong scaling); `weak` adds each rank running a whole chunk of
    its own, and `tp_ffn` the chunk's FFN tensor-parallel over the ranks."""
    import torch
    if args.profile:
        os.environ["LIGHTX2V_PROFILE"] = "1"
    from lightx2v_cuda import F32, CudaBackend

    torch.cuda.set_device(local_rank)
    host_cpus = bind_host_to_gpu(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist_mod
        from datetime import timedelta
        dist = dist_mod
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))

    be = CudaBackend(local_rank)
    ext = torch.cuda.ExternalStream(be.stream(), device=torch.device("cuda", local_rank))
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=f"cuda:{local_rank}")
    M = M_TOKENS
    r0, r1 = chunk_rows(M, rank, world)
    m = r1 - r0
    ws, x, h, mods, _ = make_inputs(M)
    dw = {name: (be.weight_fp8(q), be.upload(b)) for name, (q, b) in ws.items()}
    xs = x.reshape(M, DIM)[r0:r1].reshape(-1)
    hs = h.reshape(M, DIM)[r0:r1].reshape(-1)
    strong = LinearSet(be, dw, m, xs, hs, mods)

    def barrier():
        be.sync()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(vals):
        if not dist:
            return [float(v) for v in vals]
        t = torch.tensor(vals, dtype=torch.float64, device=f"cuda:{local_rank}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(v) for v in t.tolist()]

    for _ in range(max(args.warmup, 3)):
        strong.step()
    barrier()

    # --- device-resident timing (strong: the chunk's rows split over the ranks) ---------
    launches0 = be.launch_count()
    with ClockSampler(local_rank) as clk:
        time.sleep(0.01)  # first NVML samples before the region
        clk.start_region()
        step_ms = timed_steps(be, ext, flush, strong.step, args.steps)
        clk.end_region()
    barrier()
    launches = be.launch_count() - launches0
    total_ms = float(sum(step_ms))

    # --- weak scaling: every rank a whole chunk of its own -------------------------------
    full = strong if world == 1 else None
    weak_ms = total_ms
    if world > 1:
        from lightx2v_cuda import rng
        full = LinearSet(be, dw, M, rng.normal(11 + rank, M * DIM), rng.normal(12 + rank, M * DIM), mods)
        for _ in range(max(args.warmup, 3)):
            full.step()
        barrier()
        weak_ms = float(sum(timed_steps(be, ext, flush, full.step, args.steps)))
        barrier()

    # --- per-linear timing on a whole chunk, for the roofline ----------------------------
    kern_ms = {name: [] for name, *_ in LINEARS}
    for _ in range(max(3, min(args.steps, 20))):
        for name, *_ in LINEARS:
            kern_ms[name] += timed_steps(be, ext, flush, lambda: full.linear(name), 1)
    per_kernel = {}
    for name, n, k, act, _s in LINEARS:
        ms = float(np.mean(kern_ms[name]))
        per_kernel[name] = {"ms": ms, "tflops": 2.0 * M * n * k / (ms * 1e-3) / 1e12}
    gemm_ms = sum(v["ms"] for v in per_kernel.values())

    # --- end to end through the C ABI with host buffers (strong split) ------------------
    # Every step writes this rank's x and h rows from page-locked host memory,
    # runs the four linears and reads h back. Steps are pipelined the way a
    # serving loop would run them: the writes go out on the library's copy
    # stream as soon as the buffers they overwrite are free, the read-back is
    # queued without blocking, and h alternates between two device buffers,
    # so step i+1's uploads overlap step i's kernels and read-back.
    x_host = torch.from_numpy(np.ascontiguousarray(xs)).pin_memory()
    h_host = torch.from_numpy(np.ascontiguousarray(hs)).pin_memory()
    h_outs = [torch.empty(m * DIM, dtype=torch.float32).pin_memory() for _ in range(2)]
    hbs = [strong.hb, be.alloc(m * DIM, F32)]

    def e2e_step(i):
        hbi = hbs[i % 2]
        be.write_ptr(strong.xb, x_host.data_ptr(), m * DIM)
        strong.linear("qkv")
        strong.linear("out")
        strong.linear("ffn1")
        be.write_ptr(hbi, h_host.data_ptr(), m * DIM)
        strong.linear("ffn2", hb=hbi)
        be.download_ptr_async(hbi, h_outs[i % 2].data_ptr(), m * DIM)

    for i in range(2):
        e2e_step(i)
    barrier()
    e_a, e_b = ev(), ev()
    e_a.record(ext)
    for i in range(args.steps):
        e2e_step(i)
    e_b.record(ext)
    be.sync()
    barrier()
    e2e_ms = float(e_a.elapsed_time(e_b))

    total_ms, weak_ms, e2e_ms, gemm_ms = max_over_ranks([total_ms, weak_ms, e2e_ms, gemm_ms])

    # --- the chunk's FFN tensor-parallel over the ranks ----------------------------------
    if world > 1:
        uid = [be.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        be.comm_init(uid[0], rank, world)
    try:  # after the headline, like the chunk step below: an error is reported in the line
        tp = tp_ffn_measure(args, be, ext, flush, rank, world, dist, max_over_ranks, barrier)
    except Exception as e:  # noqa: BLE001 - reported, not hidden
        tp = {"n_gpus": world, "error": f"{type(e).__name__}: {e}"[:400]}

    # --- the whole 1.3B chunk step (C4), tensor-parallel on several GPUs -------------------
    chunk = None
    if not args.no_chunk:
        barrier()
        # measured after the headline: an error here (the same on every rank,
        # e.g. a shape a rank count makes unsupported) is reported in the line
        # instead of losing it
        try:
            chunk = chunk_step_measure(args, be, ext, flush, "c4", "fp8", 30, rank, world,
                                       max_over_ranks if world > 1 else None)
            prof = chunk.pop("_profile", None)
            if args.profile:
                chunk["profile_ms_per_step"] = prof
        except Exception as e:  # noqa: BLE001 - reported, not hidden
            chunk = {"n_gpus": world, "error": f"{type(e).__name__}: {e}"[:400]}
        barrier()

    flops_step = step_flops(M)
    value = flops_step * args.steps / (total_ms * 1e-3) / 1e12
    weak_value = flops_step * world * args.steps / (weak_ms * 1e-3) / 1e12
    e2e_value = flops_step * args.steps / (e2e_ms * 1e-3) / 1e12
    peak, hbm, peak_src = measured_peaks()
    achieved = flops_step / (gemm_ms * 1e-3) / 1e12

    configs = None
    cpu = None
    if world == 1:
        configs = measure_configs(be, ext, flush, args, peak, hbm, peak_src)
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            rows = args.cpu_rows
            idx = cpu_sample_rows(M, rows)
            dt = run_cpu_linear_set(ws, x, idx, threads=1)
            cpu = {"value": step_flops(rows) / dt / 1e12, "unit": "TFLOP/s", "cores": 1, "kind": "port",
                   "sample": f"{rows} of {M} token rows through all four linears, single thread "
                             f"({dt:.1f} s); CpuBackend::linear restated in C (oracle/)"}
        clocks = clk.summary()
        line = {
            "metric": "fp8_linear_set_tflops", "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "tokens": M, "tokens_per_gpu": m, "dim": DIM,
                       "ffn": FFN, "weights": "fp8-e4m3 group-128 (reference quantizer)",
                       "linears": [f"{nm} {k}->{n}{' gelu' if a else ''}" for nm, n, k, a, _ in LINEARS]
                       + ["ffn2 fused gated residual into f32 h"],
                       "l2": "flushed (256 MB write) before every timed step, outside the timed region",
                       "parallelism": f"dp{world}: the chunk's token rows split over the ranks, weights "
                                      f"replicated, no collective in the data path"},
            "weak": {"value": weak_value, "unit": "TFLOP/s", "ms_per_step": weak_ms / args.steps,
                     "note": "every rank runs a whole 4680-token chunk of its own (independent replicas)"},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": 2 * M * DIM * 4,
                    "d2h_bytes_per_step": M * DIM * 4,
                    "path": "C ABI, steps pipelined: lx2v_buf_write_f32 x and h rows from pinned host (copy "
                            "stream), 4 linears, lx2v_buf_download_f32_async h; h alternates between two "
                            "device buffers; one event pair around all steps, no L2 flush (each step's "
                            "inputs arrive from the host); bytes summed over ranks",
                    "host_cores": (f"{len(host_cpus)} cores local to the GPU (NVML CPU affinity)" if host_cpus
                                   else "unbound (NVML CPU affinity unavailable)")},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "peak_source": f"bf16 dense burst, {peak_src}",
                         "traffic": profile_traffic(),
                         "kernel": "gemm_ss_pair_kernel (tcgen05.mma cta_group::2, both operands TMA-staged in "
                                   "shared memory) after dequant_bf16_kernel<FP8>; achieved counts both kernels' "
                                   "time, on a whole 4680-token chunk",
                         "per_linear": per_kernel},
            "tp_ffn": tp,
            "chunk_step": chunk,
            "configs": configs,
            "cpu_baseline": cpu,
            "gpu_launches": int(launches),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)

    if dist:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------------------------
def tp_ffn_measure(args, be, ext, flush, rank, world, dist, max_over_ranks, barrier):
    """The chunk's FFN (M = 4680: 1536 -> 8960 GELU -> 1536 + gated residual,
    Q8 weights) tensor-parallel over the ranks (lightx2v_cuda/tp.py: FFN1
    column-split, FFN2 row-split, the partials summed over NVLink): strong
    scaling, the same total work at every N. Time per step = max over ranks
    of the mean CUDA-event time, L2 flushed before each step. Rank 0 also runs
    the unsplit FFN on its own GPU and reports the rel-L2 of the split one's
    h update against it."""
    from lightx2v_cuda import BF16, F32, Act, quant, rng
    from lightx2v_cuda.tp import TensorParallelFFN
    m = M_TOKENS
    # Q8: the kernels' work per element is the FP8 set's apart from the decode
    # pass, and the reference's FP8 quantizer's NaN codes would make every
    # row of the summed h NaN (nothing left to compare)
    w1 = quant.Q8.quantize(rng.normal(103, FFN * DIM, 0.02), FFN, DIM)
    w2 = quant.Q8.quantize(rng.normal(104, DIM * FFN, 0.02), DIM, FFN)
    b1, b2 = rng.normal(1103, FFN, 0.01), rng.normal(1104, DIM, 0.01)
    ffn = TensorParallelFFN(be, rank, world, w1, b1, w2, b2)
    x, h0 = rng.normal(11, m * DIM), rng.normal(12, m * DIM)
    xb = be.upload(x, BF16)
    hb = be.upload(h0, F32)
    mb = be.upload(rng.normal(13, 6 * DIM, 0.01), F32)
    for _ in range(max(args.warmup, 3)):
        ffn.forward(xb, m, hb, mb, GATE_FFN)
    barrier()
    ms = float(np.mean(timed_steps(be, ext, flush, lambda: ffn.forward(xb, m, hb, mb, GATE_FFN), args.steps)))
    barrier()
    # parity: one more step from a fresh h on every rank, against the unsplit FFN
    be.write(hb, h0)
    ffn.forward(xb, m, hb, mb, GATE_FFN)
    got = be.download(hb)
    rel = None
    if rank == 0:
        d1, d2 = be.weight_q8(w1), be.weight_q8(w2)
        hid = be.alloc(m * FFN, BF16)
        be.linear(xb, 0, m, d1, be.upload(b1, F32), Act.GELU_TANH, hid, 0)
        hr = be.upload(h0, F32)
        be.linear_gate_residual(hid, 0, m, d2, be.upload(b2, F32), Act.NONE, hr, 0, mb, GATE_FFN)
        want = be.download(hr) - h0
        upd = got - h0
        fin = ~np.isnan(want)
        rel = float(np.linalg.norm(upd[fin] - want[fin]) / np.linalg.norm(want[fin]))
    (ms,) = max_over_ranks([ms])
    flops = 2.0 * 2.0 * m * DIM * FFN
    return {"value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms, "scaling": "strong",
            "n_gpus": world, "rel_l2_vs_one_gpu": rel,
            "collective": ffn.collective_desc(),
            "workload": f"FFN of the 1.3B chunk, M={m}: {DIM}->{FFN} GELU -> {DIM} + gated residual into f32 h, "
                        "Q8 weights; FFN1 column-split, FFN2 row-split",
            "timing": "max over ranks of the mean CUDA-event time per step; L2 flushed before each"}


# ---------------------------------------------------------------------------------------------
def measure_configs(be, ext, flush, args, peak, hbm, src, which=("c1", "c3")):
    """The other BASELINE configs on one GPU: C1 (Q8 FFN up-projection,
    M = 1560, bias, f32 out) and the C3 Q4 sweep (group 64, HQQ on, quantized
    once) at M in {1, 16, 4680} (`--config c3` runs the whole sweep) at
    K x N = 1536 x 8960 and 8960 x 1536. Device-resident inputs, one
    CUDA-event pair per call on the library's stream, L2 flushed (256 MB
    write) before every call outside the timed region. M <= 16 is judged
    against HBM bandwidth (weight bytes + x + y per call), larger M against
    the bf16 dense tensor peak. The few-token entries add a dependent chain of
    40 linears replayed as a CUDA graph."""
    from lightx2v_cuda import BF16, F32, quant, rng
    cases = []
    if "c1" in which:
        cases.append(("c1", "q8", 1560, 1536, 8960))
    if "c3" in which:
        ms_ = (1, 16, 4680) if "c3full" not in which else (1, 16, 256, 1560, 4680, 18720)
        if getattr(args, "m", None):
            ms_ = tuple(m for m in ms_ if m in args.m)
        cases += [("c3", "q4", m, k, n) for (k, n) in ((1536, 8960), (8960, 1536)) for m in ms_]
        if "c3full" not in which:
            # NVFP4 (no reference counterpart) on the C3 shape at the chunk's token count
            cases.append(("nvfp4", "nvfp4", 4680, 1536, 8960))
    weights, hostq = {}, {}
    for _c, fmt, m, k, n in cases:
        if (fmt, k, n) in weights:
            continue
        if fmt == "q8":  # C1: W seed 2, N(0, 0.02)
            q = quant.Q8.quantize(rng.normal(2, n * k, 0.02), n, k)
            wbytes = n * k + n * (k // q.group) * 4
            weights[(fmt, k, n)] = (be.weight_q8(q), wbytes, "Q8 (reference quantizer)")
        elif fmt == "nvfp4":
            q = quant.Nvfp4.quantize(rng.normal(7 + k, n * k, 0.02), n, k)
            weights[(fmt, k, n)] = (be.weight_nvfp4(q), q.bytes(), "NVFP4 (e2m1 codes, e4m3 block-16 scales)")
        else:
            q = quant.Q4.quantize(rng.normal(7 + k, n * k, 0.02), n, k, 64, True)
            wbytes = n * k // 2 + n * (k // 64) * 4
            weights[(fmt, k, n)] = (be.weight_q4(q), wbytes, "Q4 group 64, HQQ on (reference quantizer)")
        hostq[(fmt, k, n)] = q
    out = {}
    for cname, fmt, m, k, n in cases:
        dw, wbytes, wdesc = weights[(fmt, k, n)]
        if cname == "c1":
            xb, bb = be.upload(rng.normal(1, m * k)), be.upload(rng.normal(3, n, 0.01), F32)
        else:
            xb, bb = be.upload(rng.normal(11, m * k)), be.upload(rng.normal(12, n, 0.01), F32)
        y_f32 = fmt == "q8"
        yb = be.alloc(m * n, F32 if y_f32 else BF16)
        for _ in range(max(args.warmup, 3)):
            be.linear(xb, 0, m, dw, bb, 0, yb, 0)
        be.sync()
        steps = args.steps if m < 4680 else max(3, args.steps // 2)
        ms = float(np.median(timed_steps(be, ext, flush, lambda: be.linear(xb, 0, m, dw, bb, 0, yb, 0), steps,
                                         cushion=4 if m <= 16 else 1)))
        flops = 2.0 * m * n * k
        nbytes = wbytes + m * k * 2 + m * n * (4 if y_f32 else 2) + n * 4
        tflops = flops / (ms * 1e-3) / 1e12
        gbs = nbytes / (ms * 1e-3) / 1e9
        small = m <= 16
        entry = {"workload": f"{fmt} linear M={m} K={k} N={n}", "weights": wdesc, "ms": ms, "tflops": tflops,
                 "gbs": gbs, "steps": steps,
                 "path": ("few-token Q4 kernel (gemv_q4_kernel: codes exact in mma.sync, group affine after)"
                          if fmt == "q4" else "few-token kernel (gemv_kernel)") if small else
                 ("two-pass (dequant_bf16_kernel + gemm_ss_pair_kernel)" if m >= 1024 else "tensor-core"),
                 "roofline": {"bound": "hbm" if small else "tensor", "achieved": gbs if small else tflops,
                              "peak": hbm if small else peak, "unit": "GB/s" if small else "TFLOP/s",
                              "frac": (gbs / hbm) if small else (tflops / peak), "peak_source": src,
                              "bytes_per_call": nbytes}}
        if small and fmt == "q4" and k == 1536 and ("q4", 8960, 1536) in hostq:
            entry["chain"] = q4_chain(be, ext, hostq, m, hbm)
        out[f"{cname}_m{m}_k{k}_n{n}"] = entry
        del xb, bb, yb
    return out


def config_arm(args, local_rank: int):
    """`--config c1` / `--config c3`: one JSON line per shape (c3 runs the whole
    M sweep, M in {1, 16, 256, 1560, 4680, 18720})."""
    import torch
    from lightx2v_cuda import CudaBackend
    torch.cuda.set_device(local_rank)
    be = CudaBackend(local_rank)
    ext = torch.cuda.ExternalStream(be.stream(), device=torch.device("cuda", local_rank))
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=f"cuda:{local_rank}")
    peak, hbm, src = measured_peaks()
    which = ("c1",) if args.config == "c1" else ("c3", "c3full")
    for name, entry in measure_configs(be, ext, flush, args, peak, hbm, src, which).items():
        print(json.dumps({"config": args.config, "case": name, "data": "synthetic",
                          "l2": "flushed (256 MB write) before every call, outside the timed region", **entry}),
              flush=True)


def q4_chain(be, ext, hostq, m, hbm):
    """Sustained few-token throughput: a dependent chain of 40 Q4 linears
    alternating 1536 -> 8960 and 8960 -> 1536 (each reads the previous one's
    output, as consecutive layers of a decode step do), over 20 device copies
    of each weight (310 MB of weights, more than L2 holds, so every launch
    streams its weights from HBM), replayed as one CUDA graph."""
    import torch
    from lightx2v_cuda import BF16, rng
    ups = [be.weight_q4(hostq[("q4", 1536, 8960)]) for _ in range(20)]
    downs = [be.weight_q4(hostq[("q4", 8960, 1536)]) for _ in range(20)]
    a_buf = be.upload(rng.normal(21, m * 1536), BF16)
    b_buf = be.alloc(m * 8960, BF16)

    def chain():
        for i in range(20):
            be.linear(a_buf, 0, m, ups[i], None, 0, b_buf, 0)
            be.linear(b_buf, 0, m, downs[i], None, 0, a_buf, 0)

    chain()
    be.sync()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=ext):
        chain()
    with torch.cuda.stream(ext):  # replay() launches on the current stream
        for _ in range(3):
            g.replay()
        torch.cuda.current_stream().synchronize()
        evs = []
        for _ in range(10):
            e0, e1 = ev(), ev()
            e0.record(ext)
            g.replay()
            e1.record(ext)
            evs.append((e0, e1))
    be.sync()
    ms = float(np.median([e0.elapsed_time(e1) for e0, e1 in evs]))
    wbytes = 20 * (8960 * 1536 // 2 + 8960 * (1536 // 64) * 4) * 2
    gbs = wbytes / (ms * 1e-3) / 1e9
    del g
    return {"launches": 40, "ms": ms, "us_per_launch": ms * 1e3 / 40, "weight_gbs": gbs, "frac_hbm": gbs / hbm,
            "note": "one CUDA graph of 40 dependent linears; weight bytes only in the GB/s"}


def attention_arm(args, local_rank: int):
    """`--config attn`: the causal attention of one 1.3B chunk layer (12 heads x
    128, 4680 queries of latent frames 9-11 against a 12-frame cache of 18720
    keys, key visible when its frame <= the query's: the MemRoPE mask of
    dit.rs:645-657) through lx2v_causal_attention_temporal; bf16 q/k/v,
    device-resident, CUDA events per call, L2 flushed before each. FLOPs:
    4 * d per visible (query, key) pair and head (QK^T and PV)."""
    import torch
    from lightx2v_cuda import BF16, CudaBackend, rng
    torch.cuda.set_device(local_rank)
    be = CudaBackend(local_rank)
    ext = torch.cuda.ExternalStream(be.stream(), device=torch.device("cuda", local_rank))
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=f"cuda:{local_rank}")
    heads, d, frame = 12, 128, 1560
    sq, sk = 3 * frame, 12 * frame
    qb = be.upload(rng.normal(71, heads * sq * d), BF16)
    kb = be.upload(rng.normal(72, heads * sk * d), BF16)
    vb = be.upload(rng.normal(73, heads * sk * d), BF16)
    ob = be.alloc(sq * heads * d, BF16)
    tq = (9 + np.arange(sq) // frame).astype(np.int32)
    tk = (np.arange(sk) // frame).astype(np.int32)
    visible = int(sum(int(np.sum(tk <= t)) for t in (9, 10, 11)) * frame)
    for _ in range(max(args.warmup, 3)):
        be.causal_attention_temporal(qb, kb, vb, heads, sq, sk, d, tq, tk, ob)
    be.sync()
    ms = float(np.median(timed_steps(be, ext, flush, lambda: be.causal_attention_temporal(
        qb, kb, vb, heads, sq, sk, d, tq, tk, ob), args.steps)))
    peak, _hbm, src = measured_peaks()
    flops = 4.0 * d * heads * visible
    dense = 4.0 * d * heads * sq * sk
    print(json.dumps({"config": "attn", "workload": "causal attention, 1.3B chunk layer: 12 heads x 128, sq 4680, "
                                                   "sk 18720, frame-causal mask", "ms": ms,
                      "tflops": flops / (ms * 1e-3) / 1e12, "dense_equivalent_tflops": dense / (ms * 1e-3) / 1e12,
                      "visible_fraction": visible / (sq * sk), "roofline": {"bound": "tensor", "peak": peak,
                      "frac": flops / (ms * 1e-3) / 1e12 / peak, "peak_source": src}, "steps": args.steps}),
          flush=True)


# The chunk-step configs of BASELINE.json: (WanConfig fields, latent frame h x w)
CHUNK_PRESETS = {
    # Wan2.1-T2V-1.3B, 832 x 480 -> latent 104 x 60 -> 52 x 30 patches = 1560 tokens / frame
    "c4": ({"heads": 12, "head_dim": 128, "ffn_dim": 8960, "in_channels": 16, "out_channels": 16}, (60, 104)),
    # Wan2.2-TI2V-5B shape, 1280 x 704 -> latent 80 x 44 (48 channels) -> 40 x 22 = 880 tokens / frame;
    # WanConfig has no 5B preset, so the model is built from these fields directly
    "c5": ({"heads": 24, "head_dim": 128, "ffn_dim": 14336, "in_channels": 48, "out_channels": 48}, (44, 80)),
}


def chunk_step_measure(args, be, ext, flush, preset: str = "c4", fmt: str = "fp8", layers: int = 30,
                       rank: int = 0, world: int = 1, max_over_ranks=None):
    """BASELINE configs C4 / C5: one denoising step of a 3-latent-frame chunk
    through all blocks and the output head, at start frame 12 with each
    layer's MemRoPE cache holding 12 frames after its update. Weights: one
    synthetic block N(0, 0.02) quantized with the reference's quantizer,
    uploaded as `layers` separate device copies; prompt K/V from a random
    512 x 4096 text embedding. The caches are filled by running the chunks
    at start frames 0, 3, 6 and 9 first; every timed step re-runs the chunk
    at frame 12 (the next DMD step of the same chunk overwrites its own
    cache rows). ms per step from CUDA events on the library's stream, L2
    flushed before each. With world > 1 every block runs tensor-parallel
    over the ranks (lightx2v_cuda/tp.py TensorParallelDit; the backend has
    joined the group) and the time is the max over ranks."""
    from lightx2v_cuda import F32, quant, rng
    from lightx2v_cuda.dit import LightDitCuda, WanConfig, synthetic_block
    from lightx2v_cuda.tp import TensorParallelDit
    fields, (lh, lw) = CHUNK_PRESETS[preset]
    cfg = WanConfig(layers=layers, **fields)
    d = cfg.dim
    qz = {"fp8": lambda w, r, c: quant.Fp8E4M3.quantize(w, r, c),
          "q8": lambda w, r, c: quant.Q8.quantize(w, r, c)}[fmt]
    t0 = time.perf_counter()
    block = synthetic_block(cfg, 3, qz)
    mat = lambda seed, r, c: (rng.normal(seed, r * c, 0.02), rng.normal(seed + 1, r, 0.01))
    wargs = (cfg, [block] * layers, mat(901, d, cfg.patch_in), mat(903, d, cfg.text_dim), mat(905, d, d),
             mat(907, cfg.patch_out, d))
    if world == 1:
        model = LightDitCuda(be, *wargs)
    else:
        import torch.distributed as dist

        def exchange(blob):  # the CUDA IPC handles of the shared buffers
            got = [None] * world
            dist.all_gather_object(got, blob)
            return got

        model = TensorParallelDit(be, rank, world, *wargs, exchange=exchange)
    prompt = model.prepare_prompt(rng.normal(911, cfg.text_len * cfg.text_dim))
    ft, frames = (lh // cfg.patch) * (lw // cfg.patch), 3
    s = ft * frames
    ang = rng.normal(931, s * cfg.head_dim // 2, 1.0)
    ws = model.workspace(frames, ft, np.cos(ang), np.sin(ang))
    mods = [be.upload(rng.normal(920 + l % 7, 6 * d, 0.1), F32) for l in range(layers)]
    head = be.upload(rng.normal(930, 2 * d, 0.1), F32)
    out = be.alloc(s * cfg.patch_out, F32)
    latent = be.upload(rng.normal(950, cfg.in_channels * frames * lh * lw), F32)
    setup_s = time.perf_counter() - t0

    def step(start):
        model.patch_embed(ws, latent, cfg.in_channels, frames, lh, lw)
        model.forward_chunk(ws, mods, head, prompt, start, out)

    for start in (0, 3, 6, 9):
        step(start)
    for _ in range(max(args.warmup, 3)):
        step(12)
    be.sync()
    n = max(3, min(args.steps, 10))
    ms = float(np.median(timed_steps(be, ext, flush, lambda: step(12), n)))
    if max_over_ranks is not None:
        (ms,) = max_over_ranks([ms])
    prof = None
    if getattr(args, "profile", False):
        # per-op device time of one more step (the context records events
        # around every op when LIGHTX2V_PROFILE is set)
        be.profile_reset()
        step(12)
        be.sync()
        prof = {k: round(v["ms"], 3) for k, v in sorted(be.profile().items(), key=lambda kv: -kv[1]["ms"])}
    sk = be.kv_cache_len(ws.caches[0])
    # FLOPs: block linears 2 M N K each layer, patch embed and head once;
    # self-attention 4 d per visible (query, key) pair and head (queries of
    # frame 12 + i see the cached frames up to their own); cross-attention
    # 4 d x 512 keys per query and head
    blk = 2.0 * s * d * (3 * d + d + d + d + 2 * cfg.ffn_dim)
    ends = 2.0 * s * cfg.patch_in * d + 2.0 * s * d * cfg.patch_out
    tk = np.array(be.kv_cache_temporal(ws.caches[0]))
    visible = int(sum(int(np.sum(tk <= t)) for t in (12, 13, 14)) * ft)
    att = 4.0 * cfg.head_dim * cfg.heads * (visible + s * cfg.text_len)
    flops = layers * (blk + att) + ends
    return {"n_gpus": world, "parallelism": ("one GPU" if world == 1 else
                                             f"tp{world}: heads and FFN features split; token rows owned per rank, partials reduced and "
                                             "normalised rows gathered over NVLink peer memory (CUDA IPC)"),
            "workload": f"{preset}: {layers} blocks (dim {d}, {cfg.heads} x {cfg.head_dim} heads, FFN {cfg.ffn_dim}) + "
                        f"patch embed + head, {s} tokens ({frames} frames x {ft}), start frame 12, {fmt} block "
                        f"weights, 12-frame MemRoPE cache", "ms_per_step": ms,
            "tflops": flops / (ms * 1e-3) / 1e12, "flop_per_step": flops, "cache_keys": sk,
            "visible_pairs_per_head": visible, "steps": n, "setup_s": setup_s, "_profile": prof,
            "note": "one step = patch_embed + forward_chunk (self-attention over the cache, cross-attention, FFN, "
                    "head) through the C ABI from Python; the caches were filled by four earlier chunks"}


def chunk_arm(args, local_rank: int):
    import torch
    if args.profile:
        os.environ["LIGHTX2V_PROFILE"] = "1"
    from lightx2v_cuda import CudaBackend
    torch.cuda.set_device(local_rank)
    be = CudaBackend(local_rank)
    ext = torch.cuda.ExternalStream(be.stream(), device=torch.device("cuda", local_rank))
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=f"cuda:{local_rank}")
    r = chunk_step_measure(args, be, ext, flush, args.config, args.chunk_format)
    prof = r.pop("_profile", None)
    if args.profile:
        r["profile_ms_per_step"] = prof
    print(json.dumps({"config": args.config, "metric": "chunk_step_ms", "value": r["ms_per_step"], "unit": "ms",
                      "higher_is_better": False, "data": "synthetic", **r}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    ap.add_argument("--cpu-rows", type=int, default=96)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-chunk", action="store_true", help="skip the C4 chunk step in the default line")
    ap.add_argument("--m", type=int, nargs="*", default=None,
                    help="with --config c3: only these token counts of the sweep")
    ap.add_argument("--chunk-format", default="fp8", choices=["fp8", "q8"],
                    help="with --config c4 / c5: the block weights' format")
    ap.add_argument("--profile", action="store_true",
                    help="with --config c4 / c5: add the per-op device times of one step")
    ap.add_argument("--config", default="c2", choices=["c2", "c1", "c3", "attn", "c4", "c5"],
                    help="c2 (default): the headline FP8 linear set, with C1 / C3 and the tensor-parallel FFN as "
                         "extra keys; c1 / c3: those configs alone, one line per shape (c3: the whole M sweep)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank, world)
    elif args.config == "attn":
        if rank == 0:
            attention_arm(args, local_rank)
    elif args.config in ("c4", "c5"):
        if rank == 0:
            chunk_arm(args, local_rank)
    elif args.config != "c2":
        if rank == 0:
            config_arm(args, local_rank)
    else:
        cuda_arm(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
