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
One step = those four linears. Every arithmetic op is bf16 x bf16 -> f32 on
tcgen05 tensor cores after exact in-register dequantisation.

value  TFLOP/s with inputs resident in HBM, device-timed with CUDA events per
       step on the library's stream; L2 is flushed (256 MB write) before every
       timed step, outside the timed region.
e2e    the same TFLOP/s through the C ABI with host buffers: every step uploads
       x and h from pinned f32 host memory and downloads h (f32) back.
Multi-GPU (torchrun): weak scaling, each rank runs its own 4680-token chunk
with replicated weights and no collective in the data path; time = max over
ranks.

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
def cuda_arm(args, rank: int, world: int, local_rank: int):
    import torch
    from lightx2v_cuda import BF16, F32, CudaBackend

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist_mod
        from datetime import timedelta
        dist = dist_mod
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))

    be = CudaBackend(local_rank)
    ext = torch.cuda.ExternalStream(be.stream(), device=torch.device("cuda", local_rank))
    m = M_TOKENS
    ws, x, h, mods, _ = make_inputs(m, seed_offset=rank)
    dw = {name: (be.weight_fp8(q), be.upload(b)) for name, (q, b) in ws.items()}
    xb = be.upload(x)                     # bf16 activations (the CUDA backend's precision)
    hb = be.upload(h, F32)                # f32 residual stream
    mb = be.upload(mods)
    qkv = be.alloc(m * 3 * DIM)
    tmp = be.alloc(m * DIM)
    hid = be.alloc(m * FFN)

    def step():
        be.linear(xb, 0, m, dw["qkv"][0], dw["qkv"][1], 0, qkv, 0)
        be.linear(xb, 0, m, dw["out"][0], dw["out"][1], 0, tmp, 0)
        be.linear(xb, 0, m, dw["ffn1"][0], dw["ffn1"][1], 1, hid, 0)
        be.linear_gate_residual(hid, 0, m, dw["ffn2"][0], dw["ffn2"][1], 0, hb, 0, mb, GATE_FFN)

    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=f"cuda:{local_rank}")

    def flush_l2():
        with torch.cuda.stream(ext):
            flush.zero_()

    def ev():
        return torch.cuda.Event(enable_timing=True)

    for _ in range(max(args.warmup, 3)):
        step()
    be.sync()

    # --- device-resident timing -----------------------------------------------------------
    def barrier():
        be.sync()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    barrier()
    launches0 = be.launch_count()
    pairs = []
    with ClockSampler(local_rank) as clk:
        time.sleep(0.01)  # first NVML samples before the region
        clk.start_region()
        for _ in range(args.steps):
            flush_l2()
            a, b = ev(), ev()
            a.record(ext)
            step()
            b.record(ext)
            pairs.append((a, b))
        be.sync()
        clk.end_region()
    barrier()
    launches = be.launch_count() - launches0
    step_ms = [a.elapsed_time(b) for a, b in pairs]
    total_ms = float(sum(step_ms))

    # --- per-kernel timing for the roofline (same launches, one event pair each) ----------
    kern_ms = {name: [] for name, *_ in LINEARS}
    for _ in range(max(3, min(args.steps, 20))):
        for name, n, k, act, _s in LINEARS:
            flush_l2()
            a, b = ev(), ev()
            a.record(ext)
            if name == "qkv":
                be.linear(xb, 0, m, dw["qkv"][0], dw["qkv"][1], 0, qkv, 0)
            elif name == "out":
                be.linear(xb, 0, m, dw["out"][0], dw["out"][1], 0, tmp, 0)
            elif name == "ffn1":
                be.linear(xb, 0, m, dw["ffn1"][0], dw["ffn1"][1], 1, hid, 0)
            else:
                be.linear_gate_residual(hid, 0, m, dw["ffn2"][0], dw["ffn2"][1], 0, hb, 0, mb, GATE_FFN)
            b.record(ext)
            kern_ms[name].append((a, b))
    be.sync()
    per_kernel = {}
    for name, n, k, act, _s in LINEARS:
        ms = float(np.mean([a.elapsed_time(b) for a, b in kern_ms[name]]))
        per_kernel[name] = {"ms": ms, "tflops": 2.0 * m * n * k / (ms * 1e-3) / 1e12}
    gemm_ms = sum(v["ms"] for v in per_kernel.values())

    # --- end to end through the C ABI with host buffers ------------------------------------
    # Every step writes x and h from page-locked host memory, runs the four
    # linears and reads h back. Steps are pipelined the way a serving loop
    # would run them: the writes go out on the library's copy stream as soon
    # as the buffers they overwrite are free, the read-back is queued without
    # blocking, and h alternates between two device buffers, so step i+1's
    # uploads overlap step i's kernels and read-back.
    x_host = torch.from_numpy(x).pin_memory()
    h_host = torch.from_numpy(h).pin_memory()
    h_outs = [torch.empty(m * DIM, dtype=torch.float32).pin_memory() for _ in range(2)]
    hbs = [hb, be.alloc(m * DIM, F32)]

    def e2e_step(i):
        hbi = hbs[i % 2]
        be.write_ptr(xb, x_host.data_ptr(), m * DIM)
        be.linear(xb, 0, m, dw["qkv"][0], dw["qkv"][1], 0, qkv, 0)
        be.linear(xb, 0, m, dw["out"][0], dw["out"][1], 0, tmp, 0)
        be.linear(xb, 0, m, dw["ffn1"][0], dw["ffn1"][1], 1, hid, 0)
        be.write_ptr(hbi, h_host.data_ptr(), m * DIM)
        be.linear_gate_residual(hid, 0, m, dw["ffn2"][0], dw["ffn2"][1], 0, hbi, 0, mb, GATE_FFN)
        be.download_ptr_async(hbi, h_outs[i % 2].data_ptr(), m * DIM)

    for i in range(2):
        e2e_step(i)
    be.sync()
    barrier()
    e_a, e_b = ev(), ev()
    e_a.record(ext)
    for i in range(args.steps):
        e2e_step(i)
    e_b.record(ext)
    be.sync()
    barrier()
    e2e_ms = float(e_a.elapsed_time(e_b))

    # --- max over ranks --------------------------------------------------------------------
    if dist:
        t = torch.tensor([total_ms, e2e_ms, gemm_ms], dtype=torch.float64, device=f"cuda:{local_rank}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_ms, gemm_ms = (float(v) for v in t.tolist())

    flops_all = step_flops(m) * args.steps * world
    value = flops_all / (total_ms * 1e-3) / 1e12
    e2e_value = flops_all / (e2e_ms * 1e-3) / 1e12
    peak, _hbm, peak_src = measured_peaks()
    achieved = step_flops(m) / (gemm_ms * 1e-3) / 1e12

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            rows = args.cpu_rows
            idx = cpu_sample_rows(m, rows)
            dt = run_cpu_linear_set(ws, x, idx, threads=1)
            cpu = {"value": step_flops(rows) / dt / 1e12, "unit": "TFLOP/s", "cores": 1, "kind": "port",
                   "sample": f"{rows} of {m} token rows through all four linears, single thread "
                             f"({dt:.1f} s); CpuBackend::linear restated in C (oracle/)"}
        clocks = clk.summary()
        line = {
            "metric": "fp8_linear_set_tflops", "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "tokens_per_gpu": m, "global_tokens": m * world, "dim": DIM,
                       "ffn": FFN, "weights": "fp8-e4m3 group-128 (reference quantizer)",
                       "linears": [f"{nm} {k}->{n}{' gelu' if a else ''}" for nm, n, k, a, _ in LINEARS]
                       + ["ffn2 fused gated residual into f32 h"],
                       "l2": "flushed (256 MB write) before every timed step, outside the timed region",
                       "parallelism": f"dp{world} (token rows; weights replicated; no collective)"},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": 2 * m * DIM * 4,
                    "d2h_bytes_per_step": m * DIM * 4,
                    "path": "C ABI, steps pipelined: lx2v_buf_write_f32 x and h from pinned host (copy "
                            "stream), 4 linears, lx2v_buf_download_f32_async h; h alternates between two "
                            "device buffers; one event pair around all steps, no L2 flush (each step's "
                            "inputs arrive from the host)"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "peak_source": f"bf16 dense burst, {peak_src}",
                         "traffic": profile_traffic(),
                         "kernel": "gemm_ss_pair_kernel (tcgen05.mma cta_group::2, both operands TMA-staged in "
                                   "shared memory) after dequant_bf16_kernel<FP8>; achieved counts both kernels' time",
                         "per_linear": per_kernel},
            "cpu_baseline": cpu,
            "gpu_launches": int(launches),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)

    del pairs
    if dist:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------------------------
def config_arm(args, local_rank: int):
    """The other BASELINE configs as single-GPU parity/throughput cases, one JSON
    line per shape: C1 (Q8 FFN up-projection, M = 1560) and the C3 Q4 sweep
    (M in {1, 16, 256, 1560, 4680, 18720} at K x N = 1536 x 8960 and
    8960 x 1536). Device-resident inputs, one CUDA-event pair per call on the
    library's stream, L2 flushed (256 MB write) before every call outside the
    timed region. M <= 16 is judged against HBM bandwidth (weight bytes + x +
    y per call), larger M against the bf16 dense tensor peak."""
    import torch
    from lightx2v_cuda import BF16, F32, CudaBackend, quant, rng

    torch.cuda.set_device(local_rank)
    be = CudaBackend(local_rank)
    ext = torch.cuda.ExternalStream(be.stream(), device=torch.device("cuda", local_rank))
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=f"cuda:{local_rank}")
    peak, hbm, src = measured_peaks()
    if args.config == "c1":
        cases = [("q8", 1560, 1536, 8960)]
    else:
        cases = [("q4", m, k, n) for (k, n) in ((1536, 8960), (8960, 1536))
                 for m in (1, 16, 256, 1560, 4680, 18720)]
    weights, hostq = {}, {}
    for fmt, m, k, n in cases:
        if (fmt, k, n) in weights:
            continue
        w = rng.normal(7 + k, n * k, 0.02)
        if fmt == "q8":
            q = quant.Q8.quantize(w, n, k)
            wbytes = n * k + n * (k // q.group) * 4
            weights[(fmt, k, n)] = (be.weight_q8(q), wbytes, "Q8 (reference quantizer)")
        else:
            # HQQ refinement changes the scale/zero values, not the packed
            # format or the kernel's work; skipped to keep the run short
            q = quant.Q4.quantize(w, n, k, 64, False)
            wbytes = n * k // 2 + n * (k // 64) * 4
            weights[(fmt, k, n)] = (be.weight_q4(q), wbytes, "Q4 group 64 (reference quantizer, HQQ off)")
        hostq[(fmt, k, n)] = q
    for fmt, m, k, n in cases:
        dw, wbytes, wdesc = weights[(fmt, k, n)]
        xb = be.upload(rng.normal(11, m * k))
        bb = be.upload(rng.normal(12, n, 0.01), F32)
        y_f32 = fmt == "q8"
        yb = be.alloc(m * n, F32 if y_f32 else BF16)
        for _ in range(max(args.warmup, 3)):
            be.linear(xb, 0, m, dw, bb, 0, yb, 0)
        be.sync()
        evs = []
        steps = args.steps if m < 4680 else max(3, args.steps // 4)
        for _ in range(steps):
            with torch.cuda.stream(ext):
                flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(ext)
            be.linear(xb, 0, m, dw, bb, 0, yb, 0)
            b.record(ext)
            evs.append((a, b))
        be.sync()
        ms = float(np.median([a.elapsed_time(b) for a, b in evs]))
        flops = 2.0 * m * n * k
        nbytes = wbytes + m * k * 2 + m * n * (4 if y_f32 else 2) + n * 4
        tflops = flops / (ms * 1e-3) / 1e12
        gbs = nbytes / (ms * 1e-3) / 1e9
        small = m <= 16
        line = {"config": args.config, "workload": f"{fmt} linear M={m} K={k} N={n}", "weights": wdesc,
                "ms": ms, "tflops": tflops, "gbs": gbs, "steps": steps, "data": "synthetic",
                "l2": "flushed (256 MB write) before every call, outside the timed region",
                "path": "few-token kernel" if small else ("two-pass (decode + gemm_ss_pair_kernel)"
                                                          if m >= 1024 else "tensor-core single-CTA kernel"),
                "roofline": {"bound": "hbm" if small else "tensor",
                             "achieved": gbs if small else tflops,
                             "peak": hbm if small else peak, "unit": "GB/s" if small else "TFLOP/s",
                             "frac": (gbs / hbm) if small else (tflops / peak), "peak_source": src,
                             "bytes_per_call": nbytes}}
        if small and fmt == "q4" and (fmt, 8960, 1536) in hostq and (fmt, 1536, 8960) in hostq and k == 1536:
            line["chain"] = q4_chain(be, ext, hostq, m, hbm)
        print(json.dumps(line), flush=True)
        del xb, bb, yb


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
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
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


# ---------------------------------------------------------------------------------------------
def tpffn_arm(args, rank: int, world: int, local_rank: int):
    """The chunk's FFN (M = 4680, 1536 -> 8960 GELU -> 1536 + gated residual, Q8)
    tensor-parallel over the torchrun ranks (lightx2v_cuda/tp.py: FFN1
    column-split, FFN2 row-split, one NCCL all-reduce through the C ABI):
    strong scaling, the same total work at every N. Time per step = max over
    ranks of CUDA-event times on each library stream, L2 flushed before every
    step outside the timed region."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from lightx2v_cuda import BF16, F32, CudaBackend, quant, rng
    from lightx2v_cuda.tp import TensorParallelFFN

    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))  # id exchange and timing max
    be = CudaBackend(local_rank)
    if world > 1:
        uid = [be.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        be.comm_init(uid[0], rank, world)
    m = M_TOKENS
    # Q8 (quantized in well under a second; the kernels' work per element is
    # the same as FP8's apart from the decode pass)
    w1 = quant.Q8.quantize(rng.normal(103, FFN * DIM, 0.02), FFN, DIM)
    w2 = quant.Q8.quantize(rng.normal(104, DIM * FFN, 0.02), DIM, FFN)
    ffn = TensorParallelFFN(be, rank, world, w1, rng.normal(1103, FFN, 0.01), w2, rng.normal(1104, DIM, 0.01))
    xb = be.upload(rng.normal(11, m * DIM), BF16)
    hb = be.upload(rng.normal(12, m * DIM), F32)
    mb = be.upload(rng.normal(13, 6 * DIM, 0.01), F32)
    ext = torch.cuda.ExternalStream(be.stream(), device=torch.device("cuda", local_rank))
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=f"cuda:{local_rank}")
    for _ in range(max(args.warmup, 3)):
        ffn.forward(xb, m, hb, mb, GATE_FFN)
    be.sync()
    if world > 1:
        dist.barrier()
    evs = []
    for _ in range(args.steps):
        with torch.cuda.stream(ext):
            flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(ext)
        ffn.forward(xb, m, hb, mb, GATE_FFN)
        b.record(ext)
        evs.append((a, b))
    be.sync()
    ms = float(np.mean([a.elapsed_time(b) for a, b in evs]))
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    flops = 2.0 * 2.0 * m * DIM * FFN
    if rank == 0:
        print(json.dumps({"config": "tpffn", "metric": "tp_ffn_tflops", "value": flops / (ms * 1e-3) / 1e12,
                          "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "ms_per_step": ms,
                          "scaling": "strong", "dtype": "bf16", "data": "synthetic",
                          "workload": f"FFN of the 1.3B chunk, M={m}: {DIM}->{FFN} GELU -> {DIM} + gated residual, "
                                      "Q8 weights; FFN1 column-split, FFN2 row-split, NCCL all-reduce (f32)",
                          "timing": "max over ranks of the mean CUDA-event time per step; L2 flushed before each"}),
              flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    ap.add_argument("--cpu-rows", type=int, default=96)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", default="c2", choices=["c2", "c1", "c3", "tpffn"],
                    help="c2 (default): the headline FP8 linear set; c1 / c3: the other configs, one line per "
                         "shape; tpffn: the chunk's FFN tensor-parallel over the torchrun ranks")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank, world)
    elif args.config == "tpffn":
        tpffn_arm(args, rank, world, local_rank)
    elif args.config != "c2":
        if rank == 0:
            config_arm(args, local_rank)
    else:
        cuda_arm(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
