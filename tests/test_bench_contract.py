"""bench.py's reference arm (the restated CpuBackend::linear timed on the host)
prints one JSON line with the keys the benchmark contract asks for."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["metric"] == "fp8_linear_set_tflops" and d["value"] > 0
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    for k in ("value", "unit", "cores", "kind", "sample"):
        assert k in d["cpu_baseline"], k
    assert d["cpu_baseline"]["value"] == d["value"]


def test_host_binding_follows_the_gpu_cpu_affinity(monkeypatch):
    """bench.bind_host_to_gpu reads the GPU's local cores from NVML (a fake
    here: cores 0 and 2 of the process's own set) and moves the process onto
    them; without NVML it changes nothing and returns None."""
    import types
    import torch
    sys.path.insert(0, ROOT)
    import bench
    own = sorted(os.sched_getaffinity(0))
    want = {own[0], own[-1]}
    mask = [0] * ((max(own) // 64) + 1)
    for c in want:
        mask[c // 64] |= 1 << (c % 64)
    seen = {}
    fake = types.SimpleNamespace(
        nvmlInit=lambda: None, nvmlShutdown=lambda: None,
        nvmlDeviceGetHandleByPciBusId=lambda bus: seen.setdefault("bus", bus),
        nvmlDeviceGetCpuAffinity=lambda handle, n: mask[:n] + [0] * max(0, n - len(mask)))
    props = types.SimpleNamespace(pci_domain_id=0, pci_bus_id=0x1B, pci_device_id=0)
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda i: props)
    try:
        assert bench.bind_host_to_gpu(0) == sorted(want)
        assert os.sched_getaffinity(0) == want
        assert seen["bus"] == "00000000:1b:00.0"
    finally:
        os.sched_setaffinity(0, own)
    monkeypatch.setitem(sys.modules, "pynvml", None)  # import fails: no binding
    assert bench.bind_host_to_gpu(0) is None
    assert sorted(os.sched_getaffinity(0)) == own
