"""A quantized checkpoint in the reference's stored layout, loaded and
uploaded as stored (lightx2v_cuda/weights.py), drives the linear to the
oracle's result on the dequantised weight (backend.rs:199-212)."""
import numpy as np
import pytest

from lightx2v_cuda import F32, Act, quant
from lightx2v_cuda.weights import SafetensorsDir, upload_stored, write_quantized

pytestmark = pytest.mark.gpu


def test_loaded_checkpoint_linears_match_the_oracle(be, oracle, tmp_path):
    N, K, M = 384, 512, 300
    lin = {
        "a": quant.Q8.quantize(oracle.normal(91, N * K, 0.02), N, K),
        "b": quant.Q4.quantize(oracle.normal(92, N * K, 0.02), N, K, 64, True),
        "c": quant.Fp8E4M3.quantize(oracle.normal(93, N * K, 0.02), N, K),
    }
    path = str(tmp_path / "ckpt.safetensors")
    write_quantized(path, lin)
    src = SafetensorsDir(path)
    x = oracle.normal(94, M * K)
    xb = be.upload(x)
    for key, w in lin.items():
        dw = upload_stored(be, src.stored(key))
        yb = be.alloc(M * N, F32)
        be.linear(xb, 0, M, dw, None, Act.NONE, yb, 0)
        got = be.download(yb)
        want = oracle.linear(x, M, w.dequantize(), N, K, threads=8).reshape(-1)
        fin = ~np.isnan(want)  # the reference's FP8 decode gives NaN for its NaN codes
        assert np.array_equal(np.isnan(got), ~fin), key
        assert np.linalg.norm(got[fin] - want[fin]) / np.linalg.norm(want[fin]) <= 1e-2, key
