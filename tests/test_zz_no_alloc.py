"""lx2v_linear_noalloc: the linear for callers that cannot have the library
allocate device memory while they run (a serving loop whose VRAM was planned
up front, or a caller that cannot afford cudaMalloc's device-wide
synchronisation). Its stream-K scratch is a fixed array inside the library,
shared by every call on a device, so this file is collected last: if it
fails, a run that stops at the first failure has already run everything else.

The check: on two calls in a row (the second reuses the array with the first
call's contents still in it), the output equals lx2v_linear's on the same
inputs within the tolerance the GPU tests use for two kernels with the same
bf16 operands and a different f32 summation order, with identical NaN masks.
"""
import numpy as np
import pytest

from lightx2v_cuda import F32, Act, quant

pytestmark = pytest.mark.gpu

SAME_OPERANDS_REL_L2 = 1e-5


def _rel_l2(got, want):
    got = np.asarray(got, np.float64).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    nan_g, nan_w = np.isnan(got), np.isnan(want)
    assert np.array_equal(nan_g, nan_w), f"NaN masks differ: {nan_g.sum()} vs {nan_w.sum()}"
    fin = ~nan_w
    return np.linalg.norm(got[fin] - want[fin]) / np.linalg.norm(want[fin])


@pytest.mark.parametrize("fmt,M,N,K", [("fp8", 1000, 1536, 1536), ("q8", 700, 768, 4096)])
def test_noalloc_linear_matches_linear_twice(be, oracle, fmt, M, N, K):
    w = oracle.normal(201, N * K, 0.02)
    q = quant.Fp8E4M3.quantize(w, N, K) if fmt == "fp8" else quant.Q8.quantize(w, N, K)
    dw = be.weight_fp8(q) if fmt == "fp8" else be.weight_q8(q)
    x = oracle.normal(202, (M + 3) * K)
    b = oracle.normal(203, N, 0.01)
    xb, bb = be.upload(x), be.upload(b)
    ref = be.alloc((M + 5) * N, F32)
    be.linear(xb, 3, M, dw, bb, Act.GELU_TANH, ref, 5)
    want = be.download(ref).reshape(M + 5, N)[5:]
    for call in range(2):
        yb = be.alloc((M + 5) * N, F32)
        be.linear_noalloc(xb, 3, M, dw, bb, Act.GELU_TANH, yb, 5)
        got = be.download(yb).reshape(M + 5, N)
        assert np.all(got[:5] == 0), call           # rows outside [y_row, y_row + rows) untouched
        assert _rel_l2(got[5:], want) <= SAME_OPERANDS_REL_L2, call
