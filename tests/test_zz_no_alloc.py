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


def test_noalloc_rejects_shapes_it_cannot_run_and_writes_nothing(be, oracle):
    # fewer than 16 rows: the tensor-core kernel behind the no-allocation
    # linear does not take it, so the call fails with UNSUPPORTED before any
    # launch and leaves the output as it was
    from lightx2v_cuda import _lib as L
    N, K = 512, 512
    q = quant.Q8.quantize(oracle.normal(211, N * K, 0.02), N, K)
    dw = be.weight_q8(q)
    xb = be.upload(oracle.normal(212, 8 * K))
    yb = be.alloc(8 * N, F32)
    with pytest.raises(L.Lx2vError) as e:
        be.linear_noalloc(xb, 0, 8, dw, None, Act.NONE, yb, 0)
    assert e.value.status == L.ERR_UNSUPPORTED
    be.sync()
    assert np.all(be.download(yb) == 0)


def test_noalloc_linear_replays_in_a_cuda_graph(be, oracle):
    # captured after an eager call (which looks the scratch array up); every
    # replay must follow the inputs it sees, so the split tiles' flags have to
    # be fresh on each replay even though the captured epoch is fixed
    import torch
    M, N, K = 1000, 1536, 1536
    q = quant.Fp8E4M3.quantize(oracle.normal(221, N * K, 0.02), N, K)
    dw = be.weight_fp8(q)
    x_sets = [be.upload(oracle.normal(222 + i, M * K)) for i in range(2)]
    xb = be.alloc(M * K)
    yb = be.alloc(M * N, F32)
    wants = []
    for xs in x_sets:
        be.copy(xs, 0, xb, 0, M * K)
        be.linear_noalloc(xb, 0, M, dw, None, Act.GELU_TANH, yb, 0)
        wants.append(be.download(yb))
    ref = be.alloc(M * N, F32)
    be.linear(x_sets[0], 0, M, dw, None, Act.GELU_TANH, ref, 0)
    assert _rel_l2(wants[0], be.download(ref)) <= SAME_OPERANDS_REL_L2
    ext = torch.cuda.ExternalStream(be.stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=ext):
        be.linear_noalloc(xb, 0, M, dw, None, Act.GELU_TANH, yb, 0)
    try:
        for r in range(3):
            i = r % 2
            be.copy(x_sets[i], 0, xb, 0, M * K)
            with torch.cuda.stream(ext):
                g.replay()
            assert np.array_equal(be.download(yb), wants[i], equal_nan=True), r
    finally:
        del g
