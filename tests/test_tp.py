"""Host logic of the tensor-parallel FFN (lightx2v_cuda/tp.py), on CPU.

- weight shards hold exactly the reference's codes and scales: dequantising a
  row or column shard gives the same bits as slicing the dequantised weight;
- the column-split FFN1 / row-split FFN2 composition, with the partial
  products summed by an all-reduce over two gloo ranks and b2 added once,
  equals the unsplit FFN with gated residual (dit.rs:738-760) computed by the
  oracle, up to f32 summation order.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from lightx2v_cuda import quant, tp


def test_split_points_are_even_multiples_of_the_unit():
    assert tp.split_points(8960, 2, 128) == [0, 4480, 8960]
    pts = tp.split_points(8960, 8, 128)
    sizes = np.diff(pts)
    assert pts[0] == 0 and pts[-1] == 8960 and np.all(sizes % 128 == 0)
    assert sizes.max() - sizes.min() <= 128
    assert tp.split_points(256, 4, 128) == [0, 128, 256, 256, 256]


def _weights(kind, rows, cols, seed, oracle):
    w = oracle.normal(seed, rows * cols, 0.02)
    if kind == "q8":
        return quant.Q8.quantize(w, rows, cols)
    if kind == "q4":
        return quant.Q4.quantize(w, rows, cols, 64, True)
    return quant.Fp8E4M3.quantize(w, rows, cols)


@pytest.mark.parametrize("kind", ["q8", "q4", "fp8"])
def test_shards_dequantise_to_slices_of_the_full_weight(kind, oracle):
    rows, cols = 48, 512
    w = _weights(kind, rows, cols, 41, oracle)
    full = w.dequantize().reshape(rows, cols)
    r = tp.slice_rows(w, 16, 40)
    assert np.array_equal(r.dequantize().reshape(24, cols).view(np.uint32), full[16:40].view(np.uint32))
    c = tp.slice_cols(w, 128, 384)
    assert np.array_equal(c.dequantize().reshape(rows, 256).view(np.uint32), full[:, 128:384].view(np.uint32))
    with pytest.raises(AssertionError):
        tp.slice_cols(w, 100, 384)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


D, F, M = 128, 512, 24


def _ffn_inputs(oracle):
    w1 = quant.Fp8E4M3.quantize(oracle.normal(51, F * D, 0.05), F, D)
    w2 = quant.Fp8E4M3.quantize(oracle.normal(52, D * F, 0.05), D, F)
    b1 = oracle.normal(53, F, 0.01)
    b2 = oracle.normal(54, D, 0.01)
    x = oracle.normal(55, M * D)
    h = oracle.normal(56, M * D)
    mods = oracle.normal(57, 6 * D, 0.5)
    return w1, b1, w2, b2, x, h, mods


def _rank_main(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (os.path.join(root, "lightx2v-rs_b200"), os.path.join(root, "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import oracle
    import torch
    import torch.distributed as dist
    from lightx2v_cuda import tp as tpm
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w1, b1, w2, b2, x, h, mods = _ffn_inputs(oracle)
        pts = tpm.split_points(F, world, 128)
        f0, f1 = pts[rank], pts[rank + 1]
        w1r = tpm.slice_rows(w1, f0, f1)
        w2r = tpm.slice_cols(w2, f0, f1)
        hid = oracle.linear(x, M, w1r.dequantize(), f1 - f0, D, bias=b1[f0:f1], act=1)
        part = oracle.linear(hid.reshape(-1), M, w2r.dequantize(), D, f1 - f0,
                             bias=b2 if rank == 0 else None)
        t = torch.from_numpy(np.ascontiguousarray(part, np.float32).reshape(-1))
        dist.all_reduce(t)
        out = oracle.gate_residual(h.reshape(M, D).copy(), t.numpy().reshape(M, D), M, D, mods, 5)
        q.put((rank, np.asarray(out, np.float32).reshape(-1)))
    finally:
        dist.destroy_process_group()


def test_split_ffn_over_two_gloo_ranks_equals_the_full_ffn(oracle):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    outs = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    w1, b1, w2, b2, x, h, mods = _ffn_inputs(oracle)
    hid = oracle.linear(x, M, w1.dequantize(), F, D, bias=b1, act=1)
    lin = oracle.linear(hid.reshape(-1), M, w2.dequantize(), D, F, bias=b2)
    want = np.asarray(oracle.gate_residual(h.reshape(M, D).copy(), lin, M, D, mods, 5), np.float32).reshape(-1)
    assert np.array_equal(outs[0], outs[1])  # h stays replicated
    upd, ref = outs[0] - h, want - h
    assert np.linalg.norm(upd - ref) / np.linalg.norm(ref) <= 1e-5
