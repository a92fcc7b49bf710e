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


# ---- the DiT block tensor-parallel over heads ------------------------------------------------
def test_heads_split_unevenly_earlier_ranks_first():
    assert np.diff(tp.head_split_points(12, 8)).tolist() == [2, 2, 2, 2, 1, 1, 1, 1]
    assert tp.head_split_points(24, 8) == list(range(0, 25, 3))
    assert tp.head_split_points(12, 1) == [0, 12]


@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("kind", ["native", "q8"])
def test_attention_shards_reassemble_the_block(oracle, kind, world):
    # per rank: the fused QKV / KV keep their heads' rows of every part, out1
    # / out2 their heads' input columns; across the ranks the shards hold
    # every row and column once, and the ranks' partial out1 products sum to
    # the full one
    heads, hd = 12, 128  # out1 / out2 column shards stay on Q8's 128-wide groups
    d = heads * hd
    def mat(seed, r, c):
        w = oracle.normal(seed, r * c, 0.02)
        return (quant.Q8.quantize(w, r, c) if kind == "q8" else w), oracle.normal(seed + 1, r, 0.01)
    deq = lambda w: w.dequantize() if kind == "q8" else np.asarray(w, np.float32)
    block = {"qkv": mat(1, 3 * d, d), "kv2": mat(3, 2 * d, d), "q2": mat(5, d, d), "out1": mat(7, d, d),
             "out2": mat(9, d, d), "norm_q1": oracle.normal(11, d), "norm_k1": oracle.normal(12, d),
             "norm_q2": oracle.normal(13, d), "norm_k2": oracle.normal(14, d)}
    pts = tp.head_split_points(heads, world)
    shards = [tp.shard_block(block, d, hd, pts[r], pts[r + 1]) for r in range(world)]
    full_qkv = deq(block["qkv"][0]).reshape(3, heads, hd, d)
    got_qkv = np.concatenate([deq(sh["qkv"][0]).reshape(3, -1, hd, d) for sh in shards], axis=1)
    assert np.array_equal(got_qkv, full_qkv)
    full_b = np.asarray(block["qkv"][1]).reshape(3, heads, hd)
    assert np.array_equal(np.concatenate([sh["qkv"][1].reshape(3, -1, hd) for sh in shards], axis=1), full_b)
    assert np.array_equal(np.concatenate([deq(sh["kv2"][0]).reshape(2, -1, hd, d) for sh in shards], axis=1),
                          deq(block["kv2"][0]).reshape(2, heads, hd, d))
    assert np.array_equal(np.concatenate([sh["norm_k1"] for sh in shards]), block["norm_k1"])
    w1 = deq(block["out1"][0]).reshape(d, d)
    assert np.array_equal(np.concatenate([deq(sh["out1"][0]).reshape(d, -1) for sh in shards], axis=1), w1)
    a = oracle.normal(20, 5 * d).reshape(5, d).astype(np.float64)
    parts = sum(a[:, pts[r] * hd:pts[r + 1] * hd] @ deq(shards[r]["out1"][0]).reshape(d, -1).T.astype(np.float64)
                for r in range(world))
    assert np.allclose(parts, a @ w1.T.astype(np.float64), rtol=1e-10, atol=1e-12)


def test_row_sumsq_over_head_shards_is_the_row_sumsq(oracle):
    # the cross-head RMS under head sharding: per-rank sums of squares over
    # their heads' columns, summed, equal the full row's (cpu lib.rs:433-438)
    heads, hd, world = 12, 128, 8
    pts = tp.head_split_points(heads, world)
    x = oracle.normal(30, 7 * heads * hd).reshape(7, -1).astype(np.float64)
    parts = sum((x[:, pts[r] * hd:pts[r + 1] * hd] ** 2).sum(1) for r in range(world))
    assert np.allclose(parts, (x ** 2).sum(1), rtol=1e-12)
