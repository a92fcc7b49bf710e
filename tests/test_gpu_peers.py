"""The tensor-parallel peer entry points on one GPU (include/lightx2v_cuda.h,
csrc/peer.cu). A group of one rank runs the same kernels as a group of
several, with its own buffers as the "peers": lx2v_tp_reduce_norm must equal
the trait's residual_norm / gate_residual + layer_norm on the rows it owns,
and lx2v_row_sumsq_peers + lx2v_head_split_rms_parts must equal head_split's
own RMS. The barrier's bounded wait is checked with a group whose other rank
never arrives: the wait runs out, the next sync reports LX2V_ERR_DEVICE and
the context keeps working (no fault, no hang). The two-GPU case is
tests/test_gpu_tp.py."""
import numpy as np
import pytest

from lightx2v_cuda import BF16, F32

pytestmark = pytest.mark.gpu


def rel_l2(got, want):
    got = np.asarray(got, np.float64).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    return np.linalg.norm(got - want) / np.linalg.norm(want)


def one_rank_group(be):
    flags = be.alloc(1, F32)
    be.sync()
    return be.peers_create(0, 1, [flags])


@pytest.mark.parametrize("gate", [None, 2])
@pytest.mark.parametrize("part_dtype", [BF16, F32])
def test_reduce_norm_on_one_rank_is_residual_norm(be, oracle, gate, part_dtype):
    rows, dim, r0, r1 = 300, 1536, 40, 250
    g = one_rank_group(be)
    h0 = oracle.normal(201, rows * dim)
    a = oracle.normal(202, rows * dim)
    mods = oracle.normal(203, 6 * dim, 0.5)
    w, b = oracle.normal(204, dim, 0.5), oracle.normal(205, dim, 0.5)
    mb, wb, bb = be.upload(mods, F32), be.upload(w, F32), be.upload(b, F32)
    part = be.upload(a, part_dtype)
    # reference: the trait's residual_norm on the same rows
    h_ref, n_ref = be.upload(h0, F32), be.alloc(rows * dim)
    be.residual_norm(h_ref, part, rows, dim, mb, gate, ("affine", wb, bb), 1e-6, n_ref)
    h, normed = be.upload(h0, F32), be.alloc(rows * dim)
    be.peers_barrier(g)
    be.tp_reduce_norm(g, [part], h, r0, r1, dim, mb, gate, ("affine", wb, bb), None, 1e-6, [normed])
    be.peers_barrier(g)
    got_h = be.download(h).reshape(rows, dim)
    got_n = be.download(normed).reshape(rows, dim)
    want_h = be.download(h_ref).reshape(rows, dim)
    want_n = be.download(n_ref).reshape(rows, dim)
    assert np.array_equal(got_h[:r0], h0.reshape(rows, dim)[:r0])  # rows outside the range untouched
    assert np.array_equal(got_h[r1:], h0.reshape(rows, dim)[r1:])
    assert np.all(got_n[:r0] == 0) and np.all(got_n[r1:] == 0)
    assert rel_l2(got_h[r0:r1], want_h[r0:r1]) <= 1e-6
    assert rel_l2(got_n[r0:r1], want_n[r0:r1]) <= 1e-2


def test_reduce_norm_without_parts_is_layer_norm(be, oracle):
    rows, dim = 128, 3072
    g = one_rank_group(be)
    x = oracle.normal(211, rows * dim)
    mods = oracle.normal(212, 6 * dim, 0.3)
    xb, mb = be.upload(x, F32), be.upload(mods, F32)
    want = be.alloc(rows * dim)
    be.layer_norm(xb, rows, dim, ("mod", 1, 0), mb, 1e-6, want)
    got = be.alloc(rows * dim)
    be.tp_reduce_norm(g, None, xb, 0, rows, dim, None, None, ("mod", 1, 0), mb, 1e-6, [got])
    assert np.array_equal(be.download(xb), x.astype(np.float32))  # no parts: h is only read
    assert rel_l2(be.download(got), be.download(want)) <= 1e-2


def test_peer_row_sums_feed_head_split_like_its_own_rms(be, oracle):
    rows, heads, hd = 200, 4, 128
    g = one_rank_group(be)
    src = be.upload(oracle.normal(221, rows * 3 * heads * hd))
    rms_w = be.upload(oracle.normal(222, heads * hd, 0.5), F32)
    ss = be.alloc(rows, F32)
    be.row_sumsq_peers(g, src, rows, 3 * heads * hd, heads * hd, heads * hd, [ss])
    want, got = be.alloc(rows * heads * hd), be.alloc(rows * heads * hd)
    be.head_split(src, rows, 3 * heads * hd, heads * hd, heads, hd, rms_w, None, 1e-6, want)
    be.head_split_rms_parts(src, rows, 3 * heads * hd, heads * hd, heads, hd, rms_w, ss, 1, heads * hd, None,
                            1e-6, got)
    assert rel_l2(be.download(got), be.download(want)) <= 1e-2


def test_barrier_whose_peer_never_arrives_runs_out_and_the_context_survives(be, oracle):
    from lightx2v_cuda import _lib as L
    own, absent = be.alloc(2, F32), be.alloc(2, F32)  # nobody writes rank 1's slot of `own`
    be.sync()
    g = be.peers_create(0, 2, [own, absent])
    be.set_wait_limit_ns(1_000_000)  # 1 ms
    try:
        be.peers_barrier(g)
        with pytest.raises(L.Lx2vError) as e:
            be.sync()
        assert e.value.status == L.ERR_DEVICE
    finally:
        be.set_wait_limit_ns(2_000_000_000)
    be.sync()  # the error word was cleared
    # rank 0 stored its epoch into both arrays before waiting
    assert be.download(own)[0] != 0 and be.download(absent)[0] != 0
    x = oracle.normal(231, 64 * 256)
    xb, out = be.upload(x, F32), be.alloc(64 * 256)
    mods = be.upload(oracle.normal(232, 2 * 256, 0.1), F32)
    be.layer_norm(xb, 64, 256, ("mod", 1, 0), mods, 1e-6, out)
    assert np.isfinite(be.download(out)).all()
