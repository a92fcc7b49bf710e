"""GPU parity of the attention ops against the C oracle (attention_impl,
crates/lightx2v-cpu/src/lib.rs:170-208), through the C ABI.

- The reference's own check cases (crates/lightx2v-model/src/check.rs:
  137-225): attention and the lower-triangular causal mask, head_dim 4, f32
  buffers (the CUDA-core kernel), with the reference's tolerances.
- The tensor-core kernel (head_dim 128, bf16 q/k/v): no mask, a boolean
  mask, and the MemRoPE rule tk <= tq given by temporal indices, on ragged
  shapes (partial query tiles and key blocks), and at the 1.3B chunk's shape
  (12 heads, 4680 queries against an 18720-key cache) on sampled query rows.
  The oracle gets the bf16 values the device holds, so the comparison
  measures the kernel (bf16 P, f32 sums in another order) against rel-L2
  <= 1e-2 (the north star's tolerance), NaN-aware.
"""
import numpy as np
import pytest

from lightx2v_cuda import BF16, F32

pytestmark = pytest.mark.gpu

REL_L2 = 1e-2


def rel_l2(got, want):
    got = np.asarray(got, np.float64).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    nan_g, nan_w = np.isnan(got), np.isnan(want)
    assert np.array_equal(nan_g, nan_w), f"NaN masks differ: {nan_g.sum()} vs {nan_w.sum()}"
    fin = ~nan_w
    return np.linalg.norm(got[fin] - want[fin]) / np.linalg.norm(want[fin])


def device_values(be, a, dtype=BF16):
    """Upload, then read back: the values the kernel sees (bf16-rounded)."""
    b = be.upload(a, dtype)
    return b, be.download(b)


# ---- the reference's check cases (check.rs:137-225), f32 buffers --------------------------
def test_check_attention_hand_case(be, oracle):
    heads, sq, sk, d = 1, 2, 3, 4
    r = oracle.normal(3, heads * (sq + 2 * sk) * d)  # Rng::new(3): q, then k, then v
    q, k, v = r[:8], r[8:20], r[20:32]
    qb, kb, vb = be.upload(q, F32), be.upload(k, F32), be.upload(v, F32)
    ob = be.alloc(sq * d, F32)
    be.attention(qb, kb, vb, heads, sq, sk, d, ob)
    got = be.download(ob)
    sc = (q.reshape(sq, d).astype(np.float64) @ k.reshape(sk, d).T.astype(np.float64)) / np.sqrt(d)
    p = np.exp(sc - sc.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    want = (p @ v.reshape(sk, d)).reshape(-1)
    assert np.abs(got - want).max() <= 1e-6                       # check.rs:169-173
    assert np.abs(got - oracle.attention(q, k, v, heads, sq, sk, d).reshape(-1)).max() <= 1e-6


def test_check_causal_attention_mask(be, oracle):
    heads, sq, sk, d = 1, 3, 3, 4
    r = oracle.normal(5, heads * (sq + 2 * sk) * d)
    q, k, v = r[:12], r[12:24], r[24:36]
    mask = np.tril(np.ones((sq, sk), bool))
    qb, kb, vb = be.upload(q, F32), be.upload(k, F32), be.upload(v, F32)
    ob = be.alloc(sq * d, F32)
    be.causal_attention(qb, kb, vb, heads, sq, sk, d, mask, ob)
    got = be.download(ob)
    want = oracle.attention(q, k, v, heads, sq, sk, d, mask).reshape(-1)
    err = max(np.abs(got - want).max(), np.abs(got[:d] - v[:d]).max())
    assert err <= 1e-5                                              # check.rs:216-224
    # the same mask as temporal indices: query i sees keys j <= i
    tb = be.alloc(sq * d, F32)
    be.causal_attention_temporal(qb, kb, vb, heads, sq, sk, d, np.arange(sq), np.arange(sk), tb)
    assert np.abs(be.download(tb) - want).max() <= 1e-5


# ---- tensor-core kernel --------------------------------------------------------------------
def _qkv(be, oracle, heads, sq, sk, seed):
    qb, q = device_values(be, oracle.normal(seed, heads * sq * 128))
    kb, k = device_values(be, oracle.normal(seed + 1, heads * sk * 128))
    vb, v = device_values(be, oracle.normal(seed + 2, heads * sk * 128))
    return qb, kb, vb, q, k, v


@pytest.mark.parametrize("heads,sq,sk", [(1, 128, 128), (2, 300, 333), (3, 1, 1000), (12, 256, 1408)])
def test_tensor_core_attention_matches_oracle(be, oracle, heads, sq, sk):
    qb, kb, vb, q, k, v = _qkv(be, oracle, heads, sq, sk, 11 + sq)
    for odt in (BF16, F32):
        ob = be.alloc(sq * heads * 128, odt)
        be.attention(qb, kb, vb, heads, sq, sk, 128, ob)
        got = be.download(ob)
        want = oracle.attention(q, k, v, heads, sq, sk, 128)
        assert rel_l2(got, want) <= REL_L2, (heads, sq, sk, odt)


@pytest.mark.parametrize("heads,sq,sk", [(2, 200, 300), (4, 384, 1000)])
def test_tensor_core_attention_with_boolean_mask(be, oracle, heads, sq, sk):
    qb, kb, vb, q, k, v = _qkv(be, oracle, heads, sq, sk, 21 + sk)
    rng = np.random.default_rng(sk)
    mask = rng.random((sq, sk)) < 0.7
    mask[:, 0] = True  # every query sees a key
    ob = be.alloc(sq * heads * 128, F32)
    be.causal_attention(qb, kb, vb, heads, sq, sk, 128, mask, ob)
    want = oracle.attention(q, k, v, heads, sq, sk, 128, mask)
    assert rel_l2(be.download(ob), want) <= REL_L2


def frame_causal(sq, sk, frame, q_frame0):
    """The MemRoPE mask of a chunk: key k belongs to frame k // frame, query i
    to frame q_frame0 + i // frame; a query sees keys of its own and earlier
    frames (dit.rs:645-657)."""
    tk = np.arange(sk) // frame
    tq = q_frame0 + np.arange(sq) // frame
    return tq.astype(np.int32), tk.astype(np.int32)


@pytest.mark.parametrize("heads,sq,sk,frame,q0", [(2, 300, 500, 100, 2), (3, 640, 1280, 160, 4), (1, 200, 333, 37, 0)])
def test_tensor_core_attention_temporal_mask(be, oracle, heads, sq, sk, frame, q0):
    # frames smaller than, equal to and not aligned with the 128-wide tiles:
    # skipped, fully visible and mixed key blocks all occur
    qb, kb, vb, q, k, v = _qkv(be, oracle, heads, sq, sk, 31 + sq)
    tq, tk = frame_causal(sq, sk, frame, q0)
    ob = be.alloc(sq * heads * 128, F32)
    be.causal_attention_temporal(qb, kb, vb, heads, sq, sk, 128, tq, tk, ob)
    got = be.download(ob)
    mask = tk[None, :] <= tq[:, None]
    want = oracle.attention(q, k, v, heads, sq, sk, 128, mask)
    assert rel_l2(got, want) <= REL_L2
    # the boolean form of the same mask gives the same result
    bb = be.alloc(sq * heads * 128, F32)
    be.causal_attention(qb, kb, vb, heads, sq, sk, 128, mask, bb)
    assert rel_l2(be.download(bb), got) <= 1e-5


def test_query_that_sees_no_key_is_nan(be, oracle):
    # the reference's softmax of an all -inf row is NaN (0 / 0); both kernels agree
    heads, sq, sk = 2, 130, 256
    qb, kb, vb, q, k, v = _qkv(be, oracle, heads, sq, sk, 41)
    mask = np.ones((sq, sk), bool)
    mask[5] = False
    mask[129] = False
    ob = be.alloc(sq * heads * 128, F32)
    be.causal_attention(qb, kb, vb, heads, sq, sk, 128, mask, ob)
    got = be.download(ob).reshape(sq, -1)
    assert np.isnan(got[5]).all() and np.isnan(got[129]).all()
    want = oracle.attention(q, k, v, heads, sq, sk, 128, mask)
    assert rel_l2(got, want) <= REL_L2
    # temporal form: queries of frame -1 see nothing
    tq = np.zeros(sq, np.int32)
    tq[:3] = -1
    tk = np.zeros(sk, np.int32)
    tb = be.alloc(sq * heads * 128, F32)
    be.causal_attention_temporal(qb, kb, vb, heads, sq, sk, 128, tq, tk, tb)
    t = be.download(tb).reshape(sq, -1)
    assert np.isnan(t[:3]).all() and np.isfinite(t[3:]).all()


def test_tensor_core_and_generic_kernels_agree(be, oracle):
    # the same bf16 values through the tensor-core kernel (bf16 buffers) and
    # the CUDA-core kernel (f32 buffers holding those values)
    heads, sq, sk = 2, 200, 400
    qb, kb, vb, q, k, v = _qkv(be, oracle, heads, sq, sk, 51)
    tc = be.alloc(sq * heads * 128, F32)
    be.attention(qb, kb, vb, heads, sq, sk, 128, tc)
    gen = be.alloc(sq * heads * 128, F32)
    be.attention(be.upload(q, F32), be.upload(k, F32), be.upload(v, F32), heads, sq, sk, 128, gen)
    want = oracle.attention(q, k, v, heads, sq, sk, 128)
    assert rel_l2(be.download(gen), want) <= 1e-5
    assert rel_l2(be.download(tc), want) <= REL_L2


def test_attention_at_the_chunk_shape(be, oracle):
    # 1.3B chunk: 12 heads x 128, 3 frames of 1560 queries (frames 9-11)
    # against a 12-frame cache of 18720 keys; sampled query rows
    heads, sq, sk, frame = 12, 4680, 18720, 1560
    qb, kb, vb, q, k, v = _qkv(be, oracle, heads, sq, sk, 61)
    tq, tk = frame_causal(sq, sk, frame, 9)
    ob = be.alloc(sq * heads * 128, BF16)
    be.causal_attention_temporal(qb, kb, vb, heads, sq, sk, 128, tq, tk, ob)
    got = be.download(ob).reshape(sq, heads * 128)
    rows = np.array([0, 1, 777, 1559, 1560, 2000, 3119, 3120, 4000, 4679])
    qs = q.reshape(heads, sq, 128)[:, rows].reshape(-1)
    mask = tk[None, :] <= tq[rows][:, None]
    want = oracle.attention(qs, k, v, heads, len(rows), sk, 128, mask)
    assert rel_l2(got[rows], want) <= REL_L2
    assert np.isfinite(got).all()


def test_attention_argument_errors(be):
    from lightx2v_cuda import _lib as L
    qb = be.alloc(2 * 8 * 128)
    kb = be.alloc(2 * 8 * 128)
    ob = be.alloc(8 * 2 * 128)
    with pytest.raises(L.Lx2vError) as e:
        be.attention(qb, kb, kb, 2, 8, 16, 128, ob)    # k holds 8 rows, not 16
    assert e.value.status == L.ERR_INVALID
    with pytest.raises(L.Lx2vError) as e:
        be.attention(qb, kb, kb, 2, 8, 8, 128, qb)     # output aliases q
    assert e.value.status == L.ERR_INVALID


# ---- sparse attention (backend.rs:309-331; VSA, cpu lib.rs:496-606) -------------------------
def test_check_sparse_is_dense_at_zero_sparsity(be, oracle):
    # crates/lightx2v-model/src/check.rs:227-255, tolerance 1e-5: sparsity 0
    # keeps every tile, gate 0 removes the coarse term
    from lightx2v_cuda import vsa
    heads, d, grid = 1, 8, (4, 4, 4)
    seq = 64
    x = oracle.normal(11, 3 * heads * seq * d)  # q, k, v drawn in turn from one stream
    q, k, v = np.split(x, 3)
    qb, kb, vb = be.upload(q, F32), be.upload(k, F32), be.upload(v, F32)
    gb = be.upload(np.zeros(heads * seq * d), F32)
    sp = be.sparse_prepare(vsa.SparseSpec.new(grid, heads, d, 0.0))
    ob, ob2 = be.alloc(seq * d, F32), be.alloc(seq * d, F32)
    be.sparse_attention(qb, kb, vb, gb, sp, ob)
    be.attention(qb, kb, vb, heads, seq, seq, d, ob2)
    assert np.max(np.abs(be.download(ob) - be.download(ob2))) <= 1e-5


@pytest.mark.parametrize("grid,heads,d,sparsity,dtype", [
    ((4, 8, 8), 2, 8, 0.5, F32),      # 4 tiles, keep 2
    ((5, 6, 7), 2, 8, 0.6, F32),      # partial tiles, 8 of them, keep 4
    ((4, 8, 12), 3, 128, 0.5, BF16),  # tensor-core fine stage, 6 tiles, keep 3
])
def test_sparse_attention_matches_oracle(be, oracle, grid, heads, d, sparsity, dtype):
    from lightx2v_cuda import vsa
    spec = vsa.SparseSpec.new(grid, heads, d, sparsity)
    seq = spec.plan.seq
    n = heads * seq * d
    q, k, v = (oracle.normal(60 + i, n) for i in range(3))
    gate = oracle.normal(63, n, 0.5)
    qb, kb, vb = (be.upload(a, dtype) for a in (q, k, v))
    gb = be.upload(gate, F32)
    sp = be.sparse_prepare(spec)
    ob = be.alloc(seq * heads * d, F32)
    be.sparse_attention(qb, kb, vb, gb, sp, ob)
    got = be.download(ob)
    # the oracle on the values the device holds
    qh, kh, vh = (be.download(b) for b in (qb, kb, vb))
    want = oracle.sparse_attention(qh, kh, vh, gate, spec.plan.slot_src, spec.plan.block_sizes, seq, heads, d,
                                   spec.topk, spec.scale).reshape(-1)
    tol = 1e-4 if dtype == F32 else REL_L2
    assert rel_l2(got, want) <= tol
    assert np.isfinite(got).all()
