"""The VSA plan the sparse-attention entry points take (lightx2v_cuda/vsa.py,
restating crates/lightx2v-core/src/sparse.rs), checked with the reference's
own test values (sparse.rs:104-131), and the oracle's restatement of the CPU
VSA against dense attention at zero sparsity with a zero gate (the property
check.rs:227-255 asserts). No GPU."""
import numpy as np

from lightx2v_cuda import vsa


def test_short_480p_plan_matches_the_reference_test():
    p = vsa.TilePlan.new((21, 30, 52))
    assert p.tiles == (6, 8, 13)
    assert p.num_tiles() == 624
    assert vsa.topk_for(0.8, 624) == 125
    real = p.slot_src[p.slot_src != vsa.PAD]
    assert np.array_equal(np.sort(real), np.arange(p.seq))  # every token in exactly one slot
    assert int(p.block_sizes.sum()) == p.seq
    assert int(p.block_sizes[-1]) == 1 * 2 * 4


def test_topk_is_clamped():
    assert vsa.topk_for(0.0, 7) == 7 and vsa.topk_for(1.0, 7) == 1 and vsa.topk_for(0.99, 3) == 1


def test_oracle_vsa_is_dense_at_zero_sparsity(oracle):
    heads, d, grid = 2, 8, (4, 4, 8)
    spec = vsa.SparseSpec.new(grid, heads, d, 0.0)
    seq = spec.plan.seq
    x = oracle.normal(11, 3 * heads * seq * d)
    q, k, v = np.split(x, 3)
    got = oracle.sparse_attention(q, k, v, np.zeros(heads * seq * d), spec.plan.slot_src, spec.plan.block_sizes,
                                  seq, heads, d, spec.topk, spec.scale)
    want = oracle.attention(q, k, v, heads, seq, seq, d)
    assert np.max(np.abs(got - want)) <= 1e-5
