"""GPU parity at the shapes the reference actually calls the linear with, each
against the C oracle (CpuBackend::linear, crates/lightx2v-cpu/src/lib.rs:
296-326, on weights dequantized by quant.rs), through the C ABI.

- The Q4 sweep of the benchmark configs: Q4 group 64 with HQQ on (the
  shipped `int4-hqq-g64` format), M in {1, 16, 256, 1560, 4680, 18720} at
  K x N = 1536 x 8960 and 8960 x 1536; every kernel the dispatcher picks on
  the way (few-token, single-CTA, two-pass) is covered, and M = 18720 is the
  largest tile count the benchmarks run.
- Fused QKV / cross-attention KV weights stacked from separately quantized
  parts, as load_linear stores them (crates/lightx2v-model/src/dit.rs:61-157):
  Q8::concat, Q4::concat and the inline FP8 stacking.
- The DiT's other linear call sites (dit.rs:450-475, 550-560, 772-781):
  patch_embed 64 -> 1536 and proj_out 1536 -> 64 on native weights over a
  chunk, the text MLP 4096 -> 1536 (GELU) -> 1536 and the cross-attention
  KV 1536 -> 3072 over the 512 text tokens.

Bars: rel-L2 <= 1e-2 against the f32 oracle with identical NaN masks (the
north star's tolerance), on sampled rows where the full oracle would take
minutes; dequantisation of stacked weights bit-exact.
"""
import numpy as np
import pytest

from lightx2v_cuda import BF16, F32, Act, quant

pytestmark = pytest.mark.gpu

REL_L2 = 1e-2


def rel_l2(got, want):
    got = np.asarray(got, np.float64).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    nan_g, nan_w = np.isnan(got), np.isnan(want)
    assert np.array_equal(nan_g, nan_w), f"NaN masks differ: {nan_g.sum()} vs {nan_w.sum()}"
    fin = ~nan_w
    d = np.linalg.norm(got[fin] - want[fin])
    n = np.linalg.norm(want[fin])
    return d / n if n > 0 else d


def sampled_rows(M, n=32):
    return np.array(sorted(set(np.linspace(0, M - 1, min(n, M)).astype(int).tolist() + [M - 1])))


def oracle_rows(oracle, x, K, rows, w_deq, N, bias=None, act=0):
    """The oracle on the sampled token rows only (gathered, then one call)."""
    xs = np.ascontiguousarray(x.reshape(-1, K)[rows])
    return oracle.linear(xs, len(rows), w_deq, N, K, bias=bias, act=act, threads=8)


def q4_hqq(oracle, rows, cols, seed):
    """Q4::quantize(w, rows, cols, 64, hqq = true) by the C restatement (the
    numpy mirror is bit-identical but takes ~100 s on a full matrix)."""
    w = oracle.normal(seed, rows * cols, 0.02)
    q, s, z, g = oracle.q4_quantize(w, rows, cols, 64, True)
    return quant.Q4(q, s, z, rows, cols, g)


# ---- the Q4 sweep, HQQ on -------------------------------------------------------------------
@pytest.fixture(scope="module")
def q4_sweep_weights(be, oracle):
    out = {}
    for K, N, seed in ((1536, 8960, 7 + 1536), (8960, 1536, 7 + 8960)):
        q = q4_hqq(oracle, N, K, seed)
        out[(K, N)] = (q, be.weight_q4(q), oracle.q4_dequantize(q.q, q.scales, q.zeros, q.group))
    return out


@pytest.mark.parametrize("K,N", [(1536, 8960), (8960, 1536)])
@pytest.mark.parametrize("M", [1, 16, 256, 1560, 4680, 18720])
def test_q4_hqq_sweep_matches_oracle(be, oracle, q4_sweep_weights, M, K, N):
    q, dw, deq = q4_sweep_weights[(K, N)]
    x = oracle.normal(11 + M, M * K)
    b = oracle.normal(12, N, 0.01)
    xb, bb = be.upload(x), be.upload(b, F32)
    yb = be.alloc(M * N, BF16)
    be.linear(xb, 0, M, dw, bb, Act.NONE, yb, 0)
    y = be.download(yb).reshape(M, N)
    rows = sampled_rows(M)
    want = oracle_rows(oracle, x, K, rows, deq, N, bias=b)
    assert rel_l2(y[rows], want) <= REL_L2, (M, K, N)
    # the bf16 output holds every row the call covers (no row left unwritten)
    assert np.isfinite(y).all()


# ---- fused QKV / KV stacked from separately quantized parts ---------------------------------
def _parts(fmt, oracle, n_parts, rows, cols, seed):
    parts, deqs = [], []
    for i in range(n_parts):
        w = oracle.normal(seed + i, rows * cols, 0.02)
        if fmt == "q8":
            p = quant.Q8.quantize(w, rows, cols)
            d = oracle.q8_dequantize(p.q, p.scales, p.group)
        elif fmt == "q4":
            q, s, z, g = oracle.q4_quantize(w, rows, cols, 64, True)
            p = quant.Q4(q, s, z, rows, cols, g)
            d = oracle.q4_dequantize(q, s, z, g)
        else:
            p = quant.Fp8E4M3.quantize(w, rows, cols)
            d = oracle.fp8_dequantize(p.q, p.scales, p.group)
        parts.append(p)
        deqs.append(d)
    return parts, np.concatenate(deqs)


def _upload(be, fmt, q):
    return {"q8": be.weight_q8, "q4": be.weight_q4, "fp8": be.weight_fp8}[fmt](q)


@pytest.mark.parametrize("fmt", ["q8", "q4", "fp8"])
@pytest.mark.parametrize("site,n_parts,M", [("qkv", 3, 4680), ("cross_kv", 2, 512)])
def test_stacked_projection_matches_oracle(be, oracle, fmt, site, n_parts, M):
    D = 1536
    parts, deq = _parts(fmt, oracle, n_parts, D, D, seed=300 + n_parts)
    stacked = {"q8": quant.Q8, "q4": quant.Q4, "fp8": quant.Fp8E4M3}[fmt].concat(parts)
    assert stacked.rows == n_parts * D and stacked.cols == D
    dw = _upload(be, fmt, stacked)
    # the stack decodes to the parts' own dequantisations, row block by row block
    got = be.weight_dequant_f32(dw)
    assert np.array_equal(np.isnan(got), np.isnan(deq))
    fin = ~np.isnan(deq)
    assert np.array_equal(got[fin].view(np.uint32), deq[fin].view(np.uint32))
    N = n_parts * D
    x = oracle.normal(310, M * D)
    b = np.concatenate([oracle.normal(320 + i, D, 0.01) for i in range(n_parts)])
    xb, bb = be.upload(x), be.upload(b, F32)
    yb = be.alloc(M * N, BF16)
    be.linear(xb, 0, M, dw, bb, Act.NONE, yb, 0)
    y = be.download(yb).reshape(M, N)
    rows = sampled_rows(M)
    want = oracle_rows(oracle, x, D, rows, deq, N, bias=b)
    assert rel_l2(y[rows], want) <= REL_L2


# ---- the DiT's other call sites ------------------------------------------------------------
@pytest.mark.parametrize("site,M,K,N,act,fmt", [
    ("patch_embed", 4680, 64, 1536, Act.NONE, "native"),      # dit.rs:550-560
    ("proj_out", 4680, 1536, 64, Act.NONE, "native"),         # dit.rs:772-781
    ("text_mlp1", 512, 4096, 1536, Act.GELU_TANH, "native"),  # dit.rs:450-459
    ("text_mlp2", 512, 1536, 1536, Act.NONE, "native"),       # dit.rs:460-469
    ("cross_kv_fp8", 512, 1536, 3072, Act.NONE, "fp8"),       # dit.rs:474
    ("cross_kv_q8", 512, 1536, 3072, Act.NONE, "q8"),
])
def test_dit_call_site_matches_oracle(be, oracle, site, M, K, N, act, fmt):
    w = oracle.normal(400 + K + N, N * K, 0.02)
    if fmt == "native":
        dw, deq = be.weight(w, N, K), w
    elif fmt == "q8":
        q = quant.Q8.quantize(w, N, K)
        dw, deq = be.weight_q8(q), oracle.q8_dequantize(q.q, q.scales, q.group)
    else:
        q = quant.Fp8E4M3.quantize(w, N, K)
        dw, deq = be.weight_fp8(q), oracle.fp8_dequantize(q.q, q.scales, q.group)
    x = oracle.normal(401, M * K)
    b = oracle.normal(402, N, 0.01)
    xb, bb = be.upload(x), be.upload(b, F32)
    for ydt in (BF16, F32):
        yb = be.alloc(M * N, ydt)
        be.linear(xb, 0, M, dw, bb, act, yb, 0)
        y = be.download(yb).reshape(M, N)
        rows = sampled_rows(M, 48)
        want = oracle_rows(oracle, x, K, rows, deq, N, bias=b, act=act)
        assert rel_l2(y[rows], want) <= REL_L2, (site, ydt)
