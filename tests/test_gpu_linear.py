"""GPU parity of the quantized linear against the C oracle (restating
CpuBackend::linear, crates/lightx2v-cpu/src/lib.rs:296-326, on weights
dequantized by quant.rs). All calls go through the C ABI (lightx2v_cuda).

Tolerances: dequantisation bit-exact; GEMM outputs
rel-L2 <= 1e-2 against the f32 oracle, NaN-aware for FP8 (identical NaN
masks, rel-L2 over the finite entries).
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


def make_weight(fmt, rows, cols, seed, std=0.02, group=64, hqq=True, oracle=None):
    w = oracle.normal(seed, rows * cols, std)
    if fmt == "q8":
        q = quant.Q8.quantize(w, rows, cols)
    elif fmt == "q4":
        q = quant.Q4.quantize(w, rows, cols, group, hqq)
    elif fmt == "fp8":
        q = quant.Fp8E4M3.quantize(w, rows, cols)
    else:
        q = None
    return w, q


def oracle_dequant(oracle, fmt, q, w):
    if fmt == "q8":
        return oracle.q8_dequantize(q.q, q.scales, q.group)
    if fmt == "q4":
        return oracle.q4_dequantize(q.q, q.scales, q.zeros, q.group)
    if fmt == "fp8":
        return oracle.fp8_dequantize(q.q, q.scales, q.group)
    return w


def upload_weight(be, fmt, q, w, rows, cols):
    if fmt == "q8":
        return be.weight_q8(q)
    if fmt == "q4":
        return be.weight_q4(q)
    if fmt == "fp8":
        return be.weight_fp8(q)
    return be.weight(w, rows, cols)


# ---- dequantisation: bit-exact -------------------------------------------------
@pytest.mark.parametrize("fmt,rows,cols,group", [
    ("q8", 8960, 1536, None), ("q8", 1536, 8960, None), ("q8", 33, 200, None),
    ("fp8", 4608, 1536, None), ("fp8", 1536, 8960, None), ("fp8", 17, 96, None),
    ("q4", 8960, 1536, 64), ("q4", 64, 256, 16), ("q4", 9, 200, 64), ("q4", 8, 24, 8),
])
def test_dequant_bit_exact(be, oracle, fmt, rows, cols, group):
    w, q = make_weight(fmt, rows, cols, seed=11 + rows, group=group or 64, hqq=(rows < 4096),
                       oracle=oracle)
    dw = upload_weight(be, fmt, q, w, rows, cols)
    got = be.weight_dequant_f32(dw)
    want = oracle_dequant(oracle, fmt, q, w)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    fin = ~np.isnan(want)
    assert np.array_equal(got[fin].view(np.uint32), want[fin].view(np.uint32))


def test_fp8_special_codes_bit_exact(be, oracle):
    # every code byte, including the NaN codes and the exponent-field-0 codes
    # the reference decodes as m/8 * 2^-9, with fast and slow scales
    rows, cols = 8, 256
    codes = np.tile(np.arange(256, dtype=np.uint8), rows * cols // 256)
    for scales in (np.full(rows * cols // 128, 0.01, np.float32),
                   np.full(rows * cols // 128, 300.0, np.float32)):
        q = quant.Fp8E4M3(codes.copy(), scales, rows, cols, 128)
        got = be.weight_dequant_f32(be.weight_fp8(q))
        want = oracle.fp8_dequantize(codes, scales, 128)
        assert np.array_equal(np.isnan(got), np.isnan(want))
        fin = ~np.isnan(want)
        assert np.array_equal(got[fin].view(np.uint32), want[fin].view(np.uint32))


# ---- linear: small shapes against the oracle ------------------------------------------
@pytest.mark.parametrize("fmt", ["q8", "q4", "fp8", "native"])
@pytest.mark.parametrize("M", [1, 3, 17, 129, 300])
def test_linear_small_shapes(be, oracle, fmt, M):
    N, K = 384, 256
    w, q = make_weight(fmt, N, K, seed=3, oracle=oracle)
    dw = upload_weight(be, fmt, q, w, N, K)
    x = oracle.normal(1, M * K)
    b = oracle.normal(2, N, 0.01)
    xb, bb = be.upload(x), be.upload(b)
    for act in (Act.NONE, Act.GELU_TANH):
        for ydt in (BF16, F32):
            yb = be.alloc(M * N, ydt)
            be.linear(xb, 0, M, dw, bb, act, yb, 0)
            got = be.download(yb).reshape(M, N)
            want = oracle.linear(x, M, oracle_dequant(oracle, fmt, q, w), N, K, bias=b, act=act,
                                 threads=8)
            assert rel_l2(got, want) <= REL_L2, (fmt, M, act, ydt)


@pytest.mark.parametrize("fmt", ["q8", "q4", "fp8"])
def test_tensor_core_path_matches_generic_path(be, oracle, fmt):
    M, N, K = 300, 640, 512
    w, q = make_weight(fmt, N, K, seed=5, oracle=oracle)
    dw = upload_weight(be, fmt, q, w, N, K)
    xb = be.upload(oracle.normal(6, M * K))
    bb = be.upload(oracle.normal(7, N, 0.01))
    outs = []
    for path in (1, 3):
        be.set_linear_path(path)
        yb = be.alloc(M * N, F32)
        be.linear(xb, 0, M, dw, bb, Act.GELU_TANH, yb, 0)
        outs.append(be.download(yb))
    be.set_linear_path(0)
    # same bf16 operands, different f32 summation order
    assert rel_l2(outs[0], outs[1]) <= 1e-5


def test_row_offsets_write_only_their_rows(be, oracle):
    # linear(x, x_row, rows, ..., y, y_row) as the FFN chunk loop calls it
    # (crates/lightx2v-model/src/dit.rs:735-759): other rows stay untouched.
    N, K, M = 256, 256, 200
    w, q = make_weight("q8", N, K, seed=8, oracle=oracle)
    dw = be.weight_q8(q)
    x = oracle.normal(9, M * K)
    xb = be.upload(x)
    sentinel = np.full(M * N, 7.0, np.float32)
    yb = be.upload(sentinel, F32)
    be.linear(xb, 40, 100, dw, None, Act.NONE, yb, 60)
    y = be.download(yb).reshape(M, N)
    assert np.all(y[:60] == 7.0) and np.all(y[160:] == 7.0)
    want = oracle.linear(x, 100, q.dequantize(), N, K, x_row=40, threads=8)
    assert rel_l2(y[60:160], want) <= REL_L2


# ---- BASELINE shapes: sampled rows against the oracle -------------------------------------
def sampled_rows(M, n=24):
    rows = sorted(set(np.linspace(0, M - 1, n).astype(int).tolist() + [M - 1]))
    return np.array(rows)


def test_config1_q8_ffn_up(be, oracle):
    # Q8, X [1560,1536] ~ N(0,1) seed 1, W [8960,1536] ~ N(0,0.02)
    # seed 2, bias ~ N(0,0.01) seed 3, f32 output.
    M, K, N = 1560, 1536, 8960
    x = oracle.normal(1, M * K)
    w = oracle.normal(2, N * K, 0.02)
    b = oracle.normal(3, N, 0.01)
    q = quant.Q8.quantize(w, N, K)
    dw = be.weight_q8(q)
    xb, bb = be.upload(x), be.upload(b)
    yb = be.alloc(M * N, F32)
    be.linear(xb, 0, M, dw, bb, Act.NONE, yb, 0)
    y = be.download(yb).reshape(M, N)
    rows = sampled_rows(M)
    want = np.stack([oracle.linear(x, 1, q.dequantize(), N, K, bias=b, x_row=int(r), threads=8)[0]
                     for r in rows])
    assert rel_l2(y[rows], want) <= REL_L2
    assert np.isfinite(y).all()


@pytest.mark.parametrize("name,N,K,act", [("qkv", 4608, 1536, Act.NONE), ("out", 1536, 1536, Act.NONE),
                                          ("ffn1", 8960, 1536, Act.GELU_TANH),
                                          ("ffn2", 1536, 8960, Act.NONE)])
def test_config2_fp8_linear_set(be, oracle, name, N, K, act):
    # FP8 e4m3 weights (the reference's group-128 layout),
    # bf16 N(0,1) activations, M = 4680.
    M = 4680
    x = oracle.normal(21, M * K)
    w = oracle.normal(22 + N + K, N * K, 0.02)
    b = oracle.normal(23, N, 0.01)
    q = quant.Fp8E4M3.quantize(w, N, K)
    dw = be.weight_fp8(q)
    xb, bb = be.upload(x), be.upload(b)
    yb = be.alloc(M * N, BF16)
    be.linear(xb, 0, M, dw, bb, act, yb, 0)
    y = be.download(yb).reshape(M, N)
    rows = sampled_rows(M, 16)
    deq = q.dequantize()
    want = np.stack([oracle.linear(x, 1, deq, N, K, bias=b, act=act, x_row=int(r), threads=8)[0]
                     for r in rows])
    assert rel_l2(y[rows], want) <= REL_L2


def test_fused_gate_residual_matches_reference_sequence(be, oracle):
    # dit.rs:748-760: FFN2 into tmp, then gate_residual(h += tmp * mods[GATE_FFN]).
    M, N, K = 777, 1536, 1024
    w, q = make_weight("fp8", N, K, seed=31, oracle=oracle)
    dw = be.weight_fp8(q)
    x = oracle.normal(32, M * K)
    h0 = oracle.normal(33, M * N)
    mods = oracle.normal(34, 6 * N, 0.5)
    b = oracle.normal(35, N, 0.01)
    xb, bb, mb = be.upload(x), be.upload(b), be.upload(mods, F32)
    want = oracle.gate_residual(h0, oracle.linear(x, M, q.dequantize(), N, K, bias=b, threads=8),
                                M, N, mods, 5)
    h0m = h0.reshape(M, N)
    for hdt in (F32, BF16):
        # an f32 residual stream resolves the update itself; a bf16 one only
        # to its own rounding, so it is compared as a whole
        check = (lambda g: rel_l2(g - h0m, want - h0m)) if hdt == F32 else (lambda g: rel_l2(g, want))
        hb = be.upload(h0, hdt)
        be.linear_gate_residual(xb, 0, M, dw, bb, Act.NONE, hb, 0, mb, 5)
        assert check(be.download(hb).reshape(M, N)) <= REL_L2, hdt
        # the unfused sequence through the trait ops gives the same result
        hb2 = be.upload(h0, hdt)
        tmp = be.alloc(M * N, F32)
        be.linear(xb, 0, M, dw, bb, Act.NONE, tmp, 0)
        be.gate_residual(hb2, tmp, M, N, mb, 5)
        assert check(be.download(hb2).reshape(M, N)) <= REL_L2, hdt


# ---- the reference's conformance case and edge cases ----------------------------------------
def test_check_linear_hand_case(be):
    # crates/lightx2v-model/src/check.rs:74-103, tolerance 1e-6
    x = np.array([1, 2, 3, 4, 5, 6], np.float32)
    w = np.array([1, 0, -1, 0.5, 1, 0.5, 2, -1, 0, 0, 1, 2], np.float32)
    b = np.array([0.5, -0.5, 1.0, 0.0], np.float32)
    xb, yb, wb, bb = be.upload(x), be.alloc(8), be.weight(w, 4, 3), be.upload(b)
    be.linear(xb, 0, 2, wb, bb, Act.NONE, yb, 0)
    got = be.download(yb)
    want = [b[o] + sum(x[r * 3 + i] * w[o * 3 + i] for i in range(3)) for r in range(2) for o in range(4)]
    assert np.abs(got - np.array(want, np.float32)).max() <= 1e-6


def test_zero_rows_and_empty_is_noop(be, oracle):
    w, q = make_weight("q8", 128, 128, seed=1, oracle=oracle)
    dw = be.weight_q8(q)
    xb = be.upload(np.ones(128, np.float32))
    yb = be.upload(np.full(128, 3.0, np.float32))
    be.linear(xb, 0, 0, dw, None, Act.NONE, yb, 0)
    assert np.all(be.download(yb) == 3.0)


def test_errors_are_reported(be, oracle):
    from lightx2v_cuda import _lib as L
    w, q = make_weight("q8", 128, 128, seed=1, oracle=oracle)
    dw = be.weight_q8(q)
    xb = be.upload(np.ones(10 * 128, np.float32))
    yb = be.alloc(10 * 128)
    with pytest.raises(L.Lx2vError) as e:
        be.linear(xb, 5, 10, dw, None, Act.NONE, yb, 0)  # x too short
    assert e.value.status == L.ERR_INVALID
    with pytest.raises(L.Lx2vError) as e:
        be.linear(xb, 0, 10, dw, None, Act.NONE, xb, 0)  # output aliases input
    assert e.value.status == L.ERR_INVALID
    with pytest.raises(L.Lx2vError) as e:
        be.linear(xb, 0, 10, dw, None, 7, yb, 0)
    assert e.value.status == L.ERR_INVALID
    with pytest.raises(L.Lx2vError):
        be.weight_q4(quant.Q4(np.zeros(256, np.uint8), np.array([0.1], np.float32),
                              np.array([0.0], np.float32), 1, 256, 256))  # 0.1 is not an f16 value


def test_profile_report_lists_linear(be, oracle):
    import os
    import subprocess
    import sys
    code = (
        "import sys; sys.path.insert(0, 'lightx2v-rs_b200');"
        "import numpy as np; from lightx2v_cuda import CudaBackend, Act, quant;"
        "be = CudaBackend(0); q = quant.Q8.quantize(np.ones(256*256, np.float32), 256, 256);"
        "w = be.weight_q8(q); x = be.upload(np.ones(64*256, np.float32)); y = be.alloc(64*256);"
        "be.linear(x, 0, 64, w, None, Act.NONE, y, 0); be.sync();"
        "p = be.profile(); assert p['linear']['calls'] == 1 and p['linear']['ms'] > 0, p;"
        "print(be.profile_report())")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True,
                       env={**os.environ, "LIGHTX2V_PROFILE": "1"}, timeout=300)
    assert r.returncode == 0, r.stderr
    assert "linear" in r.stdout


def test_expired_wait_is_reported_and_context_survives(be, oracle):
    """A pipeline wait that runs out stops the kernel with an error status
    the host reads (no trap, no hang); the context stays usable."""
    from lightx2v_cuda import _lib as L
    M, N, K = 2048, 2048, 1536
    w, q = make_weight("q8", N, K, seed=41, oracle=oracle)
    dw = be.weight_q8(q)
    x = oracle.normal(42, M * K)
    xb = be.upload(x)
    yb = be.alloc(M * N, F32)
    be.sync()
    be.set_wait_limit_ns(1)  # every wait that does not succeed at once expires
    try:
        be.linear(xb, 0, M, dw, None, Act.NONE, yb, 0)
        with pytest.raises(L.Lx2vError) as e:
            be.sync()
        assert e.value.status == L.ERR_DEVICE
    finally:
        be.set_wait_limit_ns(2_000_000_000)
    be.sync()  # error word was cleared
    be.linear(xb, 0, M, dw, None, Act.NONE, yb, 0)
    y = be.download(yb).reshape(M, N)
    rows = sampled_rows(M, 8)
    want = np.stack([oracle.linear(x, 1, q.dequantize(), N, K, x_row=int(r), threads=8)[0] for r in rows])
    assert rel_l2(y[rows], want) <= REL_L2


# ---- the CTA-pair (cta_group::2) tensor-core kernel ---------------------------------------
@pytest.mark.parametrize("fmt", ["fp8", "q8", "q4", "native"])
@pytest.mark.parametrize("M,N,K,bt", [(512, 256, 128, 256), (700, 640, 448, 192), (1000, 384, 1024, 128),
                                      (257, 1536, 256, 256)])
def test_pair_kernel_matches_oracle_and_single_cta(be, oracle, fmt, M, N, K, bt):
    w, q = make_weight(fmt, N, K, seed=51 + M, oracle=oracle)
    dw = upload_weight(be, fmt, q, w, N, K)
    x = oracle.normal(52, M * K)
    b = oracle.normal(53, N, 0.01)
    xb, bb = be.upload(x), be.upload(b)
    outs = {}
    try:
        be.set_token_tile(bt)
        for path in (4, 5, 1):
            be.set_linear_path(path)
            yb = be.alloc(M * N, F32)
            be.linear(xb, 0, M, dw, bb, Act.GELU_TANH, yb, 0)
            outs[path] = be.download(yb).reshape(M, N)
    finally:
        be.set_linear_path(0)
        be.set_token_tile(0)
    want = oracle.linear(x, M, oracle_dequant(oracle, fmt, q, w), N, K, bias=b, act=1, threads=8)
    for path in (4, 5):
        assert rel_l2(outs[path], want) <= REL_L2, path
        # same bf16 operands, different summation order
        assert rel_l2(outs[path], outs[1]) <= 1e-5, path


@pytest.mark.parametrize("path", [4, 5])
def test_pair_kernel_gated_residual_and_offsets(be, oracle, path):
    M, N, K = 900, 768, 512
    w, q = make_weight("fp8", N, K, seed=61, oracle=oracle)
    dw = be.weight_fp8(q)
    x = oracle.normal(62, (M + 40) * K)
    h0 = oracle.normal(63, (M + 7) * N)
    mods = oracle.normal(64, 6 * N, 0.5)
    xb, mb = be.upload(x), be.upload(mods, F32)
    hb = be.upload(h0, F32)
    try:
        be.set_linear_path(path)
        be.linear_gate_residual(xb, 40, M, dw, None, Act.NONE, hb, 7, mb, 5)
    finally:
        be.set_linear_path(0)
    got = be.download(hb).reshape(M + 7, N)
    lin = oracle.linear(x, M, q.dequantize(), N, K, x_row=40, threads=8)
    want = h0.reshape(M + 7, N).copy()
    want[7:] = oracle.gate_residual(h0.reshape(M + 7, N)[7:], lin, M, N, mods, 5)
    assert np.array_equal(got[:7], h0.reshape(M + 7, N)[:7])
    assert rel_l2(got[7:] - h0.reshape(M + 7, N)[7:], want[7:] - h0.reshape(M + 7, N)[7:]) <= REL_L2


# ---- two-pass linear (weight decoded once to bf16, then both operands from smem) ----------
@pytest.mark.parametrize("fmt", ["fp8", "q4"])
@pytest.mark.parametrize("M,N,K,bt", [(4680, 1536, 1536, 128), (4680, 4608, 1536, 256), (2100, 1552, 8960, 192),
                                      (1030, 8960, 704, 256)])
def test_two_pass_matches_one_pass_at_chunk_shapes(be, oracle, fmt, M, N, K, bt):
    # the token tiles and k-block groupings of the 1.3B chunk's linears, plus
    # ragged N / M and K without 128-column groups (704 = 11 k-blocks)
    w, q = make_weight(fmt, N, K, seed=131 + N, oracle=oracle)
    dw = upload_weight(be, fmt, q, w, N, K)
    x = oracle.normal(132, M * K)
    b = oracle.normal(133, N, 0.01)
    xb, bb = be.upload(x), be.upload(b)
    outs = {}
    try:
        be.set_token_tile(bt)
        for path in (5, 4):
            be.set_linear_path(path)
            for rep in range(2 if path == 5 else 1):  # the second call reuses the decoded-weight workspace
                yb = be.alloc(M * N, F32)
                be.linear(xb, 0, M, dw, bb, Act.GELU_TANH, yb, 0)
                outs[(path, rep)] = be.download(yb).reshape(M, N)
    finally:
        be.set_linear_path(0)
        be.set_token_tile(0)
    assert np.array_equal(outs[(5, 0)], outs[(5, 1)], equal_nan=True)
    # same bf16 operands, f32 sums possibly in another order
    assert rel_l2(outs[(5, 0)], outs[(4, 0)]) <= 1e-5
    rows = sampled_rows(M, 32)
    want = np.stack([oracle.linear(x, 1, oracle_dequant(oracle, fmt, q, w), N, K, bias=b, act=1,
                                   x_row=int(r), threads=8)[0] for r in rows])
    assert rel_l2(outs[(5, 0)][rows], want) <= REL_L2


# ---- GEMM operand decode: bit-exact through a one-hot activation --------------------------
def bf16_round(v):
    """f32 -> bf16 round-to-nearest-even, returned as f32 (NaN kept NaN)."""
    b = np.asarray(v, np.float32).view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32).copy()
    out[np.isnan(v)] = np.nan
    return out


def fp8_all_codes_weight(N, K, seed):
    """Codes cover all 256 bytes; rows >= N - 16 keep the NaN codes, the
    others have them replaced; scales mix the fast range with values far
    outside it (which take the reference-formula path)."""
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 256, N * K, dtype=np.uint8).reshape(N, K)
    codes[: N - 16][(codes[: N - 16] & 0x7F) == 0x7F] ^= 0x01
    codes[: N - 16, :64] = np.arange(256, dtype=np.uint8).reshape(4, 64).repeat((N - 16) // 4 + 1, 0)[: N - 16] & 0xFE
    groups = N * K // 128
    scales = rng.choice(np.array([0.01, 3e-4, 1.5, 300.0, 1e-33, 2.0 ** -101, 2.0 ** 7], np.float32), groups)
    return quant.Fp8E4M3(codes.reshape(-1).copy(), scales.astype(np.float32), N, K, 128)


@pytest.mark.parametrize("fmt", ["fp8_all", "fp8", "q8", "q4", "native"])
@pytest.mark.parametrize("path", [1, 4, 5, 3])
def test_gemm_operands_are_bf16_of_exact_dequant(be, oracle, fmt, path):
    # x = identity (K tokens, one-hot): y[m][n] = operand(w[n][m]) exactly,
    # since every other product is 0 * w. Rows holding a NaN code are NaN.
    N, K = 512, 256
    if fmt == "fp8_all":
        q = fp8_all_codes_weight(N, K, 7)
        dw = be.weight_fp8(q)
        deq = oracle.fp8_dequantize(q.q, q.scales, q.group).reshape(N, K)
    else:
        w, q = make_weight(fmt, N, K, seed=71, group=64, oracle=oracle)
        dw = upload_weight(be, fmt, q, w, N, K)
        deq = oracle_dequant(oracle, fmt, q, w).reshape(N, K)
    x = np.eye(K, dtype=np.float32).reshape(-1)
    xb = be.upload(x)
    yb = be.alloc(K * N, F32)
    try:
        be.set_linear_path(path)
        be.linear(xb, 0, K, dw, None, Act.NONE, yb, 0)
        got = be.download(yb).reshape(K, N)
    finally:
        be.set_linear_path(0)
    want = bf16_round(deq.reshape(-1)).reshape(N, K).T.copy()
    nan_rows = np.isnan(deq).any(axis=1)
    want[:, nan_rows] = np.nan
    assert np.array_equal(np.isnan(got), np.isnan(want))
    # values below the f32 normal range may be flushed inside the tensor
    # core; everything else must match to the bit
    tiny = ~np.isnan(want) & (np.abs(np.nan_to_num(want)) < 2.0 ** -126)
    fin = ~np.isnan(want) & ~tiny
    bad = np.flatnonzero(got[fin] != want[fin])
    assert bad.size == 0, (fmt, path, bad.size, got[fin][bad[:4]], want[fin][bad[:4]])
    assert np.all(np.abs(got[tiny]) <= 2.0 ** -126)



# ---- stream-K work split of the CTA-pair kernel ------------------------------------------
@pytest.mark.parametrize("fmt", ["fp8", "q8", "q4", "native"])
@pytest.mark.parametrize("M,N,K,bt", [(4680, 1536, 1536, 256), (1000, 512, 8960, 256), (700, 640, 4480, 192),
                                      (2500, 1552, 704, 128), (19200, 256, 768, 256)])
@pytest.mark.parametrize("path", [4, 5])
def test_stream_k_matches_whole_tiles_and_oracle(be, oracle, fmt, M, N, K, bt, path):
    # tiles split over several CTA pairs, several partial tiles added into one
    # (1000 x 512 x 8960: ~10 pairs per tile), ragged M and N; 19200 x 256 x
    # 768: 75 tiles on 74 pairs, whose leftover tile alone has fewer k-block
    # groups than there are pairs (the two-pass kernel then splits one more
    # wave)
    w, q = make_weight(fmt, N, K, seed=101 + K, oracle=oracle)
    dw = upload_weight(be, fmt, q, w, N, K)
    x = oracle.normal(102, M * K)
    b = oracle.normal(103, N, 0.01)
    xb, bb = be.upload(x), be.upload(b)
    outs = {}
    try:
        be.set_linear_path(path)
        be.set_token_tile(bt)
        for mode in (2, 1):
            be.set_split_mode(mode)
            for rep in range(2):  # a second launch reuses the workspace with a new epoch
                yb = be.alloc(M * N, F32)
                be.linear(xb, 0, M, dw, bb, Act.GELU_TANH, yb, 0)
                outs[(mode, rep)] = be.download(yb).reshape(M, N)
    finally:
        be.set_split_mode(0)
        be.set_token_tile(0)
        be.set_linear_path(0)
    assert np.array_equal(outs[(2, 0)], outs[(2, 1)], equal_nan=True)
    assert rel_l2(outs[(2, 0)], outs[(1, 0)]) <= 1e-5
    rows = sampled_rows(M, 64)
    want = np.stack([oracle.linear(x, 1, oracle_dequant(oracle, fmt, q, w), N, K, bias=b, act=1,
                                   x_row=int(r), threads=8)[0] for r in rows])
    assert rel_l2(outs[(2, 0)][rows], want) <= REL_L2


@pytest.mark.parametrize("M,N,K", [(4680, 1536, 8960), (1800, 768, 4096)])
def test_k_split_gated_residual_matches_whole_tiles(be, oracle, M, N, K):
    """The two-pass kernel cuts the tiles of a gated residual into k-ranges
    that reduce-add into f32 h on their own (the 1.3B chunk's FFN2: 114
    tiles on 74 pairs become 342 items of a third of a tile); the bias is
    added by the first range only. Same bf16 operands as whole tiles (f32
    sums in another order), and the oracle on sampled rows."""
    w, q = make_weight("fp8", N, K, seed=151 + K, oracle=oracle)
    dw = be.weight_fp8(q)
    x = oracle.normal(152, (M + 40) * K)
    h0 = oracle.normal(153, (M + 7) * N)
    mods = oracle.normal(154, 6 * N, 0.5)
    b = oracle.normal(155, N, 0.01)
    xb, mb, bb = be.upload(x), be.upload(mods, F32), be.upload(b, F32)
    outs = {}
    try:
        be.set_linear_path(5)
        for mode in (0, 1):  # automatic (k-split), whole tiles
            be.set_split_mode(mode)
            hb = be.upload(h0, F32)
            be.linear_gate_residual(xb, 40, M, dw, bb, Act.NONE, hb, 7, mb, 5)
            outs[mode] = be.download(hb).reshape(M + 7, N)
    finally:
        be.set_split_mode(0)
        be.set_linear_path(0)
    h0 = h0.reshape(M + 7, N)
    assert np.array_equal(outs[0][:7], h0[:7])
    assert rel_l2(outs[0][7:] - h0[7:], outs[1][7:] - h0[7:]) <= 1e-5
    rows = sampled_rows(M, 32)
    lin = np.stack([oracle.linear(x, 1, q.dequantize(), N, K, bias=b, x_row=40 + int(r), threads=8)[0]
                    for r in rows])
    want = oracle.gate_residual(h0[7:][rows].copy(), lin, len(rows), N, mods, 5)
    assert rel_l2(outs[0][7:][rows] - h0[7:][rows], want - h0[7:][rows]) <= REL_L2


@pytest.mark.parametrize("path", [4, 5])
def test_stream_k_gated_residual_with_offsets(be, oracle, path):
    M, N, K = 1800, 768, 4096
    w, q = make_weight("fp8", N, K, seed=111, oracle=oracle)
    dw = be.weight_fp8(q)
    x = oracle.normal(112, (M + 40) * K)
    h0 = oracle.normal(113, (M + 7) * N)
    mods = oracle.normal(114, 6 * N, 0.5)
    xb, mb = be.upload(x), be.upload(mods, F32)
    hb = be.upload(h0, F32)
    try:
        be.set_linear_path(path)
        be.set_split_mode(2)
        be.linear_gate_residual(xb, 40, M, dw, None, Act.NONE, hb, 7, mb, 5)
    finally:
        be.set_split_mode(0)
        be.set_linear_path(0)
    got = be.download(hb).reshape(M + 7, N)
    h0 = h0.reshape(M + 7, N)
    assert np.array_equal(got[:7], h0[:7])
    rows = sampled_rows(M, 48)
    lin = np.stack([oracle.linear(x, 1, q.dequantize(), N, K, x_row=40 + int(r), threads=8)[0] for r in rows])
    want = oracle.gate_residual(h0[7:][rows].copy(), lin, len(rows), N, mods, 5)
    assert rel_l2(got[7:][rows] - h0[7:][rows], want - h0[7:][rows]) <= REL_L2


# ---- few-token kernel (M <= 16, bandwidth-bound) --------------------------------------------
@pytest.mark.parametrize("fmt", ["fp8", "q8", "q4", "native"])
@pytest.mark.parametrize("M,N,K", [(1, 8960, 1536), (16, 1536, 8960), (7, 640, 4096), (3, 200, 256), (16, 4608, 1536)])
def test_few_token_kernel_matches_generic_and_oracle(be, oracle, fmt, M, N, K):
    w, q = make_weight(fmt, N, K, seed=121 + N, oracle=oracle)
    dw = upload_weight(be, fmt, q, w, N, K)
    x = oracle.normal(122, (M + 2) * K)
    b = oracle.normal(123, N, 0.01)
    xb, bb = be.upload(x), be.upload(b)
    outs = {}
    try:
        for path in (2, 3):
            be.set_linear_path(path)
            for rep in range(2):  # split-K arrival counters must be back at zero
                yb = be.alloc((M + 1) * N, F32)
                be.linear(xb, 2, M, dw, bb, Act.GELU_TANH, yb, 1)
                outs[(path, rep)] = be.download(yb).reshape(M + 1, N)
    finally:
        be.set_linear_path(0)
    assert np.all(outs[(2, 0)][0] == 0)
    assert np.array_equal(outs[(2, 0)], outs[(2, 1)], equal_nan=True)
    want = oracle.linear(x, M, oracle_dequant(oracle, fmt, q, w), N, K, bias=b, act=1, x_row=2, threads=8)
    assert rel_l2(outs[(2, 0)][1:], want) <= REL_L2
    if fmt == "q4" and K % 64 == 0:
        # Q4 few-token kernel: codes multiplied exactly, each group's scale and
        # zero applied after the products, so no bf16 rounding of the weight;
        # it is at least as close to the f32 oracle as the generic kernel's
        # bf16-rounded weights, and near it
        assert rel_l2(outs[(2, 0)][1:], want) <= rel_l2(outs[(3, 0)][1:], want) * 1.02
        assert rel_l2(outs[(2, 0)][1:], outs[(3, 0)][1:]) <= 5e-3
    else:
        assert rel_l2(outs[(2, 0)][1:], outs[(3, 0)][1:]) <= 1e-5


@pytest.mark.parametrize("M,N,K,group,x_f32,y_f32", [
    (1, 8960, 1536, 64, False, False),    # C3, one CTA per row group
    (16, 1536, 8960, 64, False, True),    # C3, k split over a cluster
    (16, 8960, 1536, 64, True, True),     # two token tiles, f32 x
    (9, 1000, 4096, 128, False, False),   # ragged rows, group 128
    (5, 200, 64, 64, True, False),        # one chunk
    (12, 1024, 14336, 64, False, True),   # long k (the 5B FFN2 depth)
])
def test_few_token_q4_kernel_matches_oracle(be, oracle, M, N, K, group, x_f32, y_f32):
    """The Q4 few-token kernel (gemv_q4.cu) against the f32 oracle on the
    reference's dequantised weights, rows offset on both sides, bias + GELU;
    two calls in a row give identical bits (fixed summation order)."""
    w, q = make_weight("q4", N, K, seed=141 + N + K, group=group, oracle=oracle)
    dw = be.weight_q4(q)
    x = oracle.normal(142, (M + 3) * K)
    b = oracle.normal(143, N, 0.01)
    xb = be.upload(x, F32 if x_f32 else BF16)
    bb = be.upload(b, F32)
    outs = []
    for _ in range(2):
        yb = be.alloc((M + 2) * N, F32 if y_f32 else BF16)
        be.linear(xb, 3, M, dw, bb, Act.GELU_TANH, yb, 2)
        outs.append(be.download(yb).reshape(M + 2, N))
    assert np.array_equal(outs[0], outs[1])
    assert np.all(outs[0][:2] == 0)
    xr = be.download(xb)  # the bf16 values the device holds when x is bf16
    want = oracle.linear(xr, M, oracle_dequant(oracle, "q4", q, w), N, K, bias=b, act=1, x_row=3, threads=8)
    assert rel_l2(outs[0][2:], want) <= (REL_L2 if not y_f32 else 5e-3)


def test_few_token_kernel_is_the_automatic_choice_and_fuses_the_gate(be, oracle):
    M, N, K = 4, 1536, 8960
    w, q = make_weight("q4", N, K, seed=131, oracle=oracle)
    dw = be.weight_q4(q)
    x = oracle.normal(132, M * K)
    h0 = oracle.normal(133, M * N)
    mods = oracle.normal(134, 6 * N, 0.5)
    xb, mb = be.upload(x), be.upload(mods, F32)
    hb = be.upload(h0, F32)
    n0 = be.launch_count()
    be.linear_gate_residual(xb, 0, M, dw, None, Act.NONE, hb, 0, mb, 5)
    assert be.launch_count() == n0 + 1
    got = be.download(hb).reshape(M, N)
    lin = oracle.linear(x, M, oracle_dequant(oracle, "q4", q, None), N, K, threads=8)
    want = oracle.gate_residual(h0.reshape(M, N).copy(), lin, M, N, mods, 5)
    assert rel_l2(got - h0.reshape(M, N), want - h0.reshape(M, N)) <= REL_L2


# ---- CUDA graph replay of stream-K launches ----------------------------------------------
def replay_follows_inputs(be, run, xb, x_sets, yb, wants, replays=3):
    """Capture `run` (which reads xb and writes yb) on the library's stream,
    then replay it with the inputs switched between replays: every replay must
    equal the eager result for the inputs it saw. A stream-K launch whose
    flags still held the previous replay's epoch would add partial tiles left
    from the earlier inputs (or still being written) and fail this."""
    import torch
    ext = torch.cuda.ExternalStream(be.stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=ext):
        run()
    try:
        for r in range(replays):
            i = r % len(x_sets)
            be.copy(x_sets[i], 0, xb, 0, be.buf_len(xb))
            with torch.cuda.stream(ext):
                g.replay()
            got = be.download(yb)
            assert np.array_equal(got, wants[i], equal_nan=True), (r, i)
    finally:
        del g


@pytest.mark.parametrize("path", [4, 5])
def test_stream_k_linear_replays_in_a_cuda_graph(be, oracle, path):
    M, N, K = 1000, 1536, 1536
    w, q = make_weight("fp8", N, K, seed=81, oracle=oracle)
    dw = be.weight_fp8(q)
    x_sets = [be.upload(oracle.normal(82 + i, M * K)) for i in range(2)]
    xb = be.alloc(M * K)
    bb = be.upload(oracle.normal(84, N, 0.01), F32)
    yb = be.alloc(M * N, F32)
    try:
        be.set_linear_path(path)
        be.set_split_mode(2)

        def run():
            be.linear(xb, 0, M, dw, bb, Act.GELU_TANH, yb, 0)

        wants = []
        for xs in x_sets:  # eager: also the first call that sizes every workspace
            be.copy(xs, 0, xb, 0, M * K)
            run()
            wants.append(be.download(yb))
        be.sync()
        replay_follows_inputs(be, run, xb, x_sets, yb, wants)
    finally:
        be.set_linear_path(0)
        be.set_split_mode(0)
    want = oracle.linear(be.download(x_sets[0]), M, q.dequantize(), N, K, bias=be.download(bb), act=1, threads=8)
    assert rel_l2(wants[0].reshape(M, N), want) <= REL_L2


# ---- NVFP4 (no reference counterpart; the format's own definition as the oracle) -----------
def test_nvfp4_device_decode_is_bit_exact(be, oracle):
    rows, cols = 96, 1536
    q = quant.Nvfp4.quantize(oracle.normal(161, rows * cols, 0.02), rows, cols)
    got = be.weight_dequant_f32(be.weight_nvfp4(q))
    assert np.array_equal(got.view(np.uint32), q.dequantize().view(np.uint32))


@pytest.mark.parametrize("M,N,K", [(4680, 1536, 1536), (300, 8960, 1536), (40, 200, 512), (4, 512, 256)])
def test_nvfp4_linear_matches_oracle(be, oracle, M, N, K):
    # two-pass (bf16 decode + CTA-pair GEMM) for the first two, the generic kernel for the others
    q = quant.Nvfp4.quantize(oracle.normal(171 + N, N * K, 0.02), N, K)
    dw = be.weight_nvfp4(q)
    x = oracle.normal(172, (M + 1) * K)
    b = oracle.normal(173, N, 0.01)
    xb, bb = be.upload(x), be.upload(b, F32)
    yb = be.alloc(M * N, F32)
    be.linear(xb, 1, M, dw, bb, Act.GELU_TANH, yb, 0)
    y = be.download(yb).reshape(M, N)
    rows = sampled_rows(M, 24)
    want = np.stack([oracle.linear(x, 1, q.dequantize(), N, K, bias=b, act=1, x_row=1 + int(r), threads=8)[0]
                     for r in rows])
    assert rel_l2(y[rows], want) <= REL_L2


def test_nvfp4_is_refused_by_the_kernels_that_do_not_take_it(be, oracle):
    from lightx2v_cuda import _lib as L
    q = quant.Nvfp4.quantize(oracle.normal(181, 512 * 512, 0.02), 512, 512)
    dw = be.weight_nvfp4(q)
    xb, yb = be.upload(oracle.normal(182, 512 * 512)), be.alloc(512 * 512, F32)
    try:
        for path in (1, 2, 4):
            be.set_linear_path(path)
            with pytest.raises(L.Lx2vError) as e:
                be.linear(xb, 0, 512, dw, None, Act.NONE, yb, 0)
            assert e.value.status == L.ERR_UNSUPPORTED
    finally:
        be.set_linear_path(0)
