"""The host-side mirror of lightx2v-core::quant / Rng (lightx2v_cuda.quant, .rng)
against the C oracle, bit for bit, on BASELINE-sized matrices."""
import numpy as np
import pytest

from lightx2v_cuda import quant, rng


def test_rng_u64_stream_and_uniform_exact(oracle):
    # rng.rs:20-36: the integer stream and uniform() are exact.
    for seed in (0, 1, 17, 2 ** 63 + 5):
        assert np.array_equal(rng.uniform(seed, 4097, 1.0), oracle.uniform(seed, 4097, 1.0))


def test_rng_normal_within_four_ulp(oracle):
    a = oracle.normal(3, 200001)
    b = rng.normal(3, 200001)
    ulp = np.spacing(np.maximum(np.abs(a), np.abs(b)).astype(np.float32))
    # r and cos/sin can each be one ulp off glibc, so the product a few ulp
    assert np.all(np.abs(a - b) <= 4 * ulp)
    assert (a == b).mean() > 0.97


@pytest.mark.parametrize("rows,cols", [(8960, 1536), (1536, 8960), (7, 200), (3, 128)])
def test_q8_exact(oracle, rows, cols):
    w = oracle.normal(2, rows * cols, 0.02)
    m = quant.Q8.quantize(w, rows, cols)
    q, s, g = oracle.q8_quantize(w, rows, cols)
    assert m.group == g and np.array_equal(m.q, q) and np.array_equal(m.scales, s)
    assert np.array_equal(m.dequantize().view(np.uint32), oracle.q8_dequantize(q, s, g).view(np.uint32))


@pytest.mark.parametrize("rows,cols", [(8960, 1536), (4608, 1536), (7, 200), (5, 384)])
def test_fp8_exact(oracle, rows, cols):
    w = oracle.normal(4, rows * cols, 0.02)
    m = quant.Fp8E4M3.quantize(w, rows, cols)
    q, s, g = oracle.fp8_quantize(w, rows, cols)
    assert m.group == g and np.array_equal(m.q, q) and np.array_equal(m.scales, s)
    d = oracle.fp8_dequantize(q, s, g)
    md = m.dequantize()
    assert np.array_equal(np.isnan(md), np.isnan(d))
    fin = ~np.isnan(d)
    assert np.array_equal(md[fin].view(np.uint32), d[fin].view(np.uint32))


def test_fp8_encoder_edge_values(oracle):
    vals = np.array([0.0, -0.0, 1.0, -1.0, 448.0, 464.0, 463.99, 1e-3, 2.0 ** -9, 2.0 ** -8,
                     2.0 ** -7, 2.0 ** -10, 2.0 ** -12, 3e-5, 1e-8, np.inf, -np.inf, np.nan,
                     255.9, 0.0078125 * 1.875, 0.0039, -0.005], np.float32)
    got = quant.f32_to_e4m3(vals)
    want = np.array([oracle.f32_to_e4m3(float(v)) for v in vals], np.uint8)
    assert np.array_equal(got, want)
    # every decode of the table equals the oracle's decode
    t = quant.e4m3_decode_table()
    for c in range(256):
        o = oracle.e4m3_to_f32(c)
        assert (np.isnan(t[c]) and np.isnan(o)) or t[c] == o


@pytest.mark.parametrize("hqq", [False, True])
@pytest.mark.parametrize("rows,cols,group", [(512, 1536, 64), (96, 8960, 64), (16, 256, 16),
                                             (8, 200, 64)])
def test_q4_exact(oracle, rows, cols, group, hqq):
    w = oracle.normal(5, rows * cols, 0.02)
    m = quant.Q4.quantize(w, rows, cols, group, hqq)
    q, s, z, g = oracle.q4_quantize(w, rows, cols, group, hqq)
    assert m.group == g
    assert np.array_equal(m.q, q)
    assert np.array_equal(m.scales, s) and np.array_equal(m.zeros, z)
    assert np.array_equal(m.packed(), oracle.q4_pack(q))
    assert np.array_equal(quant.Q4.from_packed(m.packed(), s, z, rows, cols).q, q)


def test_weight_quant_parse_and_for_key():
    # quant.rs:45-132 and the parse cases of quant.rs:513-525
    WQ = quant.WeightQuant
    assert WQ.parse("int4-hqq-g32") == WQ("int4", 32, True, False)
    assert WQ.parse("fp8") == WQ("fp8")
    assert WQ.parse("int4-hqq-g64-ffn").attn() == WQ("int8")
    assert str(WQ.parse("int4-hqq-g64")) == "int4-hqq-g64"
    with pytest.raises(ValueError):
        WQ.parse("int4-g12")
    q = WQ.parse("int4-hqq-g64-ffn")
    assert q.for_key("blocks.3.ffn.net.0.proj") == q
    assert q.for_key("blocks.3.attn1.to_q") == WQ("int8")
    assert q.for_key("blocks.3.norm2") == WQ("native")
    assert q.for_key("proj_out") == WQ("native")


@pytest.mark.parametrize("fmt", ["q8", "q4", "fp8"])
def test_concat_stacks_rows_like_load_linear(oracle, fmt):
    # fused QKV: parts quantized one by one and stacked by rows, codes then
    # scales (quant.rs:189-199, 339-350; FP8 inline in dit.rs:127-147)
    rows, cols = 8, 256
    ws = [oracle.normal(40 + i, rows * cols, 0.02) for i in range(3)]
    if fmt == "q8":
        parts = [quant.Q8.quantize(w, rows, cols) for w in ws]
        st = quant.Q8.concat(parts)
    elif fmt == "q4":
        parts = [quant.Q4.quantize(w, rows, cols, 64, True) for w in ws]
        st = quant.Q4.concat(parts)
        assert np.array_equal(st.zeros, np.concatenate([p.zeros for p in parts]))
    else:
        parts = [quant.Fp8E4M3.quantize(w, rows, cols) for w in ws]
        st = quant.Fp8E4M3.concat(parts)
    assert (st.rows, st.cols, st.group) == (3 * rows, cols, parts[0].group)
    assert np.array_equal(st.q, np.concatenate([p.q for p in parts]))
    assert np.array_equal(st.scales, np.concatenate([p.scales for p in parts]))
    deq = st.dequantize()
    want = np.concatenate([p.dequantize() for p in parts])
    assert np.array_equal(np.isnan(deq), np.isnan(want))
    assert np.array_equal(deq[~np.isnan(want)], want[~np.isnan(want)])


def test_fp8_concat_rejects_mismatched_parts(oracle):
    a = quant.Fp8E4M3.quantize(oracle.normal(1, 4 * 256), 4, 256)
    b = quant.Fp8E4M3.quantize(oracle.normal(2, 4 * 128), 4, 128)
    with pytest.raises(AssertionError):
        quant.Fp8E4M3.concat([a, b])


# ---- NVFP4 (no counterpart in the reference: the format's definition) ---------------------
def test_nvfp4_codes_lie_on_the_e2m1_grid_times_the_block_scale(oracle):
    rows, cols = 48, 512
    w = oracle.normal(61, rows * cols, 0.02)
    q = quant.Nvfp4.quantize(w, rows, cols)
    assert q.q.size == rows * cols // 2 and q.scales.size == rows * cols // 16
    d = q.dequantize().reshape(-1, 16)
    eff = (quant.e4m3_ocp_table()[q.scales] * np.float32(q.global_scale)).astype(np.float32)
    c = q.codes().astype(np.int64).reshape(-1, 16)
    val = np.where(c & 8, -1.0, 1.0).astype(np.float32) * quant.E2M1_VALUES[c & 7]
    assert np.array_equal(d, (val * eff[:, None]).astype(np.float32))  # w = e2m1(code) x (block x global)
    ratio = val
    # nearest grid point: the error is at most half the widest gap (6 - 4) times the scale
    err = np.abs(d - np.asarray(w, np.float32).reshape(-1, 16))
    assert np.all(err <= eff[:, None] * 1.0 + 1e-12)
    assert np.linalg.norm(d.reshape(-1) - w) / np.linalg.norm(w) < 0.12
    # the largest value of a block uses (nearly) the top of the e2m1 range
    assert np.max(np.abs(ratio)) == 6.0


def test_nvfp4_zero_weight_and_ocp_e4m3_table():
    q = quant.Nvfp4.quantize(np.zeros(4 * 64, np.float32), 4, 64)
    assert np.all(q.dequantize() == 0)
    t = quant.e4m3_ocp_table()
    assert t[0x7E] == 448.0 and t[0x08] == 2.0 ** -6 and t[0x01] == 2.0 ** -9
    assert np.isnan(t[0x7F]) and np.isnan(t[0xFF]) and t[0xBE] == -1.75
