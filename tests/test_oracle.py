"""Pins the C oracle to the reference's own known-answer tests and bounds.

Every case restates a test of the Rust reference (path:line given) with the
same inputs; the reference cannot be compiled here (no Rust toolchain), so
these are the oracle's anchor.
"""
import math

import numpy as np
import pytest


def test_e4m3_spot_values(oracle):
    # crates/lightx2v-core/src/quant.rs:529-538
    o = oracle
    assert o.f32_to_e4m3(0.0) == 0x00
    assert o.f32_to_e4m3(1.0) == 0x38
    assert o.f32_to_e4m3(-1.0) == 0xB8
    assert o.f32_to_e4m3(448.0) == 0x7E
    assert o.f32_to_e4m3(2.0) == 0x40
    assert abs(o.e4m3_to_f32(0x38) - 1.0) < 1e-7
    assert abs(o.e4m3_to_f32(0x40) - 2.0) < 1e-7
    assert abs(o.e4m3_to_f32(0x01) - 2.0 ** -9 / 8.0) < 1e-9


def test_e4m3_defect_is_restated(oracle):
    # quant.rs:396: `(e + 7) as u8` wraps for e = -8 / -9, and `exp << 3` on a
    # u8 drops the high bits: |v| in [2^-9, 2^-7) encodes to 0xF0..0xFF / 0x70..0x7F.
    o = oracle
    assert o.f32_to_e4m3(2.0 ** -8) == 0xF8        # e = -8 -> exp 255 -> 0xF8
    assert o.f32_to_e4m3(-(2.0 ** -8)) == 0xF8     # sign bit already set by the wrap
    assert o.f32_to_e4m3(2.0 ** -9) == 0xF0        # e = -9 -> exp 254 -> 0xF0
    assert o.f32_to_e4m3(1.875 * 2.0 ** -8) == 0xFF  # mantissa 7 -> NaN code
    assert math.isnan(o.e4m3_to_f32(0xFF)) and math.isnan(o.e4m3_to_f32(0x7F))
    # exponent-field-0 codes decode as m/8 * 2^-9 (quant.rs:413-414)
    for m in range(8):
        assert o.e4m3_to_f32(m) == m / 8.0 * 2.0 ** -9
    # saturation (quant.rs:382-385, 393-395)
    assert o.f32_to_e4m3(1e9) == 0x7E and o.f32_to_e4m3(-1e9) == 0xFE
    assert o.f32_to_e4m3(float("inf")) == 0x7E


def test_q8_round_trip_error_is_half_a_step(oracle):
    # quant.rs:466-479
    rows, cols = 8, 256
    i = np.arange(rows * cols)
    w = (((i * 7919 % 1000).astype(np.float32) / np.float32(500.0) - np.float32(1.0)) *
         (1 + i // cols).astype(np.float32)).astype(np.float32)
    q, s, group = oracle.q8_quantize(w, rows, cols)
    assert group == 128 and s.size == rows * 2
    d = oracle.q8_dequantize(q, s, group)
    assert np.all(np.abs(w - d) <= s[i // 128] * 0.5 + 1e-6)


def _q4_test_matrix():
    rows, cols = 16, 256
    i = np.arange(rows * cols)
    u = (i * 7919 % 1009).astype(np.float32) / np.float32(1009.0) - np.float32(0.5)
    w = np.where(i % 97 == 0, u * np.float32(8.0), u * np.float32(0.3)).astype(np.float32)
    return w, rows, cols


def test_q4_round_trip_and_hqq_does_not_hurt(oracle):
    # quant.rs:481-526
    w, rows, cols = _q4_test_matrix()
    q, s, z, g = oracle.q4_quantize(w, rows, cols, 64, False)
    assert q.max() <= 15
    d = oracle.q4_dequantize(q, s, z, g)
    i = np.arange(w.size)
    assert np.all(np.abs(w - d) <= s[i // 64] * 0.52 + 1e-5)
    qh, sh, zh, gh = oracle.q4_quantize(w, rows, cols, 64, True)
    assert qh.max() <= 15
    err = lambda dd: float(((w - dd) ** 2).sum())
    assert err(oracle.q4_dequantize(qh, sh, zh, gh)) <= err(d) * 1.05


def test_fp8_round_trip_error_is_half_an_e4m3_step(oracle):
    # quant.rs:540-554
    rows, cols = 4, 256
    i = np.arange(rows * cols)
    w = (((i * 7919 % 1000).astype(np.float32) / np.float32(500.0) - np.float32(1.0)) *
         np.float32(0.7)).astype(np.float32)
    q, s, g = oracle.fp8_quantize(w, rows, cols)
    d = oracle.fp8_dequantize(q, s, g)
    tol = np.abs(w) * 0.0625 + s[i // 128] * 0.5 + 1e-6
    assert np.all(np.abs(w - d) <= tol)


def test_check_quant(oracle):
    # crates/lightx2v-model/src/check.rs:294-320 (Rng seed 17, uniform +-1, 8x256, tol 0.2)
    w = oracle.uniform(17, 8 * 256, 1.0)
    q, s, g = oracle.q8_quantize(w, 8, 256)
    e8 = np.abs(w - oracle.q8_dequantize(q, s, g)).max()
    q4, s4, z4, g4 = oracle.q4_quantize(w, 8, 256, 64, True)
    e4 = np.abs(w - oracle.q4_dequantize(q4, s4, z4, g4)).max()
    qf, sf, gf = oracle.fp8_quantize(w, 8, 256)
    ef = (np.abs(w - oracle.fp8_dequantize(qf, sf, gf)) / (np.abs(w) + 1e-6)).max()
    assert max(e8, e4, ef) <= 0.2


def test_check_linear_hand_case(oracle):
    # crates/lightx2v-model/src/check.rs:74-103 (tol 1e-6)
    x = np.array([1, 2, 3, 4, 5, 6], np.float32)
    w = np.array([1, 0, -1, 0.5, 1, 0.5, 2, -1, 0, 0, 1, 2], np.float32)
    b = np.array([0.5, -0.5, 1.0, 0.0], np.float32)
    got = oracle.linear(x, 2, w, 4, 3, bias=b)
    want = np.array([[b[o] + sum(x[r * 3 + i] * w[o * 3 + i] for i in range(3)) for o in range(4)]
                     for r in range(2)], np.float32)
    assert np.abs(got - want).max() <= 1e-6


def test_rng_deterministic_and_gaussian(oracle):
    # crates/lightx2v-core/src/rng.rs:59-69
    a = oracle.normal(7, 1000)
    assert np.array_equal(a, oracle.normal(7, 1000))
    assert not np.array_equal(oracle.normal(8, 16), oracle.normal(7, 16))
    assert abs(a.mean()) < 0.1 and abs(a.var() - 1.0) < 0.15


def test_gelu_tanh_and_gate_residual(oracle):
    # crates/lightx2v-cpu/src/lib.rs:151-153, 394-404
    for v in (-3.0, -0.5, 0.0, 0.7, 4.0):
        ref = 0.5 * v * (1 + math.tanh(math.sqrt(2 / math.pi) * (v + 0.044715 * v ** 3)))
        assert abs(oracle.gelu_tanh(v) - ref) < 1e-6
    h = np.arange(6, dtype=np.float32).reshape(2, 3)
    a = np.ones((2, 3), np.float32)
    mods = np.arange(12, dtype=np.float32)
    out = oracle.gate_residual(h, a, 2, 3, mods, 2)
    assert np.array_equal(out, h + mods[6:9])


@pytest.mark.parametrize("threads", [1, 3])
def test_linear_threads_do_not_change_bits(oracle, threads):
    x = oracle.normal(1, 7 * 64)
    w = oracle.normal(2, 40 * 64, 0.02)
    b = oracle.normal(3, 40, 0.01)
    y1 = oracle.linear(x, 7, w, 40, 64, bias=b, act=1, threads=1)
    yt = oracle.linear(x, 7, w, 40, 64, bias=b, act=1, threads=threads)
    assert np.array_equal(y1, yt)
