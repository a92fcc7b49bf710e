"""Host-side mirror of lightx2v-core's weight formats (crates/lightx2v-core/src/quant.rs).

These are the structs `Backend::weight_q8 / weight_q4 / weight_fp8` receive,
with the reference's quantizers restated in vectorised numpy so that
benchmarks and the model harness can make weights of BASELINE's sizes in
seconds. The arithmetic is kept f32 and in the reference's order:
  - Rust `f32::round` (half away from zero) is done exactly in f64;
  - sequential f32 accumulations (HQQ's err / zsum) stay sequential;
  - log2f / powf are evaluated in f64 and rounded once to f32 (a correctly
    rounded result, which glibc's log2f / powf return for these inputs).
tests/test_quant_mirror.py checks every format bit-for-bit against the C
restatement in oracle/ on BASELINE-sized matrices.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np

Q8_GROUP = 128  # quant.rs:19
FP8_GROUP = 128  # quant.rs:21
FP8_E4M3_MAX = np.float32(448.0)  # quant.rs:23

_F32 = np.float32


def _round_away(x: np.ndarray) -> np.ndarray:
    """Rust `f32::round`: half away from zero, exact for every f32."""
    x64 = x.astype(np.float64)
    return np.trunc(x64 + np.copysign(0.5, x64)).astype(np.float32)


def _as_i8(x: np.ndarray) -> np.ndarray:
    """Rust `f as i8` on values already clamped to [-127, 127]; NaN -> 0."""
    return np.nan_to_num(x, nan=0.0).astype(np.int8)


def _as_u8(x: np.ndarray) -> np.ndarray:
    """Rust `f as u8`: saturating, NaN -> 0."""
    return np.clip(np.nan_to_num(x, nan=0.0), 0, 255).astype(np.uint8)


def _amax(g: np.ndarray) -> np.ndarray:
    # fold(0.0, |m, v| m.max(v.abs())): f32::max ignores NaN, like np.fmax.
    return np.fmax.reduce(np.abs(g), axis=1, initial=_F32(0.0)).astype(_F32)


@dataclass
class Q8:
    """`Q8` (quant.rs:144-205): int8 codes, one f32 scale per group of columns."""
    q: np.ndarray       # i8 [rows*cols]
    scales: np.ndarray  # f32 [rows * cols/group]
    rows: int
    cols: int
    group: int

    @staticmethod
    def quantize(data, rows: int, cols: int) -> "Q8":
        w = np.ascontiguousarray(data, _F32).reshape(-1)
        assert w.size == rows * cols
        group = Q8_GROUP if cols % Q8_GROUP == 0 else cols
        g = w.reshape(-1, group)
        amax = _amax(g)
        s = np.where(amax > 0, amax / _F32(127.0), _F32(1.0)).astype(_F32)
        r = _round_away((g / s[:, None]).astype(_F32))
        q = _as_i8(np.clip(r, _F32(-127.0), _F32(127.0)))
        return Q8(q.reshape(-1), s, rows, cols, group)

    def dequantize(self) -> np.ndarray:
        return (self.q.astype(_F32).reshape(-1, self.group) * self.scales[:, None]).reshape(-1)

    @staticmethod
    def concat(parts) -> "Q8":
        a = parts[0]
        for b in parts[1:]:
            assert (a.cols, a.group) == (b.cols, b.group)
        return Q8(np.concatenate([p.q for p in parts]), np.concatenate([p.scales for p in parts]),
                  sum(p.rows for p in parts), a.cols, a.group)

    def bytes(self) -> int:
        return self.q.size + 4 * self.scales.size


def _f16(x: np.ndarray) -> np.ndarray:
    """half::f16::from_f32(v).to_f32(): IEEE round-to-nearest-even."""
    return x.astype(np.float16).astype(_F32)


def _hqq_block(g: np.ndarray, is_: np.ndarray, z: np.ndarray) -> np.ndarray:
    """HQQ zero refinement (quant.rs:248-276) of a block of groups: rows of g
    with their inverse scales and initial zeros; returns the best zeros.
    Each group iterates on its own, so only the groups still improving are
    computed in each round (most stop within a few rounds)."""
    p, kappa = _F32(0.7), _F32(1.01)
    pm1 = np.float64(p - _F32(1.0))
    n = _F32(g.shape[1])
    z = z.copy()
    best_z = z.copy()
    best = np.full(z.shape, _F32(3.4028235e38), _F32)
    beta = np.full(z.shape, _F32(10.0), _F32)
    idx = np.arange(z.size)
    for _ in range(20):
        gi, si, zi, bi = g[idx], is_[idx], z[idx], beta[idx]
        v = (gi * si[:, None]).astype(_F32) + zi[:, None]
        c = np.clip(_round_away(v.astype(_F32)), _F32(0.0), _F32(15.0))
        r = ((c - zi[:, None]) / si[:, None]).astype(_F32)
        e = (gi - r).astype(_F32)
        a = np.abs(e)
        with np.errstate(divide="ignore", invalid="ignore"):
            pw = np.power(a.astype(np.float64), pm1).astype(_F32)
            t = np.fmax((a - (pw / bi[:, None]).astype(_F32)).astype(_F32), _F32(0.0))
        sh = np.where(a > 0, np.where(e > 0, t, -t), _F32(0.0)).astype(_F32)
        term = (c - ((gi - sh).astype(_F32) * si[:, None]).astype(_F32)).astype(_F32)
        err = np.zeros(idx.size, _F32)
        zsum = np.zeros(idx.size, _F32)
        for i in range(g.shape[1]):  # sequential f32 sums, as the reference
            err = (err + a[:, i]).astype(_F32)
            zsum = (zsum + term[:, i]).astype(_F32)
        err = (err / n).astype(_F32)
        upd = ~(err >= best[idx])
        idx = idx[upd]
        if idx.size == 0:
            break
        best[idx] = err[upd]
        best_z[idx] = zi[upd]
        z[idx] = (zsum[upd] / n).astype(_F32)
        beta[idx] = (bi[upd] * kappa).astype(_F32)
    return best_z


def _hqq_zeros(g: np.ndarray, is_: np.ndarray, z: np.ndarray) -> np.ndarray:
    """_hqq_block over blocks of groups on a thread pool (numpy's array
    operations release the GIL); results do not depend on the split."""
    blocks = max(1, min(os.cpu_count() or 1, 16, g.shape[0] // 4096))
    if blocks == 1:
        return _hqq_block(g, is_, z)
    from concurrent.futures import ThreadPoolExecutor
    cuts = np.linspace(0, g.shape[0], blocks + 1).astype(int)
    with ThreadPoolExecutor(blocks) as ex:
        parts = list(ex.map(lambda i: _hqq_block(g[cuts[i]:cuts[i + 1]], is_[cuts[i]:cuts[i + 1]],
                                                   z[cuts[i]:cuts[i + 1]]), range(blocks)))
    return np.concatenate(parts)


@dataclass
class Q4:
    """`Q4` (quant.rs:212-356): 4-bit codes (one per byte in memory) with an f16-exact
    (scale, zero) per group: w = (q - z) * s."""
    q: np.ndarray       # u8 [rows*cols], one code per byte
    scales: np.ndarray  # f32 (f16-exact) [rows * cols/group]
    zeros: np.ndarray
    rows: int
    cols: int
    group: int

    @staticmethod
    def quantize(data, rows: int, cols: int, group: int, hqq: bool) -> "Q4":
        w = np.ascontiguousarray(data, _F32).reshape(-1)
        assert w.size == rows * cols
        if cols % group != 0:
            group = cols
        g = w.reshape(-1, group)
        lo = np.fmin.reduce(g, axis=1, initial=_F32(3.4028235e38)).astype(_F32)
        hi = np.fmax.reduce(g, axis=1, initial=_F32(-3.4028235e38)).astype(_F32)
        is_ = np.where(hi > lo, _F32(15.0) / (hi - lo), _F32(1.0)).astype(_F32)
        z = (-lo * is_).astype(_F32)

        def code(zz):
            v = (g * is_[:, None]).astype(_F32) + zz[:, None]
            return np.clip(_round_away(v.astype(_F32)), _F32(0.0), _F32(15.0))

        if hqq:  # quant.rs:248-276, vectorised across groups
            z = _hqq_zeros(g, is_, z)
        q = _as_u8(code(z))
        scales = _f16((_F32(1.0) / is_).astype(_F32))
        zeros = _f16(z)
        return Q4(q.reshape(-1), scales, zeros, rows, cols, group)

    def dequantize(self) -> np.ndarray:
        c = self.q.astype(_F32).reshape(-1, self.group)
        return ((c - self.zeros[:, None]) * self.scales[:, None]).astype(_F32).reshape(-1)

    def packed(self) -> np.ndarray:
        """Two codes per byte, element 2i in the low nibble (quant.rs:306-311)."""
        q = self.q
        if q.size % 2:
            q = np.concatenate([q, np.zeros(1, np.uint8)])
        return (q[0::2] | (q[1::2] << 4)).astype(np.uint8)

    @staticmethod
    def from_packed(packed, scales, zeros, rows: int, cols: int) -> "Q4":
        n = rows * cols
        packed = np.asarray(packed, np.uint8)
        assert packed.size == (n + 1) // 2
        q = np.empty(2 * packed.size, np.uint8)
        q[0::2] = packed & 15
        q[1::2] = packed >> 4
        scales = np.asarray(scales, _F32)
        zeros = np.asarray(zeros, _F32)
        assert scales.size and scales.size == zeros.size and n % scales.size == 0
        return Q4(q[:n], scales, zeros, rows, cols, n // scales.size)

    @staticmethod
    def concat(parts) -> "Q4":
        a = parts[0]
        for b in parts[1:]:
            assert (a.cols, a.group) == (b.cols, b.group)
        return Q4(np.concatenate([p.q for p in parts]), np.concatenate([p.scales for p in parts]),
                  np.concatenate([p.zeros for p in parts]), sum(p.rows for p in parts), a.cols,
                  a.group)

    def bytes(self) -> int:
        return (self.q.size + 1) // 2 + 4 * self.scales.size


# ---- FP8 e4m3 (quant.rs:358-460) ------------------------------------------------
def e4m3_decode_table() -> np.ndarray:
    """e4m3_to_f32 for all 256 codes (quant.rs:409-420): exponent-field-0 codes
    decode as m/8 * 2^-9, 0x7F / 0xFF as NaN."""
    t = np.empty(256, _F32)
    for c in range(256):
        sign = -1.0 if c & 0x80 else 1.0
        e, m = (c >> 3) & 0xF, c & 7
        if e == 0:
            t[c] = sign * (m / 8.0) * 2.0 ** -9
        elif e == 0xF and m == 7:
            t[c] = np.nan
        else:
            t[c] = sign * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


_E4M3 = e4m3_decode_table()


def f32_to_e4m3(v: np.ndarray) -> np.ndarray:
    """f32_to_e4m3 (quant.rs:376-406), vectorised, with the reference's
    small-magnitude defect: `(e + 7) as u8` wraps for e < -7 and the u8 shift
    drops the high bits."""
    v = np.asarray(v, _F32)
    sign = np.where(np.signbit(v), 0x80, 0x00).astype(np.int64)
    a = np.abs(v)
    out = np.zeros(v.shape, np.int64)
    zero = v == 0
    sat = ~np.isfinite(a) | (a >= 464.0)
    rest = ~zero & ~sat
    with np.errstate(divide="ignore", invalid="ignore"):
        l2 = np.log2(a.astype(np.float64)).astype(_F32)  # log2f, correctly rounded
    e = np.floor(l2)
    e = np.where(rest, e, 0).astype(np.int64)
    sub = rest & (e < -9)
    big = rest & (e > 8)
    nrm = rest & ~sub & ~big
    # subnormal branch: (a / (2^-9 / 8)).round() as u8, min 7
    m_sub = np.minimum(_as_u8(_round_away((a / _F32(2.0 ** -12)).astype(_F32))), 7).astype(np.int64)
    # normal branch
    p2 = np.ldexp(np.ones(v.shape, _F32), np.where(nrm, e, 0)).astype(_F32)
    mant = _as_u8(_round_away((((a / p2).astype(_F32) - _F32(1.0)) * _F32(8.0)).astype(_F32)))
    mant = mant.astype(np.int64)
    exp = (e + 7) & 0xFF  # `as u8` wraps
    bump = mant >= 8
    code_n = np.where(bump, np.where(exp >= 15, 0x7E, ((exp + 1) << 3) & 0xFF),
                      ((exp << 3) & 0xFF) | mant)
    out = np.where(zero, sign, out)
    out = np.where(sat | big, sign | 0x7E, out)
    out = np.where(sub, sign | m_sub, out)
    out = np.where(nrm, sign | code_n, out)
    return out.astype(np.uint8)


@dataclass
class Fp8E4M3:
    """`Fp8E4M3` (quant.rs:365-460): e4m3 codes with one f32 scale per group of
    FP8_GROUP elements (the repo's layout: groups along K, not per channel)."""
    q: np.ndarray       # u8 [rows*cols]
    scales: np.ndarray  # f32 [rows*cols/group]
    rows: int
    cols: int
    group: int

    @staticmethod
    def quantize(data, rows: int, cols: int) -> "Fp8E4M3":
        w = np.ascontiguousarray(data, _F32).reshape(-1)
        assert w.size == rows * cols
        group = FP8_GROUP if cols % FP8_GROUP == 0 else cols
        g = w.reshape(-1, group)
        amax = _amax(g)
        s = np.where(amax > 0, amax / FP8_E4M3_MAX, _F32(1.0)).astype(_F32)
        scaled = (g / s[:, None]).astype(_F32)
        # element-wise: blocks of groups on a thread pool (numpy releases the
        # GIL), the same codes whatever the split
        blocks = max(1, min(os.cpu_count() or 1, 16, g.shape[0] // 8192))
        if blocks == 1:
            q = f32_to_e4m3(scaled)
        else:
            from concurrent.futures import ThreadPoolExecutor
            cuts = np.linspace(0, g.shape[0], blocks + 1).astype(int)
            with ThreadPoolExecutor(blocks) as ex:
                q = np.concatenate(list(ex.map(lambda i: f32_to_e4m3(scaled[cuts[i]:cuts[i + 1]]), range(blocks))))
        return Fp8E4M3(q.reshape(-1), s, rows, cols, group)

    def dequantize(self) -> np.ndarray:
        return (_E4M3[self.q].reshape(-1, self.group) * self.scales[:, None]).astype(_F32).reshape(-1)

    @staticmethod
    def concat(parts) -> "Fp8E4M3":
        """Rows of several FP8 matrices stacked, codes then scales in part
        order, with the first part's cols and group: the fused QKV / KV
        stacking of load_linear (crates/lightx2v-model/src/dit.rs:127-147),
        which has no method of its own in quant.rs. Unlike Q8/Q4 concat the
        reference does not assert that cols and group agree; a stack whose
        parts differ would be mis-shaped, so this mirror rejects it."""
        a = parts[0]
        for b in parts[1:]:
            assert (a.cols, a.group) == (b.cols, b.group)
        return Fp8E4M3(np.concatenate([p.q for p in parts]), np.concatenate([p.scales for p in parts]),
                       sum(p.rows for p in parts), a.cols, a.group)

    def bytes(self) -> int:
        return self.q.size + 4 * self.scales.size


# ---- NVFP4 (no counterpart in the reference) ----------------------------------------
# The reference names NVFP4 (micro-block fp4 e2m1 codes, one e4m3 scale per 16
# values, one f32 global scale) as its next quantisation (docs/design.md:
# 137-145, quant.rs:13-16, 361-364) but does not implement it, so this is the
# format's definition here: w = e2m1(code) * (e4m3(block scale) * global), the
# bracket rounded to f32 once, e4m3 as the OCP format (exponent-field-0 codes
# are subnormals m/8 * 2^-6). The device decode (lx2v_weight_nvfp4) matches
# `dequantize` bit for bit.
E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)
NVFP4_BLOCK = 16


def e4m3_ocp_table() -> np.ndarray:
    """The 256 OCP e4m3 codes as f32 (0x7F / 0xFF NaN)."""
    c = np.arange(256, dtype=np.uint32)
    sign = np.where(c & 0x80, -1.0, 1.0)
    e, m = (c >> 3) & 0xF, (c & 7).astype(np.float64)
    v = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1.0 + m / 8.0) * 2.0 ** (e.astype(np.float64) - 7))
    v = (sign * v).astype(np.float32)
    v[(c & 0x7F) == 0x7F] = np.nan
    return v


def _nearest_code(x: np.ndarray, values: np.ndarray) -> np.ndarray:
    """Index of the nearest entry of the ascending `values` (ties to the lower)."""
    hi = np.clip(np.searchsorted(values, x), 1, len(values) - 1)
    lo = hi - 1
    return np.where(np.abs(x - values[lo]) <= np.abs(values[hi] - x), lo, hi)


@dataclass
class Nvfp4:
    q: np.ndarray          # u8 packed, element 2i in the low nibble [rows * cols / 2]
    scales: np.ndarray     # u8 e4m3 block scales [rows * cols / 16]
    global_scale: float
    rows: int
    cols: int

    @staticmethod
    def quantize(data, rows: int, cols: int) -> "Nvfp4":
        """The usual two-level recipe: global = amax / (6 * 448), block scale
        = e4m3(block amax / 6 / global) (nearest, at most 448), code = nearest
        e2m1 of w / (block scale * global)."""
        assert cols % 32 == 0, cols
        w = np.asarray(data, np.float32).reshape(rows, cols)
        amax = float(np.max(np.abs(w))) if w.size else 0.0
        gs = np.float32(amax / (6.0 * 448.0)) if amax > 0 else np.float32(1.0)
        blocks = w.reshape(rows, cols // NVFP4_BLOCK, NVFP4_BLOCK)
        bmax = np.max(np.abs(blocks), axis=2)
        table = e4m3_ocp_table()
        pos = table[:0x7F]                        # codes 0x00..0x7E, ascending 0 .. 448
        want = np.minimum(bmax / np.float32(6.0) / gs, np.float32(448.0)).astype(np.float32)
        sc = _nearest_code(want, pos).astype(np.uint8)
        eff = (pos[sc] * gs).astype(np.float32)  # block scale x global, one f32 rounding
        safe = np.where(eff > 0, eff, np.float32(1.0))
        r = (blocks / safe[:, :, None]).astype(np.float32)
        mag = _nearest_code(np.minimum(np.abs(r), np.float32(6.0)), E2M1_VALUES).astype(np.uint8)
        code = (mag | np.where(r < 0, 8, 0).astype(np.uint8)).reshape(-1)
        code[np.repeat(eff.reshape(-1) == 0, NVFP4_BLOCK)] = 0
        packed = (code[0::2] | (code[1::2] << 4)).astype(np.uint8)
        return Nvfp4(packed, sc.reshape(-1), float(gs), rows, cols)

    def codes(self) -> np.ndarray:
        c = np.empty(self.rows * self.cols, np.uint8)
        c[0::2], c[1::2] = self.q & 0xF, self.q >> 4
        return c

    def dequantize(self) -> np.ndarray:
        c = self.codes().astype(np.int64)
        val = np.where(c & 8, -1.0, 1.0).astype(np.float32) * E2M1_VALUES[c & 7]
        eff = (e4m3_ocp_table()[self.scales] * np.float32(self.global_scale)).astype(np.float32)
        return (val.reshape(-1, NVFP4_BLOCK) * eff[:, None]).astype(np.float32).reshape(-1)

    def bytes(self) -> int:
        return self.q.size + self.scales.size + 4


# ---- WeightQuant (quant.rs:27-132) ------------------------------------------------
@dataclass(frozen=True)
class WeightQuant:
    kind: str = "native"      # native | int8 | int4 | fp8
    group: int = 64
    hqq: bool = False
    ffn_only: bool = False

    def attn(self) -> "WeightQuant":
        """quant.rs:47-52: with `-ffn`, the attention linears use int8."""
        if self.kind == "int4" and self.ffn_only:
            return WeightQuant("int8")
        return self

    def for_key(self, key: str) -> "WeightQuant":
        """quant.rs:57-71."""
        if not key.startswith("blocks.") or "." not in key[len("blocks."):]:
            return WeightQuant("native")
        role = key[len("blocks."):].split(".", 1)[1]
        if role in ("ffn.net.0.proj", "ffn.net.2"):
            return self
        if role in ("attn1.to_q", "attn1.to_k", "attn1.to_v", "attn1.to_out.0", "attn2.to_q",
                    "attn2.to_k", "attn2.to_v", "attn2.to_out.0", "to_gate_compress"):
            return self.attn()
        return WeightQuant("native")

    @staticmethod
    def parse(s: str) -> "WeightQuant":
        """FromStr (quant.rs:94-132)."""
        if s in ("native", "bf16", "f16"):
            return WeightQuant("native")
        if s in ("int8", "q8"):
            return WeightQuant("int8")
        if s in ("fp8", "fp8-e4m3"):
            return WeightQuant("fp8")
        ffn_only = s.endswith("-ffn")
        if ffn_only:
            s = s[: -len("-ffn")]
        if not s.startswith("int4"):
            raise ValueError(f"unknown weight format `{s}` (native | int8 | fp8 | int4[-hqq][-gN][-ffn])")
        rest = s[len("int4"):]
        hqq = rest.startswith("-hqq")
        if hqq:
            rest = rest[len("-hqq"):]
        if rest.startswith("-g"):
            try:
                group = int(rest[2:])
            except ValueError:
                raise ValueError(f"bad group in `{s}`") from None
        elif rest == "":
            group = 64
        else:
            raise ValueError(f"bad weight format `{s}`")
        if group == 0 or group % 8 != 0:
            raise ValueError(f"int4 group must be a multiple of 8, got {group}")
        return WeightQuant("int4", group, hqq, ffn_only)

    def __str__(self) -> str:
        if self.kind == "int4":
            return f"int4{'-hqq' if self.hqq else ''}-g{self.group}{'-ffn' if self.ffn_only else ''}"
        return {"native": "native", "int8": "int8", "fp8": "fp8-e4m3"}[self.kind]
