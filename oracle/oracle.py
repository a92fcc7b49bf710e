"""ctypes wrapper of the C oracle (lx2v_oracle.c).

TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA library. Only
tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs
import this module. Each function names the reference function it restates
(path:line inside the lightx2v-rs project).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblx2v_oracle.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i8p = ctypes.POINTER(ctypes.c_int8)
_sz = ctypes.c_size_t


def build() -> str:
    """Compile the oracle with its Makefile (fast; a no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.orc_normal.argtypes = [ctypes.c_uint64, _sz, ctypes.c_float, _f32p]
        L.orc_uniform.argtypes = [ctypes.c_uint64, _sz, ctypes.c_float, _f32p]
        L.orc_q8_quantize.argtypes = [_f32p, _sz, _sz, _i8p, _f32p]
        L.orc_q8_quantize.restype = _sz
        L.orc_q8_dequantize.argtypes = [_i8p, _f32p, _sz, _sz, _f32p]
        L.orc_q4_quantize.argtypes = [_f32p, _sz, _sz, _sz, ctypes.c_int, _u8p, _f32p, _f32p]
        L.orc_q4_quantize.restype = _sz
        L.orc_q4_dequantize.argtypes = [_u8p, _f32p, _f32p, _sz, _sz, _f32p]
        L.orc_q4_pack.argtypes = [_u8p, _sz, _u8p]
        L.orc_q4_unpack.argtypes = [_u8p, _sz, _u8p]
        L.orc_f32_to_e4m3.argtypes = [ctypes.c_float]
        L.orc_f32_to_e4m3.restype = ctypes.c_uint8
        L.orc_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.orc_e4m3_to_f32.restype = ctypes.c_float
        L.orc_fp8_quantize.argtypes = [_f32p, _sz, _sz, _u8p, _f32p]
        L.orc_fp8_quantize.restype = _sz
        L.orc_fp8_dequantize.argtypes = [_u8p, _f32p, _sz, _sz, _f32p]
        L.orc_gelu_tanh.argtypes = [ctypes.c_float]
        L.orc_gelu_tanh.restype = ctypes.c_float
        L.orc_linear.argtypes = [_f32p, _sz, _sz, _f32p, _sz, _sz, _f32p, ctypes.c_int,
                                 _f32p, _sz, ctypes.c_int]
        L.orc_gate_residual.argtypes = [_f32p, _f32p, _sz, _sz, _f32p, _sz]
        L.orc_openmp_threads.restype = ctypes.c_int
        L.orc_attention.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _u8p, _f32p, ctypes.c_int]
        L.orc_layer_norm.argtypes = [_f32p, _sz, _sz, ctypes.c_int, _f32p, _f32p, _f32p, _sz, _sz,
                                     ctypes.c_float, _f32p]
        L.orc_residual_norm.argtypes = [_f32p, _f32p, _sz, _sz, _f32p, ctypes.c_long, ctypes.c_int, _f32p,
                                        _f32p, _sz, _sz, ctypes.c_float, _f32p]
        L.orc_head_split.argtypes = [_f32p, _sz, _sz, _sz, _sz, _sz, _f32p, _f32p, _f32p, ctypes.c_float,
                                     _f32p]
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(t)


# ---- rng.rs:8-53 --------------------------------------------------------
def normal(seed: int, n: int, std: float = 1.0) -> np.ndarray:
    """`std * Rng::new(seed).normal(n)` (rng.rs:39-52)."""
    out = np.empty(n, np.float32)
    lib().orc_normal(seed, n, std, _p(out, _f32p))
    return out


def uniform(seed: int, n: int, a: float) -> np.ndarray:
    """`Rng::new(seed).uniform(n, a)` (rng.rs:34-36)."""
    out = np.empty(n, np.float32)
    lib().orc_uniform(seed, n, a, _p(out, _f32p))
    return out


# ---- quant.rs -------------------------------------------------------------
def q8_quantize(w: np.ndarray, rows: int, cols: int):
    """Q8::quantize (quant.rs:154-178) -> (codes i8 [rows*cols], scales f32, group)."""
    w = np.ascontiguousarray(w, np.float32).reshape(-1)
    group = 128 if cols % 128 == 0 else cols
    q = np.empty(rows * cols, np.int8)
    s = np.empty(rows * cols // group, np.float32)
    g = lib().orc_q8_quantize(_p(w, _f32p), rows, cols, _p(q, _i8p), _p(s, _f32p))
    assert g == group
    return q, s, group


def q8_dequantize(q, scales, group) -> np.ndarray:
    """Q8::dequantize (quant.rs:180-186)."""
    q = np.ascontiguousarray(q, np.int8)
    scales = np.ascontiguousarray(scales, np.float32)
    out = np.empty(q.size, np.float32)
    lib().orc_q8_dequantize(_p(q, _i8p), _p(scales, _f32p), q.size, group, _p(out, _f32p))
    return out


def q4_quantize(w: np.ndarray, rows: int, cols: int, group: int, hqq: bool):
    """Q4::quantize (quant.rs:226-292) -> (codes u8 one per byte, scales, zeros, group)."""
    w = np.ascontiguousarray(w, np.float32).reshape(-1)
    g_used = group if cols % group == 0 else cols
    q = np.empty(rows * cols, np.uint8)
    s = np.empty(rows * cols // g_used, np.float32)
    z = np.empty_like(s)
    g = lib().orc_q4_quantize(_p(w, _f32p), rows, cols, group, int(hqq), _p(q, _u8p),
                              _p(s, _f32p), _p(z, _f32p))
    assert g == g_used
    return q, s, z, g_used


def q4_dequantize(q, scales, zeros, group) -> np.ndarray:
    """Q4::dequantize (quant.rs:294-303), codes one per byte."""
    q = np.ascontiguousarray(q, np.uint8)
    scales = np.ascontiguousarray(scales, np.float32)
    zeros = np.ascontiguousarray(zeros, np.float32)
    out = np.empty(q.size, np.float32)
    lib().orc_q4_dequantize(_p(q, _u8p), _p(scales, _f32p), _p(zeros, _f32p), q.size, group,
                            _p(out, _f32p))
    return out


def q4_pack(q) -> np.ndarray:
    """Q4::packed (quant.rs:306-311)."""
    q = np.ascontiguousarray(q, np.uint8)
    out = np.empty((q.size + 1) // 2, np.uint8)
    lib().orc_q4_pack(_p(q, _u8p), q.size, _p(out, _u8p))
    return out


def q4_unpack(packed, n) -> np.ndarray:
    """Q4::from_packed's code unpacking (quant.rs:324-326)."""
    packed = np.ascontiguousarray(packed, np.uint8)
    out = np.empty(n, np.uint8)
    lib().orc_q4_unpack(_p(packed, _u8p), n, _p(out, _u8p))
    return out


def f32_to_e4m3(v: float) -> int:
    """f32_to_e4m3 (quant.rs:376-406), defect included."""
    return int(lib().orc_f32_to_e4m3(v))


def e4m3_to_f32(code: int) -> float:
    """e4m3_to_f32 (quant.rs:409-420)."""
    return float(lib().orc_e4m3_to_f32(code))


def fp8_quantize(w: np.ndarray, rows: int, cols: int):
    """Fp8E4M3::quantize (quant.rs:423-447) -> (codes u8, scales f32, group)."""
    w = np.ascontiguousarray(w, np.float32).reshape(-1)
    group = 128 if cols % 128 == 0 else cols
    q = np.empty(rows * cols, np.uint8)
    s = np.empty(rows * cols // group, np.float32)
    g = lib().orc_fp8_quantize(_p(w, _f32p), rows, cols, _p(q, _u8p), _p(s, _f32p))
    assert g == group
    return q, s, group


def fp8_dequantize(q, scales, group) -> np.ndarray:
    """Fp8E4M3::dequantize (quant.rs:449-455)."""
    q = np.ascontiguousarray(q, np.uint8)
    scales = np.ascontiguousarray(scales, np.float32)
    out = np.empty(q.size, np.float32)
    lib().orc_fp8_dequantize(_p(q, _u8p), _p(scales, _f32p), q.size, group, _p(out, _f32p))
    return out


# ---- crates/lightx2v-cpu/src/lib.rs ----------------------------------------
def gelu_tanh(x: float) -> float:
    """gelu_tanh (lib.rs:151-153)."""
    return float(lib().orc_gelu_tanh(x))


def linear(x: np.ndarray, rows: int, w: np.ndarray, n: int, k: int, bias=None, act: int = 0,
           x_row: int = 0, threads: int = 1) -> np.ndarray:
    """CpuBackend::linear (lib.rs:296-326) on a dequantized f32 weight `w` [n, k].

    Returns y [rows, n] (the rows the call writes, y_row = 0)."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    w = np.ascontiguousarray(w, np.float32).reshape(-1)
    assert w.size == n * k and x.size >= (x_row + rows) * k
    y = np.empty(rows * n, np.float32)
    bp = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, np.float32)
        bp = _p(bias, _f32p)
    lib().orc_linear(_p(x, _f32p), x_row, rows, _p(w, _f32p), n, k, bp, act, _p(y, _f32p), 0,
                     threads)
    return y.reshape(rows, n)


def gate_residual(h: np.ndarray, a: np.ndarray, rows: int, dim: int, mods: np.ndarray,
                  gate: int) -> np.ndarray:
    """CpuBackend::gate_residual (lib.rs:394-404); returns the updated copy of h."""
    h = np.array(h, np.float32, copy=True).reshape(-1)
    a = np.ascontiguousarray(a, np.float32).reshape(-1)
    mods = np.ascontiguousarray(mods, np.float32).reshape(-1)
    lib().orc_gate_residual(_p(h, _f32p), _p(a, _f32p), rows, dim, _p(mods, _f32p), gate)
    return h.reshape(rows, dim)


def openmp_threads() -> int:
    return int(lib().orc_openmp_threads())


# ---- attention / norms / head_split (cpu lib.rs:155-208, 328-459) -----------------------------
def _f(a):
    return np.ascontiguousarray(a, np.float32).reshape(-1)


def attention(q, k, v, heads: int, sq: int, sk: int, d: int, mask=None, threads: int = 8) -> np.ndarray:
    """attention_impl (cpu lib.rs:170-208): q [heads, sq, d], k / v [heads, sk, d], mask
    [sq, sk] bool (True = allowed) or None -> out [sq, heads * d]."""
    q, k, v = _f(q), _f(k), _f(v)
    assert q.size == heads * sq * d and k.size == heads * sk * d and v.size == heads * sk * d
    out = np.empty(sq * heads * d, np.float32)
    mp = None
    if mask is not None:
        m = np.ascontiguousarray(np.asarray(mask, bool).reshape(sq, sk)).view(np.uint8)
        mp = _p(m, _u8p)
    lib().orc_attention(_p(q, _f32p), _p(k, _f32p), _p(v, _f32p), heads, sq, sk, d, mp, _p(out, _f32p), threads)
    return out.reshape(sq, heads * d)


def layer_norm(x, rows: int, dim: int, eps: float, w=None, b=None, mods=None, scale: int = 0,
               shift: int = 0) -> np.ndarray:
    """CpuBackend::layer_norm (cpu lib.rs:328-362): Affine when w/b are given, else Mod
    (mods [slots, dim], rows `scale` and `shift`)."""
    x = _f(x)
    out = np.empty(rows * dim, np.float32)
    kind = 0 if w is not None else 1
    w = _f(w) if w is not None else np.zeros(1, np.float32)
    b = _f(b) if b is not None else np.zeros(1, np.float32)
    mods = _f(mods) if mods is not None else np.zeros(1, np.float32)
    lib().orc_layer_norm(_p(x, _f32p), rows, dim, kind, _p(w, _f32p), _p(b, _f32p), _p(mods, _f32p), scale,
                         shift, eps, _p(out, _f32p))
    return out.reshape(rows, dim)


def residual_norm(h, a, rows: int, dim: int, mods, gate, eps: float, w=None, b=None, scale: int = 0,
                  shift: int = 0):
    """CpuBackend::residual_norm (cpu lib.rs:364-392) -> (updated h, normed)."""
    h = np.array(_f(h), copy=True)
    a = _f(a)
    mods = _f(mods)
    out = np.empty(rows * dim, np.float32)
    kind = 0 if w is not None else 1
    w = _f(w) if w is not None else np.zeros(1, np.float32)
    b = _f(b) if b is not None else np.zeros(1, np.float32)
    lib().orc_residual_norm(_p(h, _f32p), _p(a, _f32p), rows, dim, _p(mods, _f32p), -1 if gate is None else gate,
                            kind, _p(w, _f32p), _p(b, _f32p), scale, shift, eps, _p(out, _f32p))
    return h.reshape(rows, dim), out.reshape(rows, dim)


def head_split(src, rows: int, src_stride: int, col_off: int, heads: int, head_dim: int, rms_w=None,
               rope=None, eps: float = 1e-6) -> np.ndarray:
    """CpuBackend::head_split (cpu lib.rs:406-459) -> [heads, rows, head_dim]."""
    src = _f(src)
    out = np.empty(heads * rows * head_dim, np.float32)
    w = _f(rms_w) if rms_w is not None else None
    c, s_ = (_f(rope[0]), _f(rope[1])) if rope is not None else (None, None)
    wp = _p(w, _f32p) if w is not None else None
    cp = _p(c, _f32p) if c is not None else None
    sp = _p(s_, _f32p) if s_ is not None else None
    lib().orc_head_split(_p(src, _f32p), rows, src_stride, col_off, heads, head_dim, wp, cp, sp, eps,
                         _p(out, _f32p))
    return out.reshape(heads, rows, head_dim)


# ---- KV cache / MemRoPE (cpu lib.rs:607-806; memrope.rs ema_update) ----------------------------
SINK, LONG_EMA, SHORT_EMA, RECENT, NEW = range(5)


class KvCacheRef:
    """CpuBackend's KvCache restated in numpy: k / v rows [rows, heads * head_dim]
    f32 (a token row holds all its heads, as the reference's flat Vec does),
    one temporal index and slot kind per row."""

    def __init__(self, heads: int, head_dim: int):
        self.heads, self.head_dim = heads, head_dim
        self.k = np.zeros((0, heads * head_dim), np.float32)
        self.v = np.zeros((0, heads * head_dim), np.float32)
        self.temporal: list[int] = []
        self.kinds: list[int] = []

    def rows(self) -> int:
        return len(self.temporal)

    @staticmethod
    def _rows_of(x, heads, rows, hd):
        # [heads, rows, head_dim] -> [rows, heads * head_dim]
        return np.asarray(x, np.float32).reshape(heads, rows, hd).transpose(1, 0, 2).reshape(rows, heads * hd)

    def append(self, k, v, rows: int, temporal):
        """kv_cache_append, lib.rs:620-648."""
        self.k = np.concatenate([self.k, self._rows_of(k, self.heads, rows, self.head_dim)])
        self.v = np.concatenate([self.v, self._rows_of(v, self.heads, rows, self.head_dim)])
        self.temporal += [int(t) for t in temporal]
        self.kinds += [NEW] * rows

    def put(self, k, v, rows: int, temporal):
        """kv_cache_put, lib.rs:650-678."""
        temporal = [int(t) for t in temporal]
        pos = next((i for i, (t, kd) in enumerate(zip(self.temporal, self.kinds))
                    if t == temporal[0] and kd not in (LONG_EMA, SHORT_EMA)), None)
        if pos is not None and all(pos + i < self.rows() and self.temporal[pos + i] == temporal[i]
                                   for i in range(rows)):
            self.k[pos:pos + rows] = self._rows_of(k, self.heads, rows, self.head_dim)
            self.v[pos:pos + rows] = self._rows_of(v, self.heads, rows, self.head_dim)
            return
        self.append(k, v, rows, temporal)

    def kv(self):
        """kv_cache_kv, lib.rs:690-706: [heads, rows, head_dim] each."""
        r = self.rows()
        f = lambda a: a.reshape(r, self.heads, self.head_dim).transpose(1, 0, 2).copy()
        return f(self.k), f(self.v)

    def memrope_update(self, cache_frames: int, sink_frames: int, new_frames: int, alpha_long: float,
                       alpha_short: float, ft: int):
        """kv_cache_memrope_update, lib.rs:708-806."""
        def n_frames():
            return self.rows() // ft

        def frame_kinds():
            return [self.kinds[f * ft] for f in range(n_frames())]

        if n_frames() == 0:
            return
        fk = frame_kinds()
        if LONG_EMA not in fk and n_frames() > sink_frames:
            at = sink_frames * ft
            t = self.temporal[min(at, max(self.rows() - 1, 0))]
            zero = np.zeros((ft, self.k.shape[1]), np.float32)
            for kind in (SHORT_EMA, LONG_EMA):
                self.k = np.concatenate([self.k[:at], zero, self.k[at:]])
                self.v = np.concatenate([self.v[:at], zero, self.v[at:]])
                self.temporal[at:at] = [t] * ft
                self.kinds[at:at] = [kind] * ft
                fk = frame_kinds()
        news = [i for i, kd in enumerate(fk) if kd == NEW]
        if len(news) > new_frames:
            for f in news[:len(news) - new_frames]:
                self.kinds[f * ft:(f + 1) * ft] = [RECENT] * ft
        while n_frames() > cache_frames:
            kn = frame_kinds()
            f = kn.index(RECENT) if RECENT in kn else (kn.index(NEW) if NEW in kn else None)
            if f is None:
                break
            ev_k = self.k[f * ft:(f + 1) * ft].copy()
            ev_v = self.v[f * ft:(f + 1) * ft].copy()
            for kind, alpha in ((LONG_EMA, alpha_long), (SHORT_EMA, alpha_short)):
                if kind in kn:
                    sf = kn.index(kind)
                    a = np.float32(alpha)
                    one_m = np.float32(1.0) - a
                    for arr, ev in ((self.k, ev_k), (self.v, ev_v)):
                        e = arr[sf * ft:(sf + 1) * ft]
                        arr[sf * ft:(sf + 1) * ft] = (one_m * e).astype(np.float32) + (a * ev).astype(np.float32)
            self.k = np.concatenate([self.k[:f * ft], self.k[(f + 1) * ft:]])
            self.v = np.concatenate([self.v[:f * ft], self.v[(f + 1) * ft:]])
            del self.temporal[f * ft:(f + 1) * ft]
            del self.kinds[f * ft:(f + 1) * ft]
        for f in range(min(sink_frames, n_frames())):
            self.kinds[f * ft:(f + 1) * ft] = [SINK] * ft


def sparse_attention(q, k, v, gate, slot_src, block_sizes, seq: int, heads: int, d: int, topk: int,
                     scale: float) -> np.ndarray:
    """CpuBackend::sparse_attention, crates/lightx2v-cpu/src/lib.rs:500-606 (the
    VSA of crates/lightx2v-core/src/sparse.rs): per head, tile means (x / n
    added in slot order), coarse softmax attention over the tiles
    (softmax_row, lib.rs:155-166), the top-k key tiles per query tile (higher
    score first, ties to the lower tile), fine attention from every token to
    the selected tiles' tokens, out = coarse * gate + fine, [seq, heads * d].
    q, k, v, gate are f32 [heads, seq, d]. Loops over tiles and tokens as the
    reference runs them; the dot products and the fine softmax in f32."""
    q, k, v, gate = (np.asarray(a, np.float32).reshape(heads, seq, d) for a in (q, k, v, gate))
    nt = len(block_sizes)
    tile_tokens = [[int(s) for s in slot_src[t * 64:t * 64 + int(block_sizes[t])]] for t in range(nt)]
    token_tile = np.zeros(seq, np.int64)
    for t, toks in enumerate(tile_tokens):
        token_tile[toks] = t
    out = np.zeros((seq, heads, d), np.float32)
    sc = np.float32(scale)

    def softmax(row):
        m = np.float32(-np.inf)
        for x in row:
            m = max(m, x)
        e = np.exp((row - m).astype(np.float32)).astype(np.float32)
        s = np.float32(0.0)
        for x in e:
            s = np.float32(s + x)
        return (e * (np.float32(1.0) / s)).astype(np.float32)

    for h in range(heads):
        cq = np.zeros((nt, d), np.float32)
        ck = np.zeros((nt, d), np.float32)
        cv = np.zeros((nt, d), np.float32)
        for t, toks in enumerate(tile_tokens):
            n = np.float32(max(len(toks), 1))
            for tok in toks:
                cq[t] = (cq[t] + q[h, tok] / n).astype(np.float32)
                ck[t] = (ck[t] + k[h, tok] / n).astype(np.float32)
                cv[t] = (cv[t] + v[h, tok] / n).astype(np.float32)
        coarse = np.zeros((nt, d), np.float32)
        selected = []
        for qi in range(nt):
            row = np.array([np.float32(np.dot(cq[qi], ck[ki])) * sc for ki in range(nt)], np.float32)
            row = softmax(row)
            coarse[qi] = (row[:, None] * cv).sum(axis=0, dtype=np.float32)
            order = sorted(range(nt), key=lambda ki: (-row[ki], ki))
            selected.append(order[:topk])
        for tok in range(seq):
            qt = int(token_tile[tok])
            keys = [kt for t in selected[qt] for kt in tile_tokens[t]]
            s = (k[h, keys] @ q[h, tok]).astype(np.float32) * sc
            p = softmax(s.astype(np.float32))
            fine = (p[:, None] * v[h, keys]).sum(axis=0, dtype=np.float32)
            out[tok, h] = coarse[qt] * gate[h, tok] + fine
    return out.reshape(seq, heads * d)
