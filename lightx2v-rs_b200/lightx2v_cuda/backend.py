"""`CudaBackend`: the reference's `Backend` trait (crates/lightx2v-core/src/backend.rs:145-446)
for the quantized-linear path, over the C ABI of liblightx2v_cuda.so.

Method names, argument order and meaning follow the trait:
  alloc / upload / write / download / buf_len / copy            backend.rs:160-177
  weight / weight_q8 / weight_q4 / weight_fp8 / sync             backend.rs:178-190
  profile_report / profile_reset                                 backend.rs:192-196
  linear                                                         backend.rs:199-212
  gate_residual                                                  backend.rs:244-253
plus `linear_gate_residual`, the fused form of the FFN2 linear followed by
gate_residual (crates/lightx2v-model/src/dit.rs:748-760).

Like the reference, misuse raises (the reference panics: `assert!` in the
backends); the availability probe `try_new` returns None when no B200 answers
(WgpuBackend::try_new, crates/lightx2v-wgpu/src/lib.rs:285-290).
"""
from __future__ import annotations

import ctypes
import json

import numpy as np

from . import _lib as L
from .quant import Fp8E4M3, Q4, Q8


class Act:
    """`Act` (backend.rs:38-43)."""
    NONE = L.ACT_NONE
    GELU_TANH = L.ACT_GELU_TANH


class Buf:
    """A flat device buffer of activations (bf16 or f32 elements)."""

    def __init__(self, be: "CudaBackend", handle: int, length: int, dtype: int):
        self._be = be
        self.handle = ctypes.c_void_p(handle)
        self.len = length
        self.dtype = dtype

    def __del__(self):
        be = getattr(self, "_be", None)
        if be is not None and be._ctx and self.handle:
            be._lib.lx2v_buf_free(be._ctx, self.handle)
            self.handle = ctypes.c_void_p(0)

    @property
    def dev_ptr(self) -> int:
        p = ctypes.c_void_p()
        self._be._check(self._be._lib.lx2v_buf_info(self._be._ctx, self.handle, None,
                                                     ctypes.byref(p)))
        return p.value or 0


class Weight:
    """A `[rows, cols]` matrix (nn.Linear layout `[out, in]`) on the device."""

    def __init__(self, be: "CudaBackend", handle: int, rows: int, cols: int, fmt: int, group: int):
        self._be = be
        self.handle = ctypes.c_void_p(handle)
        self.rows, self.cols, self.format, self.group = rows, cols, fmt, group

    def __del__(self):
        be = getattr(self, "_be", None)
        if be is not None and be._ctx and self.handle:
            be._lib.lx2v_weight_free(be._ctx, self.handle)
            self.handle = ctypes.c_void_p(0)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).reshape(-1)


class KvCache:
    """A device KV cache handle (Backend::KvCache); freed with the object."""

    def __init__(self, be: "CudaBackend", handle: int, heads: int, head_dim: int):
        self.be, self.handle, self.heads, self.head_dim = be, handle, heads, head_dim

    def __del__(self):
        if getattr(self, "handle", None) and getattr(self.be, "_ctx", None):
            self.be._lib.lx2v_kv_cache_free(self.be._ctx, self.handle)
            self.handle = None


class Sparse:
    """Sparse-attention state of one token grid (lx2v_sparse)."""

    def __init__(self, be: "CudaBackend", handle: int, spec):
        self.be, self.handle, self.spec = be, ctypes.c_void_p(handle), spec

    def __del__(self):
        if getattr(self, "handle", None) and self.handle.value and getattr(self.be, "_ctx", None):
            self.be._lib.lx2v_sparse_free(self.be._ctx, self.handle)
            self.handle = ctypes.c_void_p(0)


class Peers:
    """A tensor-parallel peer group (lx2v_peers): this rank, the group size
    and the flag buffers its barrier uses (kept alive with it)."""

    def __init__(self, be: "CudaBackend", handle: int, rank: int, world: int, flag_bufs: list):
        self.be, self.handle, self.rank, self.world = be, ctypes.c_void_p(handle), rank, world
        self._flags = flag_bufs

    def __del__(self):
        if getattr(self, "handle", None) and self.handle.value:
            self.be._lib.lx2v_peers_free(self.handle)
            self.handle = ctypes.c_void_p(0)


class CudaBackend:
    """The CUDA backend for one device. Buffers default to bf16, the CUDA
    backend's activation precision (backend.rs:9-11)."""

    def __init__(self, device: int = 0, lib_path: str | None = None):
        self._lib = L.load(lib_path)
        ctx = ctypes.c_void_p()
        st = self._lib.lx2v_init(device, ctypes.byref(ctx))
        if st != L.OK:
            raise L.Lx2vError(st, self._lib.lx2v_last_error(None).decode())
        self._ctx = ctx
        self.device = device

    @classmethod
    def try_new(cls, device: int = 0):
        """None when no usable B200 answers (the reference's skip-not-fail)."""
        try:
            return cls(device)
        except L.Lx2vError as e:
            if e.status == L.ERR_NO_DEVICE:
                return None
            raise

    def close(self):
        if getattr(self, "_ctx", None):
            self._lib.lx2v_free_ctx(self._ctx)
            self._ctx = None

    def __del__(self):
        # Buffers and weights hold a reference to the backend, so the context
        # outlives them.
        self.close()

    def _check(self, st: int):
        if st != L.OK:
            raise L.Lx2vError(st, self._lib.lx2v_last_error(self._ctx).decode())

    # ---- backend.rs:158 -------------------------------------------------------
    def name(self) -> str:
        buf = ctypes.create_string_buffer(320)
        self._check(self._lib.lx2v_name(self._ctx, buf, 320))
        return buf.value.decode()

    # ---- memory, backend.rs:160-190 -------------------------------------------
    def alloc(self, length: int, dtype: int = L.BF16) -> Buf:
        h = ctypes.c_void_p()
        self._check(self._lib.lx2v_buf_alloc(self._ctx, length, dtype, ctypes.byref(h)))
        return Buf(self, h.value, length, dtype)

    def upload(self, data, dtype: int = L.BF16) -> Buf:
        a = _f32(data)
        h = ctypes.c_void_p()
        self._check(self._lib.lx2v_buf_upload_f32(self._ctx, a.ctypes.data, a.size, dtype,
                                                  ctypes.byref(h)))
        return Buf(self, h.value, a.size, dtype)

    def upload_ptr(self, host_ptr: int, length: int, dtype: int = L.BF16) -> Buf:
        """upload() from a raw host address of `length` f32 values (e.g. pinned memory)."""
        h = ctypes.c_void_p()
        self._check(self._lib.lx2v_buf_upload_f32(self._ctx, host_ptr, length, dtype,
                                                  ctypes.byref(h)))
        return Buf(self, h.value, length, dtype)

    def write(self, buf: Buf, data):
        a = _f32(data)
        self._check(self._lib.lx2v_buf_write_f32(self._ctx, buf.handle, a.ctypes.data, a.size))

    def write_ptr(self, buf: Buf, host_ptr: int, length: int):
        self._check(self._lib.lx2v_buf_write_f32(self._ctx, buf.handle, host_ptr, length))

    def download(self, buf: Buf) -> np.ndarray:
        out = np.empty(buf.len, np.float32)
        self._check(self._lib.lx2v_buf_download_f32(self._ctx, buf.handle, out.ctypes.data,
                                                    buf.len))
        return out

    def download_ptr(self, buf: Buf, host_ptr: int, length: int):
        self._check(self._lib.lx2v_buf_download_f32(self._ctx, buf.handle, host_ptr, length))

    def download_ptr_async(self, buf: Buf, host_ptr: int, length: int):
        """download_ptr() queued without waiting: the host memory holds the data
        after the next sync() (no reference counterpart; for pipelined steps)."""
        self._check(self._lib.lx2v_buf_download_f32_async(self._ctx, buf.handle, host_ptr, length))

    def buf_len(self, buf: Buf) -> int:
        n = ctypes.c_size_t()
        self._check(self._lib.lx2v_buf_len(self._ctx, buf.handle, ctypes.byref(n)))
        return n.value

    def copy(self, src: Buf, src_off: int, dst: Buf, dst_off: int, length: int):
        self._check(self._lib.lx2v_buf_copy(self._ctx, src.handle, src_off, dst.handle, dst_off,
                                            length))

    def weight(self, data, rows: int, cols: int) -> Weight:
        a = _f32(data)
        assert a.size == rows * cols, "weight: data length != rows * cols"
        h = ctypes.c_void_p()
        self._check(self._lib.lx2v_weight_f32(self._ctx, a.ctypes.data, rows, cols,
                                              ctypes.byref(h)))
        return Weight(self, h.value, rows, cols, L.W_BF16, cols)

    def weight_q8(self, q: Q8) -> Weight:
        codes = np.ascontiguousarray(q.q, np.int8)
        scales = np.ascontiguousarray(q.scales, np.float32)
        h = ctypes.c_void_p()
        self._check(self._lib.lx2v_weight_q8(self._ctx, codes.ctypes.data, scales.ctypes.data,
                                             q.rows, q.cols, q.group, ctypes.byref(h)))
        return Weight(self, h.value, q.rows, q.cols, L.W_Q8, q.group)

    def weight_q4(self, q: Q4) -> Weight:
        packed = np.ascontiguousarray(q.packed(), np.uint8)
        scales = np.ascontiguousarray(q.scales, np.float32)
        zeros = np.ascontiguousarray(q.zeros, np.float32)
        h = ctypes.c_void_p()
        self._check(self._lib.lx2v_weight_q4(self._ctx, packed.ctypes.data, scales.ctypes.data,
                                             zeros.ctypes.data, q.rows, q.cols, q.group,
                                             ctypes.byref(h)))
        return Weight(self, h.value, q.rows, q.cols, L.W_Q4, q.group)

    def weight_fp8(self, q: Fp8E4M3) -> Weight:
        codes = np.ascontiguousarray(q.q, np.uint8)
        scales = np.ascontiguousarray(q.scales, np.float32)
        h = ctypes.c_void_p()
        self._check(self._lib.lx2v_weight_fp8(self._ctx, codes.ctypes.data, scales.ctypes.data,
                                              q.rows, q.cols, q.group, ctypes.byref(h)))
        return Weight(self, h.value, q.rows, q.cols, L.W_FP8, q.group)

    def weight_nvfp4(self, q) -> Weight:
        """NVFP4 weight (no reference counterpart): packed e2m1 codes, e4m3 block
        scales, f32 global scale (lightx2v_cuda.quant.Nvfp4)."""
        packed = np.ascontiguousarray(q.q, np.uint8)
        scales = np.ascontiguousarray(q.scales, np.uint8)
        h = ctypes.c_void_p()
        self._check(self._lib.lx2v_weight_nvfp4(self._ctx, packed.ctypes.data, scales.ctypes.data,
                                                float(q.global_scale), q.rows, q.cols, ctypes.byref(h)))
        return Weight(self, h.value, q.rows, q.cols, L.W_NVFP4, 16)

    def weight_dequant_f32(self, w: Weight) -> np.ndarray:
        """Test hook: the device's decode of `w` as f32 [rows*cols]."""
        out = np.empty(w.rows * w.cols, np.float32)
        self._check(self._lib.lx2v_weight_dequant_f32(self._ctx, w.handle, out.ctypes.data))
        return out

    def sync(self):
        self._check(self._lib.lx2v_sync(self._ctx))

    def stream(self) -> int:
        return self._lib.lx2v_stream(self._ctx) or 0

    # ---- profiling, backend.rs:192-196 ------------------------------------------
    def profile_report(self) -> str | None:
        prof = self.profile()
        if not prof:
            return None
        total = sum(v["ms"] for v in prof.values()) or 1.0
        lines = ["cuda profile (LIGHTX2V_PROFILE=1; device time per op):",
                 "op                     calls      total_ms   mean_us   share"]
        for name, v in sorted(prof.items(), key=lambda kv: -kv[1]["ms"]):
            lines.append(f"{name:<20} {v['calls']:>8} {v['ms']:>12.3f} "
                         f"{v['ms'] * 1e3 / max(v['calls'], 1):>9.1f} {v['ms'] / total * 100:>6.1f}%")
        return "\n".join(lines) + "\n"

    def profile(self) -> dict:
        n = ctypes.c_size_t()
        self._check(self._lib.lx2v_profile_json(self._ctx, None, 0, ctypes.byref(n)))
        buf = ctypes.create_string_buffer(n.value)
        self._check(self._lib.lx2v_profile_json(self._ctx, buf, n.value, ctypes.byref(n)))
        return json.loads(buf.value.decode())

    def profile_reset(self):
        self._check(self._lib.lx2v_profile_reset(self._ctx))

    # ---- transformer, backend.rs:199-253 ------------------------------------------
    def linear(self, x: Buf, x_row: int, rows: int, w: Weight, bias: Buf | None, act: int,
               y: Buf, y_row: int):
        """y[y_row + i, :] = act(x[x_row + i, :] . W^T + b) for i < rows."""
        self._check(self._lib.lx2v_linear(self._ctx, x.handle, x_row, rows, w.handle,
                                          bias.handle if bias is not None else None, act,
                                          y.handle, y_row))

    def linear_noalloc(self, x: Buf, x_row: int, rows: int, w: Weight, bias: Buf | None, act: int,
                       y: Buf, y_row: int):
        """linear() for callers that cannot have the library allocate device
        memory mid-run (a pre-planned VRAM budget, or no tolerance for
        cudaMalloc's device-wide synchronisation): the stream-K scratch lives
        in a fixed LX2V_NOALLOC_SCRATCH_BYTES array inside the library. Calls
        that may overlap on one GPU share that array and race; the first call
        on a device looks the array up, so make it before any stream capture."""
        self._check(self._lib.lx2v_linear_noalloc(self._ctx, x.handle, x_row, rows, w.handle,
                                                  bias.handle if bias is not None else None, act,
                                                  y.handle, y_row))

    def linear_gate_residual(self, x: Buf, x_row: int, rows: int, w: Weight, bias: Buf | None,
                             act: int, h: Buf, h_row: int, mods: Buf, gate: int):
        """h[h_row + i, j] += act(x[x_row + i, :] . W^T + b)[j] * mods[gate * N + j]."""
        self._check(self._lib.lx2v_linear_gate_residual(
            self._ctx, x.handle, x_row, rows, w.handle,
            bias.handle if bias is not None else None, act, h.handle, h_row, mods.handle, gate))

    def attention(self, q: Buf, k: Buf, v: Buf, heads: int, sq: int, sk: int, head_dim: int, out: Buf):
        """backend.rs:275-289: softmax(q k^T / sqrt(d)) v per head; q [heads, sq, d],
        k/v [heads, sk, d], out [sq, heads * d]."""
        self._check(self._lib.lx2v_attention(self._ctx, q.handle, k.handle, v.handle, heads, sq, sk,
                                             head_dim, out.handle))

    def causal_attention(self, q: Buf, k: Buf, v: Buf, heads: int, sq: int, sk: int, head_dim: int,
                         mask, out: Buf):
        """backend.rs:291-307: `mask` is a [sq, sk] boolean array (True = allowed) or None."""
        m = None
        if mask is not None:
            m = np.ascontiguousarray(np.asarray(mask, dtype=bool).reshape(sq, sk)).view(np.uint8)
        self._check(self._lib.lx2v_causal_attention(self._ctx, q.handle, k.handle, v.handle, heads, sq, sk,
                                                    head_dim, m.ctypes.data if m is not None else None,
                                                    out.handle))

    def causal_attention_temporal(self, q: Buf, k: Buf, v: Buf, heads: int, sq: int, sk: int, head_dim: int,
                                  tq, tk, out: Buf):
        """causal_attention with the mask tk[key] <= tq[query] (the DiT's MemRoPE
        mask, dit.rs:645-657) given by the temporal indices."""
        tq = np.ascontiguousarray(tq, np.int32)
        tk = np.ascontiguousarray(tk, np.int32)
        assert tq.size == sq and tk.size == sk
        self._check(self._lib.lx2v_causal_attention_temporal(self._ctx, q.handle, k.handle, v.handle, heads,
                                                             sq, sk, head_dim, tq.ctypes.data,
                                                             tk.ctypes.data, out.handle))

    # ---- norms / head_split / patchify / dmd_step, backend.rs:214-273, 392-428 -----
    @staticmethod
    def _norm(norm):
        """NormKind as ("affine", w, b) or ("mod", scale, shift) -> C arguments."""
        if norm[0] == "affine":
            return 0, norm[1].handle, norm[2].handle, 0, 0
        assert norm[0] == "mod"
        return 1, None, None, norm[1], norm[2]

    def layer_norm(self, x: Buf, rows: int, dim: int, norm, mods: Buf | None, eps: float, out: Buf):
        kind, w, b, scale, shift = self._norm(norm)
        self._check(self._lib.lx2v_layer_norm(self._ctx, x.handle, rows, dim, kind, w, b, scale, shift,
                                              mods.handle if mods is not None else None, eps, out.handle))

    def residual_norm(self, h: Buf, a: Buf, rows: int, dim: int, mods: Buf, gate: int | None, norm, eps: float,
                      normed: Buf):
        kind, w, b, scale, shift = self._norm(norm)
        self._check(self._lib.lx2v_residual_norm(self._ctx, h.handle, a.handle, rows, dim, mods.handle,
                                                 -1 if gate is None else gate, kind, w, b, scale, shift, eps,
                                                 normed.handle))

    def head_split(self, src: Buf, rows: int, src_stride: int, col_off: int, heads: int, head_dim: int,
                   rms_w: Buf | None, rope, eps: float, out: Buf):
        cos, sin = (rope[0].handle, rope[1].handle) if rope is not None else (None, None)
        self._check(self._lib.lx2v_head_split(self._ctx, src.handle, rows, src_stride, col_off, heads, head_dim,
                                              rms_w.handle if rms_w is not None else None, cos, sin, eps,
                                              out.handle))

    def row_sumsq(self, src: Buf, rows: int, src_stride: int, col_off: int, width: int, out: Buf):
        """out[r] = sum of squares of columns [col_off, col_off + width) of row r (f32)."""
        self._check(self._lib.lx2v_row_sumsq(self._ctx, src.handle, rows, src_stride, col_off, width, out.handle))

    def head_split_rms(self, src: Buf, rows: int, src_stride: int, col_off: int, heads: int, head_dim: int,
                       rms_w: Buf, sumsq: Buf, rms_dim: int, rope, eps: float, out: Buf):
        """head_split with the RMS statistic given (rows' sums of squares over
        rms_dim values, summed across tensor-parallel ranks)."""
        cos, sin = (rope[0].handle, rope[1].handle) if rope is not None else (None, None)
        self._check(self._lib.lx2v_head_split_rms(self._ctx, src.handle, rows, src_stride, col_off, heads, head_dim,
                                                  rms_w.handle, sumsq.handle, rms_dim, cos, sin, eps, out.handle))

    def patchify(self, latent: Buf, c: int, t: int, h: int, w: int, p: int, out: Buf):
        self._check(self._lib.lx2v_patchify(self._ctx, latent.handle, c, t, h, w, p, out.handle))

    def unpatchify(self, x: Buf, c: int, t: int, h: int, w: int, p: int, out: Buf):
        self._check(self._lib.lx2v_unpatchify(self._ctx, x.handle, c, t, h, w, p, out.handle))

    def dmd_step(self, x: Buf, v: Buf, noise: Buf | None, sigma_t: float, sigma_next: float, n: int):
        self._check(self._lib.lx2v_dmd_step(self._ctx, x.handle, v.handle,
                                            noise.handle if noise is not None else None, sigma_t, sigma_next, n))

    # ---- KV cache / MemRoPE, backend.rs:334-390 ------------------------------------
    def kv_cache_new(self, heads: int, head_dim: int, capacity_tokens: int) -> "KvCache":
        h = ctypes.c_void_p()
        self._check(self._lib.lx2v_kv_cache_new(self._ctx, heads, head_dim, capacity_tokens, ctypes.byref(h)))
        return KvCache(self, h.value, heads, head_dim)

    def kv_cache_append(self, cache: "KvCache", k: Buf, v: Buf, rows: int, temporal):
        t = np.ascontiguousarray(temporal, np.uint64)
        assert t.size == rows
        self._check(self._lib.lx2v_kv_cache_append(self._ctx, cache.handle, k.handle, v.handle, rows,
                                                   t.ctypes.data))

    def kv_cache_put(self, cache: "KvCache", k: Buf, v: Buf, rows: int, temporal):
        t = np.ascontiguousarray(temporal, np.uint64)
        assert t.size == rows
        self._check(self._lib.lx2v_kv_cache_put(self._ctx, cache.handle, k.handle, v.handle, rows, t.ctypes.data))

    def kv_cache_len(self, cache: "KvCache") -> int:
        n = ctypes.c_size_t()
        self._check(self._lib.lx2v_kv_cache_len(self._ctx, cache.handle, ctypes.byref(n)))
        return n.value

    def kv_cache_temporal(self, cache: "KvCache") -> np.ndarray:
        n = self.kv_cache_len(cache)
        out = np.zeros(max(n, 1), np.uint64)
        self._check(self._lib.lx2v_kv_cache_temporal(self._ctx, cache.handle, out.ctypes.data, out.size))
        return out[:n].astype(np.int64)

    def kv_cache_kv(self, cache: "KvCache", dtype: int = L.BF16):
        n = cache.heads * self.kv_cache_len(cache) * cache.head_dim
        k, v = self.alloc(n, dtype), self.alloc(n, dtype)
        self._check(self._lib.lx2v_kv_cache_kv(self._ctx, cache.handle, k.handle, v.handle))
        return k, v

    def kv_cache_memrope_update(self, cache: "KvCache", cfg, frame_tokens: int):
        """cfg: any object with cache_frames, sink_frames, ema_alpha_long, ema_alpha_short
        (MemRopeConfig, config.rs:265-300); new_frames() is 3 unless cfg says otherwise."""
        new_frames = cfg.new_frames() if hasattr(cfg, "new_frames") else 3
        self._check(self._lib.lx2v_kv_cache_memrope_update(self._ctx, cache.handle, cfg.cache_frames,
                                                           cfg.sink_frames, new_frames, cfg.ema_alpha_long,
                                                           cfg.ema_alpha_short, frame_tokens))

    def kv_cache_attention(self, q: Buf, sq: int, tq, cache: "KvCache", out: Buf):
        tq = np.ascontiguousarray(tq, np.int32)
        assert tq.size == sq
        self._check(self._lib.lx2v_kv_cache_attention(self._ctx, q.handle, sq, tq.ctypes.data, cache.handle,
                                                      out.handle))

    def gate_residual(self, h: Buf, a: Buf, rows: int, dim: int, mods: Buf, gate: int):
        """In place on h: h += a * mods[gate] (backend.rs:244-253)."""
        self._check(self._lib.lx2v_gate_residual(self._ctx, h.handle, a.handle, rows, dim,
                                                 mods.handle, gate))

    # ---- tensor parallelism (no reference counterpart) -----------------------------
    def comm_unique_id(self) -> bytes:
        """NCCL id for a new tensor-parallel group (made on one rank, passed to all)."""
        buf = ctypes.create_string_buffer(L.COMM_ID_BYTES)
        st = self._lib.lx2v_comm_unique_id(buf, L.COMM_ID_BYTES)
        if st != L.OK:  # a context-free call: its message is the library-wide one
            raise L.Lx2vError(st, self._lib.lx2v_last_error(None).decode())
        return buf.raw

    def comm_init(self, uid: bytes, rank: int, world: int):
        assert len(uid) == L.COMM_ID_BYTES
        self._check(self._lib.lx2v_comm_init(self._ctx, uid, rank, world))

    def all_reduce_sum(self, buf: Buf, length: int | None = None):
        """In place: buf[:length] = sum over the group (on this context's stream)."""
        self._check(self._lib.lx2v_all_reduce_sum(self._ctx, buf.handle, buf.len if length is None else length))

    # ---- sparse attention, backend.rs:309-331 -------------------------------------------
    def sparse_prepare(self, spec) -> Sparse:
        """spec: lightx2v_cuda.vsa.SparseSpec (the reference's SparseSpec)."""
        p = spec.plan
        slots = np.ascontiguousarray(p.slot_src, np.uint32)
        sizes = np.ascontiguousarray(p.block_sizes, np.uint32)
        h = ctypes.c_void_p()
        self._check(self._lib.lx2v_sparse_prepare(self._ctx, slots.ctypes.data, sizes.ctypes.data, p.num_tiles(),
                                                  p.seq, spec.heads, spec.head_dim, spec.topk, spec.scale,
                                                  ctypes.byref(h)))
        return Sparse(self, h.value, spec)

    def sparse_attention(self, q: Buf, k: Buf, v: Buf, gate: Buf, sp: Sparse, out: Buf):
        self._check(self._lib.lx2v_sparse_attention(self._ctx, q.handle, k.handle, v.handle, gate.handle,
                                                    sp.handle, out.handle))

    # ---- tensor parallelism over NVLink peer memory (no reference counterpart) --------
    def ipc_handle(self, buf: Buf) -> bytes:
        """CUDA IPC handle of an own buffer, for the other processes of a group."""
        out = ctypes.create_string_buffer(L.IPC_HANDLE_BYTES)
        self._check(self._lib.lx2v_buf_ipc_handle(self._ctx, buf.handle, out, L.IPC_HANDLE_BYTES))
        return out.raw

    def open_ipc(self, handle: bytes, length: int, dtype: int) -> Buf:
        """A peer's buffer mapped into this context (freeing it unmaps it)."""
        assert len(handle) == L.IPC_HANDLE_BYTES
        h = ctypes.c_void_p()
        self._check(self._lib.lx2v_buf_open_ipc(self._ctx, handle, length, dtype, ctypes.byref(h)))
        return Buf(self, h.value, length, dtype)

    def peers_create(self, rank: int, world: int, flag_bufs: list) -> "Peers":
        """A peer group; flag_bufs[r] is rank r's flag buffer (own one at index rank)."""
        arr = (ctypes.c_void_p * world)(*[b.handle.value for b in flag_bufs])
        h = ctypes.c_void_p()
        self._check(self._lib.lx2v_peers_create(self._ctx, rank, world, arr, ctypes.byref(h)))
        return Peers(self, h.value, rank, world, flag_bufs)

    def peers_barrier(self, g: "Peers"):
        self._check(self._lib.lx2v_peers_barrier(self._ctx, g.handle))

    def row_sumsq_peers(self, g: "Peers", src: Buf, rows: int, src_stride: int, col_off: int, width: int,
                        outs: list):
        """This rank's row sums of squares into its slot of every rank's [world][rows] buffer."""
        oa = (ctypes.c_void_p * g.world)(*[o.handle.value for o in outs])
        self._check(self._lib.lx2v_row_sumsq_peers(self._ctx, g.handle, src.handle, rows, src_stride, col_off,
                                                   width, oa))

    def head_split_rms_parts(self, src: Buf, rows: int, src_stride: int, col_off: int, heads: int, head_dim: int,
                             rms_w: Buf, sumsq: Buf, parts: int, rms_dim: int, rope, eps: float, out: Buf):
        cos, sin = (rope[0].handle, rope[1].handle) if rope is not None else (None, None)
        self._check(self._lib.lx2v_head_split_rms_parts(self._ctx, src.handle, rows, src_stride, col_off, heads,
                                                        head_dim, rms_w.handle, sumsq.handle, parts, rms_dim, cos,
                                                        sin, eps, out.handle))

    def tp_reduce_norm(self, g: "Peers", parts: list | None, h: Buf, row0: int, row1: int, dim: int,
                       gate_mods: Buf | None, gate: int | None, norm, norm_mods: Buf | None, eps: float,
                       normed: list):
        """Rows [row0, row1) owned by this rank: h += gate * sum of every rank's
        partial, then the norm into every rank's output (see the C header)."""
        kind, w, b, scale, shift = self._norm(norm)
        n = g.world
        pa = (ctypes.c_void_p * n)(*[p.handle.value for p in parts]) if parts is not None else None
        oa = (ctypes.c_void_p * n)(*[o.handle.value for o in normed])
        self._check(self._lib.lx2v_tp_reduce_norm(
            self._ctx, g.handle, pa, h.handle, row0, row1, dim, gate_mods.handle if gate_mods is not None else None,
            -1 if gate is None else gate, kind, w, b, norm_mods.handle if norm_mods is not None else None,
            scale, shift, eps, oa))

    # ---- knobs ---------------------------------------------------------------------
    def set_linear_path(self, path: int):
        """0 automatic, 1 tensor-core GEMM, 2 small-M GEMV, 3 generic CUDA-core kernel,
        4 CTA-pair tensor-core GEMM, 5 two-pass (bf16 decode + CTA-pair GEMM)."""
        self._check(self._lib.lx2v_set_linear_path(self._ctx, path))

    def set_token_tile(self, tokens: int):
        """Tokens per tensor-core tile: 0 automatic, or 128 / 192 / 256."""
        self._check(self._lib.lx2v_set_token_tile(self._ctx, tokens))

    def set_split_mode(self, mode: int):
        """Work split of the CTA-pair kernel: 0 automatic, 1 whole tiles, 2 stream-K."""
        self._check(self._lib.lx2v_set_split_mode(self._ctx, mode))

    def set_wait_limit_ns(self, ns: int):
        self._check(self._lib.lx2v_set_wait_limit_ns(self._ctx, ns))

    def launch_count(self) -> int:
        n = ctypes.c_uint64()
        self._check(self._lib.lx2v_launch_count(self._ctx, ctypes.byref(n)))
        return n.value
