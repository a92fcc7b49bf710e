"""Tensor-parallel FFN of a DiT block over P GPUs (one process per GPU).

The reference runs a block's FFN on one device (crates/lightx2v-model/src/
dit.rs:738-760): hid = GELU(x W1^T + b1), then h += gate * (hid W2^T + b2).
Split over P ranks:
  - FFN1 column-split: rank r owns hidden features [f_r, f_{r+1}) — rows of
    W1 and the matching entries of b1 — so GELU stays local;
  - FFN2 row-split: rank r owns the same range of W2's K columns and
    computes a partial [M, D] product over its hidden features;
  - the partials are summed with one all-reduce (NCCL over NVLink, on the
    backend's stream), b2 is added once (by rank 0, inside its partial), and
    the gated residual h += gate * sum is applied on every rank, which keeps
    h replicated. The partials are bf16 by default (the activation precision
    of the CUDA backend, half the bytes on NVLink; each partial is rounded
    once, within the north star's 1e-2) or f32 on request.
Hidden features are split on boundaries that are multiples of the FFN2
weight's quantization group (and of 128), so every rank's W2 slice is a
whole number of the reference's groups: the shard holds exactly the
reference's codes and scales, and the sum of the partials equals the full
product up to f32 summation order.
"""
from __future__ import annotations

import dataclasses

import numpy as np

from . import _lib as L
from .quant import Fp8E4M3, Q4, Q8


def split_points(total: int, parts: int, unit: int) -> list[int]:
    """Boundaries [0 = b_0 <= ... <= b_parts = total] in multiples of `unit`,
    as even as possible (earlier parts take the extra units)."""
    assert total % unit == 0, (total, unit)
    units = total // unit
    base, extra = divmod(units, parts)
    pts = [0]
    for r in range(parts):
        pts.append(pts[-1] + (base + (1 if r < extra else 0)) * unit)
    return pts


def slice_rows(w, r0: int, r1: int):
    """Rows [r0, r1) of a quantized weight (codes and per-row scale groups)."""
    g = w.cols // w.group  # groups per row
    kw = {"q": w.q[r0 * w.cols:r1 * w.cols].copy(), "scales": w.scales[r0 * g:r1 * g].copy(), "rows": r1 - r0}
    if isinstance(w, Q4):
        kw["zeros"] = w.zeros[r0 * g:r1 * g].copy()
    return dataclasses.replace(w, **kw)


def slice_cols(w, k0: int, k1: int):
    """Columns [k0, k1) of a quantized weight; both ends on group boundaries."""
    assert k0 % w.group == 0 and k1 % w.group == 0, (k0, k1, w.group)
    g = w.cols // w.group
    q = w.q.reshape(w.rows, w.cols)[:, k0:k1].reshape(-1).copy()
    sl = slice(k0 // w.group, k1 // w.group)
    kw = {"q": q, "scales": w.scales.reshape(w.rows, g)[:, sl].reshape(-1).copy(), "cols": k1 - k0}
    if isinstance(w, Q4):
        kw["zeros"] = w.zeros.reshape(w.rows, g)[:, sl].reshape(-1).copy()
    return dataclasses.replace(w, **kw)


def upload_weight(be, w):
    if isinstance(w, Fp8E4M3):
        return be.weight_fp8(w)
    if isinstance(w, Q8):
        return be.weight_q8(w)
    if isinstance(w, Q4):
        return be.weight_q4(w)
    raise TypeError(type(w))


class TensorParallelFFN:
    """This rank's shard of a DiT FFN. `w1` [F, D] and `w2` [D, F] are the full
    quantized weights (every rank holds the same host copy), `b1` [F] and
    `b2` [D] f32. The backend must have joined the group (`comm_init`)."""

    def __init__(self, be, rank: int, world: int, w1, b1, w2, b2, partial_dtype: int = L.BF16):
        self.be, self.rank, self.world = be, rank, world
        self.partial_dtype = partial_dtype
        self.dim, self.ffn = w1.cols, w1.rows
        assert w2.rows == self.dim and w2.cols == self.ffn
        unit = int(np.lcm(w2.group, 128))
        pts = split_points(self.ffn, world, unit)
        self.f0, self.f1 = pts[rank], pts[rank + 1]
        self.local = self.f1 - self.f0
        self.w1 = upload_weight(be, slice_rows(w1, self.f0, self.f1))
        self.b1 = be.upload(np.asarray(b1, np.float32)[self.f0:self.f1], L.F32)
        self.w2 = upload_weight(be, slice_cols(w2, self.f0, self.f1))
        self.b2 = be.upload(np.asarray(b2, np.float32), L.F32) if rank == 0 else None
        self._bufs = {}

    def collective_desc(self) -> str:
        if self.world == 1:
            return "none (one rank)"
        dt = "f32" if self.partial_dtype == L.F32 else "bf16"
        return (f"one NCCL all-reduce (sum) of the {dt} [rows, {self.dim}] FFN2 partials per step, on the "
                "backend's stream")

    def _scratch(self, rows: int):
        if rows not in self._bufs:
            self._bufs[rows] = (self.be.alloc(rows * self.local, L.BF16),
                                self.be.alloc(rows * self.dim, self.partial_dtype))
        return self._bufs[rows]

    def forward(self, x, rows: int, h, mods, gate: int):
        """h[:rows] += mods[gate] * (GELU(x W1^T + b1) W2^T + b2), summed over the
        group; x bf16 [rows, D] and h f32 [rows, D] replicated on every rank."""
        hid, part = self._scratch(rows)
        self.be.linear(x, 0, rows, self.w1, self.b1, L.ACT_GELU_TANH, hid, 0)
        self.be.linear(hid, 0, rows, self.w2, self.b2, L.ACT_NONE, part, 0)
        if self.world > 1:
            self.be.all_reduce_sum(part, rows * self.dim)
        self.be.gate_residual(h, part, rows, self.dim, mods, gate)
