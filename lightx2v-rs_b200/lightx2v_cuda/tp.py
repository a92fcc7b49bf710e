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


# ---- the DiT block tensor-parallel over heads and FFN features ----------------------------------
def _rows(w, r0: int, r1: int, cols: int):
    """Rows [r0, r1) of a quantized struct or of a flat f32 [rows * cols] array."""
    if isinstance(w, (Q8, Q4, Fp8E4M3)):
        return slice_rows(w, r0, r1)
    return np.ascontiguousarray(np.asarray(w, np.float32).reshape(-1, cols)[r0:r1]).reshape(-1)


def _cols(w, k0: int, k1: int, cols: int):
    """Columns [k0, k1) of a quantized struct (group boundaries) or of an f32 array."""
    if isinstance(w, (Q8, Q4, Fp8E4M3)):
        return slice_cols(w, k0, k1)
    return np.ascontiguousarray(np.asarray(w, np.float32).reshape(-1, cols)[:, k0:k1]).reshape(-1)


def _stack(parts):
    """Rows of several matrices stacked (the fused QKV / KV layout, dit.rs:106-149)."""
    a = parts[0]
    if isinstance(a, (Q8, Q4, Fp8E4M3)):
        return type(a).concat(parts)
    return np.concatenate([np.asarray(p, np.float32).reshape(-1) for p in parts])


def head_split_points(heads: int, world: int) -> list[int]:
    """Heads per rank, earlier ranks taking the extra ones (12 heads on 8 GPUs:
    2, 2, 2, 2, 1, 1, 1, 1)."""
    return split_points(heads, world, 1)


def shard_block(block: dict, dim: int, head_dim: int, h0: int, h1: int):
    """This rank's attention weights of one block (host side): the fused QKV
    and the cross-attention KV keep only the rows of heads [h0, h1) of each
    of their parts, q2 likewise; out1 / out2 keep the matching input columns
    (their partial products are summed over the ranks); the q/k RMS weights
    keep those heads' channels. FFN and norm2 are handled elsewhere."""
    c0, c1 = h0 * head_dim, h1 * head_dim
    wq, bq = block["qkv"]
    wkv, bkv = block["kv2"]
    bq, bkv = np.asarray(bq, np.float32), np.asarray(bkv, np.float32)
    sel = lambda v: np.asarray(v, np.float32)[c0:c1]
    return {
        "qkv": (_stack([_rows(wq, p * dim + c0, p * dim + c1, dim) for p in range(3)]),
                np.concatenate([bq[p * dim + c0:p * dim + c1] for p in range(3)])),
        "norm_q1": sel(block["norm_q1"]), "norm_k1": sel(block["norm_k1"]),
        "out1": (_cols(block["out1"][0], c0, c1, dim), np.asarray(block["out1"][1], np.float32)),
        "q2": (_rows(block["q2"][0], c0, c1, dim), sel(block["q2"][1])),
        "kv2": (_stack([_rows(wkv, p * dim + c0, p * dim + c1, dim) for p in range(2)]),
                np.concatenate([bkv[p * dim + c0:p * dim + c1] for p in range(2)])),
        "norm_q2": sel(block["norm_q2"]), "norm_k2": sel(block["norm_k2"]),
        "out2": (_cols(block["out2"][0], c0, c1, dim), np.asarray(block["out2"][1], np.float32)),
    }


class TensorParallelDit:
    """LightDit's chunk step (crates/lightx2v-model/src/dit.rs:440-782) with each
    block tensor-parallel over the group, one process per GPU:

      attention  rank r owns heads [h_r, h_{r+1}): the fused QKV keeps those
                 heads' rows, so q, k, v, the KV cache and the attention are
                 local; the q/k RMS norm spans all heads (cpu lib.rs:433-438),
                 so each rank writes its per-row sum of squares over its heads
                 into every rank's [world][rows] array (peer memory), and
                 head_split adds the ranks' sums in order; out1 is split by its input columns and leaves a
                 partial product on every rank (bias on rank 0);
      cross-attn q2 and the prompt's K/V the same way (the prompt K RMS too);
                 out2 split like out1;
      FFN        FFN1 column-split (GELU local), FFN2 row-split into a partial;
      rows       rank r owns token rows [r0, r1) of the chunk: after each
                 partial it adds its rows of every rank's partial (over NVLink
                 peer memory, CUDA IPC) into its rows of the residual stream h
                 and writes them normalised into every rank's activation
                 buffer (lx2v_tp_reduce_norm between two lx2v_peers_barrier),
                 so the norms run once per row instead of on every rank;
      the rest   patch embed and the output head run on all rows on every
                 rank (the head's input is gathered like the others), so every
                 rank ends a step with the same output.

    `blocks` etc. are the host weights of lightx2v_cuda.dit.LightDitCuda; every
    rank holds the same host copy and uploads only its shard."""

    def __init__(self, be, rank: int, world: int, cfg, blocks, patch, text1, text2, proj_out, memrope=None,
                 partial_dtype: int = L.BF16, exchange=None):
        from .dit import Block, Linear, MemRopeConfig, upload_weight as up
        self.be, self.rank, self.world, self.cfg = be, rank, world, cfg
        # exchange(bytes) -> [bytes of rank 0, ..., rank world-1]: the host
        # channel that carries the CUDA IPC handles of the shared buffers
        # (torch.distributed, a launcher's store, ...); needed for world > 1
        assert world == 1 or exchange is not None, "a tensor-parallel group needs an exchange for IPC handles"
        self.exchange = exchange
        self.memrope = memrope or MemRopeConfig()
        self.partial_dtype = partial_dtype
        d, hd = cfg.dim, cfg.head_dim
        pts = head_split_points(cfg.heads, world)
        self.h0, self.h1 = pts[rank], pts[rank + 1]
        self.nl = self.h1 - self.h0
        self.dl = self.nl * hd
        dl = self.dl

        def lin(p, rows, cols, bias=True):
            b = be.upload(np.asarray(p[1], np.float32), L.F32) if bias else None
            return Linear(up(be, p[0], rows, cols), b)

        def vec(a):
            return be.upload(np.asarray(a, np.float32), L.F32)

        self.patch = lin(patch, d, cfg.patch_in)
        self.text1 = lin(text1, d, cfg.text_dim)
        self.text2 = lin(text2, d, d)
        self.proj_out = lin(proj_out, cfg.patch_out, d)
        self.blocks, self.ffns = [], []
        for b in blocks:
            sh = shard_block(b, d, hd, self.h0, self.h1)
            self.blocks.append(Block(
                qkv=lin(sh["qkv"], 3 * dl, d), norm_q1=vec(sh["norm_q1"]), norm_k1=vec(sh["norm_k1"]),
                out1=lin(sh["out1"], d, dl, bias=rank == 0), q2=lin(sh["q2"], dl, d), kv2=lin(sh["kv2"], 2 * dl, d),
                norm_q2=vec(sh["norm_q2"]), norm_k2=vec(sh["norm_k2"]), out2=lin(sh["out2"], d, dl, bias=rank == 0),
                norm2_w=vec(b["norm2_w"]), norm2_b=vec(b["norm2_b"]), ffn1=None, ffn2=None))
            self.ffns.append(TensorParallelFFN(be, rank, world, b["ffn1"][0], b["ffn1"][1], b["ffn2"][0],
                                               b["ffn2"][1], partial_dtype=partial_dtype))

    def _reduce(self, buf, n):
        if self.world > 1:
            self.be.all_reduce_sum(buf, n)

    def prepare_prompt(self, embeds):
        be, c = self.be, self.cfg
        n, d, dl = c.text_len, c.dim, self.dl
        x = be.upload(np.asarray(embeds, np.float32))
        mid, ctx = be.alloc(n * d), be.alloc(n * d)
        be.linear(x, 0, n, self.text1.w, self.text1.b, L.ACT_GELU_TANH, mid, 0)
        be.linear(mid, 0, n, self.text2.w, self.text2.b, L.ACT_NONE, ctx, 0)
        kv, ss = be.alloc(n * 2 * dl), be.alloc(n, L.F32)
        out = []
        for b in self.blocks:
            be.linear(ctx, 0, n, b.kv2.w, b.kv2.b, L.ACT_NONE, kv, 0)
            k, v = be.alloc(n * dl), be.alloc(n * dl)
            be.row_sumsq(kv, n, 2 * dl, 0, dl, ss)
            self._reduce(ss, n)
            be.head_split_rms(kv, n, 2 * dl, 0, self.nl, c.head_dim, b.norm_k2, ss, d, None, c.eps, k)
            be.head_split(kv, n, 2 * dl, dl, self.nl, c.head_dim, None, None, c.eps, v)
            out.append((k, v))
        return out

    def _share(self, buf):
        """Every rank's instance of `buf` (a collective over the group): own
        buffer at index rank, the peers' mapped by CUDA IPC."""
        if self.world == 1:
            return [buf]
        handles = self.exchange(self.be.ipc_handle(buf))
        return [buf if r == self.rank else self.be.open_ipc(hd, buf.len, buf.dtype) for r, hd in enumerate(handles)]

    def workspace(self, chunk_frames: int, frame_tokens: int, rope_cos, rope_sin):
        """Buffers of one chunk. Each rank owns rows [r0, r1) of the chunk's
        tokens (sequence parallelism): it keeps those rows of the residual
        stream h current and normalises them for every rank; the partial
        products, the normalised activations and the barrier flags are shared
        with the peers by CUDA IPC (a collective: every rank calls this in
        the same order)."""
        from types import SimpleNamespace
        be, c = self.be, self.cfg
        s, d, dl = chunk_frames * frame_tokens, c.dim, self.dl
        cap = self.memrope.cache_frames * frame_tokens
        rows = split_points(s, self.world, 1)
        part, normed = be.alloc(s * d, self.partial_dtype), be.alloc(s * d)
        ws = SimpleNamespace(
            tokens=s, frame_tokens=frame_tokens, r0=rows[self.rank], r1=rows[self.rank + 1],
            caches=[be.kv_cache_new(self.nl, c.head_dim, cap) for _ in self.blocks],
            h=be.alloc(s * d, L.F32), normed=normed, qkv=be.alloc(s * 3 * dl), q=be.alloc(s * dl),
            k=be.alloc(s * dl), v=be.alloc(s * dl), attn=be.alloc(s * dl), q2=be.alloc(s * dl),
            hid=be.alloc(s * self.ffns[0].local), part=part,
            patches=be.alloc(s * max(c.patch_in, c.patch_out)),
            rope_cos=be.upload(np.asarray(rope_cos, np.float32), L.F32),
            rope_sin=be.upload(np.asarray(rope_sin, np.float32), L.F32))
        ws.parts, ws.normeds = self._share(part), self._share(normed)
        # the ranks' per-row q / k sums of squares, [world][rows] on every rank
        ws.ssq, ws.ssk = (self._share(be.alloc(self.world * s, L.F32)) for _ in range(2))
        flags = be.alloc(self.world, L.F32)  # u32 barrier slots, zeroed
        be.sync()  # zeroed before any peer's first barrier can write it
        ws.peers = be.peers_create(self.rank, self.world, self._share(flags))
        return ws

    def row_range(self, ws) -> tuple[int, int]:
        """The chunk rows whose residual stream this rank keeps current."""
        return ws.r0, ws.r1

    def patch_embed(self, ws, latent, c: int, t: int, h: int, w: int):
        be = self.be
        be.patchify(latent, c, t, h, w, self.cfg.patch, ws.patches)
        be.linear(ws.patches, 0, ws.tokens, self.patch.w, self.patch.b, L.ACT_NONE, ws.h, 0)

    def forward_chunk(self, ws, mods, head_mods, prompt, start_frame: int, out):
        """dit.rs:569-782 on this rank's shard; out ends replicated, h current
        on this rank's rows [ws.r0, ws.r1).

        After each row-split linear (out1, out2, FFN2) every rank holds a
        partial product of all rows; between two barriers, one kernel per rank
        adds its rows of every rank's partial (gated) into h and writes those
        rows normalised into every rank's activation buffer, which is what the
        next column-split linear (q2, FFN1, the next block's QKV, the head)
        reads. The FFN's gated residual and the next block's (or the head's)
        layer_norm are one such step."""
        from .dit import GATE_FFN, GATE_MSA, SCALE_FFN, SCALE_MSA, SHIFT_FFN, SHIFT_MSA
        be, c = self.be, self.cfg
        s, d, hd, nl, dl, eps = ws.tokens, c.dim, c.head_dim, self.nl, self.dl, c.eps
        r0, r1, g = ws.r0, ws.r1, ws.peers
        rope = (ws.rope_cos, ws.rope_sin)
        token_temporal = start_frame + np.arange(s) // ws.frame_tokens
        tq = token_temporal.astype(np.int32)

        def step(parts, gate_mods, gate, norm, norm_mods):
            be.peers_barrier(g)  # every rank's partial (and the previous readers of the outputs) done
            be.tp_reduce_norm(g, parts, ws.h, r0, r1, d, gate_mods, gate, norm, norm_mods, eps, ws.normeds)
            be.peers_barrier(g)  # every rank's rows of the output written

        step(None, None, None, ("mod", SCALE_MSA, SHIFT_MSA), mods[0])
        n_blocks = len(self.blocks)
        for li, (bl, m) in enumerate(zip(self.blocks, mods)):
            be.linear(ws.normed, 0, s, bl.qkv.w, bl.qkv.b, L.ACT_NONE, ws.qkv, 0)
            be.row_sumsq_peers(g, ws.qkv, s, 3 * dl, 0, dl, ws.ssq)
            be.row_sumsq_peers(g, ws.qkv, s, 3 * dl, dl, dl, ws.ssk)
            be.peers_barrier(g)
            me = self.rank
            be.head_split_rms_parts(ws.qkv, s, 3 * dl, 0, nl, hd, bl.norm_q1, ws.ssq[me], self.world, d, rope, eps,
                                    ws.q)
            be.head_split_rms_parts(ws.qkv, s, 3 * dl, dl, nl, hd, bl.norm_k1, ws.ssk[me], self.world, d, rope, eps,
                                    ws.k)
            be.head_split(ws.qkv, s, 3 * dl, 2 * dl, nl, hd, None, None, eps, ws.v)
            cache = ws.caches[li]
            be.kv_cache_put(cache, ws.k, ws.v, s, token_temporal)
            be.kv_cache_memrope_update(cache, self.memrope, ws.frame_tokens)
            be.kv_cache_attention(ws.q, s, tq, cache, ws.attn)
            be.linear(ws.attn, 0, s, bl.out1.w, bl.out1.b, L.ACT_NONE, ws.part, 0)
            step(ws.parts, m, GATE_MSA, ("affine", bl.norm2_w, bl.norm2_b), None)
            k2, v2 = prompt[li]
            be.linear(ws.normed, 0, s, bl.q2.w, bl.q2.b, L.ACT_NONE, ws.q2, 0)
            # every rank read ssq (its QKV head_split) before the out1 step's barriers
            be.row_sumsq_peers(g, ws.q2, s, dl, 0, dl, ws.ssq)
            be.peers_barrier(g)
            be.head_split_rms_parts(ws.q2, s, dl, 0, nl, hd, bl.norm_q2, ws.ssq[me], self.world, d, None, eps, ws.q)
            be.attention(ws.q, k2, v2, nl, s, c.text_len, hd, ws.attn)
            be.linear(ws.attn, 0, s, bl.out2.w, bl.out2.b, L.ACT_NONE, ws.part, 0)
            step(ws.parts, m, None, ("mod", SCALE_FFN, SHIFT_FFN), m)
            ffn = self.ffns[li]
            be.linear(ws.normed, 0, s, ffn.w1, ffn.b1, L.ACT_GELU_TANH, ws.hid, 0)
            be.linear(ws.hid, 0, s, ffn.w2, ffn.b2, L.ACT_NONE, ws.part, 0)
            if li + 1 < n_blocks:
                step(ws.parts, m, GATE_FFN, ("mod", SCALE_MSA, SHIFT_MSA), mods[li + 1])
            else:
                step(ws.parts, m, GATE_FFN, ("mod", 1, 0), head_mods)
        be.linear(ws.normed, 0, s, self.proj_out.w, self.proj_out.b, L.ACT_NONE, out, 0)
