"""The DiT chunk step of lightx2v-rs on the CUDA backend.

A host-side mirror of crates/lightx2v-model/src/dit.rs (LightDit::
prepare_prompt :440-493, workspace :498-535, patch_embed :539-560,
forward_chunk :569-782): the same op sequence, called through this
package's C ABI, so that a whole denoising step of a chunk runs on one B200
with every op (linears, norms, head_split, KV cache / MemRoPE, attention)
on the device. A Rust caller keeps the reference's own dit.rs and binds the
same entry points through the `Backend` trait; this module is what the
tests and the benchmark drive.

Weights come from the caller (quantized structs of lightx2v_cuda.quant or
f32 arrays); the module does not read checkpoints itself (weights.py does).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import _lib as L

# rows of a block's [6, dim] modulation table (dit.rs:30-35)
SHIFT_MSA, SCALE_MSA, GATE_MSA, SHIFT_FFN, SCALE_FFN, GATE_FFN = range(6)


@dataclass
class WanConfig:
    """WanConfig (crates/lightx2v-core/src/config.rs:30-91), the fields the DiT reads."""
    heads: int = 12
    head_dim: int = 128
    ffn_dim: int = 8960
    layers: int = 30
    text_dim: int = 4096
    text_len: int = 512
    in_channels: int = 16
    out_channels: int = 16
    patch: int = 2
    eps: float = 1e-6

    @property
    def dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def patch_in(self) -> int:
        return self.in_channels * self.patch * self.patch

    @property
    def patch_out(self) -> int:
        return self.out_channels * self.patch * self.patch


@dataclass
class MemRopeConfig:
    """MemRopeConfig::default_memrope (config.rs:282-295)."""
    cache_frames: int = 12
    sink_frames: int = 3
    ema_alpha_long: float = 0.01
    ema_alpha_short: float = 0.1

    def new_frames(self) -> int:
        return 3


@dataclass
class Linear:
    w: object  # device Weight
    b: object  # device Buf (f32)


@dataclass
class Block:
    qkv: Linear
    norm_q1: object
    norm_k1: object
    out1: Linear
    q2: Linear
    kv2: Linear
    norm_q2: object
    norm_k2: object
    out2: Linear
    norm2_w: object
    norm2_b: object
    ffn1: Linear
    ffn2: Linear


@dataclass
class Workspace:
    """Activation buffers of one chunk (dit.rs:208-232), reused by every block."""
    tokens: int
    frame_tokens: int
    caches: list
    h: object
    normed: object
    qkv: object
    q: object
    k: object
    v: object
    attn: object
    tmp: object
    hid: object
    patches: object
    rope_cos: object
    rope_sin: object


def upload_weight(be, w, rows: int, cols: int):
    """A quantized struct (Q8 / Q4 / Fp8E4M3) or an f32 array -> device weight."""
    from .quant import Fp8E4M3, Q4, Q8
    if isinstance(w, Q8):
        return be.weight_q8(w)
    if isinstance(w, Q4):
        return be.weight_q4(w)
    if isinstance(w, Fp8E4M3):
        return be.weight_fp8(w)
    return be.weight(w, rows, cols)


class LightDitCuda:
    """LightDit on the CUDA backend. `blocks` is a list of dicts of host weights
    with the keys of Block (linears as (weight, bias) pairs; norm vectors as f32
    arrays); `patch`, `text1`, `text2`, `proj_out` are (weight, bias) pairs."""

    def __init__(self, be, cfg: WanConfig, blocks, patch, text1, text2, proj_out,
                 memrope: MemRopeConfig | None = None):
        self.be, self.cfg = be, cfg
        self.memrope = memrope or MemRopeConfig()
        d, f = cfg.dim, cfg.ffn_dim

        def lin(p, rows, cols):
            return Linear(upload_weight(be, p[0], rows, cols), be.upload(np.asarray(p[1], np.float32), L.F32))

        def vec(a):
            return be.upload(np.asarray(a, np.float32), L.F32)

        self.patch = lin(patch, d, cfg.patch_in)
        self.text1 = lin(text1, d, cfg.text_dim)
        self.text2 = lin(text2, d, d)
        self.proj_out = lin(proj_out, cfg.patch_out, d)
        self.blocks = [Block(qkv=lin(b["qkv"], 3 * d, d), norm_q1=vec(b["norm_q1"]), norm_k1=vec(b["norm_k1"]),
                             out1=lin(b["out1"], d, d), q2=lin(b["q2"], d, d), kv2=lin(b["kv2"], 2 * d, d),
                             norm_q2=vec(b["norm_q2"]), norm_k2=vec(b["norm_k2"]), out2=lin(b["out2"], d, d),
                             norm2_w=vec(b["norm2_w"]), norm2_b=vec(b["norm2_b"]), ffn1=lin(b["ffn1"], f, d),
                             ffn2=lin(b["ffn2"], d, f))
                       for b in blocks]

    # ---- dit.rs:440-493 ----------------------------------------------------------------
    def prepare_prompt(self, embeds):
        """Text embeds [text_len, text_dim] -> per-block cross-attention (k, v),
        each [heads, text_len, head_dim]."""
        be, c = self.be, self.cfg
        n, d = c.text_len, c.dim
        x = be.upload(np.asarray(embeds, np.float32))
        mid, ctx = be.alloc(n * d), be.alloc(n * d)
        be.linear(x, 0, n, self.text1.w, self.text1.b, L.ACT_GELU_TANH, mid, 0)
        be.linear(mid, 0, n, self.text2.w, self.text2.b, L.ACT_NONE, ctx, 0)
        kv = be.alloc(n * 2 * d)
        out = []
        for b in self.blocks:
            be.linear(ctx, 0, n, b.kv2.w, b.kv2.b, L.ACT_NONE, kv, 0)
            k, v = be.alloc(n * d), be.alloc(n * d)
            be.head_split(kv, n, 2 * d, 0, c.heads, c.head_dim, b.norm_k2, None, c.eps, k)
            be.head_split(kv, n, 2 * d, d, c.heads, c.head_dim, None, None, c.eps, v)
            out.append((k, v))
        return out

    # ---- dit.rs:498-535 -----------------------------------------------------------------
    def workspace(self, chunk_frames: int, frame_tokens: int, rope_cos, rope_sin) -> Workspace:
        """rope_cos / rope_sin: [tokens, head_dim / 2] tables of the chunk's
        tokens (rope.rs rope_table_for_indices)."""
        be, c = self.be, self.cfg
        s, d = chunk_frames * frame_tokens, c.dim
        cap = self.memrope.cache_frames * frame_tokens
        return Workspace(
            tokens=s, frame_tokens=frame_tokens,
            caches=[be.kv_cache_new(c.heads, c.head_dim, cap) for _ in range(len(self.blocks))],
            h=be.alloc(s * d, L.F32), normed=be.alloc(s * d), qkv=be.alloc(s * 3 * d), q=be.alloc(s * d),
            k=be.alloc(s * d), v=be.alloc(s * d), attn=be.alloc(s * d), tmp=be.alloc(s * d),
            hid=be.alloc(s * c.ffn_dim), patches=be.alloc(s * max(c.patch_in, c.patch_out)),
            rope_cos=be.upload(np.asarray(rope_cos, np.float32), L.F32),
            rope_sin=be.upload(np.asarray(rope_sin, np.float32), L.F32))

    # ---- dit.rs:539-560 -----------------------------------------------------------------
    def patch_embed(self, ws: Workspace, latent, c: int, t: int, h: int, w: int):
        be = self.be
        be.patchify(latent, c, t, h, w, self.cfg.patch, ws.patches)
        be.linear(ws.patches, 0, ws.tokens, self.patch.w, self.patch.b, L.ACT_NONE, ws.h, 0)

    # ---- dit.rs:569-782 -----------------------------------------------------------------
    def forward_chunk(self, ws: Workspace, mods, head_mods, prompt, start_frame: int, out):
        """One chunk through every block and the output head. `mods` is one
        [6, dim] device table per block, `head_mods` the [2, dim] head table;
        `out` gets [tokens, patch_out]. The per-layer caches are updated."""
        be, c = self.be, self.cfg
        s, d, hd, nh, eps = ws.tokens, c.dim, c.head_dim, c.heads, c.eps
        ft = ws.frame_tokens
        rope = (ws.rope_cos, ws.rope_sin)
        token_temporal = start_frame + np.arange(s) // ft
        tq = token_temporal.astype(np.int32)
        for li, (bl, m) in enumerate(zip(self.blocks, mods)):
            # self-attention: AdaLN, QKV, q/k RMS across heads + RoPE, v split
            be.layer_norm(ws.h, s, d, ("mod", SCALE_MSA, SHIFT_MSA), m, eps, ws.normed)
            be.linear(ws.normed, 0, s, bl.qkv.w, bl.qkv.b, L.ACT_NONE, ws.qkv, 0)
            be.head_split(ws.qkv, s, 3 * d, 0, nh, hd, bl.norm_q1, rope, eps, ws.q)
            be.head_split(ws.qkv, s, 3 * d, d, nh, hd, bl.norm_k1, rope, eps, ws.k)
            be.head_split(ws.qkv, s, 3 * d, 2 * d, nh, hd, None, None, eps, ws.v)
            # MemRoPE: write the chunk's K/V, fold / evict, attend to the cache
            # (mask tk <= tq evaluated on the device, read in place)
            cache = ws.caches[li]
            be.kv_cache_put(cache, ws.k, ws.v, s, token_temporal)
            be.kv_cache_memrope_update(cache, self.memrope, ft)
            be.kv_cache_attention(ws.q, s, tq, cache, ws.attn)
            be.linear(ws.attn, 0, s, bl.out1.w, bl.out1.b, L.ACT_NONE, ws.tmp, 0)
            be.residual_norm(ws.h, ws.tmp, s, d, m, GATE_MSA, ("affine", bl.norm2_w, bl.norm2_b), eps, ws.normed)
            # cross-attention against the prompt's K/V
            k2, v2 = prompt[li]
            be.linear(ws.normed, 0, s, bl.q2.w, bl.q2.b, L.ACT_NONE, ws.tmp, 0)
            be.head_split(ws.tmp, s, d, 0, nh, hd, bl.norm_q2, None, eps, ws.q)
            be.attention(ws.q, k2, v2, nh, s, c.text_len, hd, ws.attn)
            be.linear(ws.attn, 0, s, bl.out2.w, bl.out2.b, L.ACT_NONE, ws.tmp, 0)
            be.residual_norm(ws.h, ws.tmp, s, d, m, None, ("mod", SCALE_FFN, SHIFT_FFN), eps, ws.normed)
            # FFN; FFN2 fused with the gated residual h += gate * (hid W2^T + b2)
            be.linear(ws.normed, 0, s, bl.ffn1.w, bl.ffn1.b, L.ACT_GELU_TANH, ws.hid, 0)
            be.linear_gate_residual(ws.hid, 0, s, bl.ffn2.w, bl.ffn2.b, L.ACT_NONE, ws.h, 0, m, GATE_FFN)
        # output head: AdaLN with the [2, dim] table (shift = row 0, scale = row 1)
        be.layer_norm(ws.h, s, d, ("mod", 1, 0), head_mods, eps, ws.normed)
        be.linear(ws.normed, 0, s, self.proj_out.w, self.proj_out.b, L.ACT_NONE, out, 0)


def synthetic_block(cfg: WanConfig, seed: int, quantize, std: float = 0.02):
    """Host weights of one block with the reference's shapes: N(0, std)
    matrices through `quantize(w, rows, cols)` (or kept f32 when it is None),
    biases N(0, 0.01), norm weights 1 + N(0, 0.1)."""
    from . import rng
    d, f = cfg.dim, cfg.ffn_dim

    def mat(k, rows, cols):
        w = rng.normal(seed * 100 + k, rows * cols, std)
        return (quantize(w, rows, cols) if quantize else w), rng.normal(seed * 100 + 50 + k, rows, 0.01)

    def norm(k):
        return np.float32(1.0) + rng.normal(seed * 100 + 80 + k, d, 0.1)

    return {"qkv": mat(1, 3 * d, d), "norm_q1": norm(1), "norm_k1": norm(2), "out1": mat(2, d, d),
            "q2": mat(3, d, d), "kv2": mat(4, 2 * d, d), "norm_q2": norm(3), "norm_k2": norm(4),
            "out2": mat(5, d, d), "norm2_w": norm(5), "norm2_b": rng.normal(seed * 100 + 90, d, 0.1),
            "ffn1": mat(6, f, d), "ffn2": mat(7, d, f)}
