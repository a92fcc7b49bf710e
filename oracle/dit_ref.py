"""The DiT chunk step on the CPU oracle: LightDit (crates/lightx2v-model/src/
dit.rs:440-782) composed from the oracle's restatements of CpuBackend's ops
(linear, layer_norm, residual_norm, gate_residual, head_split, attention and
the MemRoPE KV cache). TEST INFRASTRUCTURE ONLY: the checker for the CUDA
chunk step in lightx2v_cuda/dit.py; nothing in the product imports it.

Weights are the f32 arrays the reference's CpuBackend multiplies (quantized
weights dequantized first, lib.rs:259-284).
"""
from __future__ import annotations

import numpy as np

import oracle

SHIFT_MSA, SCALE_MSA, GATE_MSA, SHIFT_FFN, SCALE_FFN, GATE_FFN = range(6)


class DitRef:
    def __init__(self, cfg, blocks, patch, text1, text2, proj_out, memrope, threads: int = 8):
        """blocks: dicts with the keys of lightx2v_cuda.dit.Block, linears as
        (f32 weight [out, in], bias) pairs, norms as f32 vectors."""
        self.cfg, self.blocks, self.patch, self.text1, self.text2, self.proj_out = (
            cfg, blocks, patch, text1, text2, proj_out)
        self.memrope = memrope
        self.t = threads

    def _lin(self, x, rows, p, n, k, act=0):
        return oracle.linear(x, rows, p[0], n, k, bias=p[1], act=act, threads=self.t)

    def prepare_prompt(self, embeds):
        c = self.cfg
        n, d = c.text_len, c.dim
        mid = self._lin(embeds, n, self.text1, d, c.text_dim, act=1)
        ctx = self._lin(mid, n, self.text2, d, d)
        out = []
        for b in self.blocks:
            kv = self._lin(ctx, n, b["kv2"], 2 * d, d)
            k = oracle.head_split(kv, n, 2 * d, 0, c.heads, c.head_dim, rms_w=b["norm_k2"], eps=c.eps)
            v = oracle.head_split(kv, n, 2 * d, d, c.heads, c.head_dim, eps=c.eps)
            out.append((k, v))
        return out

    def new_caches(self):
        return [oracle.KvCacheRef(self.cfg.heads, self.cfg.head_dim) for _ in self.blocks]

    def forward_chunk(self, caches, h, mods, head_mods, prompt, start_frame, frame_tokens, rope):
        """h: f32 [tokens, dim] (updated copy returned with the output)."""
        c = self.cfg
        s = h.size // c.dim
        d, hd, nh, eps = c.dim, c.head_dim, c.heads, c.eps
        h = np.array(h, np.float32).reshape(s, d)
        temporal = start_frame + np.arange(s) // frame_tokens
        mr = self.memrope
        for li, (b, m) in enumerate(zip(self.blocks, mods)):
            normed = oracle.layer_norm(h, s, d, eps, mods=m, scale=SCALE_MSA, shift=SHIFT_MSA)
            qkv = self._lin(normed, s, b["qkv"], 3 * d, d)
            q = oracle.head_split(qkv, s, 3 * d, 0, nh, hd, rms_w=b["norm_q1"], rope=rope, eps=eps)
            k = oracle.head_split(qkv, s, 3 * d, d, nh, hd, rms_w=b["norm_k1"], rope=rope, eps=eps)
            v = oracle.head_split(qkv, s, 3 * d, 2 * d, nh, hd, eps=eps)
            cache = caches[li]
            cache.put(k, v, s, temporal)
            cache.memrope_update(mr.cache_frames, mr.sink_frames, mr.new_frames(), mr.ema_alpha_long,
                                 mr.ema_alpha_short, frame_tokens)
            kk, vv = cache.kv()
            tk = np.array(cache.temporal)
            mask = tk[None, :] <= temporal[:, None]
            attn = oracle.attention(q, kk, vv, nh, s, cache.rows(), hd, mask, threads=self.t)
            tmp = self._lin(attn, s, b["out1"], d, d)
            h, normed = oracle.residual_norm(h, tmp, s, d, m, GATE_MSA, eps, w=b["norm2_w"], b=b["norm2_b"])
            tmp = self._lin(normed, s, b["q2"], d, d)
            q = oracle.head_split(tmp, s, d, 0, nh, hd, rms_w=b["norm_q2"], eps=eps)
            k2, v2 = prompt[li]
            attn = oracle.attention(q, k2, v2, nh, s, c.text_len, hd, threads=self.t)
            tmp = self._lin(attn, s, b["out2"], d, d)
            h, normed = oracle.residual_norm(h, tmp, s, d, m, None, eps, scale=SCALE_FFN, shift=SHIFT_FFN)
            hid = self._lin(normed, s, b["ffn1"], c.ffn_dim, d, act=1)
            tmp = self._lin(hid, s, b["ffn2"], d, c.ffn_dim)
            h = oracle.gate_residual(h, tmp, s, d, m, GATE_FFN)
        normed = oracle.layer_norm(h, s, d, eps, mods=head_mods, scale=1, shift=0)
        out = self._lin(normed, s, self.proj_out, c.patch_out, d)
        return h, out
