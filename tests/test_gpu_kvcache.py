"""GPU KV cache / MemRoPE against the oracle's restatement of CpuBackend's cache
(crates/lightx2v-cpu/src/lib.rs:607-806): the same sequence of puts (a chunk
written, then re-written on the next denoising step) and MemRoPE updates
must give the same temporal indices in the same order, exactly, and the same
K/V rows within bf16 rounding (the device stores bf16; EMA folds are f32 on
the stored values), rel-L2 <= 1e-2. Then the causal attention of a chunk
against the cache, read in place, matches the oracle's attention with the
mask dit.rs:645-657 builds.
"""
from dataclasses import dataclass

import numpy as np
import pytest

from lightx2v_cuda import BF16, F32

pytestmark = pytest.mark.gpu


@dataclass
class MemRope:  # MemRopeConfig::default_memrope (crates/lightx2v-core/src/config.rs:282-295)
    cache_frames: int = 12
    sink_frames: int = 3
    ema_alpha_long: float = 0.01
    ema_alpha_short: float = 0.1

    def new_frames(self):
        return 3


def rel_l2(got, want):
    got = np.asarray(got, np.float64).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    n = np.linalg.norm(want)
    return np.linalg.norm(got - want) / (n if n > 0 else 1.0)


def bf16(a):
    b = np.asarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return (((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


@pytest.mark.parametrize("heads,head_dim,ft", [(2, 128, 4), (3, 16, 5)])
def test_memrope_cache_follows_the_reference(be, oracle, heads, head_dim, ft):
    cfg = MemRope()
    cache = be.kv_cache_new(heads, head_dim, 4 * ft)  # small: the cache must grow
    ref = oracle.KvCacheRef(heads, head_dim)
    rows = 3 * ft
    seed = 100
    for chunk in range(7):
        temporal = [3 * chunk + i // ft for i in range(rows)]
        for step in range(2):  # the chunk's next denoising step overwrites its rows
            k = bf16(oracle.normal(seed, heads * rows * head_dim))
            v = bf16(oracle.normal(seed + 1, heads * rows * head_dim))
            seed += 2
            be.kv_cache_put(cache, be.upload(k, BF16), be.upload(v, F32), rows, temporal)
            ref.put(k, v, rows, temporal)
            be.kv_cache_memrope_update(cache, cfg, ft)
            ref.memrope_update(cfg.cache_frames, cfg.sink_frames, 3, cfg.ema_alpha_long, cfg.ema_alpha_short, ft)
            assert be.kv_cache_len(cache) == ref.rows()
            assert be.kv_cache_temporal(cache).tolist() == ref.temporal
            kb, vb = be.kv_cache_kv(cache, F32)
            rk, rv = ref.kv()
            assert rel_l2(be.download(kb), rk) <= 1e-2, (chunk, step)
            assert rel_l2(be.download(vb), rv) <= 1e-2, (chunk, step)
    assert ref.rows() == cfg.cache_frames * ft  # the cache filled and evicted


def test_append_keeps_repeated_chunks(be, oracle):
    # kv_cache_append never overwrites: the same temporal run twice is two runs
    cache = be.kv_cache_new(1, 8, 0)
    k = oracle.normal(7, 4 * 8)
    for _ in range(2):
        be.kv_cache_append(cache, be.upload(k), be.upload(k), 4, [0, 0, 1, 1])
    assert be.kv_cache_temporal(cache).tolist() == [0, 0, 1, 1, 0, 0, 1, 1]


def test_chunk_attention_against_the_cache(be, oracle):
    # a 3-frame chunk attends to a 12-frame cache (sinks, EMA slots, recent,
    # its own frames), read in place; mask tk <= tq (dit.rs:645-657)
    heads, hd, ft = 4, 128, 96
    cfg = MemRope()
    cache = be.kv_cache_new(heads, hd, 12 * ft)
    rows = 3 * ft
    for chunk in range(5):
        temporal = [3 * chunk + i // ft for i in range(rows)]
        k = bf16(oracle.normal(500 + chunk, heads * rows * hd))
        v = bf16(oracle.normal(600 + chunk, heads * rows * hd))
        be.kv_cache_put(cache, be.upload(k), be.upload(v), rows, temporal)
        be.kv_cache_memrope_update(cache, cfg, ft)
    tq = np.array(temporal, np.int32)
    qb = be.upload(oracle.normal(700, heads * rows * hd))
    q = be.download(qb)
    ob = be.alloc(rows * heads * hd, F32)
    be.kv_cache_attention(qb, rows, tq, cache, ob)
    kb, vb = be.kv_cache_kv(cache, F32)
    sk = be.kv_cache_len(cache)
    tk = be.kv_cache_temporal(cache)
    mask = tk[None, :] <= tq[:, None]
    want = oracle.attention(q, be.download(kb), be.download(vb), heads, rows, sk, hd, mask)
    got = be.download(ob)
    assert np.isfinite(got).all()
    assert rel_l2(got, want) <= 1e-2
    # the reference's own route: kv_cache_kv, then causal_attention with the boolean mask
    ob2 = be.alloc(rows * heads * hd, F32)
    kb2, vb2 = be.kv_cache_kv(cache, BF16)
    be.causal_attention(qb, kb2, vb2, heads, rows, sk, hd, mask, ob2)
    assert rel_l2(be.download(ob2), got) <= 1e-5
