"""The DiT chunk step end to end on the GPU against the oracle's composition of
CpuBackend ops (oracle/dit_ref.py): two full-width Wan2.1-1.3B blocks (dim
1536, 12 heads x 128, FFN 8960, Q8 attention/FFN weights, native patch /
text / head weights), the prompt's cross-attention K/V, and five successive
3-frame chunks through the per-layer MemRoPE caches (sinks, EMA seeding,
graduation, eviction all happen), each chunk's output and residual stream
compared with rel-L2 <= 1e-2 (the north star's tolerance). The spatial size
is reduced (64 tokens per frame) so that the oracle finishes in seconds; the
width and every op are the real ones.
"""
import numpy as np
import pytest

from lightx2v_cuda import F32, quant, rng
from lightx2v_cuda.dit import LightDitCuda, MemRopeConfig, WanConfig, synthetic_block

pytestmark = pytest.mark.gpu


def rel_l2(got, want):
    got = np.asarray(got, np.float64).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    assert np.isfinite(got).all()
    return np.linalg.norm(got - want) / np.linalg.norm(want)


def test_chunk_steps_match_the_oracle(be, oracle):
    import dit_ref
    cfg = WanConfig(layers=2)
    mr = MemRopeConfig()
    d = cfg.dim
    ft, frames = 64, 3
    s = ft * frames
    q8 = lambda w, r, c: quant.Q8.quantize(w, r, c)
    host_blocks = [synthetic_block(cfg, 10 + l, q8) for l in range(cfg.layers)]
    deq_blocks = [{k: ((v[0].dequantize(), v[1]) if isinstance(v, tuple) else v) for k, v in b.items()}
                  for b in host_blocks]
    mat = lambda seed, r, c: (rng.normal(seed, r * c, 0.02), rng.normal(seed + 1, r, 0.01))
    patch, text1, text2 = mat(901, d, cfg.patch_in), mat(903, d, cfg.text_dim), mat(905, d, d)
    proj_out = mat(907, cfg.patch_out, d)
    model = LightDitCuda(be, cfg, host_blocks, patch, text1, text2, proj_out, mr)
    ref = dit_ref.DitRef(cfg, deq_blocks, patch, text1, text2, proj_out, mr)

    embeds = rng.normal(911, cfg.text_len * cfg.text_dim)
    prompt = model.prepare_prompt(embeds)
    prompt_ref = ref.prepare_prompt(embeds)
    # the prompt's K/V (text MLP, kv2, head_split with norm_k2) agree
    for (k, v), (rk, rv) in zip(prompt, prompt_ref):
        assert rel_l2(be.download(k), rk) <= 1e-2
        assert rel_l2(be.download(v), rv) <= 1e-2

    mods_h = [rng.normal(920 + l, 6 * d, 0.1) for l in range(cfg.layers)]
    mods = [be.upload(m, F32) for m in mods_h]
    head_h = rng.normal(930, 2 * d, 0.1)
    head = be.upload(head_h, F32)
    ang = rng.normal(931, s * cfg.head_dim // 2, 1.0)
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    ws = model.workspace(frames, ft, cos, sin)
    caches = ref.new_caches()
    out = be.alloc(s * cfg.patch_out, F32)
    for chunk in range(5):
        h0 = rng.normal(940 + chunk, s * d)
        be.write(ws.h, h0)
        model.forward_chunk(ws, mods, head, prompt, 3 * chunk, out)
        h_ref, out_ref = ref.forward_chunk(caches, h0, mods_h, head_h, prompt_ref, 3 * chunk, ft, (cos, sin))
        assert be.kv_cache_temporal(ws.caches[0]).tolist() == caches[0].temporal
        assert rel_l2(be.download(ws.h) - h0, h_ref.reshape(-1) - h0) <= 1e-2, chunk
        assert rel_l2(be.download(out), out_ref) <= 1e-2, chunk
