"""GPU: the prefill state builder (skv_prefill_build) against the torch restatement
of ShadowKVCache_CPU.prefill_kv_cache (models/kvcache/shadow.py:463-544)."""
import copy
import math
import types

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import shadowkv_oracle as o

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy()


def _inputs(cfg, seed):
    from shadowkv_b200 import workload
    g = torch.Generator(device=DEV).manual_seed(seed)
    T, Hk, Hq, D = cfg.ctx, cfg.kv_heads, cfg.q_heads, 128
    U0 = torch.randn(T, cfg.r_true, generator=g, device=DEV)
    W0 = torch.randn(cfg.r_true, Hk * D, generator=g, device=DEV) / math.sqrt(math.sqrt(cfg.r_true))
    k_pre = (U0 @ W0).add_(torch.randn(T, Hk * D, generator=g, device=DEV), alpha=0.05)
    k_pre = k_pre.to(torch.bfloat16).view(1, T, Hk, D).transpose(1, 2).contiguous()
    v = torch.randn(1, Hk, T, D, generator=g, device=DEV).to(torch.bfloat16)
    q_last = torch.randn(1, Hq, 1, D, generator=g, device=DEV).to(torch.bfloat16)
    cs = workload.llama_cos_sin(T + 64, device=DEV)[:T].float()
    cos = torch.cat((cs[:, :64], cs[:, :64]), -1)
    sin = torch.cat((cs[:, 64:], cs[:, 64:]), -1)
    kf = k_pre.float()
    k_roped = (kf * cos + torch.cat((-kf[..., 64:], kf[..., :64]), -1) * sin).to(torch.bfloat16)
    return k_roped, v, q_last


def _cache(cfg):
    from shadowkv_b200.kvcache import ShadowKVCache_CPU
    conf = types.SimpleNamespace(num_attention_heads=cfg.q_heads, num_key_value_heads=cfg.kv_heads,
                                 hidden_size=cfg.q_heads * 128, num_hidden_layers=1)
    return ShadowKVCache_CPU(conf, batch_size=1, max_length=cfg.ctx, device=DEV, sparse_budget=cfg.budget,
                             rank=cfg.rank, local_chunk=cfg.local_chunk, outlier_chunk=cfg.outliers,
                             gen_len=cfg.gen_len, geometry=cfg.geometry)


@pytest.mark.parametrize("name,geometry,seed", [("tiny", "torch", 1), ("tiny", "cpu", 2), ("config0", "torch", 3)])
def test_prefill_builder_matches_torch_path(name, geometry, seed):
    from shadowkv_b200 import workload
    cfg = copy.deepcopy(workload.CONFIGS[name])
    cfg.geometry = geometry
    from shadowkv_b200._lib import device_errors
    device_errors()  # clear
    k_roped, v, q_last = _inputs(cfg, seed)
    ct, cn = _cache(cfg), _cache(cfg)
    ct.prefill_kv_cache(v, 0, k_roped, q_last)
    ws = cn.prefill_kv_cache_native(v, 0, k_roped, q_last)
    torch.cuda.synchronize()
    del ws
    assert (cn.chunks, cn.prefill_local, cn.sparse_start, cn.sparse_end) == \
        (ct.chunks, ct.prefill_local, ct.sparse_start, ct.sparse_end)
    c, nout, ps, ss, K = cn.chunks, cn.outlier_chunk, cn.prefill_local, cn.sparse_start, cn.select_sets
    H = cfg.kv_heads
    # host value store: every whole chunk of the prompt
    assert np.array_equal(bits(cn.v_cache_cpu[0]), bits(ct.v_cache_cpu[0]))
    # reference intermediates (the torch ops of shadow.py:484-488)
    ctx = k_roped[:, :, :c * 8].view(1, H, c, 8, 128)
    cand = ctx.mean(dim=-2)
    minsim = F.cosine_similarity(cand.unsqueeze(3).expand(-1, -1, -1, 8, -1), ctx, dim=-1).min(dim=-1).values
    ms = minsim.float().cpu().numpy()[0]
    lm_idx = cn.k_landmark_idx[0, 0].cpu().numpy()
    kb, vb = bits(cn.k_cache_buffer[0, 0]), bits(cn.v_cache_buffer[0, 0])
    kr, vr = bits(k_roped[0]), bits(v[0])
    for h in range(H):
        outl = np.setdiff1d(np.arange(c), lm_idx[h])
        assert len(outl) == nout
        # a valid set of the nout smallest similarities (ties at the boundary either way)
        assert ms[h, outl].max() <= np.delete(ms[h], outl).min()
        # landmarks: the means of the other chunks, in chunk order
        assert np.array_equal(lm_idx[h], np.delete(np.arange(c), outl))
        assert np.array_equal(bits(cn.k_landmark[0, 0, h]), bits(cand[0, h])[lm_idx[h]])
        # outlier rows in (similarity, chunk id) order
        order = outl[np.lexsort((outl, ms[h, outl]))]
        rows = (order[:, None] * 8 + np.arange(8)).reshape(-1)
        assert np.array_equal(kb[h, ps:ss], kr[h, rows]) and np.array_equal(vb[h, ps:ss], vr[h, rows])
        # local window
        assert np.array_equal(kb[h, :ps], kr[h, cfg.ctx - ps:]) and np.array_equal(vb[h, :ps], vr[h, cfg.ctx - ps:])
    # first selection: a top-K of the reference's (bf16-rounded) chunk scores, up to near-ties
    G = cfg.q_heads // H
    lm = cn.k_landmark[0, 0]
    att = torch.einsum("bhgd,bhcd->bhgc", q_last.view(1, H, G, 128), lm.unsqueeze(0)) / math.sqrt(128)
    sc = F.softmax(att, dim=-1, dtype=torch.float32).to(torch.bfloat16).max(dim=-2).values.float().cpu().numpy()[0]
    slots = cn.slots[0, 0].cpu().numpy()
    assert np.array_equal(cn.position_ids[0, 0].cpu().numpy(), slots.astype(np.int64))
    for h in range(H):
        assert np.array_equal(np.sort(slots[h]), slots[h])  # ascending chunk id per slot
        pos = np.searchsorted(lm_idx[h], slots[h])
        assert np.array_equal(lm_idx[h][pos], slots[h])
        assert o.topk_tie_ok(sc[h][None], pos[None], K, rtol=1e-2)
        rows = (slots[h][:, None] * 8 + np.arange(8)).reshape(-1)
        assert np.array_equal(kb[h, ss:ss + 8 * K], kr[h, rows]) and np.array_equal(vb[h, ss:ss + 8 * K], vr[h, rows])
    # with the same outlier set, the whole landmark state equals the torch path's
    if np.array_equal(cn.k_landmark_idx[0].cpu().numpy(), ct.k_landmark_idx[0].cpu().numpy()):
        assert np.array_equal(bits(cn.k_landmark[0]), bits(ct.k_landmark[0]))
    assert device_errors()[0] == 0
