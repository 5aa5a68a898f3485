"""GPU: one layer at the benchmark's full sizes, through ShadowAttention.decode_fused, vs the oracle.

config1 is the Llama-3-8B shape at 122,880 tokens of context (the headline
workload: 15,308 landmarks per head, 8-CTA selection clusters); config3 is the
GLM shape at 1,048,576 tokens (131,020 landmarks per head: the keys kernel and
16-CTA clusters, partial interleaved RoPE, correlated queries so that later
steps hit the reuse cache).  Every step is checked on the state the kernels
left: the selected chunk set of every head is a top-k of the fp32 oracle
scores (models/kvcache/shadow.py:547-576), the slot table follows the
slot-stable update, every V slot is bit-identical to its chunk in the host
store, every key in the selected region is the oracle reconstruction with
RoPE at the original positions (bf16 tolerance), and the attention output is
the oracle attention over the buffers (atol 2e-2 / rtol 1e-2).
"""
import copy

import numpy as np
import pytest
import torch

from oracle import shadowkv_oracle as o

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def f32(t):
    return t.float().cpu().numpy()


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _roped_query(q, pos, cs, glm):
    """The new token's post-RoPE query as the scoring pass computes it (bf16 op by op)."""
    qn = f32(q)[:, :, 0, :]
    c = cs[pos][:, None, :]
    if glm:
        return o.rope_glm_bf16(qn, c)
    return o.rope_rotate_half_bf16(qn, c[..., :64], c[..., 64:128])


@pytest.mark.parametrize("name", ["config1", "config3"])
def test_full_size_decode_steps_against_oracle(name):
    from shadowkv_b200 import workload
    from shadowkv_b200._lib import device_errors
    cfg = copy.deepcopy(workload.CONFIGS[name])
    layer = workload.Layer(cfg, device=DEV, seed=11)
    c, attn = layer.cache, layer.attn
    glm = cfg.rope == "glm"
    cs = f32(layer.cos_sin)
    lm = f32(c.k_landmark[0])
    lidx = c.k_landmark_idx[0].cpu().numpy()
    B, H, L, D = lm.shape
    G, K, ss = c.num_key_value_groups, c.select_sets, c.sparse_start
    # start from an empty reuse cache: the first step misses every chunk
    c.slots[0].fill_(-1)
    prev = c.slots[0].cpu().numpy()
    hits = []
    for step in range(3):
        q, k, v = layer.next_inputs()
        p = cfg.ctx + step
        pos = torch.full((B, 1), p, dtype=torch.int64, device=DEV)
        c.gen_offset = 0
        out = attn.decode_fused(q, k, v, pos, 0)
        torch.cuda.synchronize()
        assert device_errors()[0] == 0
        hits.append(c.hit_rate())
        new = c.slots[0].cpu().numpy()
        assert (new >= 0).all()
        # selection: a top-k of the fp32 scores, slot-stable against the previous table
        qr = _roped_query(q, np.full(B, p), cs, glm)
        sc = o.landmark_scores(qr.reshape(B, H, G, D), lm)
        for b in range(B):
            for h in range(H):
                order = np.argsort(lidx[b, h])
                at = order[np.searchsorted(lidx[b, h][order], np.sort(new[b, h]))]
                assert np.array_equal(lidx[b, h][at], np.sort(new[b, h]))
                assert o.topk_tie_ok(sc[b, h][None], at[None], K, rtol=1e-5)
        eslots, _, _ = o.stable_slot_update(prev, np.sort(new, -1))
        assert np.array_equal(new, eslots)
        prev = new
        # buffers: V slots bit-exact, keys = reconstruction + RoPE at the original positions
        vb = bits(c.v_cache_buffer[0])
        kb = f32(c.k_cache_buffer[0])
        for b in range(B):
            for h in range(H):
                ids = new[b, h].astype(np.int64)
                want_v = bits(c.v_cache_cpu[0][b, h].index_select(0, torch.from_numpy(ids)))
                assert np.array_equal(vb[b, h, ss:ss + 8 * K].reshape(K, 1024), want_v), "V slots"
                rows = (ids[:, None] * 8 + np.arange(8)).reshape(-1)
                Ur = f32(c.U[0][b].index_select(0, torch.from_numpy(rows).to(DEV)))
                ek = o.reconstruct_keys_rope(Ur, f32(c.SV[0][b, h]), np.arange(K), cs[rows], glm=glm)
                np.testing.assert_allclose(kb[b, h, ss:ss + 8 * K], ek, atol=2e-2, rtol=1e-2)
        # attention over the buffers: local rows, outliers, the selection and the new token
        ref = o.decode_attention(qr, kb, f32(c.v_cache_buffer[0]), c.sparse_end + 1)
        np.testing.assert_allclose(f32(out)[:, 0], ref, atol=2e-2, rtol=1e-2)
    assert hits[0] == 0.0
    if cfg.rho > 0:
        assert max(hits[1:]) > 0.0  # correlated queries reuse chunks of the previous step


def test_full_size_reference_path_config1():
    """config1 at full size through ShadowAttention.decode -- the reference's decode sequence
    (models/attention/shadow.py:22-48, models/kvcache/shadow.py:547-597, models/tensor_op.py:
    159-243) on the twelve drop-in bindings: batch_gemm_softmax + torch.topk,
    reorder_keys_and_compute_offsets, gather_copy_with_offsets, gather_copy_d2d_with_offsets,
    batch_gather_gemm and apply_rotary_pos_emb_push_cache_opt, with 15,308 landmarks per head and
    map size 256.  Checked on the state the bindings leave:

    * the new position_ids are the oracle's reorder of (previous ids, selected set) -- hits in
      old-slot order, then misses by chunk id -- bit for bit, and the cnts match;
    * the selected set is a top-k of the reference's bf16-rounded scores (ties allowed);
    * every V slot is bit-identical to its host chunk;
    * missed chunks: the gathered GEMM output (the cache's ``output`` buffer) is within one bf16
      ulp of the oracle's (fp32 accumulation order), and the keys pushed into the buffer are the
      bf16 RoPE of that output bit for bit; hit chunks keep the rows they had, bit for bit
      (the bf16 op-by-op RoPE cancels on near-zero keys, so a one-ulp GEMM difference is not
      compared through it);
    * the attention output is the oracle attention over the buffers (atol 2e-2 / rtol 1e-2).
    """
    from shadowkv_b200 import workload
    from shadowkv_b200._lib import device_errors
    cfg = copy.deepcopy(workload.CONFIGS["config1"])
    layer = workload.Layer(cfg, device=DEV, seed=13)
    c, attn = layer.cache, layer.attn
    cs = f32(layer.cos_sin)
    lm = f32(c.k_landmark[0])
    lidx = c.k_landmark_idx[0].cpu().numpy()
    B, H, L, D = lm.shape
    G, K, ss = c.num_key_value_groups, c.select_sets, c.sparse_start
    assert K == 256 and L == 15308
    U = f32(c.U[0])
    # start from an empty reuse cache (prefill's own selection holds exact keys, not
    # reconstructions): every key of the selected region is then a reconstruction
    c.position_ids[0].fill_(-1)
    prev = c.position_ids[0].cpu().numpy()
    prev_kb = bits(c.k_cache_buffer[0])
    for step in range(2):
        q, k, v = layer.next_inputs()
        p = cfg.ctx + step
        pos = torch.full((B, 1), p, dtype=torch.int64, device=DEV)
        c.gen_offset = 0
        out = attn.decode(q, k, v, pos, 0)
        torch.cuda.synchronize()
        assert device_errors()[0] == 0
        new = c.position_ids[0].cpu().numpy()
        # reorder: the oracle's order and counts, given the selected set
        want, _, want_cnts = o.reorder_keys_and_compute_offsets(prev, np.sort(new, -1))
        assert np.array_equal(new.reshape(-1, K), want), "reordered position_ids"
        assert np.array_equal(c.cnts.cpu().numpy(), want_cnts), "cnts (hits per head)"
        prev_ids = prev
        prev = new
        # selection: a top-k of the bf16-rounded scores of the CUTLASS-path restatement
        qr = _roped_query(q, np.full(B, p), cs, False)
        sc = o.landmark_scores(qr.reshape(B, H, G, D), lm)
        for b in range(B):
            for h in range(H):
                order = np.argsort(lidx[b, h])
                at = order[np.searchsorted(lidx[b, h][order], np.sort(new[b, h]))]
                assert np.array_equal(lidx[b, h][at], np.sort(new[b, h]))
                assert o.topk_tie_ok(sc[b, h][None], at[None], K, rtol=5e-2)
        vb = bits(c.v_cache_buffer[0])
        kbits = bits(c.k_cache_buffer[0])
        gemm = f32(c.output)
        cnts = c.cnts.cpu().numpy().reshape(B, H)
        for b in range(B):
            for h in range(H):
                ids = new[b, h].astype(np.int64)
                want_v = bits(c.v_cache_cpu[0][b, h].index_select(0, torch.from_numpy(ids)))
                assert np.array_equal(vb[b, h, ss:ss + 8 * K].reshape(K, 1024), want_v), "V slots"
                hit = int(cnts[b, h])
                miss_ids = ids[hit:]
                x = o.batch_gather_gemm(U[b:b + 1], f32(c.SV[0][b:b + 1, h:h + 1]),
                                        miss_ids[None, None].astype(np.int32), np.zeros(1, np.int32))[0, 0]
                got = gemm[b, h, 8 * hit:8 * K]
                # one bf16 ulp, plus the fp32 accumulation-order error of near-cancelling sums
                np.testing.assert_allclose(got, x, rtol=2.0 ** -7, atol=1e-5)
                rows = (miss_ids[:, None] * 8 + np.arange(8)).reshape(-1)
                ek = o.rope_rotate_half_bf16(got, cs[rows][:, :64], cs[rows][:, 64:128])
                assert np.array_equal(kbits[b, h, ss + 8 * hit:ss + 8 * K], o.f32_to_bf16_bits(ek)), "pushed keys"
                old_ids = list(prev_ids[b, h])
                for j in range(hit):
                    sl = old_ids.index(ids[j])
                    assert np.array_equal(kbits[b, h, ss + 8 * j:ss + 8 * j + 8],
                                          prev_kb[b, h, ss + 8 * sl:ss + 8 * sl + 8]), "hit keys kept"
        prev_kb = kbits
        ref = o.decode_attention(qr, f32(c.k_cache_buffer[0]), f32(c.v_cache_buffer[0]), c.sparse_end + 1)
        np.testing.assert_allclose(f32(out)[:, 0], ref, atol=2e-2, rtol=1e-2)
