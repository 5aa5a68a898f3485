"""GPU: the reference-facing classes end to end (ShadowAttention.decode / decode_fused) vs the oracle."""
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


@pytest.fixture(scope="module")
def tiny_layer():
    from shadowkv_b200 import workload
    cfg = copy.deepcopy(workload.CONFIGS["tiny"])
    return workload.Layer(cfg, device=DEV, seed=7)


@pytest.mark.parametrize("rope_mode", [0, 1])
def test_append_kernel(rope_mode):
    from shadowkv_b200 import decode as fz
    rng = np.random.default_rng(rope_mode)
    B, Hq, Hk, buf_len, row = 3, 8, 2, 100, 77
    width = 128 if rope_mode == 0 else 64
    cs = o.round_bf16(rng.uniform(-1, 1, (500, width)).astype(np.float32))
    q = o.round_bf16(rng.standard_normal((B, Hq, 128)).astype(np.float32))
    k = o.round_bf16(rng.standard_normal((B, Hk, 128)).astype(np.float32))
    v = o.round_bf16(rng.standard_normal((B, Hk, 128)).astype(np.float32))
    pos = np.array([3, 499, 250], np.int64)
    dev = lambda x: torch.from_numpy(o.f32_to_bf16_bits(x).view(np.int16)).view(torch.bfloat16).to(DEV)
    g = fz.Geometry(batch=B, kv_heads=Hk, q_heads=Hq, rank=64, select_sets=1, num_landmarks=1, num_chunks=1,
                    ctx_len=8, buf_len=buf_len, sparse_start=0, rope_mode=rope_mode, cos_sin_stride=width,
                    cos_sin_rows=500)
    kb = torch.zeros(B, Hk, buf_len, 128, dtype=torch.bfloat16, device=DEV)
    vb = torch.zeros_like(kb)
    qo = torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=DEV)
    fz.append(g, dev(q), dev(k), dev(v), torch.from_numpy(pos).to(DEV), dev(cs), qo, kb, vb, row)
    c = cs[pos][:, None, :]
    if rope_mode == 0:
        eq = o.rope_rotate_half_bf16(q, c[..., :64], c[..., 64:])
        ek = o.rope_rotate_half_bf16(k, c[..., :64], c[..., 64:])
    else:
        eq, ek = o.rope_glm_bf16(q, c), o.rope_glm_bf16(k, c)
    assert np.array_equal(bits(qo), o.f32_to_bf16_bits(eq))
    assert np.array_equal(bits(kb[:, :, row]), o.f32_to_bf16_bits(ek))
    assert np.array_equal(bits(vb[:, :, row]), o.f32_to_bf16_bits(v))
    assert (f32(kb[:, :, :row]) == 0).all() and (f32(vb[:, :, row + 1:]) == 0).all()


def _check_buffers(layer, ids_per_slot, fused):
    """V rows of every slot equal the host chunk; K rows equal the oracle reconstruction."""
    c = layer.cache
    ss = c.sparse_start
    v_host = bits(c.v_cache_cpu[0])  # [B, H, chunks, 1024]
    vb = bits(c.v_cache_buffer[0])
    kb = f32(c.k_cache_buffer[0])
    U = f32(c.U[0])
    SVt = f32(c.SV[0])
    cs = f32(layer.cos_sin)
    B, H, K = ids_per_slot.shape
    for b in range(B):
        for h in range(H):
            ids = ids_per_slot[b, h]
            got_v = vb[b, h, ss:ss + 8 * K].reshape(K, 1024)
            assert np.array_equal(got_v, v_host[b, h, ids]), "V slots"
            if fused:
                ek = o.reconstruct_keys_rope(U[b], SVt[b, h], ids, cs)
            else:
                x = o.batch_gather_gemm(U[b:b + 1], SVt[b:b + 1, h:h + 1], ids[None, None], np.zeros(1, np.int32))[0, 0]
                pos = (ids[:, None] * 8 + np.arange(8)).reshape(-1)
                ek = o.rope_rotate_half_bf16(x, cs[pos][:, :64], cs[pos][:, 64:])
            np.testing.assert_allclose(kb[b, h, ss:ss + 8 * K], ek, atol=2e-2, rtol=1e-2)


def _scores_ok(layer, q_roped, ids_per_slot, rtol):
    c = layer.cache
    lm = f32(c.k_landmark[0])
    lidx = c.k_landmark_idx[0].cpu().numpy()
    B, H, L, D = lm.shape
    G = c.num_key_value_groups
    sc = o.landmark_scores(q_roped.reshape(B, H, G, D), lm)
    for b in range(B):
        for h in range(H):
            order = np.argsort(lidx[b, h])
            pos = order[np.searchsorted(lidx[b, h][order], np.sort(ids_per_slot[b, h]))]
            assert o.topk_tie_ok(sc[b, h][None], pos[None], c.select_sets, rtol=rtol)


@pytest.mark.parametrize("path", ["fused", "fused_split", "reference"])
def test_decode_steps_against_oracle(tiny_layer, path):
    from shadowkv_b200._lib import device_errors
    layer = tiny_layer
    c, attn = layer.cache, layer.attn
    # start from an empty reuse cache: every chunk of the first step is a miss, so every key
    # in the selected region is a reconstruction (prefill wrote the exact keys of its selection)
    c.position_ids[0].fill_(-1)
    c.slots[0].fill_(-1)
    hits = []
    for step in range(4):
        q, k, v = layer.next_inputs()
        pos = torch.full((c.batch_size, 1), layer.cfg.ctx + step, dtype=torch.int64, device=DEV)
        c.gen_offset = 0
        if path in ("fused", "fused_split"):
            out = (attn.decode_fused if path == "fused" else attn.decode_fused_split)(q, k, v, pos, 0)
            ids = c.slots[0].cpu().numpy()
            hits.append(c.hit_rate())
        else:
            out = attn.decode(q, k, v, pos, 0)
            ids = c.position_ids[0].cpu().numpy()
        torch.cuda.synchronize()
        assert device_errors()[0] == 0
        # selection: fp32 scores (fused) or the bf16 softmax of the CUTLASS path (reference)
        qr = attn.apply_rotary_pos_emb(q, k, pos)[0]
        _scores_ok(layer, f32(qr)[:, :, 0, :], ids, rtol=5e-2 if path == "reference" else 1e-5)
        _check_buffers(layer, ids, fused=(path != "reference"))
        seq_len = c.sparse_end + 1
        ref = o.decode_attention(f32(qr)[:, :, 0, :], f32(c.k_cache_buffer[0]), f32(c.v_cache_buffer[0]), seq_len)
        np.testing.assert_allclose(f32(out)[:, 0], ref, atol=2e-2, rtol=1e-2)
    if path != "reference":
        assert all(0.0 <= h <= 1.0 for h in hits)


def test_repeated_query_is_all_hits_on_both_paths(tiny_layer):
    """The same query twice: the second step serves every chunk from the reuse cache."""
    layer = tiny_layer
    c, attn = layer.cache, layer.attn
    q, k, v = layer.next_inputs()
    pos = torch.full((c.batch_size, 1), layer.cfg.ctx + 9, dtype=torch.int64, device=DEV)
    full = c.batch_size * c.num_key_value_heads * c.select_sets
    c.gen_offset = 0
    out_ref = attn.decode(q, k, v, pos, 0)
    c.gen_offset = 0
    out_ref2 = attn.decode(q, k, v, pos, 0)
    assert int(c.cnts.sum().item()) == full
    torch.testing.assert_close(out_ref2, out_ref, atol=0, rtol=0)
    ref_sets = np.sort(c.position_ids[0].cpu().numpy(), -1)
    c.sync_slots_from_position_ids(0)
    c.gen_offset = 0
    out_f = attn.decode_fused(q, k, v, pos, 0)
    c.gen_offset = 0
    out_f2 = attn.decode_fused(q, k, v, pos, 0)
    assert c.hit_rate() == 1.0
    torch.testing.assert_close(out_f2, out_f, atol=0, rtol=0)
    # fp32 (fused) and bf16-rounded (reference) scores select nearly the same chunks
    f_sets = np.sort(c.slots[0].cpu().numpy(), -1)
    for b in range(f_sets.shape[0]):
        for h in range(f_sets.shape[1]):
            assert len(set(f_sets[b, h]) & set(ref_sets[b, h])) >= 0.85 * f_sets.shape[2]
    torch.testing.assert_close(out_f.float(), out_ref.float(), atol=5e-2, rtol=5e-2)


def test_append_select_equals_append_then_select(tiny_layer):
    """The fused scoring pass (RoPE + append inside) gives the same q, K/V rows and slots as the two calls."""
    from shadowkv_b200 import decode as fz
    layer = tiny_layer
    c, attn = layer.cache, layer.attn
    g = c.fused_geometry(layer.cos_sin)
    q, k, v = layer.next_inputs()
    pos = torch.full((c.batch_size,), layer.cfg.ctx + 3, dtype=torch.int64, device=DEV)
    row = c.sparse_end + 5
    slots0 = c.slots[0].clone()
    kb0, vb0 = c.k_cache_buffer[0].clone(), c.v_cache_buffer[0].clone()
    B, Hq, Hk = c.batch_size, c.num_attention_heads, c.num_key_value_heads
    q1 = torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=DEV)
    fz.append(g, q.reshape(B, Hq, 128).contiguous(), k.reshape(B, Hk, 128).contiguous(),
              v.reshape(B, Hk, 128).contiguous(), pos, layer.cos_sin, q1, c.k_cache_buffer[0],
              c.v_cache_buffer[0], row)
    fz.select(g, c._fused_ws, q1, c.k_landmark[0], c.k_landmark_idx[0], c.slots[0])
    s1 = c.slots[0].clone()
    ms1, mc1, n1 = c._fused_ws.miss_slot.clone(), c._fused_ws.miss_chunk.clone(), c._fused_ws.miss_count.clone()
    kb1, vb1 = c.k_cache_buffer[0].clone(), c.v_cache_buffer[0].clone()
    c.slots[0].copy_(slots0)
    c.k_cache_buffer[0].copy_(kb0)
    c.v_cache_buffer[0].copy_(vb0)
    q2 = torch.empty_like(q1)
    fz.append_select(g, c._fused_ws, q.reshape(B, Hq, 128).contiguous(), k.reshape(B, Hk, 128).contiguous(),
                     v.reshape(B, Hk, 128).contiguous(), pos, layer.cos_sin, q2, c.k_cache_buffer[0],
                     c.v_cache_buffer[0], row, c.k_landmark[0], c.k_landmark_idx[0], c.slots[0])
    torch.cuda.synchronize()
    assert torch.equal(q1, q2)
    assert torch.equal(c.slots[0], s1)
    assert torch.equal(c._fused_ws.miss_count, n1)
    for b in range(B * Hk):
        n = int(n1[b])
        assert torch.equal(c._fused_ws.miss_slot[b, :n], ms1[b, :n])
        assert torch.equal(c._fused_ws.miss_chunk[b, :n], mc1[b, :n])
    assert torch.equal(c.k_cache_buffer[0], kb1) and torch.equal(c.v_cache_buffer[0], vb1)


def _chained_steps(layer, n_steps, mode):
    """n_steps decode steps of all the layer's layers, layer l + 1 taking layer l's
    output as its query.  mode "sync": host synchronisation after every layer (no
    overlap between launches); "stream": one stream, kernels chained by
    programmatic dependent launch; "graph": the stream version captured once and
    replayed.  Returns the per-step outputs and the final slot tables."""
    c, attn = layer.cache, layer.attn
    cfg = layer.cfg
    B, Hq, NL = cfg.batch, cfg.q_heads, cfg.layers
    torch.manual_seed(5)
    ins = [layer.next_inputs() for _ in range(n_steps)]
    s_q, s_k, s_v = (torch.empty_like(t) for t in ins[0])
    s_pos = torch.empty(B, 1, dtype=torch.int64, device=DEV)
    s_qr = torch.empty(B, Hq, 1, 128, dtype=torch.bfloat16, device=DEV)
    mids = [torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=DEV) for _ in range(NL)]
    c.fused_geometry(attn.cos_sin_cache)

    def body(sync):
        c.gen_offset = 0
        for li in range(NL):
            q_in = s_q if li == 0 else mids[li - 1]
            qr = c.append_select_fused(li, q_in, s_k, s_v, s_pos, attn.cos_sin_cache, q_out=s_qr)
            c.sparse_attention_fused(li, qr, c.sparse_end + c._gen_offset(li), attn.cos_sin_cache, out=mids[li])
            if sync:
                torch.cuda.synchronize()
        c.gen_offset = 0

    graph = None
    outs = []
    for i in range(n_steps):
        s_q.copy_(ins[i][0]), s_k.copy_(ins[i][1]), s_v.copy_(ins[i][2])
        s_pos.fill_(c.sparse_end + 1000 + i)
        if mode == "graph":
            if graph is None:
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    body(False)
                # capture does not run the step: run the captured step for step 0
            graph.replay()
        else:
            body(mode == "sync")
        torch.cuda.synchronize()
        outs.append([bits(m) for m in mids])
    return outs, [c.slots[li].cpu().numpy().copy() for li in range(NL)]


def test_chained_layers_overlap_matches_synchronized():
    """Three layers chained in one stream (the next layer's scoring may become
    resident while the previous layer's attention drains) and the same steps as
    a CUDA graph give bit-identical outputs and slot tables to the steps run
    with a host synchronisation after every layer."""
    from shadowkv_b200 import workload
    cfg = copy.deepcopy(workload.CONFIGS["tiny"])
    cfg.layers = 3
    res = {}
    for mode in ("sync", "stream", "graph"):
        layer = workload.Layer(cfg, device=DEV, seed=11)
        res[mode] = _chained_steps(layer, 4, mode)
        del layer
    for mode in ("stream", "graph"):
        for a, b in zip(res["sync"][0], res[mode][0]):
            for x, y in zip(a, b):
                assert np.array_equal(x, y), mode
        for x, y in zip(res["sync"][1], res[mode][1]):
            assert np.array_equal(x, y), mode


def test_sparse_attention_output_into_pinned_host_memory():
    """The fused step with a page-locked CPU output (written over the host
    link by the kernel) gives the same bits as with a device output."""
    from shadowkv_b200 import workload
    cfg = copy.deepcopy(workload.CONFIGS["tiny"])
    outs = []
    for where in ("device", "host"):
        layer = workload.Layer(cfg, device=DEV, seed=13)
        c, attn = layer.cache, layer.attn
        torch.manual_seed(3)
        q, k, v = layer.next_inputs()
        pos = torch.full((cfg.batch, 1), c.sparse_end + 500, dtype=torch.int64, device=DEV)
        out = (torch.empty(cfg.batch, cfg.q_heads, 128, dtype=torch.bfloat16, device=DEV) if where == "device"
               else torch.empty(cfg.batch, cfg.q_heads, 128, dtype=torch.bfloat16).pin_memory())
        c.fused_geometry(attn.cos_sin_cache)
        qr = c.append_select_fused(0, q, k, v, pos, attn.cos_sin_cache)
        c.sparse_attention_fused(0, qr, c.sparse_end + c._gen_offset(0), attn.cos_sin_cache, out=out)
        torch.cuda.synchronize()
        outs.append(bits(out))
        del layer
    assert np.array_equal(outs[0], outs[1])
    with pytest.raises(RuntimeError):
        from shadowkv_b200 import decode as fz
        fz._req_out(torch.empty(4, dtype=torch.bfloat16))  # pageable host memory is refused


def _tiny_batch_layer(seed, batch=4):
    from shadowkv_b200 import workload
    cfg = copy.deepcopy(workload.CONFIGS["tiny"])
    cfg.batch = batch
    return workload.Layer(cfg, device=DEV, seed=seed)


def test_sparse_attention_on_fewer_ctas_matches_full_grid():
    """The fused attention with its grid capped (CTAs walking the work items in
    strides) gives the same bits as one CTA per item."""
    outs = []
    for ctas in (0, 3):
        layer = _tiny_batch_layer(17)
        c, attn = layer.cache, layer.attn
        torch.manual_seed(4)
        q, k, v = layer.next_inputs()
        pos = torch.full((4, 1), c.sparse_end + 300, dtype=torch.int64, device=DEV)
        g = c.fused_geometry(attn.cos_sin_cache)
        qr = c.append_select_fused(0, q, k, v, pos, attn.cos_sin_cache)
        from shadowkv_b200 import decode as fz
        out = torch.empty(4, g.q_heads, 128, dtype=torch.bfloat16, device=DEV)
        fz.sparse_attention(g, c._fused_ws, qr.reshape(4, g.q_heads, 128), c.U[0], c.SV[0], attn.cos_sin_cache,
                            c.v_cache_cpu[0], c.k_cache_buffer[0], c.v_cache_buffer[0], c.sparse_end + 1, out,
                            max_ctas=ctas)
        torch.cuda.synchronize()
        outs.append((bits(out), bits(c.k_cache_buffer[0]), bits(c.v_cache_buffer[0])))
        del layer
    for x, y in zip(*outs):
        assert np.array_equal(x, y)


def test_microbatched_step_matches_whole_batch():
    """The step in batch slices (selection of slice i on a high-priority stream
    beside slice i-1's capped fetch) equals the whole-batch step."""
    res = []
    for parts in (1, 2):
        layer = _tiny_batch_layer(23)
        c, attn = layer.cache, layer.attn
        torch.manual_seed(6)
        q, k, v = layer.next_inputs()
        pos = torch.full((4, 1), c.sparse_end + 200, dtype=torch.int64, device=DEV)
        out = torch.empty(4, c.num_attention_heads, 128, dtype=torch.bfloat16, device=DEV)
        c.fused_geometry(attn.cos_sin_cache)
        if parts == 1:
            qr = c.append_select_fused(0, q, k, v, pos, attn.cos_sin_cache)
            c.sparse_attention_fused(0, qr, c.sparse_end + c._gen_offset(0), attn.cos_sin_cache, out=out)
        else:
            c.decode_step_microbatched(0, q, k, v, pos, attn.cos_sin_cache, out, parts, max_ctas=5)
        torch.cuda.synchronize()
        res.append((bits(out), c.slots[0].cpu().numpy().copy()))
        del layer
    assert np.array_equal(res[0][1], res[1][1])
    assert np.array_equal(res[0][0], res[1][0])


def test_decode_fused_picks_microbatching_at_large_batch():
    """ShadowAttention.decode_fused at 8 sequences runs the step in 4 slices and
    returns the same bits as the single-slice step."""
    res = []
    for mb in (1, None):
        layer = _tiny_batch_layer(29, batch=8)
        torch.manual_seed(8)
        q, k, v = layer.next_inputs()
        pos = torch.full((8, 1), layer.cache.sparse_end + 100, dtype=torch.int64, device=DEV)
        out = layer.attn.decode_fused(q, k, v, pos, 0, microbatch=mb)
        torch.cuda.synchronize()
        res.append((bits(out), layer.cache.slots[0].cpu().numpy().copy(), getattr(layer.cache, "_mb_state", None)))
        del layer
    assert res[0][2] is None and res[1][2] is not None and res[1][2][0] == (4, 2)
    assert np.array_equal(res[0][1], res[1][1])
    assert np.array_equal(res[0][0], res[1][0])
