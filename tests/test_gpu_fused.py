"""GPU parity of the fused decode path (select / gather / reconstruct / attention)."""
import math
import os

import numpy as np
import pytest
import torch

from oracle import shadowkv_oracle as o

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def bf(a):
    return o.bf16_bits_to_f32(np.asarray(a).view(np.uint16))


def to_bf16_dev(x):
    return torch.from_numpy(o.f32_to_bf16_bits(np.asarray(x, np.float32)).view(np.int16)).view(torch.bfloat16).to(DEV)


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def no_device_errors():
    from shadowkv_b200._lib import device_errors
    torch.cuda.synchronize()
    return device_errors()[0] == 0


def make_geom(**kw):
    from shadowkv_b200.decode import Geometry
    return Geometry(**kw)


# ------------------------------------------------------------------ full step vs the reference class

@pytest.fixture(scope="module")
def fix(golden_dir):
    return np.load(os.path.join(golden_dir, "torch_class_decode.npz"))


def test_fused_step_matches_reference_torch_class(fix):
    """Three decode steps of models/kvcache/shadow.py (run by make_golden.py) through the fused kernels.

    Chunk ids and gathered V: bit-exact (fp32 scores of bf16-exact inputs).
    Reconstructed K and attention output: atol 2e-2 / rtol 1e-2 (bf16).
    """
    from shadowkv_b200 import decode as fz
    d = fix
    Hq, Hkv, T, rank = int(d["Hq"]), int(d["Hkv"]), int(d["T"]), int(d["rank"])
    K = int(d["budget"]) // 8
    ss, se = int(d["sparse_start"]), int(d["sparse_end"])
    L = d["k_landmark"].shape[2]
    gen = 8
    buf_len = se + gen
    cs = bf(d["cos_sin_bf16"])
    g = make_geom(batch=1, kv_heads=Hkv, q_heads=Hq, rank=rank, select_sets=K, num_landmarks=L,
                  num_chunks=T // 8, ctx_len=T, buf_len=buf_len, sparse_start=ss, cos_sin_rows=cs.shape[0])
    ws = fz.DecodeWorkspace(g, DEV)
    lm = torch.from_numpy(d["k_landmark"]).view(torch.bfloat16).to(DEV).contiguous()
    lidx = torch.from_numpy(d["k_landmark_idx"]).to(DEV)
    U = torch.from_numpy(d["U"]).view(torch.bfloat16).to(DEV)
    SVt = torch.from_numpy(d["SV"]).view(torch.bfloat16).to(DEV).transpose(-1, -2).contiguous()
    cos_sin = torch.from_numpy(d["cos_sin_bf16"]).view(torch.bfloat16).to(DEV)
    v_full = bf(d["v_bf16"])  # [1, H, T, 128]
    v_host = torch.from_numpy(d["v_bf16"]).view(torch.bfloat16).reshape(1, Hkv, T // 8, 1024).contiguous().pin_memory()
    kbuf = torch.zeros(1, Hkv, buf_len, 128, dtype=torch.bfloat16, device=DEV)
    vbuf = torch.zeros_like(kbuf)
    kbuf[:, :, :ss] = torch.from_numpy(d["k_prefix"]).to(DEV).to(torch.bfloat16)
    vbuf[:, :, :ss] = torch.from_numpy(d["v_prefix"]).view(torch.bfloat16).to(DEV)
    slots = torch.full((1, Hkv, K), -1, dtype=torch.int32, device=DEV)
    out = torch.empty(1, Hq, 128, dtype=torch.bfloat16, device=DEV)
    for step in range(d["q"].shape[0]):
        kbuf[:, :, se + step] = torch.from_numpy(d["k_new"][step][:, :, 0]).to(DEV).to(torch.bfloat16)
        vbuf[:, :, se + step] = torch.from_numpy(d["v_new"][step][:, :, 0]).to(DEV).to(torch.bfloat16)
        q = torch.from_numpy(d["q"][step][:, :, 0, :]).to(DEV).to(torch.bfloat16).contiguous()
        old = slots.cpu().numpy()
        fz.select(g, ws, q, lm, lidx, slots)
        fz.gather_values(g, ws, v_host, vbuf)
        fz.reconstruct_keys(g, ws, U, SVt, cos_sin, kbuf)
        seq_len = int(d["seq_len"][step])
        fz.attention(g, ws, q, kbuf, vbuf, seq_len, out)
        torch.cuda.synchronize()
        assert no_device_errors()
        sel = d["selected_chunk_idx"][step]  # [1, H, K] in the reference's topk order
        new_slots = slots.cpu().numpy()
        assert np.array_equal(np.sort(new_slots, -1), np.sort(sel, -1)), "selected chunk ids"
        eslots, emiss, ehits = o.stable_slot_update(old, np.sort(sel, -1))
        assert np.array_equal(new_slots, eslots), "slot-stable placement"
        kb = kbuf.float().cpu().numpy()
        vb = vbuf.float().cpu().numpy()
        kref = np.zeros((1, Hkv, K * 8, 128), np.float32)
        vref = np.zeros_like(kref)
        for h in range(Hkv):
            for s in range(K):
                cid = new_slots[0, h, s]
                j = int(np.where(sel[0, h] == cid)[0][0])
                kref[0, h, 8 * s: 8 * s + 8] = d["k_sparse"][step][0, h, 8 * j: 8 * j + 8]
                vref[0, h, 8 * s: 8 * s + 8] = v_full[0, h, 8 * cid: 8 * cid + 8]
        assert np.array_equal(vb[:, :, ss:se], vref), "gathered values"
        np.testing.assert_allclose(kb[:, :, ss:se], kref, atol=2e-2, rtol=1e-2)
        # attention vs the reference buffers (fp32) in the reference's slot order
        kfull = np.concatenate([d["k_prefix"], d["k_sparse"][step], d["k_gen"][0][:, :, : step + 1]], axis=2)
        vfull = np.concatenate([bf(d["v_prefix"]), bf(d["v_sparse"][step]),
                                d["v_new"][: step + 1, :, :, 0].transpose(1, 2, 0, 3)], axis=2)
        assert kfull.shape[2] == seq_len
        ref = o.decode_attention(d["q"][step][:, :, 0, :], kfull, vfull, seq_len)
        np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)


def test_config0_matches_reference_torch_class(golden_dir):
    """BASELINE configs[0] (T=8192, 8/2 heads, rank 64, budget 512, 8 outliers, fp32 in the
    reference) through the reference's ShadowKVCache (tests/golden/make_golden.py), three steps
    of the shipped kernels: scoring + selection, then value fetch + key reconstruction +
    attention in one launch.

    Chunk ids and gathered V: bit-exact.  Reconstructed keys and attention: atol 2e-2 / rtol 1e-2.
    """
    import hashlib
    from shadowkv_b200 import decode as fz
    from tests.test_oracle_golden import config0_inputs
    d = np.load(os.path.join(golden_dir, "torch_class_config0.npz"))
    v_np, cs_bits = config0_inputs(d)
    Hq, Hkv, T, rank = int(d["Hq"]), int(d["Hkv"]), int(d["T"]), int(d["rank"])
    K = int(d["budget"]) // 8
    ss, se = int(d["sparse_start"]), int(d["sparse_end"])
    L = d["k_landmark"].shape[2]
    buf_len = se + 8
    g = make_geom(batch=1, kv_heads=Hkv, q_heads=Hq, rank=rank, select_sets=K, num_landmarks=L,
                  num_chunks=T // 8, ctx_len=T, buf_len=buf_len, sparse_start=ss, cos_sin_rows=cs_bits.shape[0])
    ws = fz.DecodeWorkspace(g, DEV)
    lm = torch.from_numpy(d["k_landmark"]).view(torch.bfloat16).to(DEV).contiguous()
    lidx = torch.from_numpy(d["k_landmark_idx"]).to(DEV)
    U = torch.from_numpy(d["U"]).view(torch.bfloat16).to(DEV)
    SVt = torch.from_numpy(d["SV"]).view(torch.bfloat16).to(DEV).transpose(-1, -2).contiguous()
    cos_sin = torch.from_numpy(cs_bits).view(torch.bfloat16).to(DEV)
    v_host = torch.from_numpy(v_np).to(torch.bfloat16).reshape(1, Hkv, T // 8, 1024).contiguous().pin_memory()
    kbuf = torch.zeros(1, Hkv, buf_len, 128, dtype=torch.bfloat16, device=DEV)
    vbuf = torch.zeros_like(kbuf)
    kbuf[:, :, :ss] = torch.from_numpy(d["k_prefix"]).to(DEV).to(torch.bfloat16)
    vbuf[:, :, :ss] = torch.from_numpy(d["v_prefix"]).view(torch.bfloat16).to(DEV)
    slots = torch.full((1, Hkv, K), -1, dtype=torch.int32, device=DEV)
    out = torch.empty(1, Hq, 128, dtype=torch.bfloat16, device=DEV)
    U_f, SV_f, cs_f = bf(d["U"]), bf(d["SV"]), bf(cs_bits)
    for step in range(d["q"].shape[0]):
        kbuf[:, :, se + step] = torch.from_numpy(d["k_new"][step][:, :, 0]).to(DEV).to(torch.bfloat16)
        vbuf[:, :, se + step] = torch.from_numpy(d["v_new"][step][:, :, 0]).to(DEV).to(torch.bfloat16)
        q = torch.from_numpy(d["q"][step][:, :, 0, :]).to(DEV).to(torch.bfloat16).contiguous()
        seq_len = int(d["seq_len"][step])
        fz.select(g, ws, q, lm, lidx, slots)
        fz.sparse_attention(g, ws, q, U, SVt, cos_sin, v_host, kbuf, vbuf, seq_len, out)
        torch.cuda.synchronize()
        assert no_device_errors()
        sel = d["selected_chunk_idx"][step]  # reference topk order
        new_slots = slots.cpu().numpy()
        assert np.array_equal(np.sort(new_slots, -1), np.sort(sel, -1)), f"chunk ids, step {step}"
        vb = vbuf.float().cpu().numpy()
        kb = kbuf.float().cpu().numpy()
        # our slot-stable rows in the reference's slot order: then the reference's checksum applies
        where = {(h, int(c)): sl for h in range(Hkv) for sl, c in enumerate(new_slots[0, h])}
        v_ref_order = np.zeros((1, Hkv, 8 * K, 128), np.float32)
        k_ref_order = np.zeros_like(v_ref_order)
        for h in range(Hkv):
            for j in range(K):
                sl = where[(h, int(sel[0, h, j]))]
                v_ref_order[0, h, 8 * j: 8 * j + 8] = vb[0, h, ss + 8 * sl: ss + 8 * sl + 8]
                k_ref_order[0, h, 8 * j: 8 * j + 8] = kb[0, h, ss + 8 * sl: ss + 8 * sl + 8]
        assert hashlib.sha256(np.ascontiguousarray(v_ref_order).tobytes()).digest() == \
            d["v_sparse_sha256"][step].tobytes(), f"gathered values, step {step}"
        k_expect = d["k_sparse0"] if step == 0 else o.reconstruct_keys_fp32(U_f, SV_f, sel, cs_f)
        np.testing.assert_allclose(k_ref_order, k_expect, atol=2e-2, rtol=1e-2)
        kfull = np.concatenate([d["k_prefix"], k_expect, d["k_gen"][:, :, : step + 1]], axis=2)
        vfull = np.concatenate([bf(d["v_prefix"]), v_ref_order,
                                d["v_new"][: step + 1, :, :, 0].transpose(1, 2, 0, 3)], axis=2)
        assert kfull.shape[2] == seq_len
        ref = o.decode_attention(d["q"][step][:, :, 0, :], kfull, vfull, seq_len)
        np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)


# ------------------------------------------------------------------ kernels one by one

@pytest.mark.parametrize("G,L,K,H", [(4, 15308, 256, 3), (16, 6000, 256, 2), (1, 700, 64, 2), (4, 2000, 1000, 1),
                                     (4, 40000, 256, 2), (16, 131072, 256, 1),
                                     # long contexts through the keys kernel: G = 8 and a G that is
                                     # not a multiple of 4 (scalar logit loads)
                                     (8, 50000, 512, 2), (6, 40000, 256, 2)])
def test_select_topk_and_slot_update(G, L, K, H):
    from shadowkv_b200 import decode as fz
    rng = np.random.default_rng(G * 1000 + L)
    chunks = L + 500
    lm = o.round_bf16(rng.standard_normal((1, H, L, 128)).astype(np.float32))
    q = o.round_bf16(rng.standard_normal((1, H * G, 128)).astype(np.float32))
    lidx = np.stack([np.sort(rng.permutation(chunks)[:L]) for _ in range(H)])[None].astype(np.int64)
    g = make_geom(batch=1, kv_heads=H, q_heads=H * G, rank=64, select_sets=K, num_landmarks=L, num_chunks=chunks,
                  ctx_len=chunks * 8, buf_len=K * 8 + 64, sparse_start=32)
    ws = fz.DecodeWorkspace(g, DEV)
    scores = o.landmark_scores(q.reshape(1, H, G, 128), lm)
    # previous slots: a mix of chunks that are selected now and ones that are not
    prev = np.stack([rng.permutation(lidx[0, h])[:K] for h in range(H)])[None].astype(np.int32)
    slots = torch.from_numpy(prev.copy()).to(DEV)
    fz.select(g, ws, to_bf16_dev(q), to_bf16_dev(lm), torch.from_numpy(lidx).to(DEV), slots)
    torch.cuda.synchronize()
    assert no_device_errors()
    new = slots.cpu().numpy()
    # selected set is a top-K of the fp32 scores (slack for fp32 summation order)
    for h in range(H):
        pos = np.searchsorted(lidx[0, h], np.sort(new[0, h]))
        assert o.topk_tie_ok(scores[0, h][None], pos[None], K, rtol=1e-5)
    eslots, emiss, ehits = o.stable_slot_update(prev, np.sort(new, -1))
    assert np.array_equal(new, eslots)
    mc = ws.miss_count.cpu().numpy()
    ms = ws.miss_slot.cpu().numpy()
    mch = ws.miss_chunk.cpu().numpy()
    for h in range(H):
        n = mc[h]
        assert n == K - ehits[0, h]
        assert np.array_equal(np.sort(ms[h, :n]), np.where(emiss[0, h])[0])
        assert np.array_equal(new[0, h, ms[h, :n]], mch[h, :n])


@pytest.mark.parametrize("n_top,n_next,L", [(50, 600, 3000), (100, 2900, 3000), (0, 3000, 3000), (7, 1200, 9000)])
def test_select_ties_lowest_landmark_first(n_top, n_next, L):
    """Tied scores at the K-th place: the lowest landmark indices win.

    Landmark rows are copies of three vectors, so their scores are bitwise
    equal; (50, 600) resolves the ties among the candidates of the boundary
    bin, (100, 2900) and (0, 3000) put more than 1024 keys in that bin and go
    through the exact radix fallback.
    """
    from shadowkv_b200 import decode as fz
    rng = np.random.default_rng(n_top + 7 * n_next)
    H, G, K = 2, 4, 256
    q = o.round_bf16(rng.standard_normal((1, H * G, 128)).astype(np.float32))
    base = o.round_bf16(rng.standard_normal((3, 128)).astype(np.float32))
    s3 = o.landmark_scores(q.reshape(1, H, G, 128), np.broadcast_to(base, (1, H, 3, 128)))
    lm = np.empty((1, H, L, 128), np.float32)
    for h in range(H):
        order = np.argsort(-s3[0, h], kind="stable")  # best, next, worst vector for this head
        kind = np.full(L, order[2])
        pos = rng.permutation(L)
        kind[pos[:n_top]] = order[0]
        kind[pos[n_top:n_top + n_next]] = order[1]
        lm[0, h] = base[kind]
    lidx = torch.arange(L, dtype=torch.int64, device=DEV).repeat(1, H, 1).contiguous()
    g = make_geom(batch=1, kv_heads=H, q_heads=H * G, rank=64, select_sets=K, num_landmarks=L, num_chunks=L,
                  ctx_len=L * 8, buf_len=K * 8, sparse_start=0)
    ws = fz.DecodeWorkspace(g, DEV)
    slots = torch.full((1, H, K), -1, dtype=torch.int32, device=DEV)
    fz.select(g, ws, to_bf16_dev(q), to_bf16_dev(lm), lidx, slots)
    torch.cuda.synchronize()
    assert no_device_errors()
    sc = o.landmark_scores(q.reshape(1, H, G, 128), lm)
    for h in range(H):
        expect = np.sort(np.argsort(-sc[0, h], kind="stable")[:K])
        assert np.array_equal(np.sort(slots[0, h].cpu().numpy()), expect)


def test_select_repeated_query_is_all_hits():
    from shadowkv_b200 import decode as fz
    rng = np.random.default_rng(0)
    H, G, L, K = 2, 4, 3000, 128
    lm = to_bf16_dev(rng.standard_normal((1, H, L, 128)))
    q = to_bf16_dev(rng.standard_normal((1, H * G, 128)))
    lidx = torch.arange(L, dtype=torch.int64, device=DEV).repeat(1, H, 1).contiguous()
    g = make_geom(batch=1, kv_heads=H, q_heads=H * G, rank=64, select_sets=K, num_landmarks=L, num_chunks=L,
                  ctx_len=L * 8, buf_len=K * 8, sparse_start=0)
    ws = fz.DecodeWorkspace(g, DEV)
    slots = torch.full((1, H, K), -1, dtype=torch.int32, device=DEV)
    fz.select(g, ws, q, lm, lidx, slots)
    assert (ws.miss_count.cpu().numpy() == K).all()
    first = slots.clone()
    fz.select(g, ws, q, lm, lidx, slots)
    assert (ws.miss_count.cpu().numpy() == 0).all()
    assert torch.equal(first, slots)


def test_gather_values_exact():
    from shadowkv_b200 import decode as fz
    rng = np.random.default_rng(1)
    B, H, K, chunks = 2, 3, 256, 5000
    g = make_geom(batch=B, kv_heads=H, q_heads=H * 4, rank=64, select_sets=K, num_landmarks=K, num_chunks=chunks,
                  ctx_len=chunks * 8, buf_len=K * 8 + 100, sparse_start=60)
    ws = fz.DecodeWorkspace(g, DEV)
    host = rng.integers(0, 1 << 16, (B, H, chunks, 1024), dtype=np.uint16)
    host_t = torch.from_numpy(host.view(np.int16)).view(torch.bfloat16).pin_memory()
    buf0 = rng.integers(0, 1 << 16, (B, H, K * 8 + 100, 128), dtype=np.uint16)
    buf = torch.from_numpy(buf0.view(np.int16)).view(torch.bfloat16).to(DEV)
    expect = buf0.copy()
    cnt = rng.integers(0, K + 1, B * H).astype(np.int32)
    ms = np.zeros((B * H, K), np.int32)
    mc = np.zeros((B * H, K), np.int32)
    for i in range(B * H):
        ms[i, : cnt[i]] = rng.permutation(K)[: cnt[i]]
        mc[i, : cnt[i]] = rng.permutation(chunks)[: cnt[i]]
        b, h = divmod(i, H)
        for j in range(cnt[i]):
            r0 = 60 + 8 * ms[i, j]
            expect[b, h, r0: r0 + 8] = host[b, h, mc[i, j]].reshape(8, 128)
    ws.miss_slot.copy_(torch.from_numpy(ms))
    ws.miss_chunk.copy_(torch.from_numpy(mc))
    ws.miss_count.copy_(torch.from_numpy(cnt))
    fz.gather_values(g, ws, host_t, buf)
    assert np.array_equal(bits(buf), expect)


@pytest.mark.parametrize("rope_mode,rank", [(0, 160), (1, 160), (0, 64), (1, 16), (0, 256)])
def test_reconstruct_keys_with_rope(rope_mode, rank):
    from shadowkv_b200 import decode as fz
    rng = np.random.default_rng(rope_mode + 3 + rank)
    B, H, K, T = 1, 4, 256, 16384
    chunks = T // 8
    width = 128 if rope_mode == 0 else 64
    U = o.round_bf16((rng.standard_normal((B, T, rank)) / 8).astype(np.float32))
    SVt = o.round_bf16(rng.standard_normal((B, H, 128, rank)).astype(np.float32))
    cs = o.round_bf16(rng.uniform(-1, 1, (T + 64, width)).astype(np.float32))
    g = make_geom(batch=B, kv_heads=H, q_heads=H * 4, rank=rank, select_sets=K, num_landmarks=K, num_chunks=chunks,
                  ctx_len=T, buf_len=K * 8 + 40, sparse_start=40, rope_mode=rope_mode, cos_sin_stride=width,
                  cos_sin_rows=T + 64)
    ws = fz.DecodeWorkspace(g, DEV)
    cnt = np.array([K, 0, 37, 200], np.int32)
    ms = np.zeros((H, K), np.int32)
    mc = np.zeros((H, K), np.int32)
    for h in range(H):
        ms[h, : cnt[h]] = rng.permutation(K)[: cnt[h]]
        mc[h, : cnt[h]] = rng.permutation(chunks)[: cnt[h]]
    ws.miss_slot.copy_(torch.from_numpy(ms))
    ws.miss_chunk.copy_(torch.from_numpy(mc))
    ws.miss_count.copy_(torch.from_numpy(cnt))
    kbuf = torch.full((B, H, K * 8 + 40, 128), 7.0, dtype=torch.bfloat16, device=DEV)
    fz.reconstruct_keys(g, ws, to_bf16_dev(U), to_bf16_dev(SVt), to_bf16_dev(cs), kbuf)
    got = kbuf.float().cpu().numpy()
    expect = np.full_like(got, 7.0)
    for h in range(H):
        ids = mc[h, : cnt[h]]
        if len(ids) == 0:
            continue
        rot = o.reconstruct_keys_rope(U[0], SVt[0, h], ids, cs, glm=rope_mode == 1)
        for j in range(len(ids)):
            r0 = 40 + 8 * ms[h, j]
            expect[0, h, r0: r0 + 8] = rot[8 * j: 8 * j + 8]
    untouched = expect == 7.0
    assert np.array_equal(got[untouched], expect[untouched])
    np.testing.assert_allclose(got, expect, atol=2e-2, rtol=1e-2)
    # fp32 accumulation + fp32 RoPE + one rounding: within one bf16 ulp of the float64 result
    assert (np.abs(got - expect) <= np.abs(expect) * 2.0 ** -7 + 1e-6).mean() > 0.999


@pytest.mark.parametrize("B,Hq,Hkv,S", [(1, 32, 8, 2464), (2, 32, 2, 700), (3, 8, 8, 65), (1, 32, 8, 1)])
def test_attention(B, Hq, Hkv, S):
    from shadowkv_b200 import decode as fz
    rng = np.random.default_rng(S)
    buf_len = S + 33
    q = o.round_bf16(rng.standard_normal((B, Hq, 128)).astype(np.float32))
    k = o.round_bf16(rng.standard_normal((B, Hkv, buf_len, 128)).astype(np.float32))
    v = o.round_bf16(rng.standard_normal((B, Hkv, buf_len, 128)).astype(np.float32))
    g = make_geom(batch=B, kv_heads=Hkv, q_heads=Hq, rank=64, select_sets=1, num_landmarks=1, num_chunks=1,
                  ctx_len=8, buf_len=buf_len, sparse_start=0)
    ws = fz.DecodeWorkspace(g, DEV)
    out = torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=DEV)
    fz.attention(g, ws, to_bf16_dev(q), to_bf16_dev(k), to_bf16_dev(v), S, out)
    ref = o.decode_attention(q, k, v, S)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("B,Hkv,G,rank,K,ss,extra,rope_mode,pattern", [
    (1, 2, 4, 64, 64, 40, 1, 0, "mixed"),
    (2, 2, 16, 160, 128, 32, 5, 0, "all"),
    (1, 3, 8, 96, 256, 416, 130, 1, "mixed"),
    (1, 2, 4, 160, 256, 416, 1, 0, "none"),
    (1, 1, 1, 32, 16, 8, 1, 0, "all"),
])
def test_sparse_attention_fetch_reconstruct_attend(B, Hkv, G, rank, K, ss, extra, rope_mode, pattern):
    """One launch = gather_values + reconstruct_keys + attention: buffers and output vs the oracle."""
    from shadowkv_b200 import decode as fz
    rng = np.random.default_rng(K + rank + extra)
    T = 4096
    chunks = T // 8
    width = 128 if rope_mode == 0 else 64
    se = ss + 8 * K
    seq_len = se + extra
    buf_len = seq_len + 3
    Hq = Hkv * G
    U = o.round_bf16((rng.standard_normal((B, T, rank)) / 8).astype(np.float32))
    SVt = o.round_bf16(rng.standard_normal((B, Hkv, 128, rank)).astype(np.float32))
    cs = o.round_bf16(rng.uniform(-1, 1, (T + 64, width)).astype(np.float32))
    host = o.round_bf16(rng.standard_normal((B, Hkv, chunks, 1024)).astype(np.float32))
    host_t = torch.from_numpy(o.f32_to_bf16_bits(host).view(np.int16)).view(torch.bfloat16).pin_memory()
    kb0 = o.round_bf16(rng.standard_normal((B, Hkv, buf_len, 128)).astype(np.float32))
    vb0 = o.round_bf16(rng.standard_normal((B, Hkv, buf_len, 128)).astype(np.float32))
    q = o.round_bf16(rng.standard_normal((B, Hq, 128)).astype(np.float32))
    g = make_geom(batch=B, kv_heads=Hkv, q_heads=Hq, rank=rank, select_sets=K, num_landmarks=K, num_chunks=chunks,
                  ctx_len=T, buf_len=buf_len, sparse_start=ss, rope_mode=rope_mode, cos_sin_stride=width,
                  cos_sin_rows=T + 64)
    ws = fz.DecodeWorkspace(g, DEV)
    ms = np.zeros((B * Hkv, K), np.int32)
    mc = np.zeros((B * Hkv, K), np.int32)
    cnt = np.zeros(B * Hkv, np.int32)
    for i in range(B * Hkv):
        n = {"all": K, "none": 0, "mixed": int(rng.integers(1, K))}[pattern]
        cnt[i] = n
        ms[i, :n] = np.sort(rng.permutation(K)[:n])
        mc[i, :n] = rng.permutation(chunks)[:n]
    ws.miss_slot.copy_(torch.from_numpy(ms))
    ws.miss_chunk.copy_(torch.from_numpy(mc))
    ws.miss_count.copy_(torch.from_numpy(cnt))
    kbuf, vbuf = to_bf16_dev(kb0), to_bf16_dev(vb0)
    out = torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=DEV)
    args = (g, ws, to_bf16_dev(q), to_bf16_dev(U), to_bf16_dev(SVt), to_bf16_dev(cs), host_t, kbuf, vbuf, seq_len)
    fz.sparse_attention(*args, out)
    torch.cuda.synchronize()
    assert no_device_errors()
    ek, ev = kb0.copy(), vb0.copy()
    for i in range(B * Hkv):
        b, h = divmod(i, Hkv)
        n = cnt[i]
        if n == 0:
            continue
        rot = o.reconstruct_keys_rope(U[b], SVt[b, h], mc[i, :n], cs, glm=rope_mode == 1)
        for j in range(n):
            r0 = ss + 8 * ms[i, j]
            ek[b, h, r0:r0 + 8] = rot[8 * j:8 * j + 8]
            ev[b, h, r0:r0 + 8] = host[b, h, mc[i, j]].reshape(8, 128)
    gk = kbuf.float().cpu().numpy()
    assert np.array_equal(vbuf.float().cpu().numpy(), ev), "fetched values"
    untouched = ek == kb0
    assert np.array_equal(gk[untouched], ek[untouched])
    np.testing.assert_allclose(gk, ek, atol=2e-2, rtol=1e-2)
    ref = o.decode_attention(q, gk, ev, seq_len)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)
    # the per-head tickets are back at zero: a second launch gives the same output
    out2 = torch.empty_like(out)
    fz.sparse_attention(*args, out2)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


def test_select_non_finite_query_does_not_fault():
    """Scores from a query with inf entries give non-finite keys; the selection
    still completes with an in-range slot table (which chunks it picks is unspecified)."""
    from shadowkv_b200 import decode as fz
    rng = np.random.default_rng(11)
    H, G, L, K = 2, 4, 3000, 128
    q = rng.standard_normal((1, H * G, 128)).astype(np.float32)
    q[0, 0, :4] = np.inf
    lm = to_bf16_dev(rng.standard_normal((1, H, L, 128)))
    lidx = torch.arange(L, dtype=torch.int64, device=DEV).repeat(1, H, 1).contiguous()
    g = make_geom(batch=1, kv_heads=H, q_heads=H * G, rank=64, select_sets=K, num_landmarks=L, num_chunks=L,
                  ctx_len=L * 8, buf_len=K * 8, sparse_start=0)
    ws = fz.DecodeWorkspace(g, DEV)
    slots = torch.full((1, H, K), -1, dtype=torch.int32, device=DEV)
    fz.select(g, ws, to_bf16_dev(q), lm, lidx, slots)
    torch.cuda.synchronize()
    s = slots.cpu().numpy()
    assert ((s >= 0) & (s < L)).all()
