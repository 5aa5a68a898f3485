"""GPU parity of the twelve drop-in bindings against the oracle and the reference's goldens."""
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


def to_bf16_dev(x: np.ndarray) -> torch.Tensor:
    bits = o.f32_to_bf16_bits(np.asarray(x, dtype=np.float32))
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(DEV)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.fixture(scope="module")
def skv():
    from shadowkv_b200 import shadowkv
    return shadowkv


def no_device_errors():
    from shadowkv_b200._lib import device_errors
    torch.cuda.synchronize()
    return device_errors()[0] == 0


# --------------------------------------------------------------------------- reorder

def test_reorder_reference_kat(skv):
    """kernels/test_cached_gather_copy.cu inputs (seed 12345, 192x256, 154 hits): bit-exact."""
    keys, query = o.kat_keys()
    gk, go, gc = o.golden_reorder(keys, query)
    cached = torch.from_numpy(keys.copy()).to(DEV)
    cur = torch.from_numpy(query.copy()).to(DEV)
    off = torch.zeros(192 * 256, dtype=torch.int32, device=DEV)
    cnt = torch.zeros(192, dtype=torch.int32, device=DEV)
    skv.reorder_keys_and_compute_offsets(cached, cur, off, cnt, 24, 8, 256)
    assert np.array_equal(cached.cpu().numpy(), gk)
    assert np.array_equal(off.cpu().numpy().reshape(192, 256), go)
    assert np.array_equal(cnt.cpu().numpy(), gc)


@pytest.mark.parametrize("m", [1, 7, 64, 128, 200, 256, 512, 1024])
def test_reorder_any_map_size(skv, m):
    rng = np.random.default_rng(m)
    nb = 5
    old = np.stack([rng.permutation(50000)[:m] for _ in range(nb)]).astype(np.int64)
    new = old.copy()
    for b in range(nb):
        nh = rng.integers(0, m + 1)
        keep = rng.permutation(old[b])[:nh]
        fresh = 60000 + rng.permutation(100000)[: m - nh]
        new[b] = rng.permutation(np.concatenate([keep, fresh]))
    ek, eo, ec = o.reorder_keys_and_compute_offsets(old, new)
    cached = torch.from_numpy(old.copy()).to(DEV)
    off = torch.zeros(nb * m, dtype=torch.int32, device=DEV)
    cnt = torch.zeros(nb, dtype=torch.int32, device=DEV)
    skv.reorder_keys_and_compute_offsets(cached, torch.from_numpy(new).to(DEV), off, cnt, nb, 1, m)
    assert np.array_equal(cached.cpu().numpy(), ek)
    assert np.array_equal(off.cpu().numpy().reshape(nb, m), eo)
    assert np.array_equal(cnt.cpu().numpy(), ec)


def test_reorder_initial_minus_one(skv):
    """Cached ids of -1 (the reference's initial position_ids) never hit."""
    old = -np.ones((2, 64), dtype=np.int64)
    new = np.stack([np.arange(64) * 3, np.arange(64)[::-1] * 5]).astype(np.int64)
    ek, eo, ec = o.reorder_keys_and_compute_offsets(old, new)
    cached = torch.from_numpy(old.copy()).to(DEV)
    off = torch.zeros(128, dtype=torch.int32, device=DEV)
    cnt = torch.zeros(2, dtype=torch.int32, device=DEV)
    skv.reorder_keys_and_compute_offsets(cached, torch.from_numpy(new).to(DEV), off, cnt, 1, 2, 64)
    assert (cnt.cpu().numpy() == 0).all()
    assert np.array_equal(cached.cpu().numpy(), ek)


# --------------------------------------------------------------------------- V/K reuse copies

def _kat_buffers(nb, m, cpu_chunks, hits, seed, buf_rows_extra=(40, 24)):
    rng = np.random.default_rng(seed)
    keys, query = o.kat_keys(block_num=nb, map_size=m, cpu_chunks=cpu_chunks, fake_hit_cnt=hits, seed=12345 + seed)
    cpu_len = cpu_chunks * 1024
    host = rng.integers(0, 1 << 16, size=(nb, cpu_len), dtype=np.uint16)
    pre, post = buf_rows_extra  # rows before / after the selected region, per block
    stride = (pre + m * 8 + post) * 128
    dev = rng.integers(0, 1 << 16, size=(nb, stride), dtype=np.uint16)
    for b in range(nb):
        dev[b, pre * 128: pre * 128 + m * 1024] = host[b].reshape(-1, 1024)[keys[b]].reshape(-1)
    return keys, query, host, dev, cpu_len, stride, pre * 128


@pytest.mark.parametrize("nb,m,hits", [(24, 256, 154), (3, 64, 10), (4, 128, 0), (2, 512, 512)])
def test_gather_copy_with_offsets_matches_golden(skv, nb, m, hits):
    keys, query, host, dev, cpu_len, stride, offset = _kat_buffers(nb, m, 4096, hits, nb)
    rk, off, cnt = o.reorder_keys_and_compute_offsets(keys, query)
    expect = o.gather_copy_with_offsets(host, dev, off, cnt, cpu_len, m * 1024, offset, stride, m)
    host_t = torch.from_numpy(host.view(np.int16)).view(torch.bfloat16).pin_memory()
    buf = torch.from_numpy(dev.view(np.int16)).view(torch.bfloat16).to(DEV)
    temp = torch.zeros(nb, m, 1024, dtype=torch.bfloat16, device=DEV)
    signals = torch.zeros(nb, dtype=torch.int32, device=DEV)
    off_t = torch.from_numpy(off.reshape(-1).copy()).to(DEV)
    cnt_t = torch.from_numpy(cnt.copy()).to(DEV)
    skv.gather_copy_with_offsets(host_t, buf, temp, off_t, cnt_t, signals, 1, nb, cpu_len, m * 1024, offset, stride, m)
    got = bits(buf)
    assert np.array_equal(got, expect)
    # the reference's own golden: slot-major chunks of the selected region
    golden = o.golden_cached_copy(host, dev[:, offset: offset + m * 1024], off, cnt, cpu_len, m * 1024)
    assert np.array_equal(got[:, offset: offset + m * 1024].reshape(nb, m, 1024), golden)
    assert (signals.cpu().numpy() == 0).all()
    assert no_device_errors()


@pytest.mark.parametrize("nb,m,hits", [(16, 256, 200), (2, 32, 31)])
def test_gather_copy_d2d_with_offsets(skv, nb, m, hits):
    keys, query, host, dev, cpu_len, stride, offset = _kat_buffers(nb, m, 2048, hits, 7 + nb)
    rk, off, cnt = o.reorder_keys_and_compute_offsets(keys, query)
    expect = o.gather_copy_d2d_with_offsets(dev, off, cnt, offset, stride, m)
    buf = torch.from_numpy(dev.view(np.int16)).view(torch.bfloat16).to(DEV)
    skv.gather_copy_d2d_with_offsets(buf, torch.from_numpy(off.reshape(-1).copy()).to(DEV),
                                     torch.from_numpy(cnt.copy()).to(DEV), 2, nb // 2, m * 1024, offset, stride, m)
    assert np.array_equal(bits(buf), expect)


def test_gather_copy_matches_golden(skv):
    keys, query = o.kat_keys_nohit(block_num=10, map_size=256, cpu_chunks=2048)
    rng = np.random.default_rng(9)
    cpu_len = 2048 * 1024
    host = rng.integers(0, 1 << 16, size=(10, cpu_len), dtype=np.uint16)
    golden = o.golden_gather_copy(host, query, cpu_len)
    host_t = torch.from_numpy(host.view(np.int16)).view(torch.bfloat16).pin_memory()
    gpu_len = 256 * 1024 + 4096
    buf = torch.zeros(10, gpu_len, dtype=torch.bfloat16, device=DEV)
    skv.gather_copy(host_t, buf, torch.from_numpy(query.copy()).to(DEV), 2, 5, cpu_len, gpu_len, 256)
    got = bits(buf)
    assert np.array_equal(got[:, : 256 * 1024].reshape(10, 256, 1024), golden)
    assert (got[:, 256 * 1024:] == 0).all()


def test_pageable_host_memory_is_rejected(skv):
    host = torch.zeros(1, 64 * 1024, dtype=torch.bfloat16)  # not pinned
    buf = torch.zeros(1, 64 * 1024, dtype=torch.bfloat16, device=DEV)
    ids = torch.zeros(1, 64, dtype=torch.int64, device=DEV)
    with pytest.raises(RuntimeError):
        skv.gather_copy(host, buf, ids, 1, 1, 64 * 1024, 64 * 1024, 64)


# --------------------------------------------------------------------------- RoPE

@pytest.fixture(scope="module")
def rope_fix(golden_dir):
    return np.load(os.path.join(golden_dir, "rope_bf16.npz"))


def test_rope_new_matches_reference_torch_bf16(skv, rope_fix):
    """apply_rotary_pos_emb_new vs the reference's torch RoPE run in bf16: bit-exact."""
    from shadowkv_b200.tensor_op import apply_rotary_pos_emb_cuda
    d = rope_fix
    x = torch.from_numpy(d["x"]).view(torch.bfloat16).to(DEV)
    cs = torch.from_numpy(d["cos_sin"]).view(torch.bfloat16).to(DEV)
    pos = torch.from_numpy(d["pos"]).to(DEV)
    out = apply_rotary_pos_emb_cuda(x, cs, pos)
    assert np.array_equal(bits(out), d["out_llama"].view(np.uint16))


def test_rope_separate_tables(skv, rope_fix):
    d = rope_fix
    x = torch.from_numpy(d["x"]).view(torch.bfloat16).to(DEV)
    cs = torch.from_numpy(d["cos_sin"]).view(torch.bfloat16).to(DEV)
    cos = torch.cat((cs[:, :64], cs[:, :64]), -1).contiguous()
    sin = torch.cat((cs[:, 64:], cs[:, 64:]), -1).contiguous()
    pos = torch.from_numpy(d["pos"]).to(DEV)
    out = torch.empty_like(x)
    B, H, S, D = x.shape
    skv.apply_rotary_pos_emb(x, cos, sin, pos, out, B, H, S, D, *x.stride(), cos.stride(0), sin.stride(0),
                             *pos.stride(), D // 2)
    assert np.array_equal(bits(out), d["out_llama"].view(np.uint16))


def test_rope_new_v2_chunk_ids(skv):
    rng = np.random.default_rng(4)
    B, H, S, D = 2, 3, 64, 128
    x = o.round_bf16(rng.standard_normal((B, H, S, D)).astype(np.float32))
    cs = o.round_bf16(rng.uniform(-1, 1, (1024, 128)).astype(np.float32))
    ids = rng.integers(0, 1024 // 8, (B, H, S // 8)).astype(np.int32)
    pos = ids[..., np.repeat(np.arange(S // 8), 8)] * 8 + np.tile(np.arange(8), S // 8)
    c = cs[pos]
    expect = o.rope_rotate_half_bf16(x, c[..., :64], c[..., 64:])
    xt, cst = to_bf16_dev(x), to_bf16_dev(cs)
    idt = torch.from_numpy(ids).to(DEV)
    out = torch.empty_like(xt)
    skv.apply_rotary_pos_emb_new_v2(xt, cst, idt, out, B, H, S, D, *xt.stride(), cst.stride(0), *idt.stride(),
                                    D // 2, 8)
    assert np.array_equal(bits(out), o.f32_to_bf16_bits(expect))


@pytest.mark.parametrize("glm", [False, True])
@pytest.mark.parametrize("variant", ["push_cache", "push_cache_opt"])
def test_rope_push_cache(skv, glm, variant):
    if glm and variant == "push_cache":
        pytest.skip("the GLM kernel exists only as the _opt variant")
    rng = np.random.default_rng(11)
    B, H, S, D = 2, 4, 128, 128
    width = 64 if glm else 128
    x = o.round_bf16(rng.standard_normal((B, H, S, D)).astype(np.float32))
    cs = o.round_bf16(rng.uniform(-1, 1, (4096, width)).astype(np.float32))
    ids = np.stack([[rng.permutation(500)[: S // 8] for _ in range(H)] for _ in range(B)]).astype(np.int32)
    cnts = rng.integers(0, S // 8 + 1, B * H).astype(np.int32)
    s_start, buf_len = 40, 40 + S + 16
    s_end = s_start + S - 8  # the last chunk is clipped by sparse_end
    cache = o.round_bf16(rng.standard_normal((B, H, buf_len, D)).astype(np.float32))
    expect = o.apply_rotary_pos_emb_push_cache_opt(x, cs, ids, cache, cnts, s_start, s_end, 8, glm=glm)
    xt, cst, ct = to_bf16_dev(x), to_bf16_dev(cs), to_bf16_dev(cache)
    idt, cnt_t = torch.from_numpy(ids).to(DEV), torch.from_numpy(cnts).to(DEV)
    fn = getattr(skv, f"apply_rotary_pos_emb_{variant}" + ("_glm" if glm else ""))
    fn(xt, cst, idt, ct, cnt_t, B, H, S, D, *xt.stride(), cst.stride(0), *idt.stride(), *ct.stride()[:3],
       s_start, s_end, D // 2, 8)
    assert np.array_equal(bits(ct), o.f32_to_bf16_bits(expect))


# --------------------------------------------------------------------------- GEMMs

# ranks >= 64 take the 128-byte-swizzled operand layout (160: a partial last
# k-block), 32 and 48 the 16-byte-piece layout
@pytest.mark.parametrize("rank", [160, 64, 256, 32, 48])
def test_batch_gather_gemm(skv, rank):
    rng = np.random.default_rng(rank)
    B, H, T, budget = 2, 3, 4096, 512
    M = budget // 8
    U = o.round_bf16((rng.standard_normal((B, T, rank)) / 8).astype(np.float32))
    SVt = o.round_bf16(rng.standard_normal((B, H, 128, rank)).astype(np.float32))
    ids = np.stack([[rng.permutation(T // 8)[:M] for _ in range(H)] for _ in range(B)]).astype(np.int32)
    cnts = rng.integers(0, M + 1, B * H).astype(np.int32)
    cnts[0] = 0
    expect = o.batch_gather_gemm(U, SVt, ids, cnts)
    out = torch.full((B, H, budget, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
    skv.batch_gather_gemm(to_bf16_dev(U), to_bf16_dev(SVt), None, None, torch.from_numpy(ids).to(DEV), out, B, H, T,
                          128, rank, budget, T, 8, torch.from_numpy(cnts).to(DEV))
    got = out.float().cpu().numpy()
    mask = ~np.isnan(expect)
    assert np.isnan(got[~mask]).all(), "rows of cache hits must stay untouched"
    np.testing.assert_allclose(got[mask], expect[mask], atol=2e-2, rtol=1e-2)
    # fp32 accumulation then one bf16 rounding: at most one bf16 ulp apart
    ulp = np.abs(expect[mask]) * 2.0 ** -7 + 1e-30
    assert (np.abs(got[mask] - expect[mask]) <= ulp).mean() > 0.999


@pytest.mark.parametrize("m,n", [(4, 15308), (4, 300), (16, 2000), (1, 257)])
def test_batch_gemm_softmax(skv, m, n):
    rng = np.random.default_rng(m * 7 + n)
    bsz = 3
    A = o.round_bf16(rng.standard_normal((bsz, m, 128)).astype(np.float32))
    Bm = o.round_bf16(rng.standard_normal((bsz, n, 128)).astype(np.float32))
    alpha = 1 / math.sqrt(128)
    eD, eN, eS, eP = o.batch_gemm_softmax(A, Bm, bsz, m, n, 128, alpha)
    nblk = (n + 255) // 256
    D = torch.zeros(bsz, m, n, dtype=torch.bfloat16, device=DEV)
    P = torch.zeros_like(D)
    N = torch.zeros(bsz, nblk, m, dtype=torch.float32, device=DEV)
    S = torch.zeros_like(N)
    skv.batch_gemm_softmax(to_bf16_dev(A), to_bf16_dev(Bm), D, N, S, P, bsz, m, n, 128, alpha, 0.0)
    gD = D.float().cpu().numpy()
    assert (np.abs(gD - eD) <= np.abs(eD) * 2.0 ** -7 + 1e-6).all()
    np.testing.assert_allclose(N.cpu().numpy()[:, 0], eN[:, 0], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(S.cpu().numpy()[:, 0], eS[:, 0], rtol=1e-3)
    np.testing.assert_allclose(N.cpu().numpy()[:, 1:], eN[:, 1:], rtol=1e-4, atol=1e-4)
    # the softmax is computed from the bf16 D: check it against the oracle formula on this D
    gP = P.float().cpu().numpy()
    M = eN[:, 0][:, :, None].astype(np.float64)
    inv = eS[:, 0][:, :, None].astype(np.float64)
    expect_p = o.round_bf16((np.exp(gD.astype(np.float64) - M) * inv).astype(np.float32))
    np.testing.assert_allclose(gP, expect_p, rtol=1e-2, atol=1e-6)
    np.testing.assert_allclose(gP.sum(-1), 1.0, atol=2e-2)
