"""CPU: pin the oracle against the reference's own outputs and known-answer tests."""
import os

import numpy as np
import pytest

from oracle import shadowkv_oracle as o


def bf(a):
    return o.bf16_bits_to_f32(np.asarray(a).view(np.uint16))


@pytest.fixture(scope="module")
def torch_fix(golden_dir):
    return np.load(os.path.join(golden_dir, "torch_class_decode.npz"))


@pytest.fixture(scope="module")
def rope_fix(golden_dir):
    return np.load(os.path.join(golden_dir, "rope_bf16.npz"))


def test_bf16_rounding_matches_known_values():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5, 3.0e38, 1e-40], dtype=np.float32)
    r = o.round_bf16(x)
    assert r[0] == 1.0
    assert r[1] == 1.0           # tie -> even
    assert r[2] == 1.0078125     # above the midpoint -> up
    assert r[3] == -2.5
    assert np.isfinite(r[5])


def test_selection_matches_reference_torch_class(torch_fix):
    """models/kvcache/shadow.py:208-222 run by make_golden.py: chunk ids bit-exact (fp32 scores)."""
    d = torch_fix
    Hq, Hkv = int(d["Hq"]), int(d["Hkv"])
    lm, lidx = bf(d["k_landmark"]), d["k_landmark_idx"]
    K = int(d["budget"]) // 8
    for step in range(d["q"].shape[0]):
        q = d["q"][step][:, :, 0, :].reshape(1, Hkv, Hq // Hkv, 128)
        ids, sc = o.select_chunks(q, lm, lidx, K)
        assert np.array_equal(ids, np.sort(d["selected_chunk_idx"][step], axis=-1))


def test_value_gather_matches_reference_torch_class(torch_fix):
    d = torch_fix
    v = bf(d["v_bf16"])
    for step in range(d["q"].shape[0]):
        sel = d["selected_chunk_idx"][step]
        tok = (sel[..., None] * 8 + np.arange(8)).reshape(1, sel.shape[1], -1)
        vg = np.take_along_axis(v, tok[..., None], axis=2)
        assert np.array_equal(vg, bf(d["v_sparse"][step]))


def test_key_reconstruction_matches_reference_torch_class(torch_fix):
    """shadow.py:239-256 (fp32): tolerance 1e-4."""
    d = torch_fix
    U, SV, cs = bf(d["U"]), bf(d["SV"]), bf(d["cos_sin_bf16"])
    for step in range(d["q"].shape[0]):
        kr = o.reconstruct_keys_fp32(U, SV, d["selected_chunk_idx"][step], cs)
        np.testing.assert_allclose(kr, d["k_sparse"][step], atol=1e-4, rtol=1e-4)


def test_rope_bf16_matches_reference_torch_rope(rope_fix):
    """tensor_op.py:144-156 in bf16 == rope_new.cu arithmetic restated by the oracle (bit-exact)."""
    d = rope_fix
    x = bf(d["x"])
    cs = bf(d["cos_sin"])
    pos = d["pos"]
    c = cs[pos]
    out = o.rope_rotate_half_bf16(x, c[..., :64], c[..., 64:])
    assert np.array_equal(o.f32_to_bf16_bits(out), d["out_llama"].view(np.uint16))


def test_rope_glm_bf16_matches_reference_glm_rope(rope_fix):
    """models/glm.py:207-230 in bf16 == rope_new.cu:354-371 restated (bit-exact)."""
    d = rope_fix
    x = bf(d["x"])
    cs = bf(d["cos_sin_glm"])[d["pos"]]
    out = o.rope_glm_bf16(x, cs)
    assert np.array_equal(o.f32_to_bf16_bits(out), d["out_glm"].view(np.uint16))


def test_glibc_rand_is_the_reference_generator():
    """The KAT keys depend on glibc rand(); its first outputs after srand(1) are well known."""
    import ctypes
    lib = o.load_c_oracle()
    out = (ctypes.c_int * 3)()
    lib.skv_glibc_rand_check(1, 3, out)
    assert list(out) == [1804289383, 846930886, 1681692777]


def test_reorder_oracle_equals_reference_kat_golden():
    """kernels/test_cached_gather_copy.cu: seed 12345, 192 blocks x 256, 154 forced hits."""
    keys, query = o.kat_keys()
    gk, go, gc = o.golden_reorder(keys, query)
    rk, ro, rc = o.reorder_keys_and_compute_offsets(keys, query)
    assert (gc == 154).all()
    assert np.array_equal(gk, rk) and np.array_equal(go, ro) and np.array_equal(gc, rc)


def test_reorder_oracle_hits_sorted_by_old_slot_with_unsorted_keys():
    """With unsorted cached keys the kernel order (by old slot) differs from sorting keys; check the rule."""
    rng = np.random.default_rng(3)
    old = rng.permutation(5000)[:64].reshape(1, 64)
    new = np.concatenate([old[0, rng.permutation(64)[:40]], 6000 + rng.permutation(100)[:24]]).reshape(1, 64)
    k, off, cnt = o.reorder_keys_and_compute_offsets(old, new)
    assert cnt[0] == 40
    assert (np.diff(off[0, :40]) > 0).all()
    assert np.array_equal(k[0, :40], old[0, off[0, :40]])
    assert np.array_equal(k[0, 40:], np.sort(new[0, 40:])) and np.array_equal(off[0, 40:], k[0, 40:])


def test_cached_copy_oracle_equals_reference_golden():
    """check_cached_copy (test_cached_gather_copy.cu:158-216) vs the in-place oracle."""
    rng = np.random.default_rng(0)
    keys, query = o.kat_keys(block_num=12, map_size=256, cpu_chunks=4096, fake_hit_cnt=154, seed=12345)
    nb, m = keys.shape
    cpu_len = 4096 * 1024
    host = rng.integers(0, 1 << 16, size=(nb, cpu_len), dtype=np.uint16)
    dev = np.stack([host[b].reshape(-1, 1024)[keys[b]].reshape(-1) for b in range(nb)])  # slot i holds keys[i]
    rk, off, cnt = o.reorder_keys_and_compute_offsets(keys, query)
    golden = o.golden_cached_copy(host, dev, off, cnt, cpu_len, m * 1024)
    mine = o.gather_copy_with_offsets(host, dev, off, cnt, cpu_len, m * 1024, 0, m * 1024, m)
    assert np.array_equal(golden.reshape(nb, -1), mine)
    # every slot now holds the chunk named by the reordered key
    for b in range(nb):
        assert np.array_equal(mine[b].reshape(m, 1024), host[b].reshape(-1, 1024)[rk[b]])


def test_gather_copy_oracle_equals_reference_golden():
    rng = np.random.default_rng(1)
    keys, query = o.kat_keys_nohit(block_num=6, map_size=256, cpu_chunks=2048)
    cpu_len = 2048 * 1024
    host = rng.integers(0, 1 << 16, size=(6, cpu_len), dtype=np.uint16)
    golden = o.golden_gather_copy(host, query, cpu_len)
    mine = o.gather_copy(host, np.zeros((6, 256 * 1024), np.uint16), query, cpu_len, 256 * 1024, 256)
    assert np.array_equal(golden.reshape(6, -1), mine)


def test_stable_slot_update_properties():
    rng = np.random.default_rng(5)
    old = rng.permutation(1000)[:64]
    new = np.concatenate([rng.permutation(old)[:30], 2000 + rng.permutation(500)[:34]])
    slots, miss, hits = o.stable_slot_update(old[None], new[None])
    assert hits[0] == 30
    assert set(slots[0].tolist()) == set(new.tolist())
    keep = ~miss[0]
    assert np.array_equal(slots[0][keep], old[keep])
    assert (np.diff(slots[0][miss[0]]) > 0).all()  # misses placed in ascending id order


def test_topk_tie_rule():
    s = np.array([[0.5, 0.9, 0.9, 0.1, 0.9]], dtype=np.float32)
    assert np.array_equal(o.topk_set(s, 2), [[1, 2]])
    assert o.topk_tie_ok(s, np.array([[1, 4]]), 2)
    assert not o.topk_tie_ok(s, np.array([[0, 1]]), 2)


def test_batch_gemm_softmax_oracle_rows_sum_to_one():
    rng = np.random.default_rng(2)
    A = o.round_bf16(rng.standard_normal((2, 4, 128)).astype(np.float32))
    B = o.round_bf16(rng.standard_normal((2, 700, 128)).astype(np.float32))
    D, N, S, P = o.batch_gemm_softmax(A, B, 2, 4, 700, 128, 1 / np.sqrt(128))
    assert N.shape == (2, 3, 4)
    np.testing.assert_allclose(P.sum(-1), 1.0, atol=2e-2)
    ref = o.landmark_scores(A.reshape(2, 1, 4, 128), B.reshape(2, 1, 700, 128))
    np.testing.assert_allclose(P.max(1), ref[:, 0], atol=1e-2)


# ------------------------------------------------------------------ BASELINE configs[0]

def config0_inputs(d):
    """V and the RoPE table of the config-0 fixture, regenerated and checked against its digests."""
    import hashlib
    import torch
    from tests.golden.make_golden import config0_values, cos_sin_cache
    T, Hkv = int(d["T"]), int(d["Hkv"])
    v = config0_values(T, Hkv)
    assert hashlib.sha256(v.tobytes()).digest() == d["v_sha256"].tobytes(), "regenerated V differs"
    cs = cos_sin_cache(T + 1024).to(torch.bfloat16)[: T + 64]
    cs_bits = cs.view(torch.int16).numpy()
    assert hashlib.sha256(cs_bits.tobytes()).digest() == d["cos_sin_sha256"].tobytes(), "regenerated RoPE table differs"
    return v, cs_bits


@pytest.fixture(scope="module")
def config0_fix(golden_dir):
    return np.load(os.path.join(golden_dir, "torch_class_config0.npz"))


def test_config0_selection_matches_reference_torch_class(config0_fix):
    """BASELINE configs[0] (T=8192, budget 512, fp32) through models/kvcache/shadow.py:208-229:
    the oracle's chunk ids are the reference's, bit for bit, at every step."""
    d = config0_fix
    Hq, Hkv = int(d["Hq"]), int(d["Hkv"])
    lm, lidx = bf(d["k_landmark"]), d["k_landmark_idx"]
    K = int(d["budget"]) // 8
    assert K == 64 and lm.shape[2] == 1012
    for step in range(d["q"].shape[0]):
        q = d["q"][step][:, :, 0, :].reshape(1, Hkv, Hq // Hkv, 128)
        ids, _ = o.select_chunks(q, lm, lidx, K)
        assert np.array_equal(ids, np.sort(d["selected_chunk_idx"][step], axis=-1))


def test_config0_values_and_keys_match_reference_torch_class(config0_fix):
    """shadow.py:231-256 at config 0: gathered V bit-exact (checksum of the reference's rows),
    reconstructed keys of step 0 within 1e-4 (fp32)."""
    import hashlib
    d = config0_fix
    v, cs_bits = config0_inputs(d)
    for step in range(d["q"].shape[0]):
        sel = d["selected_chunk_idx"][step]
        tok = (sel[..., None] * 8 + np.arange(8)).reshape(1, sel.shape[1], -1)
        vg = np.ascontiguousarray(np.take_along_axis(v, tok[..., None], axis=2))
        assert hashlib.sha256(vg.tobytes()).digest() == d["v_sparse_sha256"][step].tobytes()
    U, SV = bf(d["U"]), bf(d["SV"])
    kr = o.reconstruct_keys_fp32(U, SV, d["selected_chunk_idx"][0], bf(cs_bits))
    np.testing.assert_allclose(kr, d["k_sparse0"], atol=1e-4, rtol=1e-4)
