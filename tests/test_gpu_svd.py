"""The rank-r factorisation of the prompt keys (ShadowKVCache_CPU.get_svd,
models/kvcache/shadow.py:411-444) through the library's tensor-core Gram kernel.

* ``skv_gram`` against K^T K computed by torch in float64 (ragged row counts, config1 size);
* the cache's factors from the Gram path reconstruct the keys as well as the reference's own
  method (``torch.svd`` of K in fp32, rank 160, factors stored in bf16) at config1 shapes.
"""
import math
import types

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _keys(T, D, r_true, seed):
    """Pre-RoPE keys as the benchmark builds them: U0 W0 + 0.05 N(0, 1), bf16."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    U0 = torch.randn(T, r_true, generator=g, device=DEV)
    W0 = torch.randn(r_true, D, generator=g, device=DEV) / math.sqrt(math.sqrt(r_true))
    return (U0 @ W0 + 0.05 * torch.randn(T, D, generator=g, device=DEV)).to(torch.bfloat16)


# (5, 384): one 64-row slice with 59 rows past the end of K (zero-filled by the tensor copies),
# three column blocks; (64, 128): exactly one slice, the diagonal block only
@pytest.mark.parametrize("T,D", [(5000, 256), (777, 128), (122880, 1024), (5, 384), (64, 128)])
def test_gram_matches_float64(T, D):
    from shadowkv_b200 import decode
    from shadowkv_b200._lib import device_errors
    k = _keys(T, D, 32, seed=T)
    G = decode.gram(k)
    torch.cuda.synchronize()
    assert device_errors()[0] == 0
    kd = k.double()
    ref = kd.T @ kd
    assert torch.equal(G, G.T), "both triangles carry the same sums"
    # bf16 products are exact in fp32; the tensor cores accumulate a slice of up to ~30K rows in
    # fp32 (relative error growing with the slice), the slices are summed in float64
    rel = (torch.linalg.norm(G - ref) / torch.linalg.norm(ref)).item()
    assert rel < 1e-4, rel


def test_gram_of_strided_rows():
    """The first D columns of rows with a larger stride (ld > D)."""
    from shadowkv_b200 import decode
    k = _keys(3000, 512, 16, seed=3)
    G = decode.gram(k[:, :256])
    kd = k[:, :256].double()
    ref = kd.T @ kd
    assert (torch.linalg.norm(G - ref) / torch.linalg.norm(ref)).item() < 1e-4


def test_gram_factors_reconstruct_keys_like_the_svd():
    """config1 shapes: T = 122880, 8 kv heads x 128 = 1024 columns, true rank 96, rank 160."""
    from shadowkv_b200.kvcache import ShadowKVCache_CPU
    T, H, rank = 122880, 8, 160
    k = _keys(T, H * 128, 96, seed=1)
    cfg = types.SimpleNamespace(num_attention_heads=32, num_key_value_heads=H, hidden_size=32 * 128,
                                num_hidden_layers=1)
    errs = {}
    for method in ("exact", "gram"):
        c = ShadowKVCache_CPU(cfg, batch_size=1, max_length=T, device=DEV, sparse_budget=2048, rank=rank,
                              outlier_chunk=48, svd=method)
        c.get_svd(k.view(1, T, H * 128), layer_idx=0)
        U = c.U[0][0].float()                                                     # [T, r]
        SV = c.SV[0][0].float().permute(2, 0, 1).reshape(rank, H * 128)           # [r, H*128]
        rec = U @ SV
        errs[method] = (torch.linalg.norm(rec - k.float()) / torch.linalg.norm(k.float())).item()
        del c
        torch.cuda.empty_cache()
    assert errs["gram"] <= errs["exact"] * 1.01 + 1e-4, errs


@pytest.mark.parametrize("h0,hn", [(0, 1), (3, 1), (4, 4)])
def test_factors_of_a_head_range_are_the_full_factors_rows(h0, hn):
    """kv heads sharded over GPUs: a cache of heads h0 .. h0+hn-1 factorises the keys of all
    8 heads (as the reference does, U shared) and keeps U and its heads' rows of SV -- bit for bit
    the full cache's U and SV[h0 : h0+hn].  Rank 160 exceeds one head's 128 columns."""
    from shadowkv_b200.kvcache import ShadowKVCache_CPU
    T, H, rank = 8192, 8, 160
    k = _keys(T, H * 128, 96, seed=5).view(1, T, H, 128).transpose(1, 2).contiguous()  # [1, H, T, 128]

    def cache(heads):
        cfg = types.SimpleNamespace(num_attention_heads=4 * heads, num_key_value_heads=heads,
                                    hidden_size=4 * heads * 128, num_hidden_layers=1)
        return ShadowKVCache_CPU(cfg, batch_size=1, max_length=T, device=DEV, sparse_budget=512, rank=rank,
                                 outlier_chunk=8, svd="gram")

    full, part = cache(H), cache(hn)
    full.get_svd(k, 0)
    part.get_svd(k, 0, heads=(h0, hn))
    assert torch.equal(part.U, full.U)
    assert torch.equal(part.SV[0][0], full.SV[0][0][h0:h0 + hn])
    with pytest.raises(RuntimeError):
        cache(hn).get_svd(k, 0, heads=(H - hn + 1, hn))  # past the last head
