"""The one-call decode step (``skv_decode_step``), plain and pipelined over kv-head groups.

It must leave exactly the state of ``append_select`` + ``sparse_attention`` (the two-call
fused path that the other tests check against the oracle): same slots, same K/V buffer bits,
same rotated query, same miss counts -- for every head grouping, with the early value fetch
(the selection kernel fetching the missed rows and computing the attention) on and off, over
several steps (so later steps hit the reuse cache the earlier ones filled); also when the
selection concentrates in one selection CTA's landmarks, whose certain misses then exceed its
staging area and are fetched in several rounds, and for a batch of sequences.  The attention
output is the same bits without the early fetch; with it the rows are split into partials
differently (per selection CTA, 32-row tiles) and the output agrees up to fp32 summation
order and the rounding of the softmax weights to bf16: within 2^-6 relative + 2e-3.
"""
import dataclasses

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _layer(name, **kw):
    from shadowkv_b200 import workload
    cfg = dataclasses.replace(workload.CONFIGS[name], **kw)
    return workload.Layer(cfg, device=DEV, seed=7)


def _run(layer, inputs, mode, head_groups=None):
    """Steps of one layer from the same start state; returns per-step outputs and the final state."""
    cache, attn = layer.cache, layer.attn
    B, Hq = layer.cfg.batch, layer.cfg.q_heads
    outs = []
    cache.gen_offset = 0
    for i, (q, k, v) in enumerate(inputs):
        pos = torch.full((B,), layer.cfg.ctx + i, dtype=torch.int64, device=DEV)
        q_out = torch.empty(B, Hq, 1, 128, dtype=torch.bfloat16, device=DEV)
        out = torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=DEV)
        if mode == "two_calls":
            cache.append_select_fused(0, q, k, v, pos, attn.cos_sin_cache, q_out=q_out)
            seq_len = cache.sparse_end + cache._gen_offset(0)
            cache.sparse_attention_fused(0, q_out, seq_len, attn.cos_sin_cache, out=out)
            misses = cache._fused_ws.miss_count.clone()
        else:
            cache.decode_step_fused(0, q, k, v, pos, attn.cos_sin_cache, out=out, head_groups=head_groups,
                                    q_out=q_out)
            misses = cache._step_ws.miss_count.clone()
        outs.append((q_out.clone(), out.clone(), misses))
    torch.cuda.synchronize()
    return outs, (cache.k_cache_buffer[0].clone(), cache.v_cache_buffer[0].clone(), cache.slots[0].clone())


def _compare_paths(layer, inputs, groups):
    from shadowkv_b200 import decode as fz
    from shadowkv_b200._lib import device_errors
    cache = layer.cache
    start = (cache.k_cache_buffer[0].clone(), cache.v_cache_buffer[0].clone(), cache.slots[0].clone())

    def restore():
        cache.k_cache_buffer[0].copy_(start[0])
        cache.v_cache_buffer[0].copy_(start[1])
        cache.slots[0].copy_(start[2])

    ref_outs, ref_state = _run(layer, inputs, "two_calls")
    assert device_errors()[0] == 0
    before = fz.early_fetch(False)
    try:
        for early in (True, False):
            fz.early_fetch(early)
            for p in groups:
                restore()
                outs, state = _run(layer, inputs, "step", head_groups=p)
                assert device_errors()[0] == 0
                tag = f"groups {p}, early fetch {early}"
                for s, ((qr, o, m), (qr2, o2, m2)) in enumerate(zip(ref_outs, outs)):
                    assert torch.equal(qr.view(torch.int16), qr2.view(torch.int16)), f"rotated query, step {s}, {tag}"
                    if early:
                        err = (o2.float() - o.float()).abs()
                        assert (err <= o.float().abs() * 2.0 ** -6 + 2e-3).all(), f"output, step {s}, {tag}"
                    else:
                        assert torch.equal(o.view(torch.int16), o2.view(torch.int16)), f"output, step {s}, {tag}"
                    assert torch.equal(m, m2), f"miss counts, step {s}, {tag}"
                assert torch.equal(state[2], ref_state[2]), f"slots, {tag}"
                assert torch.equal(state[0].view(torch.int16), ref_state[0].view(torch.int16)), f"K buffer, {tag}"
                assert torch.equal(state[1].view(torch.int16), ref_state[1].view(torch.int16)), f"V buffer, {tag}"
    finally:
        fz.early_fetch(before)
    return ref_outs


@pytest.mark.parametrize("name,kw,groups", [
    ("tiny", {}, [1, 2]),
    # Llama-3-8B head layout (32 q / 8 kv heads) at a shorter context
    ("config1", {"ctx": 16384}, [1, 2, 4, 8]),
    # GLM partial rotary, 32 q / 2 kv heads
    ("config3", {"ctx": 16384}, [1, 2]),
    # a batch of sequences (head groups need batch 1)
    ("config1", {"ctx": 8192, "batch": 3}, [1]),
])
def test_step_matches_two_call_path(name, kw, groups):
    layer = _layer(name, **kw)
    inputs = [layer.next_inputs() for _ in range(3)]
    ref_outs = _compare_paths(layer, inputs, groups)
    # the later steps hit the reuse cache (the same query stream is not required for that:
    # consecutive random queries share part of their selection)
    assert int(ref_outs[0][2].sum()) > 0


def test_step_with_selection_in_one_cta_slice():
    """Landmarks of the first eighth of each head scaled up: the top-k falls mostly into the
    first selection CTA's slice, whose certain misses exceed its staging area (several rounds)."""
    layer = _layer("config1", ctx=32768)
    cache = layer.cache
    lm = cache.k_landmark[0]                       # [B, Hkv, L, 128]
    L = lm.shape[-2]
    lm[..., : (L + 7) // 8, :] *= 3
    inputs = [layer.next_inputs() for _ in range(2)]
    _compare_paths(layer, inputs, [1, 4])


def test_step_rejects_bad_groups():
    from shadowkv_b200 import decode as fz
    from shadowkv_b200._lib import ShadowKVError
    layer = _layer("tiny")
    g = layer.cache.fused_geometry(layer.attn.cos_sin_cache)
    with pytest.raises(ShadowKVError):
        fz.StepWorkspace(g, 3, DEV)  # 3 does not divide 2 kv heads
    gb = dataclasses.replace(g, batch=2)
    with pytest.raises(ShadowKVError):
        fz.StepWorkspace(gb, 2, DEV)  # head groups need batch 1
