"""Kernel timing of the one-call step (``skv_decode_step_timing``).

With timing on, the step's kernels stamp the GPU's global timer at every CTA's start and end
into a span pair per (kv-head group, kernel).  Its outputs and the state it leaves must equal,
bit for bit, the step without timing -- eagerly and replayed from a graph captured with timing
on -- and per group the spans must follow the kernels' order (scoring, selection, attention,
each starting after the one before it ended).
"""
import dataclasses

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
GROUPS = 4


def _bits(t):
    return t.contiguous().view(torch.int16)


def test_step_timing_leaves_results_unchanged_and_orders_the_events():
    from shadowkv_b200 import decode as fz
    from shadowkv_b200 import workload
    from shadowkv_b200._lib import ShadowKVError, device_errors
    cfg = dataclasses.replace(workload.CONFIGS["config1"], ctx=16384)
    layer = workload.Layer(cfg, device=DEV, seed=5)
    kv, attn = layer.cache, layer.attn
    q, k, v = layer.next_inputs()
    pos = torch.full((1,), cfg.ctx, dtype=torch.int64, device=DEV)
    snap = (kv.k_cache_buffer[0].clone(), kv.v_cache_buffer[0].clone(), kv.slots[0].clone())
    g0 = kv.gen_offset
    out = torch.empty(1, cfg.q_heads, 128, dtype=torch.bfloat16, device=DEV)

    def restore():
        kv.k_cache_buffer[0].copy_(snap[0])
        kv.v_cache_buffer[0].copy_(snap[1])
        kv.slots[0].copy_(snap[2])
        kv.gen_offset = g0

    def state():
        return kv.k_cache_buffer[0].clone(), kv.v_cache_buffer[0].clone(), kv.slots[0].clone()

    def eager(timing):
        restore()
        prev = fz.step_timing(timing)
        try:
            kv.decode_step_fused(0, q, k, v, pos, attn.cos_sin_cache, out=out, head_groups=GROUPS)
        finally:
            fz.step_timing(prev)
        torch.cuda.synchronize()
        return out.clone(), state()

    def check_times():
        t = fz.step_kernel_times()
        assert len(t) == GROUPS
        for spans in t:
            assert None not in spans, t
            assert all(a <= b for a, b in zip(spans, spans[1:])), t
        assert min(x[0] for x in t) == 0.0
        return t

    ref_out, ref_state = eager(False)
    got_out, got_state = eager(True)
    assert torch.equal(_bits(got_out), _bits(ref_out))
    for a, b in zip(got_state, ref_state):
        assert torch.equal(a, b)
    check_times()

    # captured with timing on: every replay records the events again
    restore()
    prev = fz.step_timing(True)
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            kv.decode_step_fused(0, q, k, v, pos, attn.cos_sin_cache, out=out, head_groups=GROUPS)
    finally:
        fz.step_timing(prev)
    try:
        for _ in range(2):
            restore()
            out.zero_()
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(_bits(out), _bits(ref_out))
            for a, b in zip(state(), ref_state):
                assert torch.equal(a, b)
            check_times()
    finally:
        del g
    assert device_errors()[0] == 0

    # the read cleared the spans, and an untimed step stamps nothing
    eager(False)
    with pytest.raises(ShadowKVError, match="no kernel of a timed step has run"):
        fz.step_kernel_times()
