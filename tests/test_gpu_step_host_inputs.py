"""The one-call step reading its inputs from page-locked host memory.

``q``, ``k_new``, ``v_new`` and ``positions`` given as page-locked CPU tensors are read over the
host link by a staging kernel at the start of the step.  Output and state must equal, bit for
bit, the same step on device inputs: eagerly (4 and 1 kv-head groups, an input only 8-byte
aligned) and replayed from a graph captured on host buffers that are refilled between replays.
"""
import dataclasses

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _bits(t):
    return t.contiguous().view(torch.int16)


def _pinned_like(t, offset_bytes=0):
    """A page-locked CPU copy of t whose data starts offset_bytes into its allocation."""
    n = t.numel() * t.element_size()
    raw = torch.zeros(n + 16, dtype=torch.uint8).pin_memory()
    view = raw[offset_bytes:offset_bytes + n].view(t.dtype).view(t.shape)
    view.copy_(t.cpu())
    return view


@pytest.fixture(scope="module")
def layer():
    from shadowkv_b200 import workload
    cfg = dataclasses.replace(workload.CONFIGS["config1"], ctx=16384)
    return workload.Layer(cfg, device=DEV, seed=9)


def _runner(layer):
    kv, attn, cfg = layer.cache, layer.attn, layer.cfg
    snap = (kv.k_cache_buffer[0].clone(), kv.v_cache_buffer[0].clone(), kv.slots[0].clone())
    g0 = kv.gen_offset

    def restore():
        kv.k_cache_buffer[0].copy_(snap[0])
        kv.v_cache_buffer[0].copy_(snap[1])
        kv.slots[0].copy_(snap[2])
        kv.gen_offset = g0

    def state():
        return kv.k_cache_buffer[0].clone(), kv.v_cache_buffer[0].clone(), kv.slots[0].clone()

    def step(q, k, v, pos, groups, out):
        kv.decode_step_fused(0, q, k, v, pos, attn.cos_sin_cache, out=out, head_groups=groups)

    return kv, cfg, restore, state, step


@pytest.mark.parametrize("groups", [4, 1])
def test_host_inputs_match_device_inputs(layer, groups):
    from shadowkv_b200._lib import device_errors
    kv, cfg, restore, state, step = _runner(layer)
    q, k, v = layer.next_inputs()
    pos = torch.full((1,), cfg.ctx, dtype=torch.int64, device=DEV)
    out = torch.empty(1, cfg.q_heads, 128, dtype=torch.bfloat16, device=DEV)
    restore()
    step(q, k, v, pos, groups, out)
    torch.cuda.synchronize()
    ref_out, ref_state = out.clone(), state()
    # host inputs; q only 8-byte aligned (8-byte pieces), the others 16-byte aligned
    for q_off in (0, 8):
        restore()
        out.zero_()
        step(_pinned_like(q, q_off), _pinned_like(k), _pinned_like(v), _pinned_like(pos), groups, out)
        torch.cuda.synchronize()
        assert torch.equal(_bits(out), _bits(ref_out)), f"output, q offset {q_off}"
        for a, b in zip(state(), ref_state):
            assert torch.equal(a, b)
    assert device_errors()[0] == 0
    restore()


def test_graph_on_host_buffers_reads_each_replays_inputs(layer):
    from shadowkv_b200._lib import device_errors
    kv, cfg, restore, state, step = _runner(layer)
    steps = [layer.next_inputs() for _ in range(2)]
    pos = torch.full((1,), cfg.ctx, dtype=torch.int64, device=DEV)
    out = torch.empty(1, cfg.q_heads, 128, dtype=torch.bfloat16, device=DEV)
    refs = []
    for q, k, v in steps:
        restore()
        step(q, k, v, pos, 4, out)
        torch.cuda.synchronize()
        refs.append((out.clone(), state()))
    hq, hk, hv, hp = (_pinned_like(t) for t in (steps[0][0], steps[0][1], steps[0][2], pos))
    restore()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step(hq, hk, hv, hp, 4, out)
    try:
        for (q, k, v), (ref_out, ref_state) in zip(reversed(steps), reversed(refs)):
            hq.copy_(q.cpu()), hk.copy_(k.cpu()), hv.copy_(v.cpu())
            restore()
            out.zero_()
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(_bits(out), _bits(ref_out))
            for a, b in zip(state(), ref_state):
                assert torch.equal(a, b)
    finally:
        del g
    assert device_errors()[0] == 0
    restore()


def test_unpinned_host_input_is_rejected(layer):
    from shadowkv_b200._lib import ShadowKVError
    kv, cfg, restore, state, step = _runner(layer)
    q, k, v = layer.next_inputs()
    pos = torch.full((1,), cfg.ctx, dtype=torch.int64, device=DEV)
    out = torch.empty(1, cfg.q_heads, 128, dtype=torch.bfloat16, device=DEV)
    with pytest.raises((ShadowKVError, RuntimeError), match="page-locked"):
        step(q.cpu(), k, v, pos, 4, out)  # pageable memory: refused before any launch
    restore()
