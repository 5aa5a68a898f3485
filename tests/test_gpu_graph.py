"""The captured multi-layer decode step (``graph.DecodeGraph``) against eager steps.

Several layers at the Llama-3-8B head layout (32 q / 8 kv heads, rank 160, budget 2048; a
shorter context keeps the test quick), several tokens in a row: the graph is captured on the
first step and replayed, the append position advancing on the device.  Every step's outputs and
the state it leaves (K/V buffers, slot tables) must equal, bit for bit, the same steps run
eagerly through ``decode_step_fused`` one layer at a time -- also with the early value fetch
(selection kernels that fetch the misses and compute the attention, reading the position from
the device).
"""
import dataclasses

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _bits(t):
    return t.contiguous().view(torch.int16)


@pytest.mark.parametrize("chain,early", [(False, False), (True, False), (True, True)])
def test_graph_replays_match_eager_steps(chain, early):
    from shadowkv_b200 import decode as fz
    before = fz.early_fetch(early)
    try:
        _graph_vs_eager(chain)
    finally:
        fz.early_fetch(before)


def _graph_vs_eager(chain):
    from shadowkv_b200 import workload
    from shadowkv_b200._lib import device_errors
    from shadowkv_b200.graph import DecodeGraph
    cfg = dataclasses.replace(workload.CONFIGS["config1"], ctx=16384, layers=3)
    layer = workload.Layer(cfg, device=DEV, seed=21)
    kv, attn = layer.cache, layer.attn
    L, B, Hq = cfg.layers, cfg.batch, cfg.q_heads
    steps = 4
    inputs = [[layer.next_inputs() for _ in range(L)] for _ in range(steps)]
    snap = [(kv.k_cache_buffer[l].clone(), kv.v_cache_buffer[l].clone(), kv.slots[l].clone()) for l in range(L)]
    g0, o0 = kv.gen_offset, kv.kv_offset

    # eager: layer by layer, step by step
    ref = []
    for s in range(steps):
        pos = torch.full((B,), cfg.ctx + s, dtype=torch.int64, device=DEV)
        outs = []
        for l in range(L):
            q = inputs[s][l][0] if (l == 0 or not chain) else outs[-1].view(B, Hq, 1, 128)
            o = kv.decode_step_fused(l, q, inputs[s][l][1], inputs[s][l][2], pos, attn.cos_sin_cache)
            outs.append(o.clone())
        ref.append(torch.stack(outs))
    torch.cuda.synchronize()
    assert device_errors()[0] == 0
    ref_state = [(kv.k_cache_buffer[l].clone(), kv.v_cache_buffer[l].clone(), kv.slots[l].clone()) for l in range(L)]
    assert kv.gen_offset == g0 + steps

    # the same steps through the captured graph
    for l in range(L):
        kv.k_cache_buffer[l].copy_(snap[l][0])
        kv.v_cache_buffer[l].copy_(snap[l][1])
        kv.slots[l].copy_(snap[l][2])
    kv.gen_offset, kv.kv_offset = g0, o0
    graph = DecodeGraph(attn, chain=chain)
    try:
        for s in range(steps):
            pos = torch.full((B,), cfg.ctx + s, dtype=torch.int64, device=DEV)
            q = torch.stack([x[0] for x in inputs[s]])
            k = torch.stack([x[1] for x in inputs[s]])
            v = torch.stack([x[2] for x in inputs[s]])
            out = graph.step(q, k, v, pos)
            torch.cuda.synchronize()
            assert torch.equal(_bits(out), _bits(ref[s])), f"outputs of step {s}"
        assert device_errors()[0] == 0
        assert graph.graph is not None and kv.gen_offset == g0 + steps
        assert int(graph.row.item()) == kv.sparse_end + kv.gen_offset
        for l in range(L):
            assert torch.equal(_bits(kv.k_cache_buffer[l]), _bits(ref_state[l][0])), f"K buffer, layer {l}"
            assert torch.equal(_bits(kv.v_cache_buffer[l]), _bits(ref_state[l][1])), f"V buffer, layer {l}"
            assert torch.equal(kv.slots[l], ref_state[l][2]), f"slots, layer {l}"
    finally:
        graph.close()
