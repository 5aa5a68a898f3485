"""GPU: attention output gathered over peer memory (kv heads split over ranks).

Two ranks are emulated in one process on one GPU: each has its own decode
state (half of the kv heads), both landing buffers live on this GPU, and every
launch goes to one stream (both merges, then both finishes), so a finish only
ever waits for arrivals that stream order has already completed.  The real
two-process, two-GPU run is ``tests/multi_gpu_peer_check.py``.
"""
import copy

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy()


def test_peer_gather_matches_local_outputs_over_steps():
    from shadowkv_b200 import workload
    from shadowkv_b200.peer import PeerOutput
    base = copy.deepcopy(workload.CONFIGS["tiny"])
    world = 2
    cfg = copy.deepcopy(base)
    cfg.kv_heads, cfg.q_heads = base.kv_heads // world, base.q_heads // world
    B, qn, Hq = cfg.batch, cfg.q_heads, base.q_heads
    ranks = [workload.Layer(cfg, device=DEV, seed=20 + r) for r in range(world)]
    twins = [workload.Layer(cfg, device=DEV, seed=20 + r) for r in range(world)]
    peers = PeerOutput.in_process(B, Hq, [r * qn for r in range(world)], merges_per_step=B * base.kv_heads)
    outs = [torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=DEV) for _ in range(world)]
    from shadowkv_b200._lib import device_errors
    device_errors()  # clear
    try:
        for step in range(5):
            refs = []
            for r in range(world):
                torch.manual_seed(100 * step + r)
                q, k, v = ranks[r].next_inputs()
                pos = torch.full((B, 1), ranks[r].cache.sparse_end + 300 + step, dtype=torch.int64, device=DEV)
                for lay, gather in ((ranks[r], True), (twins[r], False)):
                    c, attn = lay.cache, lay.attn
                    c.fused_geometry(attn.cos_sin_cache)
                    c.gen_offset = 0
                    qr = c.append_select_fused(0, q, k, v, pos, attn.cos_sin_cache)
                    sl = c.sparse_end + c._gen_offset(0)
                    if gather:
                        c.sparse_attention_gather(0, qr, sl, attn.cos_sin_cache, peers[r])
                    else:
                        refs.append(c.sparse_attention_fused(0, qr, sl, attn.cos_sin_cache))
                    c.gen_offset = 0
            for r in range(world):
                peers[r].finish(outs[r])
            torch.cuda.synchronize()
            for r in range(world):
                assert np.array_equal(bits(outs[r]), bits(outs[0])), (step, r)
                assert np.array_equal(bits(outs[0][:, r * qn:(r + 1) * qn]), bits(refs[r])), (step, r)
        assert device_errors()[0] == 0
    finally:
        for p in peers:
            p.close()


def test_peer_gather_rejects_bad_descriptions():
    from shadowkv_b200.peer import PeerOutput
    with pytest.raises(RuntimeError):
        PeerOutput(1, 8, 0, 2, 0, [0] * 9, 0)  # more ranks than supported
    p = PeerOutput.in_process(1, 8, [0, 4], merges_per_step=2)
    try:
        with pytest.raises(RuntimeError):
            p[0].finish(torch.empty(1, 4, 128, dtype=torch.bfloat16, device=DEV))  # wrong output shape
    finally:
        for x in p:
            x.close()


def test_finish_wait_runs_out_and_reports_a_status():
    """Nothing raises the arrival counter: the finish kernel's bounded wait runs out, a wait
    error is counted for the host to read, and the context stays usable.  The block's status
    is sticky: that finish copied nothing, the next finish returns at once without waiting or
    copying, and ``check`` raises until the blocks are re-created."""
    import time
    from shadowkv_b200._lib import ShadowKVError, device_errors
    from shadowkv_b200.peer import PeerOutput
    device_errors()  # clear
    (p,) = PeerOutput.in_process(1, 8, [0], merges_per_step=2)
    try:
        assert p.status() == 0
        p.check()
        out = torch.full((1, 8, 128), 7.0, dtype=torch.bfloat16, device=DEV)
        t0 = time.time()
        p.finish(out)  # no attention launch: the counter stays at zero
        torch.cuda.synchronize()
        waited = time.time() - t0
        assert device_errors() == (1, 4)  # one DEV_ERR_WAIT
        assert waited < 60
        assert p.status() == 4
        assert bool((out.float() == 7.0).all()), "a timed-out finish copies nothing"
        with pytest.raises(ShadowKVError):
            p.check()
        t0 = time.time()
        p.finish(out)  # stopped block: returns at once
        torch.cuda.synchronize()
        assert time.time() - t0 < 0.5 * max(waited, 0.2)
        assert device_errors() == (0, 0) and bool((out.float() == 7.0).all())
    finally:
        p.close()
    x = torch.arange(1024, device=DEV, dtype=torch.float32)
    assert float(x.sum().item()) == 1023 * 1024 / 2
    assert device_errors() == (0, 0)
