"""The unmodified reference offload class's binding calls, replayed through the drop-in module.

``tests/golden/offload_class_trace.npz`` is a recording of ``ShadowKVCache_CPU``
(models/kvcache/shadow.py:301-651, with the binding wrappers of models/tensor_op.py:176-243)
running prefill and three decode steps of two layers, made by ``tests/golden/make_golden.py``
with the reference checkout (which is not present where the GPU tests run).  Every call it made
to ``kernels.shadowkv`` -- same binding, same positional arguments, the same views of the same
cache tensors, the same temporaries -- is made here to ``shadowkv_b200.shadowkv`` on the rebuilt
GPU state, in order:

* each call's outputs against the oracle applied to the GPU's own state just before the call:
  bit-exact for the reuse-cache diff, both gathers and the RoPE push; within one bf16 ulp for
  the two GEMMs (fp32 accumulation order);
* the outputs that do not depend on floating-point rounding (the reordered chunk ids, offsets,
  hit counts, the V buffers, and after the last step their final state) against the digests
  the recording took of the reference class's own tensors;
* the chunks the class chose from the oracle's softmax are a valid top-k of the scores this
  library's ``batch_gemm_softmax`` produced (up to one bf16 ulp of near-ties).
"""
import os

import numpy as np
import pytest
import torch

from oracle import shadowkv_oracle as o
from tests.golden import binding_trace as bt

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
HERE = os.path.dirname(os.path.abspath(__file__))

# outputs whose recorded digests must match: integer results, and buffers of copied bf16 rows
EXACT_DIGESTS = {"reorder_keys_and_compute_offsets": (0, 2, 3), "gather_copy_with_offsets": (1,)}


def _bits(t):
    return bt.bits(t)


def test_reference_offload_class_trace_on_the_bindings():
    from shadowkv_b200 import shadowkv as skv
    from shadowkv_b200._lib import device_errors
    d = np.load(os.path.join(HERE, "golden", "offload_class_trace.npz"))
    cfg = bt.meta_of(d)["config"]
    state = bt.build_state(d, DEV, pin=True)
    assert state["v_cache_cpu"].is_pinned()
    torch.cuda.synchronize()
    G = cfg["Hq"] // cfg["Hkv"]
    budget_chunks = cfg["budget"] // 8
    pending_scores = {}
    seen = {n: 0 for n in bt.BINDINGS}

    def call(i, name, args, digests):
        pre = [a.detach().cpu().clone() if isinstance(a, torch.Tensor) else a for a in args]
        getattr(skv, name)(*args)
        torch.cuda.synchronize()
        assert device_errors()[0] == 0, f"event {i} {name}"
        expect = bt.oracle_outputs(name, pre)
        got = {k: args[k].detach().cpu() for k in expect}
        if name == "batch_gemm_softmax":
            batch, m, n = args[6], args[7], args[8]
            eD, gD = expect[2].float().numpy(), got[2].float().numpy()
            assert (np.abs(gD - eD) <= np.abs(eD) * 2.0 ** -7 + 1e-6).all(), f"event {i}: D"
            nblk = (n + 255) // 256
            eN, gN = expect[3].numpy().reshape(batch, nblk, m), got[3].numpy().reshape(batch, nblk, m)
            eS, gS = expect[4].numpy().reshape(batch, nblk, m), got[4].numpy().reshape(batch, nblk, m)
            np.testing.assert_allclose(gN, eN, rtol=1e-4, atol=1e-4)
            np.testing.assert_allclose(gS[:, 0], eS[:, 0], rtol=1e-3)
            # the softmax is computed from the bf16 D this call wrote
            gP = got[5].float().numpy().reshape(batch, m, n)
            ep = o.round_bf16((np.exp(gD.reshape(batch, m, n).astype(np.float64) - eN[:, 0][:, :, None])
                               * eS[:, 0][:, :, None].astype(np.float64)).astype(np.float32))
            np.testing.assert_allclose(gP, ep, rtol=1e-2, atol=1e-6)
            pending_scores["scores"] = gP.reshape(batch, G, n).max(axis=1)        # [B*Hkv, n]
        elif name in ("batch_gather_gemm",):
            e, g = expect[5].float().numpy(), got[5].float().numpy()
            assert (np.abs(g - e) <= np.abs(e) * 2.0 ** -7 + 1e-5).all(), f"event {i}: reconstruction"
        else:
            for k in expect:
                assert np.array_equal(_bits(got[k]), _bits(expect[k])), f"event {i} {name} argument {k}"
        for k in EXACT_DIGESTS.get(name, ()):
            assert bt.digest(got[k]) == digests[k], f"event {i} {name} argument {k} differs from the recording"
        if name == "reorder_keys_and_compute_offsets":
            # the reference class chose these chunk ids (topk over the max of the group's softmax,
            # models/kvcache/shadow.py:567-573) from the oracle's scores: they must be a top-k of ours
            scores = pending_scores.pop("scores")
            chosen_ids = pre[1].numpy().reshape(scores.shape[0], -1)
            layer = i // 7 % cfg["L"]
            lidx = state["k_landmark_idx"][layer].cpu().numpy().reshape(scores.shape[0], -1)
            chosen = np.stack([np.nonzero(np.isin(lidx[r], chosen_ids[r]))[0] for r in range(scores.shape[0])])
            assert o.topk_tie_ok(scores, chosen, budget_chunks, rtol=2.0 ** -6), f"event {i}: selection"
        seen[name] += 1

    bt.replay(d, state, DEV, call)
    assert all(v == cfg["L"] * cfg["steps"] for v in seen.values()), seen
    final = bt.meta_of(d)["final"]
    for n in ("position_ids", "offsets", "cnts", "v_cache_buffer"):
        assert bt.digest(state[n]) == final[n], f"final {n} differs from the recording"
