"""The recorded binding trace of the reference's offload class, checked on the CPU.

``tests/golden/offload_class_trace.npz`` holds every ``kernels.shadowkv`` call that the
unmodified ``ShadowKVCache_CPU`` (models/kvcache/shadow.py:301-651) made during prefill and three
decode steps of two layers, with the oracle standing in for the library.  Replaying it through
the oracle on the rebuilt state must reproduce the recording's digests bit for bit, which pins
the fixture, the rebuilt state and the adapter before the GPU tests replay the same calls
through ``shadowkv_b200.shadowkv``.
"""
import os

import numpy as np
import pytest

from tests.golden import binding_trace as bt

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def trace():
    return np.load(os.path.join(HERE, "golden", "offload_class_trace.npz"))


def test_trace_covers_the_decode_bindings(trace):
    events, _ = bt.unpack(trace)
    cfg = bt.meta_of(trace)["config"]
    names = [e["name"] for e in events]
    per_layer_step = ["append", "batch_gemm_softmax", "reorder_keys_and_compute_offsets", "gather_copy_with_offsets",
                      "gather_copy_d2d_with_offsets", "batch_gather_gemm", "apply_rotary_pos_emb_push_cache_opt"]
    assert names == per_layer_step * (cfg["L"] * cfg["steps"])


def test_oracle_replay_reproduces_the_recording(trace):
    state = bt.build_state(trace, "cpu", pin=False)
    hits = []

    def call(i, name, args, digests):
        for k, t in bt.oracle_outputs(name, args).items():
            args[k].copy_(t)
            assert bt.digest(args[k]) == digests[k], f"event {i} {name} argument {k}"
        if name == "reorder_keys_and_compute_offsets":
            hits.append(args[3].clone())

    bt.replay(trace, state, "cpu", call)
    final = bt.meta_of(trace)["final"]
    for n, dg in final.items():
        assert bt.digest(state[n]) == dg, n
    h = np.stack([x.numpy() for x in hits])
    # the trace exercises hits and misses: every block keeps some chunks and fetches others
    assert (h > 0).all() and (h < 128).all(), h
