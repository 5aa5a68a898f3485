"""CPU reference arm of bench.py (``--impl reference``) -- test infrastructure.

Times the oracle port of the reference's torch-eager ShadowKV decode step
(models/kvcache/shadow.py:208-259 + the attention of
models/attention/shadow.py:48) on the host cores, on the benchmark's
configuration.  The decode state is built here with numpy from the same
seeded recipe as the GPU workload (low-rank pre-RoPE keys + noise, rank-r
factorisation, chunk-mean landmarks, outlier chunks, first selection); it
does not use the shadowkv_b200 package.

Each timed step is one full decode step of one layer for the whole batch:
scoring of every landmark, top-k, value gather, key reconstruction with
RoPE and GQA attention.
"""
from __future__ import annotations

import math
import os
import statistics
import time

import numpy as np

from . import shadowkv_oracle as o

CONFIGS = {
    "config0": dict(ctx=8192, q_heads=8, kv_heads=2, r_true=32, rank=64, budget=512, outliers=8),
    "config1": dict(ctx=122880, q_heads=32, kv_heads=8, r_true=96, rank=160, budget=2048, outliers=48),
    "tiny": dict(ctx=2048, q_heads=8, kv_heads=2, r_true=16, rank=64, budget=256, outliers=8),
}


def cos_sin_table(n: int, theta: float = 500000.0, dim: int = 128) -> np.ndarray:
    inv = 1.0 / (theta ** (np.arange(0, dim, 2, dtype=np.float32) / dim))
    ang = np.outer(np.arange(n, dtype=np.float32), inv)
    return o.round_bf16(np.concatenate([np.cos(ang), np.sin(ang)], axis=-1).astype(np.float32))


def build_state(name: str = "config1", seed: int = 0, gen_len: int = 128):
    """Numpy prefill of one layer, B = 1, with torch-class geometry (32-token local window)."""
    c = CONFIGS[name]
    T, Hq, Hk, r_true, rank = c["ctx"], c["q_heads"], c["kv_heads"], c["r_true"], c["rank"]
    budget, n_out, D, ch = c["budget"], c["outliers"], 128, 8
    rng = np.random.default_rng(seed)
    U0 = rng.standard_normal((T, r_true), dtype=np.float32)
    W0 = rng.standard_normal((r_true, Hk * D), dtype=np.float32) / np.float32(math.sqrt(math.sqrt(r_true)))
    k = U0 @ W0
    k += np.float32(0.05) * rng.standard_normal((T, Hk * D), dtype=np.float32)
    k = o.round_bf16(k)
    del U0
    v = o.round_bf16(rng.standard_normal((1, Hk, T, D), dtype=np.float32))
    # rank-r factorisation through the Gram matrix (same leading subspace as the SVD)
    gram = (k.T @ k).astype(np.float64)
    w, vec = np.linalg.eigh(gram)
    order = np.argsort(w)[::-1][:rank]
    s = np.sqrt(np.maximum(w[order], 0.0))
    Vr = vec[:, order]
    U = o.round_bf16(((k @ Vr.astype(np.float32)) / s.astype(np.float32)).astype(np.float32))[None]
    SV = o.round_bf16((s[:, None] * Vr.T).astype(np.float32)).reshape(rank, Hk, D).transpose(1, 0, 2)[None]
    cs = cos_sin_table(T + gen_len + 1024)
    kh = k.reshape(T, Hk, D).transpose(1, 0, 2)[None]
    k_roped = o.rope_torch_fp32(kh, cs, np.arange(T))
    chunks = T // ch - 4
    prefill_local = T - chunks * ch
    ctx = k_roped[:, :, : chunks * ch].reshape(1, Hk, chunks, ch, D)
    lm_all = ctx.mean(axis=3)
    num = (lm_all[:, :, :, None, :] * ctx).sum(-1)
    den = np.linalg.norm(lm_all, axis=-1)[:, :, :, None] * np.linalg.norm(ctx, axis=-1)
    cos_min = (num / np.maximum(den, 1e-8)).min(-1)
    outl = np.argsort(cos_min, axis=-1, kind="stable")[..., :n_out]
    mask = np.ones((1, Hk, chunks), bool)
    np.put_along_axis(mask, outl, False, axis=-1)
    rest = np.stack([np.nonzero(mask[0, h])[0] for h in range(Hk)])[None]
    lm = o.round_bf16(np.take_along_axis(lm_all, rest[..., None], axis=2))
    sparse_start = prefill_local + n_out * ch
    sparse_end = sparse_start + budget
    buf_len = sparse_end + gen_len
    k_buf = np.zeros((1, Hk, buf_len, D), np.float32)
    v_buf = np.zeros_like(k_buf)
    k_buf[:, :, :prefill_local] = k_roped[:, :, -prefill_local:]
    v_buf[:, :, :prefill_local] = v[:, :, -prefill_local:]
    og = (outl[..., None] * ch + np.arange(ch)).reshape(1, Hk, -1)
    k_buf[:, :, prefill_local:sparse_start] = np.take_along_axis(k_roped, og[..., None], axis=2)
    v_buf[:, :, prefill_local:sparse_start] = np.take_along_axis(v, og[..., None], axis=2)
    st = o.TorchPathDecodeState(k_landmark=lm, k_landmark_idx=rest.astype(np.int64), U=U, SV=SV, v_full=v,
                                k_buf=k_buf, v_buf=v_buf, cos_sin=cs, sparse_start=sparse_start,
                                sparse_end=sparse_end, select_sets=budget // ch)
    return st, c, rng


def run(args, world: int, rank: int):
    """Time ``--steps`` decode steps after ``--warmup``; returns the JSON record (rank 0 only)."""
    if rank != 0:
        return None
    name = args.config if args.config in CONFIGS else "config1"
    t0 = time.perf_counter()
    st, c, rng = build_state(name)
    setup_s = time.perf_counter() - t0
    Hq, D = c["q_heads"], 128
    cores = len(os.sched_getaffinity(0))
    times = []
    for i in range(args.warmup + args.steps):
        q = o.round_bf16(rng.standard_normal((1, Hq, D), dtype=np.float32))
        seq_len = st.sparse_end + 1
        st.k_buf[:, :, st.sparse_end] = o.round_bf16(rng.standard_normal((c["kv_heads"], D), dtype=np.float32))
        st.v_buf[:, :, st.sparse_end] = o.round_bf16(rng.standard_normal((c["kv_heads"], D), dtype=np.float32))
        t = time.perf_counter()
        o.torch_path_decode_step(st, q, seq_len)
        dt = time.perf_counter() - t
        if i >= args.warmup:
            times.append(dt)
    NL = max(1, int(getattr(args, "layers", 1)))
    ms = 1e3 * statistics.mean(times) * NL  # one layer's step time x the layers of the step
    value = 1.0 / (ms / 1e3)
    return {
        "impl": "reference",
        "metric": ("sparse-attn decode tokens/s (Llama-3-8B shape, 122k ctx)" if NL == 1 else
                   f"sparse-attn decode tokens/s ({NL} attention layers, Llama-3-8B shape, 122k ctx)"),
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded; BASELINE configs[1] shapes and distributions)",
        "config": {"workload": f"{name}: one decode layer, B=1, {c['q_heads']}q/{c['kv_heads']}kv heads, "
                               f"ctx {c['ctx']}, budget {c['budget']}, rank {c['rank']}",
                   "global_batch": 1, "seq_len": c["ctx"], "parallelism": "host cores of rank 0"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} full decode steps of the numpy port of the reference's "
                                   f"torch-eager path (state build {setup_s:.1f} s, untimed)"
                                   + (f"; one layer's time x {NL} layers" if NL > 1 else "")},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
