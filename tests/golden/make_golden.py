"""Generate golden fixtures by running the reference's own Python code.

Run in the build container only (it reads the read-only reference checkout):

    python tests/golden/make_golden.py --reference /path/to/ShadowKV

What it runs:

* ``ShadowKVCache`` -- the reference's torch-eager accuracy class
  (models/kvcache/shadow.py:27-298) -- on CPU in float32, through
  ``get_svd`` -> ``prefill_kv_cache`` -> (``update_kv_cache`` ->
  ``get_retrieval_position_ids`` -> ``get_value_cache`` -> ``get_key_cache``)
  for several decode steps.  ``kernels.shadowkv`` and ``models.tensor_op``
  are replaced by stubs (the real tensor_op allocates on CUDA at import,
  models/tensor_op.py:62); the RoPE function handed to ``get_key_cache`` is
  the reference's own ``apply_rotary_pos_emb_single`` / ``rotate_half``
  (models/tensor_op.py:132-156), extracted from the source file with ``ast``.
  Attention is not part of the class (flash-attn, models/attention/
  shadow.py:48); the fixture stores the K/V buffers and the tests compute it
  with the oracle.
* ``ShadowKVCache_CPU`` -- the reference's offload class (models/kvcache/
  shadow.py:301-651), unmodified, on CPU in bf16 through ``get_svd`` ->
  ``prefill_kv_cache`` -> ``H2D`` and several decode steps of every layer.
  Its ``kernels.shadowkv`` module is ``binding_trace.Recorder``, which
  records every binding call with its arguments and computes the outputs
  with the oracle; the two wrappers it calls in models/tensor_op.py
  (``batch_gather_gemm_rotary_pos_emb_cuda``, ``apply_rotary_pos_emb_cuda_
  push_cache``) are taken from the source file with ``ast``.  The trace is
  replayed through ``shadowkv_b200.shadowkv`` by the GPU tests.
* the same torch RoPE in bf16 (llama, rotate-half) and the GLM method
  ``apply_rotary_pos_emb_single`` (models/glm.py:207-230) in bf16, which pin
  the bf16 op-by-op arithmetic of the CUDA RoPE kernels.

Inputs are rounded to bf16-representable float32 values, and ``U``, ``SV``
and the landmarks are rounded after prefill, so the same values can be fed
to bf16 CUDA kernels.  Everything is seeded.
"""
from __future__ import annotations

import argparse
import ast
import importlib.util
import math
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
_ROOT = os.path.dirname(os.path.dirname(HERE))
if _ROOT not in sys.path:  # run as a script from anywhere
    sys.path.insert(0, _ROOT)
from oracle import shadowkv_oracle as o  # noqa: E402


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


def _load_reference(ref: str):
    """Import models/kvcache/shadow.py of the reference with stubs."""
    for name in ["models", "models.kvcache", "kernels"]:
        mod = types.ModuleType(name)
        mod.__path__ = []
        sys.modules[name] = mod
    shadowkv_stub = types.ModuleType("kernels.shadowkv")
    sys.modules["kernels.shadowkv"] = shadowkv_stub
    sys.modules["kernels"].shadowkv = shadowkv_stub
    top = types.ModuleType("models.tensor_op")
    top.batch_gather_gemm_rotary_pos_emb_cuda = None
    sys.modules["models.tensor_op"] = top

    def load(name, path):
        spec = importlib.util.spec_from_file_location(name, path)
        m = importlib.util.module_from_spec(spec)
        sys.modules[name] = m
        spec.loader.exec_module(m)
        return m

    load("models.kvcache.base", os.path.join(ref, "models/kvcache/base.py"))

    class _FakeStream:
        def __init__(self, *a, **k):
            pass

    torch.cuda.Stream = _FakeStream  # the class creates a copy stream in __init__
    shadow = load("models.kvcache.shadow", os.path.join(ref, "models/kvcache/shadow.py"))

    # reference torch RoPE helpers, taken from the source file itself
    ns = {"torch": torch}
    for fname, wanted in [("models/tensor_op.py", {"rotate_half", "apply_rotary_pos_emb_single", "repeat_kv"})]:
        src = open(os.path.join(ref, fname)).read()
        tree = ast.parse(src)
        body = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in wanted]
        exec(compile(ast.Module(body=body, type_ignores=[]), fname, "exec"), ns)
    src = open(os.path.join(ref, "models/glm.py")).read()
    tree = ast.parse(src)
    glm_fn = None
    for n in ast.walk(tree):
        if isinstance(n, ast.FunctionDef) and n.name == "apply_rotary_pos_emb_single":
            n.decorator_list = []
            glm_fn = n
    exec(compile(ast.Module(body=[glm_fn], type_ignores=[]), "models/glm.py", "exec"), ns)
    glm_rope = ns["apply_rotary_pos_emb_single"]
    # the tensor_op version was overwritten by the GLM one: reload it
    ns2 = {"torch": torch}
    src = open(os.path.join(ref, "models/tensor_op.py")).read()
    tree = ast.parse(src)
    body = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in {"rotate_half", "apply_rotary_pos_emb_single"}]
    exec(compile(ast.Module(body=body, type_ignores=[]), "models/tensor_op.py", "exec"), ns2)
    return shadow, ns2["apply_rotary_pos_emb_single"], glm_rope


def _tensor_op_wrappers(ref: str, shadowkv) -> dict:
    """The reference's binding wrappers of models/tensor_op.py:176-243, from the source file,
    with ``shadowkv`` bound to the given module (the recorder)."""
    ns = {"torch": torch, "shadowkv": shadowkv}
    wanted = {"apply_rotary_pos_emb_cuda_push_cache", "batch_gather_gemm_rotary_pos_emb_cuda"}
    src = open(os.path.join(ref, "models/tensor_op.py")).read()
    tree = ast.parse(src)
    body = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in wanted]
    assert len(body) == 2
    exec(compile(ast.Module(body=body, type_ignores=[]), "models/tensor_op.py", "exec"), ns)
    return ns


def cos_sin_cache(n: int, dim: int = 128, theta: float = 500000.0) -> torch.Tensor:
    """``cat(cos[:, :64], sin[:, :64])`` as models/llama.py:137-141,167 builds it."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    t = torch.arange(n, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return torch.cat((emb.cos()[:, : dim // 2], emb.sin()[:, : dim // 2]), dim=-1)


def make_torch_class_fixture(shadow, rope_single, out_path, T=1024, Hq=8, Hkv=2, r_true=32,
                             rank=64, budget=128, outliers=8, steps=3, seed=0):
    D = 128
    g = torch.Generator().manual_seed(seed)
    U0 = torch.randn(T, r_true, generator=g)
    W0 = torch.randn(r_true, Hkv * D, generator=g) / math.sqrt(math.sqrt(r_true))
    k_pre = _bf16(U0 @ W0 + 0.05 * torch.randn(T, Hkv * D, generator=g)).unsqueeze(0)  # [1,T,Hkv*D]
    v = _bf16(torch.randn(1, Hkv, T, D, generator=g))
    cs = _bf16(cos_sin_cache(T + 1024))
    cos = torch.cat((cs[:, :64], cs[:, :64]), dim=-1)
    sin = torch.cat((cs[:, 64:], cs[:, 64:]), dim=-1)

    def rope_func(x, position_ids):
        return rope_single(x, cos, sin, position_ids)

    cfg = types.SimpleNamespace(num_attention_heads=Hq, num_key_value_heads=Hkv,
                                hidden_size=Hq * D, num_hidden_layers=1)
    cache = shadow.ShadowKVCache(cfg, batch_size=1, max_length=T, device="cpu", dtype=torch.float32,
                                 sparse_budget=budget, chunk_size=8, rank=rank)
    cache.outlier_chunk = outliers
    cache.get_svd(k_pre, layer_idx=0)
    cache.U.copy_(_bf16(cache.U))
    cache.SV.copy_(_bf16(cache.SV))
    # post-RoPE keys for prefill: torch RoPE of the pre-RoPE keys (fp32)
    k_heads = k_pre.view(1, T, Hkv, D).transpose(1, 2)
    pos = torch.arange(T)
    k_roped = k_heads * cos[pos] + torch.cat((-k_heads[..., 64:], k_heads[..., :64]), dim=-1) * sin[pos]
    q_last = _bf16(torch.randn(1, Hq, 1, D, generator=g))
    cache.prefill_kv_cache(v, 0, k_roped, q_last)
    cache.k_landmark.copy_(_bf16(cache.k_landmark))

    rec = {
        "T": T, "Hq": Hq, "Hkv": Hkv, "rank": rank, "budget": budget, "outliers": outliers,
        "sparse_start": cache.sparse_start, "sparse_end": cache.sparse_end,
        "prefill_local": cache.prefill_local, "chunks": cache.chunks,
        "k_pre_bf16": k_pre.to(torch.bfloat16).view(torch.int16).numpy(),
        "v_bf16": v.to(torch.bfloat16).view(torch.int16).numpy(),
        "cos_sin_bf16": cs[: T + 64].to(torch.bfloat16).view(torch.int16).numpy(),
        "U": cache.U[0].to(torch.bfloat16).view(torch.int16).numpy(),
        "SV": cache.SV[0].to(torch.bfloat16).view(torch.int16).numpy(),
        "k_landmark": cache.k_landmark[0].to(torch.bfloat16).view(torch.int16).numpy(),
        "k_landmark_idx": cache.k_landmark_idx[0].numpy(),
        "k_prefix": cache.k_cache_buffer[0][:, :, : cache.sparse_start].numpy(),
        "v_prefix": cache.v_cache_buffer[0][:, :, : cache.sparse_start].to(torch.bfloat16).view(torch.int16).numpy(),
    }
    qs, new_ks, new_vs, sel, kbuf, vbuf, seqlens = [], [], [], [], [], [], []
    for step in range(steps):
        q = _bf16(torch.randn(1, Hq, 1, D, generator=g))
        k_new = _bf16(torch.randn(1, Hkv, 1, D, generator=g))
        v_new = _bf16(torch.randn(1, Hkv, 1, D, generator=g))
        cache.update_kv_cache(k_new, v_new, 0)
        pid = cache.get_retrieval_position_ids(layer_idx=0, query_states=q)
        vv = cache.get_value_cache(0, pid)
        kk = cache.get_key_cache(layer_idx=0, position_ids=pid, rope_func=rope_func, cos_sin_cache=cs)
        qs.append(q.numpy())
        new_ks.append(k_new.numpy())
        new_vs.append(v_new.numpy())
        sel.append(cache.selected_chunk_idx[0].clone().numpy())
        kbuf.append(kk.clone().numpy())
        vbuf.append(vv.clone().numpy())
        seqlens.append(kk.shape[2])
    rec["q"] = np.stack(qs)
    rec["k_new"] = np.stack(new_ks)
    rec["v_new"] = np.stack(new_vs)
    rec["selected_chunk_idx"] = np.stack(sel)
    rec["seq_len"] = np.array(seqlens)
    # K/V buffer rows [sparse_start, sparse_end) in selection order, per step
    ss, se = cache.sparse_start, cache.sparse_end
    rec["k_sparse"] = np.stack([k[:, :, ss:se] for k in kbuf])
    rec["v_sparse"] = np.stack([torch.from_numpy(v_[:, :, ss:se]).to(torch.bfloat16).view(torch.int16).numpy() for v_ in vbuf])
    rec["k_gen"] = np.stack([k[:, :, se:] for k in kbuf[-1:]])
    np.savez_compressed(out_path, **rec)
    print("wrote", out_path, os.path.getsize(out_path), "bytes")


def config0_values(T=8192, Hkv=2, seed=1):
    """The value cache of the config-0 fixture, regenerated by the tests instead of stored:
    V ~ N(0, 1) from numpy's PCG64 with this seed, rounded to bf16 (as float32)."""
    v = np.random.default_rng(seed).standard_normal((1, Hkv, T, 128), dtype=np.float32)
    return _bf16(torch.from_numpy(v)).numpy()


def make_config0_fixture(shadow, rope_single, out_path, T=8192, Hq=8, Hkv=2, r_true=32, rank=64, budget=512,
                         outliers=8, steps=3, seed=0):
    """BASELINE configs[0] through the reference's ``ShadowKVCache`` on CPU in float32.

    Pre-RoPE K = U0 W0 + 0.05 N(0,1) with U0 [T, 32] ~ N(0,1) and W0 [32, 256] ~ N(0, 1/sqrt(32))
    (variance), V ~ N(0,1), q ~ N(0,1); rank-64 SVD, RoPE theta 500000, chunk 8, budget 512
    (64 chunks), 8 outlier chunks, 32-token local window.  Inputs are bf16-representable.
    V and the RoPE table are not stored (``config0_values`` and ``cos_sin_cache`` regenerate them;
    their SHA-256 digests are stored to check that);
    the reconstructed keys are stored for step 0 (the oracle is pinned on them), the chunk ids
    and gathered values' checksum for every step."""
    import hashlib
    D = 128
    rng = np.random.default_rng(seed)
    U0 = torch.from_numpy(rng.standard_normal((T, r_true), dtype=np.float32))
    W0 = torch.from_numpy(rng.standard_normal((r_true, Hkv * D), dtype=np.float32)) / math.sqrt(math.sqrt(r_true))
    noise = torch.from_numpy(rng.standard_normal((T, Hkv * D), dtype=np.float32))
    k_pre = _bf16(U0 @ W0 + 0.05 * noise).unsqueeze(0)  # [1, T, Hkv*D]
    v_np = config0_values(T, Hkv)
    v = torch.from_numpy(v_np)
    cs = _bf16(cos_sin_cache(T + 1024))
    cos = torch.cat((cs[:, :64], cs[:, :64]), dim=-1)
    sin = torch.cat((cs[:, 64:], cs[:, 64:]), dim=-1)

    def rope_func(x, position_ids):
        return rope_single(x, cos, sin, position_ids)

    cfg = types.SimpleNamespace(num_attention_heads=Hq, num_key_value_heads=Hkv,
                                hidden_size=Hq * D, num_hidden_layers=1)
    cache = shadow.ShadowKVCache(cfg, batch_size=1, max_length=T, device="cpu", dtype=torch.float32,
                                 sparse_budget=budget, chunk_size=8, rank=rank)
    cache.outlier_chunk = outliers
    cache.get_svd(k_pre, layer_idx=0)
    cache.U.copy_(_bf16(cache.U))
    cache.SV.copy_(_bf16(cache.SV))
    k_heads = k_pre.view(1, T, Hkv, D).transpose(1, 2)
    pos = torch.arange(T)
    k_roped = k_heads * cos[pos] + torch.cat((-k_heads[..., 64:], k_heads[..., :64]), dim=-1) * sin[pos]
    q_last = torch.from_numpy(rng.standard_normal((1, Hq, 1, D), dtype=np.float32))
    cache.prefill_kv_cache(v, 0, k_roped, _bf16(q_last))
    cache.k_landmark.copy_(_bf16(cache.k_landmark))
    rec = {
        "T": T, "Hq": Hq, "Hkv": Hkv, "rank": rank, "budget": budget, "outliers": outliers,
        "sparse_start": cache.sparse_start, "sparse_end": cache.sparse_end,
        "prefill_local": cache.prefill_local, "chunks": cache.chunks,
        "v_sha256": np.frombuffer(hashlib.sha256(v_np.tobytes()).digest(), dtype=np.uint8),
        # the RoPE table is regenerated by the tests (cos_sin_cache(T + 1024)[:T + 64] in bf16)
        "cos_sin_sha256": np.frombuffer(hashlib.sha256(
            cs[: T + 64].to(torch.bfloat16).view(torch.int16).numpy().tobytes()).digest(), dtype=np.uint8),
        "U": cache.U[0].to(torch.bfloat16).view(torch.int16).numpy(),
        "SV": cache.SV[0].to(torch.bfloat16).view(torch.int16).numpy(),
        "k_landmark": cache.k_landmark[0].to(torch.bfloat16).view(torch.int16).numpy(),
        "k_landmark_idx": cache.k_landmark_idx[0].numpy(),
        "k_prefix": cache.k_cache_buffer[0][:, :, : cache.sparse_start].numpy(),
        "v_prefix": cache.v_cache_buffer[0][:, :, : cache.sparse_start].to(torch.bfloat16).view(torch.int16).numpy(),
    }
    qs, new_ks, new_vs, sel, seqlens, vsums = [], [], [], [], [], []
    ss, se = cache.sparse_start, cache.sparse_end
    for step in range(steps):
        q = _bf16(torch.from_numpy(rng.standard_normal((1, Hq, 1, D), dtype=np.float32)))
        k_new = _bf16(torch.from_numpy(rng.standard_normal((1, Hkv, 1, D), dtype=np.float32)))
        v_new = _bf16(torch.from_numpy(rng.standard_normal((1, Hkv, 1, D), dtype=np.float32)))
        cache.update_kv_cache(k_new, v_new, 0)
        pid = cache.get_retrieval_position_ids(layer_idx=0, query_states=q)
        vv = cache.get_value_cache(0, pid)
        kk = cache.get_key_cache(layer_idx=0, position_ids=pid, rope_func=rope_func, cos_sin_cache=cs)
        qs.append(q.numpy())
        new_ks.append(k_new.numpy())
        new_vs.append(v_new.numpy())
        sel.append(cache.selected_chunk_idx[0].clone().numpy())
        seqlens.append(kk.shape[2])
        vb = vv[:, :, ss:se].contiguous().numpy()
        vsums.append(np.frombuffer(hashlib.sha256(vb.tobytes()).digest(), dtype=np.uint8))
        if step == 0:
            rec["k_sparse0"] = kk[:, :, ss:se].clone().numpy()
        if step == steps - 1:
            rec["k_gen"] = kk[:, :, se:].clone().numpy()
    rec["q"] = np.stack(qs)
    rec["k_new"] = np.stack(new_ks)
    rec["v_new"] = np.stack(new_vs)
    rec["selected_chunk_idx"] = np.stack(sel)
    rec["seq_len"] = np.array(seqlens)
    rec["v_sparse_sha256"] = np.stack(vsums)  # float32 rows [sparse_start, sparse_end) per step
    np.savez_compressed(out_path, **rec)
    print("wrote", out_path, os.path.getsize(out_path), "bytes")


TRACE = dict(L=2, B=2, Hq=8, Hkv=2, T=4096, r_true=24, rank=32, budget=1024, steps=3, seed=7)


def trace_inputs(L, B, Hq, Hkv, T, r_true, steps, seed, **_):
    """Inputs of the recorded offload-class trace, regenerated by the tests instead of stored.

    Per layer: pre-RoPE keys ``U0 W0 + 0.05 N(0,1)`` (U0 [B, T, r_true] ~ N(0,1), W0 ~ N(0,
    1/sqrt(r_true)) variance, products in float64), values ~ N(0,1), the last prompt query ~
    N(0,1); per decode step and layer a query (that layer's last prompt query plus 0.5 N(0,1),
    so consecutive steps share chunks), a key and a value ~ N(0,1).  All rounded to bf16 (as
    float32); keys and queries rotated by the bf16 rotate-half RoPE at their positions (prompt
    token t at t, decode step s at T + s) with the table ``cos_sin_cache(T + 1024)[:T + 64]``
    in bf16.  Returns a dict of numpy arrays."""
    D = 128
    rng = np.random.default_rng(seed)
    cs = cos_sin_cache(T + 1024).to(torch.bfloat16)[: T + 64]
    csf = cs.float().numpy()

    def rope(x, pos):
        return o.rope_rotate_half_bf16(x, csf[pos, :64], csf[pos, 64:])

    def bf(shape, scale=1.0, base=None):
        x = rng.standard_normal(shape) * scale
        if base is not None:
            x = x + base
        return o.round_bf16(x.astype(np.float32))

    k_pre, k_rot, v, q_last_pre, q_last = [], [], [], [], []
    for _ in range(L):
        U0 = rng.standard_normal((B, T, r_true))
        W0 = rng.standard_normal((B, r_true, Hkv * D)) / math.sqrt(math.sqrt(r_true))
        kp = o.round_bf16((U0 @ W0 + 0.05 * rng.standard_normal((B, T, Hkv * D))).astype(np.float32))
        kh = np.ascontiguousarray(kp.reshape(B, T, Hkv, D).transpose(0, 2, 1, 3))
        k_pre.append(kh)
        k_rot.append(rope(kh, np.arange(T)))
        v.append(bf((B, Hkv, T, D)))
        qp = bf((B, Hq, 1, D))
        q_last_pre.append(qp)
        q_last.append(rope(qp, np.array([T - 1])))
    q, k_new, v_new = [], [], []
    for s in range(steps):
        pos = np.array([T + s])
        q.append(np.stack([rope(bf((B, Hq, 1, D), 0.5, q_last_pre[l]), pos) for l in range(L)]))
        k_new.append(np.stack([rope(bf((B, Hkv, 1, D)), pos) for _ in range(L)]))
        v_new.append(np.stack([bf((B, Hkv, 1, D)) for _ in range(L)]))
    return {"k_pre": np.stack(k_pre), "k_rot": np.stack(k_rot), "v": np.stack(v), "q_last": np.stack(q_last),
            "q": np.stack(q), "k_new": np.stack(k_new), "v_new": np.stack(v_new),
            "cos_sin_bits": cs.view(torch.int16).numpy()}


class _CpuOnly:
    """The offload class allocates pinned host memory and synchronizes the device: on a machine
    without a GPU, allocate plain host memory and make the synchronizations no-ops."""

    def __enter__(self):
        self._zeros, self._sync = torch.zeros, torch.cuda.synchronize
        zeros = self._zeros

        def host_zeros(*a, pin_memory=False, **k):
            return zeros(*a, **k)

        torch.zeros = host_zeros
        torch.cuda.synchronize = lambda *a, **k: None
        return self

    def __exit__(self, *exc):
        torch.zeros, torch.cuda.synchronize = self._zeros, self._sync


def make_offload_trace(shadow, ref, out_path, L, B, Hq, Hkv, T, r_true, rank, budget, steps, seed):
    """The reference's ``ShadowKVCache_CPU`` (models/kvcache/shadow.py:301-651), unmodified, on
    CPU: prefill of every layer as ``ShadowAttention.prefill`` drives it (models/attention/
    shadow.py:8-13: ``get_svd`` of the pre-RoPE keys, then ``prefill_kv_cache`` with the rotated
    keys and the last query), ``H2D``, then ``steps`` decode steps of every layer as
    ``ShadowAttention.decode`` drives them (models/attention/shadow.py:22-46:
    ``update_kv_cache`` -> ``get_retrieval_position_ids`` -> ``get_value_cache`` ->
    ``get_key_cache``).  Writes the binding trace, the state after prefill that the inputs do
    not determine (U, SV, landmarks, the first chunk selection, the order of the outlier
    chunks) and the digest of every cache tensor after prefill."""
    import json

    from tests.golden import binding_trace as bt
    x = trace_inputs(L, B, Hq, Hkv, T, r_true, steps, seed)
    bf16 = torch.bfloat16
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(bf16)  # noqa: E731
    cs = torch.from_numpy(x["cos_sin_bits"]).view(bf16)
    D = 128
    cfg = types.SimpleNamespace(num_attention_heads=Hq, num_key_value_heads=Hkv, hidden_size=Hq * D,
                                num_hidden_layers=L)
    with _CpuOnly():
        cache = shadow.ShadowKVCache_CPU(cfg, batch_size=B, max_length=T, device="cpu", sparse_budget=budget,
                                         rank=rank)
        for l in range(L):
            cache.get_svd(t(x["k_pre"][l]), layer_idx=l)
            cache.prefill_kv_cache(t(x["v"][l]), l, t(x["k_rot"][l]), t(x["q_last"][l]))
        cache.H2D()

    names = ["v_cache_cpu", "k_cache_buffer", "v_cache_buffer", "temp", "offsets", "cnts", "signals",
             "position_ids", "output", "U", "SV", "k_landmark", "k_landmark_idx", "gemm_o", "softmax_o", "norm",
             "sum"]
    named = lambda: {**{n: getattr(cache, n) for n in names}, "cos_sin": cs}  # noqa: E731
    state = {n: {"shape": list(getattr(cache, n).shape), "dtype": str(getattr(cache, n).dtype).replace("torch.", ""),
                 "digest": bt.digest(getattr(cache, n))} for n in names}
    ps, ss, se = cache.prefill_local, cache.sparse_start, cache.sparse_end
    c = cache.chunk_size
    # the order of the outlier chunks in the buffers (the class keeps only the set): match the rows
    oc = cache.outlier_chunk
    outlier_idx = np.zeros((L, B, Hkv, oc), dtype=np.int32)
    for l in range(L):
        vch = x["v"][l][:, :, : cache.chunks * c].reshape(B, Hkv, cache.chunks, c * D)
        for b in range(B):
            for h in range(Hkv):
                for j in range(oc):
                    rows = cache.v_cache_buffer[l, b, h, ps + j * c: ps + (j + 1) * c].float().numpy().reshape(-1)
                    hit = np.nonzero((vch[b, h] == rows[None, :]).all(axis=1))[0]
                    assert hit.size == 1
                    outlier_idx[l, b, h, j] = hit[0]

    rec = bt.Recorder(named)
    shadow.shadowkv = rec
    shadow.batch_gather_gemm_rotary_pos_emb_cuda = _tensor_op_wrappers(ref, rec)["batch_gather_gemm_rotary_pos_emb_cuda"]
    initial = {"position_ids": cache.position_ids.numpy().copy(), "U": bt.bits(cache.U), "SV": bt.bits(cache.SV),
               "k_landmark": bt.bits(cache.k_landmark), "k_landmark_idx": cache.k_landmark_idx.numpy().astype(np.int32)}
    lengths = []
    with _CpuOnly():
        for s in range(steps):
            for l in range(L):
                q = t(x["q"][s][l])
                k_new, v_new = t(x["k_new"][s][l]), t(x["v_new"][s][l])
                rec.append(l, cache.sparse_end + cache.gen_offset, k_new, v_new)
                cache.update_kv_cache(k_new, v_new, l)
                pid = cache.get_retrieval_position_ids(layer_idx=l, query_states=q)
                vv = cache.get_value_cache(l, pid)
                kk = cache.get_key_cache(layer_idx=l, position_ids=pid, rope_func=None, cos_sin_cache=cs)
                lengths.append([kk.shape[-2], vv.shape[-2]])
    meta = {"config": dict(L=L, B=B, Hq=Hq, Hkv=Hkv, T=T, r_true=r_true, rank=rank, budget=budget, steps=steps,
                           seed=seed),
            "prefill_local": ps, "sparse_start": ss, "sparse_end": se, "chunks": cache.chunks,
            "state": state, "kv_lengths": lengths,
            "final": {n: bt.digest(getattr(cache, n)) for n in names}}
    out = bt.pack(rec)
    out["meta_json"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    out["outlier_idx"] = outlier_idx
    for k, v in initial.items():
        out["init_" + k] = v
    np.savez_compressed(out_path, **out)
    print("wrote", out_path, os.path.getsize(out_path), "bytes;", len(rec.events), "events")


def make_rope_fixture(rope_single, glm_rope, out_path, seed=1):
    g = torch.Generator().manual_seed(seed)
    B, H, S, D = 1, 4, 32, 128  # the reference helper broadcasts only with B=1
    x = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)
    cs = cos_sin_cache(1024).to(torch.bfloat16)
    cos = torch.cat((cs[:, :64], cs[:, :64]), dim=-1)
    sin = torch.cat((cs[:, 64:], cs[:, 64:]), dim=-1)
    pos = torch.randint(0, 1024, (B, H, S), generator=g)
    out_llama = rope_single(x, cos, sin, pos)  # bf16 tensors: each op rounds to bf16
    # GLM: cos_sin row = [cos(32) | sin(32)] (models/glm.py:132-133)
    inv = 1.0 / (10000 ** (torch.arange(0, 64, 2, dtype=torch.float32) / 64))
    ang = torch.outer(torch.arange(1024, dtype=torch.float32), inv)
    cs_glm = torch.cat((ang.cos(), ang.sin()), dim=-1).to(torch.bfloat16)
    holder = types.SimpleNamespace(cos_sin_cache=cs_glm)
    out_glm = glm_rope(holder, x, pos)
    np.savez_compressed(out_path,
                        x=x.view(torch.int16).numpy(), pos=pos.numpy(),
                        cos_sin=cs.view(torch.int16).numpy(), cos_sin_glm=cs_glm.view(torch.int16).numpy(),
                        out_llama=out_llama.contiguous().view(torch.int16).numpy(),
                        out_glm=out_glm.contiguous().view(torch.int16).numpy())
    print("wrote", out_path, os.path.getsize(out_path), "bytes")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SHADOWKV_REFERENCE"),
                    help="root of the reference checkout (or set SHADOWKV_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set SHADOWKV_REFERENCE")
    shadow, rope_single, glm_rope = _load_reference(args.reference)
    make_torch_class_fixture(shadow, rope_single, os.path.join(HERE, "torch_class_decode.npz"))
    make_config0_fixture(shadow, rope_single, os.path.join(HERE, "torch_class_config0.npz"))
    make_rope_fixture(rope_single, glm_rope, os.path.join(HERE, "rope_bf16.npz"))
    make_offload_trace(shadow, args.reference, os.path.join(HERE, "offload_class_trace.npz"), **TRACE)


if __name__ == "__main__":
    main()
