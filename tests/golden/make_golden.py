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


if __name__ == "__main__":
    main()
