"""Host helpers around the RoPE and gather-GEMM bindings.

Mirror of the three helpers of the reference's models/tensor_op.py that sit
on the decode path, with the same arguments and return values:
``apply_rotary_pos_emb_cuda`` (tensor_op.py:159-174),
``apply_rotary_pos_emb_cuda_push_cache`` (:176-204) and
``batch_gather_gemm_rotary_pos_emb_cuda`` (:206-243).  They unpack shapes and
strides and call the bindings of ``shadowkv_b200.shadowkv``.
"""
from __future__ import annotations

import torch

from . import shadowkv


def apply_rotary_pos_emb_cuda(x: torch.Tensor, cos_sin: torch.Tensor, position_ids: torch.Tensor) -> torch.Tensor:
    """RoPE of ``x`` [B, H, S, D] at int64 token positions [B, H, S]; returns a new tensor."""
    b, h, s, d = x.shape
    out = torch.empty_like(x)
    shadowkv.apply_rotary_pos_emb_new(
        x, cos_sin, position_ids, out, b, h, s, d,
        x.stride(0), x.stride(1), x.stride(2), x.stride(3), cos_sin.stride(0),
        position_ids.stride(0), position_ids.stride(1), position_ids.stride(2), d // 2)
    return out


def apply_rotary_pos_emb_cuda_push_cache(x, cos_sin, position_ids, chunk_size, cache, sparse_start, sparse_end,
                                         cnts):
    """RoPE of the missed rows of ``x`` written into ``cache`` rows ``sparse_start + s``.

    ``cos_sin`` of width 128 selects the rotate-half kernel, width 64 the GLM
    kernel; any other width raises ``ValueError`` (tensor_op.py:179-202).
    """
    b, h, s, d = x.shape
    if cos_sin.shape[-1] == 128:
        fn = shadowkv.apply_rotary_pos_emb_push_cache_opt
    elif cos_sin.shape[-1] == 64:
        fn = shadowkv.apply_rotary_pos_emb_push_cache_opt_glm
    else:
        raise ValueError(f"Invalid cos_sin shape {tuple(cos_sin.shape)}")
    fn(x, cos_sin, position_ids, cache, cnts, b, h, s, d,
       x.stride(0), x.stride(1), x.stride(2), x.stride(3), cos_sin.stride(0),
       position_ids.stride(0), position_ids.stride(1), position_ids.stride(2),
       cache.stride(0), cache.stride(1), cache.stride(2),
       int(sparse_start), int(sparse_end), d // 2, int(chunk_size))
    return cache


def batch_gather_gemm_rotary_pos_emb_cuda(a, b, cos_sin, position_ids, output, chunk_size, cache, sparse_start,
                                          sparse_end, cnts):
    """Reconstruct the missed keys (U rows x SV^T) and RoPE them into ``cache``.

    a = U [B, T, rank]; b = SV^T [B, H, D, rank]; position_ids [B, H, chunks]
    (int64 or int32 chunk ids); output [B, H, budget, D] scratch.
    """
    batch, seq_len, rank = a.shape
    _, heads, head_dim, _ = b.shape
    max_seq_len = cos_sin.shape[0]
    num_chunks = position_ids.shape[-1]
    sparse_budget = num_chunks * chunk_size
    pid32 = position_ids.to(torch.int32).contiguous()
    shadowkv.batch_gather_gemm(a.contiguous(), b.contiguous(), cos_sin, cos_sin, pid32, output, batch, heads,
                               seq_len, head_dim, rank, sparse_budget, max_seq_len, chunk_size, cnts)
    return apply_rotary_pos_emb_cuda_push_cache(output, cos_sin, pid32, chunk_size, cache, sparse_start,
                                                sparse_end, cnts)
