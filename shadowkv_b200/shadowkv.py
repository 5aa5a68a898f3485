"""Drop-in replacement of the reference's ``kernels.shadowkv`` extension.

The twelve functions below have the names, positional arguments and return
value (``None``; outputs written in place) of the reference's pybind module
(kernels/main.cu:24-37, signatures kernels/functions.h:23-121).  A host
process that did ``from kernels import shadowkv`` can use
``from shadowkv_b200 import shadowkv`` instead.

Differences a caller can observe, all deliberate:

* every call launches on ``torch.cuda.current_stream()`` (the reference used
  the legacy default stream except for ``gather_copy_with_offsets``);
* dtype / device / contiguity / size problems raise ``ShadowKVError`` (a
  ``RuntimeError``, like the reference's c10::Error) before any launch, and
  ``map_size`` may be any value in 1..1024 (the reference silently did
  nothing outside {128, 256, 512, 1024});
* ``temp`` and ``signals`` of ``gather_copy_with_offsets`` are accepted and
  left untouched (``signals`` stays zero as the reference requires);
* ``batch_gather_gemm`` does not write the output rows of cache hits (the
  reference computed whole 128-row tiles; those rows are never read).
"""
from __future__ import annotations

import torch

from ._lib import check, lib

__all__ = [
    "gather_copy", "gather_copy_d2d_with_offsets", "reorder_keys_and_compute_offsets",
    "gather_copy_with_offsets", "apply_rotary_pos_emb", "apply_rotary_pos_emb_new",
    "apply_rotary_pos_emb_new_v2", "apply_rotary_pos_emb_push_cache",
    "apply_rotary_pos_emb_push_cache_opt", "apply_rotary_pos_emb_push_cache_opt_glm",
    "batch_gather_gemm", "batch_gemm_softmax",
]


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _dev(t: torch.Tensor, name: str, dtype: torch.dtype, contiguous: bool = True) -> int:
    if not isinstance(t, torch.Tensor):
        raise RuntimeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    return t.data_ptr()


def _pinned(t: torch.Tensor, name: str) -> int:
    if not isinstance(t, torch.Tensor) or t.is_cuda:
        raise RuntimeError(f"{name} must be a page-locked CPU tensor")
    if t.dtype != torch.bfloat16:
        raise RuntimeError(f"{name} must be torch.bfloat16, got {t.dtype}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if not t.is_pinned():
        raise RuntimeError(f"{name} must be pinned (pin_memory=True)")
    return t.data_ptr()


def _need(t: torch.Tensor, n: int, name: str) -> None:
    if t.numel() < n:
        raise RuntimeError(f"{name} holds {t.numel()} elements, {n} needed")


# ---------------------------------------------------------------------------
# reuse cache
# ---------------------------------------------------------------------------

def gather_copy(values, v_cache_buffer, position_ids, batch_size, heads, cpu_v_length, gpu_v_length,
                map_size=256):
    """kernels/gather_copy.cu:47-109: copy host chunks ``position_ids`` to slots 0..map_size."""
    nb = batch_size * heads
    _need(values, nb * cpu_v_length, "values")
    _need(v_cache_buffer, nb * gpu_v_length, "v_cache_buffer")
    _need(position_ids, nb * map_size, "position_ids")
    check(lib.skv_gather_copy(_pinned(values, "values"), _dev(v_cache_buffer, "v_cache_buffer", torch.bfloat16),
                              _dev(position_ids, "position_ids", torch.int64), batch_size, heads, cpu_v_length,
                              gpu_v_length, map_size, _stream()), "gather_copy")


def gather_copy_d2d_with_offsets(keys, offsets, cnts, batch_size, heads, gpu_k_length, gpu_k_offset,
                                 gpu_k_stride, map_size=256):
    """kernels/gather_copy.cu:112-185: in-place compaction of hit chunks of the K buffer."""
    nb = batch_size * heads
    _need(keys, (nb - 1) * gpu_k_stride + gpu_k_offset + map_size * 1024, "keys")
    _need(offsets, nb * map_size, "offsets")
    _need(cnts, nb, "cnts")
    check(lib.skv_gather_copy_d2d_with_offsets(
        _dev(keys, "keys", torch.bfloat16), _dev(offsets, "offsets", torch.int32), _dev(cnts, "cnts", torch.int32),
        batch_size, heads, gpu_k_length, gpu_k_offset, gpu_k_stride, map_size, _stream()),
        "gather_copy_d2d_with_offsets")


def reorder_keys_and_compute_offsets(cached_pos_ids, cur_pos_ids, offsets, cnts, batch_size, heads, map_size=256):
    """kernels/gather_copy.cu:189-235: reuse-cache diff (hits by old slot, then misses by id)."""
    nb = batch_size * heads
    _need(cached_pos_ids, nb * map_size, "cached_pos_ids")
    _need(cur_pos_ids, nb * map_size, "cur_pos_ids")
    _need(offsets, nb * map_size, "offsets")
    _need(cnts, nb, "cnts")
    check(lib.skv_reorder_keys_and_compute_offsets(
        _dev(cached_pos_ids, "cached_pos_ids", torch.int64), _dev(cur_pos_ids, "cur_pos_ids", torch.int64),
        _dev(offsets, "offsets", torch.int32), _dev(cnts, "cnts", torch.int32), batch_size, heads, map_size,
        _stream()), "reorder_keys_and_compute_offsets")


def gather_copy_with_offsets(values, v_cache_buffer, temp, offsets, cnts, signals, batch_size, heads,
                             cpu_v_length, gpu_v_length, gpu_v_offset, gpu_v_stride, map_size=256):
    """kernels/gather_copy.cu:239-324: hits compacted in place, misses fetched from pinned host memory."""
    nb = batch_size * heads
    _need(values, nb * cpu_v_length, "values")
    _need(v_cache_buffer, (nb - 1) * gpu_v_stride + gpu_v_offset + map_size * 1024, "v_cache_buffer")
    _need(offsets, nb * map_size, "offsets")
    _need(cnts, nb, "cnts")
    check(lib.skv_gather_copy_with_offsets(
        _pinned(values, "values"), _dev(v_cache_buffer, "v_cache_buffer", torch.bfloat16),
        temp.data_ptr() if isinstance(temp, torch.Tensor) else None,
        _dev(offsets, "offsets", torch.int32), _dev(cnts, "cnts", torch.int32),
        signals.data_ptr() if isinstance(signals, torch.Tensor) else None,
        batch_size, heads, cpu_v_length, gpu_v_length, gpu_v_offset, gpu_v_stride, map_size, _stream()),
        "gather_copy_with_offsets")


# ---------------------------------------------------------------------------
# RoPE
# ---------------------------------------------------------------------------

def apply_rotary_pos_emb(x, cos, sin, position_ids, output, batch_size, heads, seq_len, embed_dim,
                         stride_xb, stride_xh, stride_xs, stride_xe, stride_cos, stride_sin,
                         stride_pid_b, stride_pid_h, stride_pid_s, half_dim):
    """kernels/rope.cu:26-87."""
    check(lib.skv_apply_rotary_pos_emb(
        _dev(x, "x", torch.bfloat16, False), _dev(cos, "cos", torch.bfloat16, False),
        _dev(sin, "sin", torch.bfloat16, False), _dev(position_ids, "position_ids", torch.int64, False),
        _dev(output, "output", torch.bfloat16, False), batch_size, heads, seq_len, embed_dim,
        stride_xb, stride_xh, stride_xs, stride_xe, stride_cos, stride_sin, stride_pid_b, stride_pid_h,
        stride_pid_s, half_dim, _stream()), "apply_rotary_pos_emb")


def apply_rotary_pos_emb_new(x, cos_sin, position_ids, output, batch_size, heads, seq_len, embed_dim,
                             stride_xb, stride_xh, stride_xs, stride_xe, stride_cos_sin,
                             stride_pid_b, stride_pid_h, stride_pid_s, half_dim):
    """kernels/rope_new.cu:26-84."""
    check(lib.skv_apply_rotary_pos_emb_new(
        _dev(x, "x", torch.bfloat16, False), _dev(cos_sin, "cos_sin", torch.bfloat16, False),
        _dev(position_ids, "position_ids", torch.int64, False), _dev(output, "output", torch.bfloat16, False),
        batch_size, heads, seq_len, embed_dim, stride_xb, stride_xh, stride_xs, stride_xe, stride_cos_sin,
        stride_pid_b, stride_pid_h, stride_pid_s, half_dim, _stream()), "apply_rotary_pos_emb_new")


def apply_rotary_pos_emb_new_v2(x, cos_sin, position_ids, output, batch_size, heads, seq_len, embed_dim,
                                stride_xb, stride_xh, stride_xs, stride_xe, stride_cos_sin,
                                stride_pid_b, stride_pid_h, stride_pid_s, half_dim, chunk_size):
    """kernels/rope_new.cu:86-144."""
    check(lib.skv_apply_rotary_pos_emb_new_v2(
        _dev(x, "x", torch.bfloat16, False), _dev(cos_sin, "cos_sin", torch.bfloat16, False),
        _dev(position_ids, "position_ids", torch.int32, False), _dev(output, "output", torch.bfloat16, False),
        batch_size, heads, seq_len, embed_dim, stride_xb, stride_xh, stride_xs, stride_xe, stride_cos_sin,
        stride_pid_b, stride_pid_h, stride_pid_s, half_dim, chunk_size, _stream()), "apply_rotary_pos_emb_new_v2")


def _push(fn, name, x, cos_sin, position_ids, output, cnts, batch_size, heads, seq_len, embed_dim,
          stride_xb, stride_xh, stride_xs, stride_xe, stride_cos_sin, stride_pid_b, stride_pid_h, stride_pid_s,
          stride_output_b, stride_output_h, stride_output_s, offset_output_s_start, offset_output_s_end,
          half_dim, chunk_size):
    check(fn(_dev(x, "x", torch.bfloat16, False), _dev(cos_sin, "cos_sin", torch.bfloat16, False),
             _dev(position_ids, "position_ids", torch.int32, False), _dev(output, "output", torch.bfloat16, False),
             _dev(cnts, "cnts", torch.int32), batch_size, heads, seq_len, embed_dim, stride_xb, stride_xh,
             stride_xs, stride_xe, stride_cos_sin, stride_pid_b, stride_pid_h, stride_pid_s, stride_output_b,
             stride_output_h, stride_output_s, offset_output_s_start, offset_output_s_end, half_dim, chunk_size,
             _stream()), name)


def apply_rotary_pos_emb_push_cache(*args):
    """kernels/rope_new.cu:146-222 (same values as the ``_opt`` variant)."""
    _push(lib.skv_apply_rotary_pos_emb_push_cache, "apply_rotary_pos_emb_push_cache", *args)


def apply_rotary_pos_emb_push_cache_opt(*args):
    """kernels/rope_new.cu:224-302: RoPE of the missed rows written into the K buffer."""
    _push(lib.skv_apply_rotary_pos_emb_push_cache_opt, "apply_rotary_pos_emb_push_cache_opt", *args)


def apply_rotary_pos_emb_push_cache_opt_glm(*args):
    """kernels/rope_new.cu:305-404: GLM partial interleaved RoPE variant."""
    _push(lib.skv_apply_rotary_pos_emb_push_cache_opt_glm, "apply_rotary_pos_emb_push_cache_opt_glm", *args)


# ---------------------------------------------------------------------------
# GEMMs
# ---------------------------------------------------------------------------

def batch_gather_gemm(a, b, cos, sin, position_ids, output, batch_size, heads, seq_len, embed_dim, rank,
                      sparse_budget, max_seq_len, chunk_size, offset_array):
    """kernels/batch_gather_gemm.cu:136-213: gathered U rows x SV^T for the missed chunks."""
    _need(a, batch_size * seq_len * rank, "a")
    _need(b, batch_size * heads * embed_dim * rank, "b")
    _need(position_ids, batch_size * heads * (sparse_budget // chunk_size), "position_ids")
    _need(output, batch_size * heads * sparse_budget * embed_dim, "output")
    _need(offset_array, batch_size * heads, "offset_array")
    check(lib.skv_batch_gather_gemm(
        _dev(a, "a", torch.bfloat16), _dev(b, "b", torch.bfloat16), None, None,
        _dev(position_ids, "position_ids", torch.int32), _dev(output, "output", torch.bfloat16),
        batch_size, heads, seq_len, embed_dim, rank, sparse_budget, max_seq_len, chunk_size,
        _dev(offset_array, "offset_array", torch.int32), _stream()), "batch_gather_gemm")


def batch_gemm_softmax(A, B, D, Norm, Sum, Softmax, batch_count, m, n, k, alpha=1.0, beta=0.0):
    """kernels/batch_gemm_softmax.cu:143-196: D = alpha*A.B^T, row softmax of the bf16 D."""
    nblk = (n + 255) // 256
    _need(A, batch_count * m * k, "A")
    _need(B, batch_count * n * k, "B")
    _need(D, batch_count * m * n, "D")
    _need(Softmax, batch_count * m * n, "Softmax")
    _need(Norm, batch_count * nblk * m, "Norm")
    _need(Sum, batch_count * nblk * m, "Sum")
    check(lib.skv_batch_gemm_softmax(
        _dev(A, "A", torch.bfloat16), _dev(B, "B", torch.bfloat16), _dev(D, "D", torch.bfloat16),
        _dev(Norm, "Norm", torch.float32), _dev(Sum, "Sum", torch.float32), _dev(Softmax, "Softmax", torch.bfloat16),
        batch_count, m, n, k, float(alpha), float(beta), _stream()), "batch_gemm_softmax")
