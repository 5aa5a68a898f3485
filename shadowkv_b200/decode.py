"""Fused decode path: thin torch wrappers of the ``skv_decode_*`` C ABI.

One layer of one decode step of ShadowKV (models/kvcache/shadow.py:547-597
and models/attention/shadow.py:22-48) as four launches groups:

1. ``select``  -- landmark scoring, top-k, slot-stable reuse diff;
2. ``gather_values`` -- zero-copy fetch of missed V chunks (copy stream);
3. ``reconstruct_keys`` -- tensor-core U x SV^T + RoPE of the missed keys;
4. ``attention`` -- split-K GQA attention over the buffer.

The slot-stable cache keeps every hit chunk where it is and refills only the
slots of chunks that dropped out, so no hit is ever moved (the reference
compacts hits in place, kernels/copy.cuh:476-479).  ``slots[b,h,s]`` names
the chunk cached in buffer rows ``sparse_start + 8s .. +8``.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from ._lib import DecodeGeom, check, lib


@dataclass
class Geometry:
    batch: int
    kv_heads: int
    q_heads: int
    rank: int
    select_sets: int
    num_landmarks: int
    num_chunks: int
    ctx_len: int
    buf_len: int
    sparse_start: int
    rope_mode: int = 0          # 0 rotate-half (cos_sin width 128), 1 GLM (width 64)
    cos_sin_stride: int = 128
    cos_sin_rows: int = 0
    head_dim: int = 128
    chunk_size: int = 8
    scale: float = 1.0 / math.sqrt(128)

    def c(self) -> DecodeGeom:
        return DecodeGeom(self.batch, self.kv_heads, self.q_heads, self.head_dim, self.rank, self.chunk_size,
                          self.select_sets, self.num_landmarks, self.num_chunks, self.ctx_len, self.buf_len,
                          self.sparse_start, self.rope_mode, self.cos_sin_stride, self.cos_sin_rows,
                          float(self.scale))


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _req_out(t: torch.Tensor):
    """An output that is a CUDA tensor or a page-locked CPU tensor (written over the host link)."""
    if t.is_cuda:
        return _req(t, "out", torch.bfloat16)
    if not t.is_pinned() or t.dtype != torch.bfloat16 or not t.is_contiguous():
        raise RuntimeError("out must be a contiguous bf16 CUDA tensor or a page-locked CPU tensor")
    return t.data_ptr()


def _req_in(t: torch.Tensor, name: str, dtype):
    """An input of ``step``: a CUDA tensor, or a page-locked CPU tensor (read over the host link)."""
    if t.is_cuda:
        return _req(t, name, dtype)
    if not t.is_pinned() or t.dtype != dtype or not t.is_contiguous():
        raise RuntimeError(f"{name} must be a contiguous {dtype} CUDA tensor or a page-locked CPU tensor")
    return t.data_ptr()


def _req(t: torch.Tensor, name: str, dtype, shape=None):
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise RuntimeError(f"{name} must be a contiguous CUDA {dtype} tensor "
                           f"(got {t.dtype}, cuda={t.is_cuda}, contiguous={t.is_contiguous()})")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise RuntimeError(f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")
    return t.data_ptr()


class DecodeWorkspace:
    """Scratch of one decode layer: selection logits and attention partials."""

    def __init__(self, geom: Geometry, device):
        self.geom = geom
        g = geom.c()
        self.select_bytes = int(lib.skv_decode_select_workspace(ctypes.byref(g)))
        self.attn_bytes = int(lib.skv_decode_attention_workspace(ctypes.byref(g), geom.buf_len))
        if self.select_bytes == 0:
            check(1, "skv_decode_select_workspace (geometry rejected)")
        self.select_ws = torch.empty(self.select_bytes, dtype=torch.uint8, device=device)
        # zero-initialised: the attention keeps per-head arrival counters here and
        # leaves them at zero after every call
        self.attn_ws = torch.zeros(max(self.attn_bytes, 256), dtype=torch.uint8, device=device)
        # fused fetch + reconstruction + attention: partials and per-head
        # tickets, zero-filled once (the kernel leaves the tickets at zero)
        self.sparse_bytes = int(lib.skv_decode_sparse_attention_workspace(ctypes.byref(g), geom.buf_len))
        self.sparse_ws = torch.zeros(max(self.sparse_bytes, 256), dtype=torch.uint8, device=device)
        bh = geom.batch * geom.kv_heads
        self.miss_slot = torch.zeros(bh, geom.select_sets, dtype=torch.int32, device=device)
        self.miss_chunk = torch.zeros(bh, geom.select_sets, dtype=torch.int32, device=device)
        self.miss_count = torch.zeros(bh, dtype=torch.int32, device=device)


class StepWorkspace:
    """Scratch of ``step`` (zero-filled once; the step leaves it ready for the next call)."""

    def __init__(self, geom: Geometry, head_groups: int, device):
        self.geom, self.head_groups = geom, head_groups
        self.nbytes = int(lib.skv_decode_step_workspace(ctypes.byref(geom.c()), int(head_groups)))
        if self.nbytes == 0:
            check(1, f"skv_decode_step_workspace (geometry or head_groups={head_groups} rejected)")
        self.buf = torch.zeros(self.nbytes, dtype=torch.uint8, device=device)
        self.miss_count = torch.zeros(geom.batch * geom.kv_heads, dtype=torch.int32, device=device)


def step(geom: Geometry, ws: StepWorkspace, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
         positions: torch.Tensor, cos_sin: torch.Tensor, q_out: torch.Tensor, k_buf: torch.Tensor,
         v_buf: torch.Tensor, row: int, landmarks: torch.Tensor, landmark_idx: torch.Tensor, slots: torch.Tensor,
         U: torch.Tensor, SVt: torch.Tensor, v_host: torch.Tensor, seq_len: int, out: torch.Tensor,
         stream=None, row_dev: torch.Tensor | None = None) -> torch.Tensor:
    """One whole decode step of a layer (``append_select`` + ``sparse_attention`` over buffer rows
    [0, seq_len)), pipelined over ``ws.head_groups`` groups of kv heads; ``ws.miss_count`` receives
    the misses per (b, kv head).  ``q``, ``k_new``, ``v_new`` and ``positions`` may be page-locked CPU
    tensors: the step then reads them over the host link itself (no separate host-to-device copy).
    ``row_dev`` (one int32 on the device): the append row read at run time, the attention then covering [0, row_dev + 1); ``row`` / ``seq_len`` are then its bounds."""
    if v_host.is_cuda or not v_host.is_pinned() or v_host.dtype != torch.bfloat16 or not v_host.is_contiguous():
        raise RuntimeError("v_host must be a contiguous pinned CPU bf16 tensor")
    g = geom.c()
    check(lib.skv_decode_step(
        ctypes.byref(g), _req_in(q, "q", torch.bfloat16), _req_in(k_new, "k_new", torch.bfloat16),
        _req_in(v_new, "v_new", torch.bfloat16), _req_in(positions, "positions", torch.int64),
        _req(cos_sin, "cos_sin", torch.bfloat16), _req(q_out, "q_out", torch.bfloat16),
        _req(k_buf, "k_buf", torch.bfloat16), _req(v_buf, "v_buf", torch.bfloat16), int(row),
        _req(row_dev, "row_dev", torch.int32, (1,)) if row_dev is not None else None,
        _req(landmarks, "landmarks", torch.bfloat16), _req(landmark_idx, "landmark_idx", torch.int64),
        _req(slots, "slots", torch.int32), _req(U, "U", torch.bfloat16), _req(SVt, "SVt", torch.bfloat16),
        v_host.data_ptr(), int(seq_len), _req_out(out), ws.miss_count.data_ptr(), int(ws.head_groups),
        ws.buf.data_ptr(), ws.nbytes, _stream(stream)), "skv_decode_step")
    return out


def early_fetch(enable: bool) -> bool:
    """Turn ``step``'s early value fetch on or off for the process (off by default): the selection
    kernel requests the certain misses' values before the selection is complete, writes keys and
    values into their slots and computes the attention itself.  Returns the previous setting.
    Both leave the same state; the outputs differ only in fp32 summation order."""
    return bool(lib.skv_decode_step_early_fetch(1 if enable else 0))


def step_timing(enable: bool) -> bool:
    """Turn ``step``'s kernel timing on or off for the process (off by default): the kernels of a
    step enqueued with it on -- eagerly, or under stream capture, then on every replay -- stamp
    the GPU's global timer at each CTA's start and end (launches and results unchanged).
    Returns the previous setting."""
    return bool(lib.skv_decode_step_timing(1 if enable else 0))


def step_kernel_times(max_groups: int = 8) -> list[tuple]:
    """Per kv-head group of the last timed step (or replay of a graph captured from one):
    ``(scoring start, scoring end, selection start, selection end, attention start, attention
    end)`` in microseconds after the step's earliest kernel start; ``None`` for a kernel that did
    not run.  Waits for the device and clears the spans."""
    us = (ctypes.c_double * (6 * max_groups))()
    n = ctypes.c_int(0)
    check(lib.skv_decode_step_kernel_times(us, max_groups, ctypes.byref(n)), "skv_decode_step_kernel_times")
    return [tuple(None if us[6 * i + k] < 0 else us[6 * i + k] for k in range(6))
            for i in range(min(n.value, max_groups))]


def append(geom: Geometry, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, positions: torch.Tensor,
           cos_sin: torch.Tensor, q_out: torch.Tensor, k_buf: torch.Tensor, v_buf: torch.Tensor, row: int,
           stream=None) -> torch.Tensor:
    """RoPE of the new token's q and k, append of k and v at buffer row ``row``; returns ``q_out``."""
    g = geom.c()
    check(lib.skv_decode_append(
        ctypes.byref(g), _req(q, "q", torch.bfloat16), _req(k_new, "k_new", torch.bfloat16),
        _req(v_new, "v_new", torch.bfloat16), _req(positions, "positions", torch.int64),
        _req(cos_sin, "cos_sin", torch.bfloat16), _req(q_out, "q_out", torch.bfloat16),
        _req(k_buf, "k_buf", torch.bfloat16), _req(v_buf, "v_buf", torch.bfloat16), int(row), _stream(stream)),
        "skv_decode_append")
    return q_out


def select(geom: Geometry, ws: DecodeWorkspace, q: torch.Tensor, landmarks: torch.Tensor,
           landmark_idx: torch.Tensor, slots: torch.Tensor, stream=None) -> None:
    g = geom.c()
    check(lib.skv_decode_select(
        ctypes.byref(g), _req(q, "q", torch.bfloat16), _req(landmarks, "landmarks", torch.bfloat16),
        _req(landmark_idx, "landmark_idx", torch.int64), _req(slots, "slots", torch.int32),
        ws.miss_slot.data_ptr(), ws.miss_chunk.data_ptr(), ws.miss_count.data_ptr(),
        ws.select_ws.data_ptr(), ws.select_bytes, _stream(stream)), "skv_decode_select")


def append_select(geom: Geometry, ws: DecodeWorkspace, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                  positions: torch.Tensor, cos_sin: torch.Tensor, q_out: torch.Tensor, k_buf: torch.Tensor,
                  v_buf: torch.Tensor, row: int, landmarks: torch.Tensor, landmark_idx: torch.Tensor,
                  slots: torch.Tensor, stream=None) -> torch.Tensor:
    """``append`` + ``select`` in one scoring pass (q pre-RoPE); returns the rotated query ``q_out``."""
    g = geom.c()
    check(lib.skv_decode_append_select(
        ctypes.byref(g), _req(q, "q", torch.bfloat16), _req(k_new, "k_new", torch.bfloat16),
        _req(v_new, "v_new", torch.bfloat16), _req(positions, "positions", torch.int64),
        _req(cos_sin, "cos_sin", torch.bfloat16), _req(q_out, "q_out", torch.bfloat16),
        _req(k_buf, "k_buf", torch.bfloat16), _req(v_buf, "v_buf", torch.bfloat16), int(row),
        _req(landmarks, "landmarks", torch.bfloat16), _req(landmark_idx, "landmark_idx", torch.int64),
        _req(slots, "slots", torch.int32), ws.miss_slot.data_ptr(), ws.miss_chunk.data_ptr(),
        ws.miss_count.data_ptr(), ws.select_ws.data_ptr(), ws.select_bytes, _stream(stream)),
        "skv_decode_append_select")
    return q_out


def gather_values(geom: Geometry, ws: DecodeWorkspace, v_host: torch.Tensor, v_buf: torch.Tensor,
                  stream=None) -> None:
    if v_host.is_cuda or not v_host.is_pinned() or v_host.dtype != torch.bfloat16 or not v_host.is_contiguous():
        raise RuntimeError("v_host must be a contiguous pinned CPU bf16 tensor")
    g = geom.c()
    check(lib.skv_decode_gather_values(
        ctypes.byref(g), v_host.data_ptr(), _req(v_buf, "v_buf", torch.bfloat16),
        ws.miss_slot.data_ptr(), ws.miss_chunk.data_ptr(), ws.miss_count.data_ptr(), _stream(stream)),
        "skv_decode_gather_values")


def reconstruct_keys(geom: Geometry, ws: DecodeWorkspace, U: torch.Tensor, SVt: torch.Tensor,
                     cos_sin: torch.Tensor, k_buf: torch.Tensor, stream=None) -> None:
    g = geom.c()
    check(lib.skv_decode_reconstruct_keys(
        ctypes.byref(g), _req(U, "U", torch.bfloat16), _req(SVt, "SVt", torch.bfloat16),
        _req(cos_sin, "cos_sin", torch.bfloat16), _req(k_buf, "k_buf", torch.bfloat16),
        ws.miss_slot.data_ptr(), ws.miss_chunk.data_ptr(), ws.miss_count.data_ptr(), _stream(stream)),
        "skv_decode_reconstruct_keys")


def attention(geom: Geometry, ws: DecodeWorkspace, q: torch.Tensor, k_buf: torch.Tensor, v_buf: torch.Tensor,
              seq_len: int, out: torch.Tensor, stream=None) -> torch.Tensor:
    g = geom.c()
    check(lib.skv_decode_attention(
        ctypes.byref(g), _req(q, "q", torch.bfloat16), _req(k_buf, "k_buf", torch.bfloat16),
        _req(v_buf, "v_buf", torch.bfloat16), int(seq_len), _req(out, "out", torch.bfloat16),
        ws.attn_ws.data_ptr(), ws.attn_bytes, _stream(stream)), "skv_decode_attention")
    return out


def sparse_attention(geom: Geometry, ws: DecodeWorkspace, q: torch.Tensor, U: torch.Tensor, SVt: torch.Tensor,
                     cos_sin: torch.Tensor, v_host: torch.Tensor, k_buf: torch.Tensor, v_buf: torch.Tensor,
                     seq_len: int, out: torch.Tensor, stream=None, max_ctas: int = 0) -> torch.Tensor:
    """``gather_values`` + ``reconstruct_keys`` + ``attention`` in one launch (after a selection);
    ``max_ctas`` > 0 caps the grid (work items walked in strides).

    ``out`` may be a page-locked CPU tensor: the kernel writes the output over
    the host link (no device-to-host copy after the launch)."""
    if v_host.is_cuda or not v_host.is_pinned() or v_host.dtype != torch.bfloat16 or not v_host.is_contiguous():
        raise RuntimeError("v_host must be a contiguous pinned CPU bf16 tensor")
    g = geom.c()
    args = [ctypes.byref(g), _req(q, "q", torch.bfloat16), _req(U, "U", torch.bfloat16),
            _req(SVt, "SVt", torch.bfloat16), _req(cos_sin, "cos_sin", torch.bfloat16), v_host.data_ptr(),
            _req(k_buf, "k_buf", torch.bfloat16), _req(v_buf, "v_buf", torch.bfloat16), ws.miss_slot.data_ptr(),
            ws.miss_chunk.data_ptr(), ws.miss_count.data_ptr(), int(seq_len), _req_out(out)]
    tail = [ws.sparse_ws.data_ptr(), ws.sparse_bytes, _stream(stream)]
    if max_ctas:
        check(lib.skv_decode_sparse_attention_ctas(*args, int(max_ctas), *tail), "skv_decode_sparse_attention_ctas")
    else:
        check(lib.skv_decode_sparse_attention(*args, *tail), "skv_decode_sparse_attention")
    return out


def gram(k: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """K^T K [D, D] float64 of K [T, D] bf16 (rows may be strided, columns contiguous) on the
    tensor cores (``skv_gram``): bf16 products, fp32 accumulation per slice of rows, float64 sum."""
    if not k.is_cuda or k.dtype != torch.bfloat16 or k.dim() != 2 or k.stride(1) != 1:
        raise RuntimeError("k must be a CUDA bf16 [T, D] tensor with contiguous rows")
    T, D = k.shape
    nbytes = int(lib.skv_gram_workspace(T, D))
    if nbytes == 0:
        check(1, f"skv_gram_workspace (T={T}, D={D}: D must be a multiple of 128)")
    if out is None:
        out = torch.empty(D, D, dtype=torch.float64, device=k.device)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=k.device)
    check(lib.skv_gram(k.data_ptr(), T, D, int(k.stride(0)), _req(out, "out", torch.float64, (D, D)),
                       ws.data_ptr(), nbytes, _stream(stream)), "skv_gram")
    return out
