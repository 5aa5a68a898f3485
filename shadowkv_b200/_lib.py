"""ctypes binding of ``libshadowkv_b200.so`` (C ABI in include/shadowkv_b200.h).

The library is built in-tree by ``shadowkv_b200/build.py``.  There is no
fallback: if the shared library is missing or a symbol is absent, importing
this module raises.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
# SKV_LIB: another build of the same library (the trace build of build.build_trace)
LIB_PATH = os.environ.get("SKV_LIB") or os.path.join(_PKG, "libshadowkv_b200.so")

SKV_OK = 0
_STATUS = {1: "invalid argument", 2: "unsupported", 3: "CUDA error", 4: "host memory not pinned/mapped"}

c_int, c_float, c_size_t, c_void_p = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p
c_char_p = ctypes.c_char_p
P = c_void_p


class DecodeGeom(ctypes.Structure):
    """``skv_decode_geom`` of include/shadowkv_b200.h."""

    _fields_ = [
        ("batch", c_int), ("kv_heads", c_int), ("q_heads", c_int), ("head_dim", c_int),
        ("rank", c_int), ("chunk_size", c_int), ("select_sets", c_int), ("num_landmarks", c_int),
        ("num_chunks", c_int), ("ctx_len", c_int), ("buf_len", c_int), ("sparse_start", c_int),
        ("rope_mode", c_int), ("cos_sin_stride", c_int), ("cos_sin_rows", c_int), ("scale", c_float),
    ]


class PrefillGeom(ctypes.Structure):
    """``skv_prefill_geom`` of include/shadowkv_b200.h."""

    _fields_ = [
        ("batch", c_int), ("kv_heads", c_int), ("q_heads", c_int), ("tokens", c_int), ("chunks", c_int),
        ("outlier_chunk", c_int), ("select_sets", c_int), ("buf_len", c_int), ("host_chunks", c_int),
    ]


SKV_MAX_PEERS = 8


class PeerGather(ctypes.Structure):
    """``skv_peer_gather`` of include/shadowkv_b200.h."""

    _fields_ = [
        ("world", c_int), ("rank", c_int), ("q_head0", c_int), ("q_heads_total", c_int),
        ("merges_per_step", c_int), ("batch", c_int), ("block", c_void_p * SKV_MAX_PEERS),
    ]


# name -> argument types (every function returns int status unless listed in _RET)
SIGNATURES = {
    "skv_last_error": [],
    "skv_version": [],
    "skv_device_errors": [P, P],
    "skv_gather_copy": [P, P, P, c_int, c_int, c_int, c_int, c_int, P],
    "skv_gather_copy_d2d_with_offsets": [P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, P],
    "skv_reorder_keys_and_compute_offsets": [P, P, P, P, c_int, c_int, c_int, P],
    "skv_gather_copy_with_offsets": [P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int, P],
    "skv_apply_rotary_pos_emb": [P, P, P, P, P] + [c_int] * 14 + [P],
    "skv_apply_rotary_pos_emb_new": [P, P, P, P] + [c_int] * 13 + [P],
    "skv_apply_rotary_pos_emb_new_v2": [P, P, P, P] + [c_int] * 14 + [P],
    "skv_apply_rotary_pos_emb_push_cache": [P, P, P, P, P] + [c_int] * 19 + [P],
    "skv_apply_rotary_pos_emb_push_cache_opt": [P, P, P, P, P] + [c_int] * 19 + [P],
    "skv_apply_rotary_pos_emb_push_cache_opt_glm": [P, P, P, P, P] + [c_int] * 19 + [P],
    "skv_batch_gather_gemm": [P, P, P, P, P, P] + [c_int] * 8 + [P, P],
    "skv_batch_gemm_softmax": [P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_float, c_float, P],
    "skv_decode_append": [ctypes.POINTER(DecodeGeom), P, P, P, P, P, P, P, P, c_int, P],
    "skv_decode_select_workspace": [ctypes.POINTER(DecodeGeom)],
    "skv_decode_select_kernels": [ctypes.POINTER(DecodeGeom)],
    "skv_decode_select": [ctypes.POINTER(DecodeGeom), P, P, P, P, P, P, P, P, c_size_t, P],
    "skv_decode_append_select": [ctypes.POINTER(DecodeGeom)] + [P] * 8 + [c_int] + [P] * 7 + [c_size_t, P],
    "skv_decode_select_noalloc": [ctypes.POINTER(DecodeGeom), P, P, P, P, P, P, P, P],
    "skv_decode_gather_values": [ctypes.POINTER(DecodeGeom), P, P, P, P, P, P],
    "skv_decode_reconstruct_keys": [ctypes.POINTER(DecodeGeom), P, P, P, P, P, P, P, P],
    "skv_decode_attention_workspace": [ctypes.POINTER(DecodeGeom), c_int],
    "skv_decode_attention": [ctypes.POINTER(DecodeGeom), P, P, P, c_int, P, P, c_size_t, P],
    "skv_decode_sparse_attention_workspace": [ctypes.POINTER(DecodeGeom), c_int],
    "skv_decode_sparse_attention": [ctypes.POINTER(DecodeGeom)] + [P] * 10 + [c_int, P, P, c_size_t, P],
    "skv_decode_sparse_attention_ctas": [ctypes.POINTER(DecodeGeom)] + [P] * 10 + [c_int, P, c_int, P, c_size_t, P],
    "skv_decode_sparse_attention_gather": [ctypes.POINTER(DecodeGeom)] + [P] * 10
                                          + [c_int, ctypes.POINTER(PeerGather), P, c_size_t, P],
    "skv_decode_step_workspace": [ctypes.POINTER(DecodeGeom), c_int],
    "skv_decode_step_early_fetch": [c_int],
    "skv_decode_step_timing": [c_int],
    "skv_decode_step_kernel_times": [P, c_int, P],
    "skv_decode_step": [ctypes.POINTER(DecodeGeom)] + [P] * 8 + [c_int] + [P] * 7 + [c_int, P, P, c_int, P, c_size_t, P],
    "skv_gram_workspace": [c_int, c_int],
    "skv_gram": [P, c_int, c_int, c_int, P, P, c_size_t, P],
    "skv_prefill_workspace": [ctypes.POINTER(PrefillGeom)],
    "skv_prefill_store_values": [ctypes.POINTER(PrefillGeom), P, P, P],
    "skv_prefill_build": [ctypes.POINTER(PrefillGeom)] + [P] * 10 + [c_size_t, P],
    "skv_peer_block_bytes": [c_int, c_int],
    "skv_peer_alloc": [c_size_t, ctypes.POINTER(c_void_p)],
    "skv_peer_free": [P],
    "skv_peer_export": [P, P],
    "skv_peer_import": [P, ctypes.POINTER(c_void_p)],
    "skv_peer_close": [P],
    "skv_peer_gather_finish": [ctypes.POINTER(PeerGather), c_int, P, P],
    "skv_peer_status": [ctypes.POINTER(PeerGather), P],
}
_RET = {"skv_last_error": c_char_p, "skv_decode_select_workspace": c_size_t,
        "skv_decode_attention_workspace": c_size_t, "skv_decode_sparse_attention_workspace": c_size_t,
        "skv_decode_step_workspace": c_size_t, "skv_gram_workspace": c_size_t,
        "skv_peer_block_bytes": c_size_t, "skv_prefill_workspace": c_size_t}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m shadowkv_b200.build` "
            "(the decode path has no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError if the symbol is absent
        fn.argtypes = args
        fn.restype = _RET.get(name, c_int)
    return lib


lib = _load()


class ShadowKVError(RuntimeError):
    """Raised when a library call returns a non-zero status."""


def check(status: int, what: str) -> None:
    if status != SKV_OK:
        msg = lib.skv_last_error().decode(errors="replace")
        raise ShadowKVError(f"{what}: {_STATUS.get(status, status)}: {msg}")


def device_errors() -> tuple[int, int]:
    """(count, first_code) of device-side index errors since the last call; clears them."""
    c = ctypes.c_uint32(0)
    f = ctypes.c_uint32(0)
    check(lib.skv_device_errors(ctypes.byref(c), ctypes.byref(f)), "skv_device_errors")
    return int(c.value), int(f.value)
