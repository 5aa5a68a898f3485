"""CPU oracle for the ShadowKV sparse decode-attention step.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (the ``shadowkv_b200``
package and its CUDA library) imports, links or executes this file.  It is
used by ``tests/`` as the parity checker, by ``__graft_entry__.smoke()`` as
the checker of one small call, and by ``bench.py`` as the timed CPU baseline
(``cpu_baseline`` and ``--impl reference``).

Every function restates, in numpy, the behaviour of one reference function of
WilliamBy/ShadowKV.  The citation in each docstring is ``file:line`` inside
the reference project.  Two families are restated:

* the torch-eager accuracy path ``ShadowKVCache`` (models/kvcache/shadow.py:
  27-298) in float32 -- pinned against fixtures produced by running that
  reference class itself (tests/golden/make_golden.py);
* the CUDA bindings used by ``ShadowKVCache_CPU`` (models/kvcache/shadow.py:
  301-651) with their exact integer semantics and bf16 rounding points --
  the reuse-cache part is pinned against the restated known-answer test of
  kernels/test_cached_gather_copy.cu (oracle/reuse_cache_oracle.c), the
  RoPE bf16 arithmetic against the reference's torch RoPE run in bf16.

bf16 values are carried as float32 arrays holding bf16-representable values
(or as uint16 bit patterns where bytes are compared).
"""
from __future__ import annotations

import math
import numpy as np

# ---------------------------------------------------------------------------
# bf16 helpers
# ---------------------------------------------------------------------------


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 -> bf16 (round to nearest even), return uint16 bits."""
    x = np.asarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + bias) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 value, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def bmul(a, b):
    """bf16 multiply with one rounding (reference: __hmul, rope_new.cu:268)."""
    return round_bf16(np.multiply(np.float32(a) if np.isscalar(a) else a, b, dtype=np.float32))


def badd(a, b):
    """bf16 add with one rounding (reference: __hadd, rope_new.cu:268).

    fp32 has more than 2*8+2 significand bits, so computing in fp32 and
    rounding once to bf16 equals the correctly rounded bf16 operation.
    """
    return round_bf16(np.add(a, b, dtype=np.float32))


# ---------------------------------------------------------------------------
# Reuse cache: reorder / gather (CUDA binding semantics)
# ---------------------------------------------------------------------------


def reorder_keys_and_compute_offsets(cached_pos_ids: np.ndarray, cur_pos_ids: np.ndarray):
    """Reuse-cache diff of the cached and the new chunk sets.

    Restates ``reorder_keys_and_mixed_offsets`` (kernels/map.cuh:475-516),
    launched by ``reorder_keys_and_compute_offsets`` (kernels/gather_copy.cu:
    189-235).  Per (b, h) block of ``map_size`` ids:

    * the cached ids map to their slot (map.cuh:86-92, 127-147);
    * a new id is a *hit* when it is cached; hits are packed first with
      value = old slot, misses after with value = chunk id
      (update_keys_and_mixed_offsets, map.cuh:341-403);
    * hits are sorted by old slot, misses by chunk id (block_sort2 with
      SORT_OFFSET, map.cuh:229-259, 503-506).

    Returns ``(reordered_ids int64, offsets int32, cnts int32)`` with the
    leading dims of the inputs flattened to blocks.  Keys are truncated to
    int32 like the kernel (map.cuh:491,496).  Cached ids are expected to be
    distinct inside a block; for duplicates the lowest slot is used.
    """
    old = np.asarray(cached_pos_ids).reshape(-1, np.asarray(cached_pos_ids).shape[-1])
    new = np.asarray(cur_pos_ids).reshape(old.shape)
    nblk, m = old.shape
    out_keys = np.empty((nblk, m), dtype=np.int64)
    out_off = np.empty((nblk, m), dtype=np.int32)
    cnts = np.empty((nblk,), dtype=np.int32)
    for k in range(nblk):
        o32 = old[k].astype(np.int64).astype(np.int32)
        n32 = new[k].astype(np.int64).astype(np.int32)
        lut = {}
        for slot in range(m):
            key = int(o32[slot])
            if key not in lut:
                lut[key] = slot
        hits = []
        misses = []
        for i in range(m):
            key = int(n32[i])
            if key in lut:
                hits.append((lut[key], key))
            else:
                misses.append(key)
        hits.sort()
        misses.sort()
        for i, (slot, key) in enumerate(hits):
            out_keys[k, i] = key
            out_off[k, i] = slot
        for j, key in enumerate(misses):
            out_keys[k, len(hits) + j] = key
            out_off[k, len(hits) + j] = key
        cnts[k] = len(hits)
    return out_keys, out_off, cnts


def gather_copy_with_offsets(values_host: np.ndarray, v_buffer: np.ndarray, offsets: np.ndarray,
                             cnts: np.ndarray, cpu_v_length: int, gpu_v_length: int,
                             gpu_v_offset: int, gpu_v_stride: int, map_size: int) -> np.ndarray:
    """Reuse-cache V update (in place on a copy of ``v_buffer``).

    Restates ``gather_copy_var_midpoint_BP`` (kernels/copy.cuh:438-498),
    launched by ``gather_copy_with_offsets`` (kernels/gather_copy.cu:239-324).
    The unit is one 2048-byte chunk (1024 bf16 = 8 tokens x 128).  For block
    ``bid`` and slot ``i``:

    * ``i < cnts[bid]`` (hit): slot ``i`` <- old slot ``offsets[i]`` of the
      same device buffer (in place; offsets are ascending so the reference's
      batched in-place move equals reading a snapshot, copy.cuh:476-479);
    * otherwise (miss): slot ``i`` <- host chunk ``offsets[i]``
      (copy.cuh:489-497).

    Element offsets: host block base ``bid*cpu_v_length``; device block base
    ``bid*gpu_v_stride + gpu_v_offset`` (copy.cuh:137-141).  ``gpu_v_length``
    only sizes the reference's temp buffer.  Arrays are bf16 bit patterns
    (uint16) or any 2-byte dtype, viewed flat.
    """
    src_h = np.asarray(values_host).reshape(-1)
    dst = np.array(v_buffer, copy=True)
    flat = dst.reshape(-1)
    snap = flat.copy()
    off = np.asarray(offsets).reshape(-1, map_size)
    cnt = np.asarray(cnts).reshape(-1)
    for bid in range(off.shape[0]):
        dbase = bid * gpu_v_stride + gpu_v_offset
        hbase = bid * cpu_v_length
        for i in range(map_size):
            o = int(off[bid, i])
            if i < cnt[bid]:
                chunk = snap[dbase + o * 1024: dbase + o * 1024 + 1024]
            else:
                chunk = src_h[hbase + o * 1024: hbase + o * 1024 + 1024]
            flat[dbase + i * 1024: dbase + i * 1024 + 1024] = chunk
    return dst


def gather_copy_d2d_with_offsets(keys: np.ndarray, offsets: np.ndarray, cnts: np.ndarray,
                                 gpu_k_offset: int, gpu_k_stride: int, map_size: int) -> np.ndarray:
    """Reuse-cache K compaction (hits only), on a copy of ``keys``.

    Restates ``gather_copy_d2d`` (kernels/copy.cuh:353-390) as launched by
    ``gather_copy_d2d_with_offsets`` (kernels/gather_copy.cu:112-185):
    slot ``i < cnts[bid]`` <- slot ``offsets[i]`` of the same buffer region
    ``bid*gpu_k_stride + gpu_k_offset``; other slots untouched.
    """
    dst = np.array(keys, copy=True)
    flat = dst.reshape(-1)
    snap = flat.copy()
    off = np.asarray(offsets).reshape(-1, map_size)
    cnt = np.asarray(cnts).reshape(-1)
    for bid in range(off.shape[0]):
        base = bid * gpu_k_stride + gpu_k_offset
        for i in range(int(cnt[bid])):
            o = int(off[bid, i])
            flat[base + i * 1024: base + i * 1024 + 1024] = snap[base + o * 1024: base + o * 1024 + 1024]
    return dst


def gather_copy(values_host: np.ndarray, v_buffer: np.ndarray, position_ids: np.ndarray,
                cpu_v_length: int, gpu_v_length: int, map_size: int) -> np.ndarray:
    """Plain chunk gather with no cache.

    Restates ``gahter_copy_fixed_start_end`` (kernels/copy.cuh:248-274) as
    launched by ``gather_copy`` (kernels/gather_copy.cu:47-109): for block
    ``bid``, slot ``i`` in ``[0, map_size)`` of the device region
    ``bid*gpu_v_length`` <- host chunk ``position_ids[bid, i]`` of region
    ``bid*cpu_v_length`` (ids truncated to int32).
    """
    src = np.asarray(values_host).reshape(-1)
    dst = np.array(v_buffer, copy=True)
    flat = dst.reshape(-1)
    pid = np.asarray(position_ids).reshape(-1, map_size).astype(np.int64).astype(np.int32)
    for bid in range(pid.shape[0]):
        for i in range(map_size):
            o = int(pid[bid, i])
            s = bid * cpu_v_length + o * 1024
            d = bid * gpu_v_length + i * 1024
            flat[d:d + 1024] = src[s:s + 1024]
    return dst


# ---------------------------------------------------------------------------
# Slot-stable reuse cache (the fused decode path of this build)
# ---------------------------------------------------------------------------


def stable_slot_update(old_slots: np.ndarray, new_ids: np.ndarray):
    """Slot-stable variant of the reuse-cache diff.

    Same hit/miss classification as ``reorder_keys_and_compute_offsets``
    (kernels/map.cuh:475-516) but hits keep their slot: the slots whose cached
    chunk is not selected any more are refilled, in ascending slot order, with
    the missed chunk ids in ascending id order.  Returns
    ``(slots int64 [.., M], miss_mask bool [.., M], hits int32 [..])``.
    """
    old = np.asarray(old_slots, dtype=np.int64)
    shp = old.shape
    old = old.reshape(-1, shp[-1])
    new = np.asarray(new_ids, dtype=np.int64).reshape(old.shape)
    slots = old.copy()
    miss = np.zeros(old.shape, dtype=bool)
    hits = np.zeros((old.shape[0],), dtype=np.int32)
    for k in range(old.shape[0]):
        nset = set(int(v) for v in new[k])
        oset = set(int(v) for v in old[k])
        free = [s for s in range(old.shape[1]) if int(old[k, s]) not in nset]
        misses = sorted(v for v in nset if v not in oset)
        assert len(free) == len(misses), "cached and new sets must have the same size"
        for s, v in zip(free, misses):
            slots[k, s] = v
            miss[k, s] = True
        hits[k] = old.shape[1] - len(misses)
    return slots.reshape(shp), miss.reshape(shp), hits.reshape(shp[:-1])


# ---------------------------------------------------------------------------
# Landmark scoring and selection
# ---------------------------------------------------------------------------


def batch_gemm_softmax(A: np.ndarray, B: np.ndarray, batch: int, m: int, n: int, k: int,
                       alpha: float, beta: float = 0.0):
    """Scoring GEMM + row softmax of the CUDA path.

    Restates ``batch_gemm_softmax`` (kernels/batch_gemm_softmax.cu:143-196)
    and its three launches (kernels/batch_gemm_softmax.h:453-511):

    * ``D = bf16(alpha * A @ B^T)`` with fp32 accumulation (``beta`` has no
      source operand, batch_gemm_softmax.cu:174);
    * per 256-column block ``j`` the partial row max ``Norm[j]`` and sum
      ``Sum[j] = sum exp(x - Norm[j])`` of the fp32 values (epilogue visitor);
    * the final reduction stores the row max in ``Norm[0]`` and ``1/sum`` in
      ``Sum[0]``;
    * ``Softmax = bf16(exp(float(D) - max) * inv_sum)`` computed from the
      bf16-rounded D (batch_gemm_softmax.h:235-246).

    A: [batch, m, k]; B: [batch, n, k] (the column-major k x n operand).
    Returns D, Norm, Sum, Softmax with Norm/Sum laid out [batch, nblk, m].
    """
    A = np.asarray(A, dtype=np.float32).reshape(batch, m, k)
    B = np.asarray(B, dtype=np.float32).reshape(batch, n, k)
    acc = np.einsum('bmk,bnk->bmn', A.astype(np.float64), B.astype(np.float64)).astype(np.float32)
    x = (np.float32(alpha) * acc).astype(np.float32)
    D = round_bf16(x)
    nblk = (n + 255) // 256
    norm = np.zeros((batch, nblk, m), dtype=np.float32)
    ssum = np.zeros((batch, nblk, m), dtype=np.float32)
    for j in range(nblk):
        blk = x[:, :, 256 * j: 256 * (j + 1)].astype(np.float64)
        mx = blk.max(axis=2)
        norm[:, j, :] = mx
        ssum[:, j, :] = np.exp(blk - mx[:, :, None]).sum(axis=2)
    gmax = norm.max(axis=1)
    gsum = (ssum.astype(np.float64) * np.exp(norm.astype(np.float64) - gmax[:, None, :])).sum(axis=1)
    norm_out = norm.copy()
    sum_out = ssum.copy()
    norm_out[:, 0, :] = gmax
    sum_out[:, 0, :] = (1.0 / gsum)
    soft = round_bf16((np.exp(D.astype(np.float64) - gmax[:, :, None]) * (1.0 / gsum)[:, :, None]).astype(np.float32))
    return D, norm_out, sum_out, soft


def landmark_scores(q: np.ndarray, landmarks: np.ndarray, scale: float = 1.0 / math.sqrt(128)) -> np.ndarray:
    """fp32 chunk scores of the torch path.

    Restates ``ShadowKVCache.get_retrieval_position_ids`` (models/kvcache/
    shadow.py:208-218) for q_len = 1: ``softmax(q.LM^T * scale)`` over
    landmarks per q head in fp32, then the max over the GQA group.
    q: [B, Hkv, G, D]; landmarks: [B, Hkv, L, D].  Returns [B, Hkv, L].
    """
    q = np.asarray(q, dtype=np.float64)
    lm = np.asarray(landmarks, dtype=np.float64)
    logits = np.einsum('bhgd,bhld->bhgl', q, lm) * scale
    logits = logits - logits.max(axis=-1, keepdims=True)
    e = np.exp(logits)
    p = e / e.sum(axis=-1, keepdims=True)
    return p.max(axis=2).astype(np.float32)


def topk_set(scores: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest scores per row, ties broken by lower index.

    ``torch.topk`` (models/kvcache/shadow.py:219,571) leaves the order of
    equal scores unspecified; this deterministic rule is what the fused CUDA
    selection implements.  Returns sorted indices [.., k].
    """
    s = np.asarray(scores)
    flat = s.reshape(-1, s.shape[-1])
    out = np.empty((flat.shape[0], k), dtype=np.int64)
    for r in range(flat.shape[0]):
        order = np.lexsort((np.arange(flat.shape[1]), -flat[r].astype(np.float64)))
        out[r] = np.sort(order[:k])
    return out.reshape(s.shape[:-1] + (k,))


def select_chunks(q, landmarks, landmark_idx, k: int, scale: float = 1.0 / math.sqrt(128)):
    """Chunk ids selected for one decode step (set semantics, sorted).

    Restates models/kvcache/shadow.py:214-222: scores, top-k, then the map
    through ``k_landmark_idx``.  Returns ``(chunk_ids [B,H,k], scores)``.
    """
    sc = landmark_scores(q, landmarks, scale)
    idx = topk_set(sc, k)
    ids = np.take_along_axis(np.asarray(landmark_idx, dtype=np.int64), idx, axis=-1)
    return np.sort(ids, axis=-1), sc


def topk_tie_ok(scores: np.ndarray, chosen: np.ndarray, k: int, rtol: float = 0.0) -> bool:
    """True when ``chosen`` is a valid top-k of ``scores`` up to ties.

    Every chosen score must be >= the k-th largest score and every unchosen
    one <= it, with a relative slack ``rtol`` for near-ties.
    """
    s = np.asarray(scores, dtype=np.float64).reshape(-1, np.asarray(scores).shape[-1])
    c = np.asarray(chosen).reshape(s.shape[0], -1)
    for r in range(s.shape[0]):
        if len(set(c[r].tolist())) != k:
            return False
        kth = np.sort(s[r])[::-1][k - 1]
        slack = abs(kth) * rtol
        mask = np.zeros(s.shape[1], dtype=bool)
        mask[c[r]] = True
        if (s[r][mask] < kth - slack).any() or (s[r][~mask] > kth + slack).any():
            return False
    return True


# ---------------------------------------------------------------------------
# Key reconstruction and RoPE
# ---------------------------------------------------------------------------


def batch_gather_gemm(U: np.ndarray, SVt: np.ndarray, chunk_ids: np.ndarray, cnts: np.ndarray,
                      chunk_size: int = 8) -> np.ndarray:
    """Gathered low-rank GEMM of the CUDA path.

    Restates ``batch_gather_gemm`` (kernels/batch_gather_gemm.cu:136-213;
    gemm_universal_batch_gather_indices.h:615-890):
    ``out[b,h,r,:] = bf16(sum_k U[b, id[r//c]*c + r%c, k] * SVt[b,h,:,k])``
    with fp32 accumulation.  Rows of hit chunks (``r//c < cnts[b*H+h]``) are
    not consumed by the reference and are returned as NaN here.
    U: [B, T, rank]; SVt: [B, H, D, rank]; chunk_ids: [B, H, nchunks].
    """
    U = np.asarray(U, dtype=np.float64)
    SVt = np.asarray(SVt, dtype=np.float64)
    ids = np.asarray(chunk_ids, dtype=np.int64)
    Bn, H, Dd, R = SVt.shape
    nch = ids.shape[-1]
    cnt = np.asarray(cnts).reshape(Bn, H)
    out = np.full((Bn, H, nch * chunk_size, Dd), np.nan, dtype=np.float32)
    for b in range(Bn):
        for h in range(H):
            rows = (ids[b, h][:, None] * chunk_size + np.arange(chunk_size)[None, :]).reshape(-1)
            res = (U[b, rows] @ SVt[b, h].T).astype(np.float32)
            res = round_bf16(res)
            lo = int(cnt[b, h]) * chunk_size
            out[b, h, lo:] = res[lo:]
    return out


def rope_rotate_half_bf16(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate-half RoPE in bf16 op-by-op arithmetic.

    Restates rope_new.cu:49-57 / 262-270:
    ``o[t] = x1*cos + (-x2)*sin``, ``o[t+64] = x2*cos + x1*sin`` with each
    multiply and add rounded to bf16.  x: [..., 128]; cos/sin: [..., 64].
    """
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    o1 = badd(bmul(x1, cos), bmul(-x2, sin))
    o2 = badd(bmul(x2, cos), bmul(x1, sin))
    return np.concatenate([o1, o2], axis=-1)


def rope_glm_bf16(x: np.ndarray, cs: np.ndarray) -> np.ndarray:
    """GLM partial interleaved RoPE in bf16 op-by-op arithmetic.

    Restates rope_new.cu:354-371: pairs (2t, 2t+1) for t < 32 with
    ``cos = cs[t]``, ``sin = cs[t+32]``; dims 64..127 pass through.
    x: [..., 128]; cs: [..., 64].
    """
    out = np.array(x, dtype=np.float32, copy=True)
    cos = cs[..., :32]
    sin = cs[..., 32:64]
    xe = x[..., 0:64:2]
    xo = x[..., 1:64:2]
    out[..., 0:64:2] = badd(bmul(xe, cos), bmul(-xo, sin))
    out[..., 1:64:2] = badd(bmul(xo, cos), bmul(xe, sin))
    return out


def apply_rotary_pos_emb_push_cache_opt(x, cos_sin, chunk_ids, cache, cnts, sparse_start: int,
                                        sparse_end: int, chunk_size: int = 8, glm: bool = False):
    """RoPE of reconstructed keys written into the K buffer (misses only).

    Restates ``apply_rotary_pos_emb_kernel_push_cache_opt`` (kernels/
    rope_new.cu:224-272) and the GLM variant (:305-374): for row ``s`` of
    head (b, h) with ``s//c >= cnts[b*H+h]`` and ``sparse_start+s <
    sparse_end``, position ``id[s//c]*c + s%c`` selects the cos/sin row and
    the rotated row is stored at ``cache[b, h, sparse_start+s]``.
    x: [B, H, S, 128]; cache: [B, H, S_buf, 128] (returned copy).
    """
    x = np.asarray(x, dtype=np.float32)
    out = np.array(cache, dtype=np.float32, copy=True)
    Bn, H, S, Dd = x.shape
    cnt = np.asarray(cnts).reshape(Bn, H)
    ids = np.asarray(chunk_ids, dtype=np.int64)
    for b in range(Bn):
        for h in range(H):
            s = np.arange(int(cnt[b, h]) * chunk_size, S)
            s = s[sparse_start + s < sparse_end]
            if s.size == 0:
                continue
            pos = ids[b, h, s // chunk_size] * chunk_size + s % chunk_size
            cs = np.asarray(cos_sin, dtype=np.float32)[pos]
            if glm:
                rows = rope_glm_bf16(x[b, h, s], cs)
            else:
                rows = rope_rotate_half_bf16(x[b, h, s], cs[:, :Dd // 2], cs[:, Dd // 2:Dd])
            out[b, h, sparse_start + s] = rows
    return out


def rope_rotate_half_fp32(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate-half RoPE in float64 math on unrounded inputs, fp32 result.

    The arithmetic of the torch path (models/tensor_op.py:132-156) without
    intermediate bf16 rounding; the fused CUDA epilogue computes this and
    rounds once.  x: [..., 128]; cos/sin: [..., 64].
    """
    x = np.asarray(x, dtype=np.float64)
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    c, s = np.asarray(cos, np.float64), np.asarray(sin, np.float64)
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1).astype(np.float32)


def rope_glm_fp32(x: np.ndarray, cs: np.ndarray) -> np.ndarray:
    """GLM partial interleaved RoPE (models/glm.py:207-230) in float64 math, fp32 result."""
    x = np.asarray(x, dtype=np.float64)
    out = x.copy()
    c, s = np.asarray(cs[..., :32], np.float64), np.asarray(cs[..., 32:64], np.float64)
    xe, xo = x[..., 0:64:2], x[..., 1:64:2]
    out[..., 0:64:2] = xe * c - xo * s
    out[..., 1:64:2] = xo * c + xe * s
    return out.astype(np.float32)


def reconstruct_keys_rope(U, SVt, chunk_ids, cos_sin, glm: bool = False, chunk_size: int = 8) -> np.ndarray:
    """Keys of the fused CUDA path: ``bf16(rope(U_rows @ SVt^T))`` with one rounding.

    Same values as the torch path (models/kvcache/shadow.py:239-256) up to
    the final bf16 rounding.  U: [T, rank]; SVt: [D, rank]; chunk_ids [n].
    Returns [n*chunk, D] float32 holding bf16 values.
    """
    ids = np.asarray(chunk_ids, dtype=np.int64)
    rows = (ids[:, None] * chunk_size + np.arange(chunk_size)).reshape(-1)
    x = np.asarray(U, np.float64)[rows] @ np.asarray(SVt, np.float64).T
    cs = np.asarray(cos_sin, np.float32)[rows]
    if glm:
        y = rope_glm_fp32(x, cs)
    else:
        y = rope_rotate_half_fp32(x, cs[:, :64], cs[:, 64:128])
    return round_bf16(y)


def rope_torch_fp32(x: np.ndarray, cos_sin: np.ndarray, positions: np.ndarray) -> np.ndarray:
    """Rotate-half RoPE in fp32 as the torch path computes it.

    Restates ``apply_rotary_pos_emb_single`` (models/tensor_op.py:144-156)
    with ``cos = cat(cs[:, :64], cs[:, :64])`` and ``sin = cat(cs[:, 64:],
    cs[:, 64:])`` (models/llama.py:167).
    """
    cs = np.asarray(cos_sin, dtype=np.float32)[np.asarray(positions)]
    h = x.shape[-1] // 2
    cos = np.concatenate([cs[..., :h], cs[..., :h]], axis=-1)
    sin = np.concatenate([cs[..., h:2 * h], cs[..., h:2 * h]], axis=-1)
    rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
    return (x * cos + rot * sin).astype(np.float32)


def reconstruct_keys_fp32(U, SV, chunk_ids, cos_sin, chunk_size: int = 8):
    """Reconstructed post-RoPE keys of the torch path (fp32).

    Restates ``ShadowKVCache.get_key_cache`` (models/kvcache/shadow.py:
    239-256): gather U rows of the selected tokens, multiply by the per-head
    ``SV`` [B, H, rank, D], then RoPE at the original positions.
    Returns [B, H, nchunks*c, D] in the order of ``chunk_ids``.
    """
    U = np.asarray(U, dtype=np.float64)
    SV = np.asarray(SV, dtype=np.float64)
    ids = np.asarray(chunk_ids, dtype=np.int64)
    Bn, H, R, Dd = SV.shape
    pos = (ids[..., None] * chunk_size + np.arange(chunk_size)).reshape(Bn, H, -1)
    out = np.empty(pos.shape + (Dd,), dtype=np.float32)
    for b in range(Bn):
        for h in range(H):
            out[b, h] = (U[b, pos[b, h]] @ SV[b, h]).astype(np.float32)
    return rope_rotate_fp32_positions(out, cos_sin, pos)


def rope_rotate_fp32_positions(x, cos_sin, pos):
    return rope_torch_fp32(np.asarray(x, dtype=np.float32), cos_sin, pos)


# ---------------------------------------------------------------------------
# Decode attention
# ---------------------------------------------------------------------------


def decode_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, seq_len: int,
                     scale: float = 1.0 / math.sqrt(128)) -> np.ndarray:
    """GQA decode attention for q_len = 1 (float64 math, fp32 result).

    Restates ``flash_attn_with_kvcache(q, k_cache, v_cache, causal=True)``
    as called by ``ShadowAttention.decode`` (models/attention/shadow.py:48)
    with the GQA head mapping of ``repeat_kv`` (models/tensor_op.py:125-130):
    q head ``i`` reads kv head ``i // G``.  With one query ``causal`` has no
    effect.  q: [B, Hq, D]; k, v: [B, Hkv, S_buf, D] of which the first
    ``seq_len`` rows are used.  Returns [B, Hq, D].
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)[:, :, :seq_len]
    v = np.asarray(v, dtype=np.float64)[:, :, :seq_len]
    Bn, Hq, Dd = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    out = np.empty((Bn, Hq, Dd), dtype=np.float32)
    for b in range(Bn):
        for hq in range(Hq):
            kk = k[b, hq // G]
            s = kk @ q[b, hq] * scale
            s -= s.max()
            p = np.exp(s)
            p /= p.sum()
            out[b, hq] = (p @ v[b, hq // G]).astype(np.float32)
    return out


# ---------------------------------------------------------------------------
# Whole decode step of the torch path (fp32) -- CPU baseline
# ---------------------------------------------------------------------------


class TorchPathDecodeState:
    """State of one layer of ``ShadowKVCache`` after prefill (numpy arrays).

    Mirrors the attributes that ``ShadowKVCache`` decode reads
    (models/kvcache/shadow.py:59-109, 149-205): ``k_landmark``,
    ``k_landmark_idx``, ``U``, ``SV`` ([B, H, rank, D]), the full value
    cache ``v_full`` [B, H, T, D], the K/V buffers and the geometry.
    """

    def __init__(self, k_landmark, k_landmark_idx, U, SV, v_full, k_buf, v_buf, cos_sin,
                 sparse_start, sparse_end, select_sets, chunk_size=8):
        self.k_landmark = k_landmark
        self.k_landmark_idx = k_landmark_idx
        self.U = U
        self.SV = SV
        self.v_full = v_full
        self.k_buf = k_buf
        self.v_buf = v_buf
        self.cos_sin = cos_sin
        self.sparse_start = sparse_start
        self.sparse_end = sparse_end
        self.select_sets = select_sets
        self.chunk_size = chunk_size


def torch_path_decode_step(st: TorchPathDecodeState, q: np.ndarray, seq_len: int):
    """One decode step of the torch path after ``update_kv_cache``.

    Restates models/attention/shadow.py:32-48 with models/kvcache/shadow.py:
    208-259: select chunks, gather V from the full value cache, reconstruct
    K with RoPE, write both into the buffers at ``[sparse_start,
    sparse_end)`` in selection order, then attention over ``seq_len`` rows.
    q: [B, Hq, D] (post-RoPE).  Returns ``(out [B,Hq,D], chunk_ids)``.
    """
    Bn, Hkv, L, Dd = st.k_landmark.shape
    G = q.shape[1] // Hkv
    ids, _ = select_chunks(q.reshape(Bn, Hkv, G, Dd), st.k_landmark, st.k_landmark_idx, st.select_sets)
    c = st.chunk_size
    pos = (ids[..., None] * c + np.arange(c)).reshape(Bn, Hkv, -1)
    v_sel = np.take_along_axis(st.v_full, pos[..., None], axis=2)
    st.v_buf[:, :, st.sparse_start:st.sparse_end] = v_sel
    st.k_buf[:, :, st.sparse_start:st.sparse_end] = reconstruct_keys_fp32(st.U, st.SV, ids, st.cos_sin, c)
    out = decode_attention(q, st.k_buf, st.v_buf, seq_len)
    return out, ids


# ---------------------------------------------------------------------------
# C part (reuse-cache known-answer tests), loaded with ctypes
# ---------------------------------------------------------------------------


def load_c_oracle():
    """ctypes handle of oracle/_build/libskv_oracle.so (built on demand)."""
    import ctypes
    import os
    from . import build_oracle
    lib = ctypes.CDLL(build_oracle.build())
    P = ctypes.c_void_p
    i = ctypes.c_int
    i64 = ctypes.c_int64
    lib.skv_glibc_rand_check.argtypes = [ctypes.c_uint, i, P]
    lib.skv_kat_keys.argtypes = [i, i, i, i, ctypes.c_uint, P, P]
    lib.skv_kat_keys_nohit.argtypes = [i, i, i, ctypes.c_uint, P, P]
    lib.skv_golden_reorder.argtypes = [i, i, P, P, P, P, P]
    lib.skv_golden_cached_copy.argtypes = [i, i, i64, i64, P, P, P, P, P]
    lib.skv_golden_gather_copy.argtypes = [i, i, i64, P, P, P]
    return lib


def kat_keys(block_num=192, map_size=256, cpu_chunks=16384, fake_hit_cnt=154, seed=12345):
    """Keys of kernels/test_cached_gather_copy.cu:220-282 (glibc rand)."""
    lib = load_c_oracle()
    keys = np.zeros(block_num * map_size, dtype=np.int64)
    query = np.zeros(block_num * map_size, dtype=np.int64)
    rc = lib.skv_kat_keys(block_num, map_size, cpu_chunks, fake_hit_cnt, seed, keys.ctypes.data, query.ctypes.data)
    assert rc == 0
    return keys.reshape(block_num, map_size), query.reshape(block_num, map_size)


def kat_keys_nohit(block_num=160, map_size=256, cpu_chunks=16384, seed=4242):
    """Keys of kernels/test_gather_copy.cu:123-167 (FAKE_HIT_CNT = 0), fixed seed."""
    lib = load_c_oracle()
    keys = np.zeros(block_num * map_size, dtype=np.int64)
    query = np.zeros(block_num * map_size, dtype=np.int64)
    rc = lib.skv_kat_keys_nohit(block_num, map_size, cpu_chunks, seed, keys.ctypes.data, query.ctypes.data)
    assert rc == 0
    return keys.reshape(block_num, map_size), query.reshape(block_num, map_size)


def golden_reorder(orig: np.ndarray, query: np.ndarray):
    """check_reorder_keys_and_mixed_offsets golden (test_cached_gather_copy.cu:70-156)."""
    lib = load_c_oracle()
    o = np.ascontiguousarray(orig, dtype=np.int64)
    q = np.ascontiguousarray(query, dtype=np.int64)
    nb, m = o.shape
    keys = np.zeros_like(o)
    offs = np.zeros((nb, m), dtype=np.int32)
    cnts = np.zeros(nb, dtype=np.int32)
    assert lib.skv_golden_reorder(nb, m, o.ctypes.data, q.ctypes.data, keys.ctypes.data, offs.ctypes.data,
                                  cnts.ctypes.data) == 0
    return keys, offs, cnts


def golden_cached_copy(host_v: np.ndarray, dev_v: np.ndarray, offsets: np.ndarray, cnts: np.ndarray,
                       cpu_v_length: int, gpu_v_length: int):
    """check_cached_copy golden (test_cached_gather_copy.cu:158-216): [blocks, map, 1024] uint16."""
    lib = load_c_oracle()
    off = np.ascontiguousarray(offsets, dtype=np.int32)
    nb, m = off.shape
    h = np.ascontiguousarray(host_v).view(np.uint16)
    d = np.ascontiguousarray(dev_v).view(np.uint16)
    out = np.zeros((nb, m, 1024), dtype=np.uint16)
    c = np.ascontiguousarray(cnts, dtype=np.int32)
    assert lib.skv_golden_cached_copy(nb, m, cpu_v_length, gpu_v_length, h.ctypes.data, d.ctypes.data,
                                      off.ctypes.data, c.ctypes.data, out.ctypes.data) == 0
    return out


def golden_gather_copy(host_v: np.ndarray, keys: np.ndarray, cpu_v_length: int):
    """check_cached_copy golden of test_gather_copy.cu:67-116: [blocks, map, 1024] uint16."""
    lib = load_c_oracle()
    k = np.ascontiguousarray(keys, dtype=np.int64)
    nb, m = k.shape
    h = np.ascontiguousarray(host_v).view(np.uint16)
    out = np.zeros((nb, m, 1024), dtype=np.uint16)
    assert lib.skv_golden_gather_copy(nb, m, cpu_v_length, h.ctypes.data, k.ctypes.data, out.ctypes.data) == 0
    return out
