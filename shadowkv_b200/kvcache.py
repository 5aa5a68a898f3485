"""``ShadowKVCache_CPU`` for B200: the reference's cache class, same API.

Mirror of ``ShadowKVCache_CPU`` (models/kvcache/shadow.py:301-651): same
constructor arguments and method names, V offloaded per layer to
page-locked host memory in 2 KiB chunks, K reconstructed from the rank-r
pre-RoPE factors.  Two decode paths share the state:

* the *reference path* -- ``get_retrieval_position_ids`` /
  ``get_value_cache`` / ``get_key_cache`` call the drop-in bindings of
  ``shadowkv_b200.shadowkv`` exactly as the reference does
  (shadow.py:547-597); buffer slots follow the reference's reorder
  (hits by old slot, then misses by chunk id);
* the *fused path* -- ``select_fused`` / ``fetch_values_fused`` /
  ``reconstruct_keys_fused`` / ``attention`` use the slot-stable kernels of
  ``shadowkv_b200.decode`` (hits never move).

``sync_slots_from_position_ids`` / ``sync_position_ids_from_slots`` convert
between the two slot orders, so one cache can be driven by either.

Prefill builds the state with the reference's algorithm (shadow.py:411-544):
``get_svd`` and ``prefill_kv_cache`` in torch on the GPU (the torch path),
``prefill_kv_cache_native`` with the library's prefill kernels.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import decode as fused
from . import shadowkv
from .tensor_op import batch_gather_gemm_rotary_pos_emb_cuda


def auto_microbatch(batch: int) -> int:
    """Slices of ``decode_step_microbatched`` for a batch: one below 8 sequences (the selection
    is short next to the fetch), else min(8, batch // 2) lowered to a divisor of the batch."""
    parts = min(8, batch // 2) if batch >= 8 else 1
    while parts > 1 and batch % parts:
        parts -= 1
    return parts


def auto_head_groups(batch: int, kv_heads: int) -> int:
    """Kv-head groups of the pipelined step (``decode_step_fused``) for one sequence: the largest
    of 4 and 2 that divides ``kv_heads`` and leaves every group at least 2 kv heads, else 1; 1 for
    a batch (sliced by sequence instead).  Groups of one head split the landmark scan without
    enough link transfer behind it to hide: at 2 kv heads and 1M tokens (GLM-4-9B shape) one
    group measured 75.8 us a step against 82.9 us for two, at 8 kv heads and 122k tokens
    (Llama-3-8B shape) four groups 112.9 us against 118 us for one."""
    if batch != 1:
        return 1
    for p in (4, 2):
        if kv_heads % p == 0 and kv_heads // p >= 2:
            return p
    return 1


class ShadowKVCache_CPU:
    """ShadowKV cache with host-offloaded values (reference models/kvcache/shadow.py:301)."""

    def __init__(self, config, batch_size: int = 1, max_length: int = 32 * 1024, device: str = "cuda:0",
                 dtype=torch.bfloat16, sparse_budget: int = 2048, chunk_size: int = 8, rank: int = 160,
                 local_chunk: int = 4, outlier_chunk: int | None = None, gen_len: int = 128,
                 geometry: str = "cpu", svd: str = "exact"):
        if dtype != torch.bfloat16:
            raise RuntimeError("the CUDA decode path is bf16 only")
        self.config = config
        self.batch_size = batch_size
        self.max_length = max_length
        self.device = torch.device(device)
        self.dtype = dtype
        self.num_key_value_groups = config.num_attention_heads // config.num_key_value_heads
        self.head_dim = config.hidden_size // config.num_attention_heads
        self.num_attention_heads = config.num_attention_heads
        self.num_key_value_heads = config.num_key_value_heads
        self.num_layers = config.num_hidden_layers
        self.sparse_budget = int(sparse_budget)
        self.chunk_size = chunk_size
        self.rank = rank
        self.local_chunk = local_chunk
        # shadow.py:329 (CPU class) derives the outlier count from the budget; the
        # torch class (shadow.py:55) fixes 48.  ``geometry`` picks the chunk rounding.
        self.outlier_chunk = int(outlier_chunk if outlier_chunk is not None else (self.sparse_budget // 1024) * 24)
        self.geometry = geometry
        self.svd_method = svd
        self.gen_len = gen_len
        self.select_sets = self.sparse_budget // self.chunk_size
        if self.select_sets * self.chunk_size != self.sparse_budget:
            raise RuntimeError(f"sparse_budget {self.sparse_budget} is not a multiple of chunk_size {chunk_size}")

        H, D, B, L = self.num_key_value_heads, self.head_dim, batch_size, self.num_layers
        self.host_chunks = max_length // chunk_size
        self.v_cache_cpu = torch.zeros(L, B, H, self.host_chunks, D * chunk_size, dtype=dtype, pin_memory=True)
        # local rows (<= (local_chunk+7) chunks after rounding) + outliers + budget + generated rows
        self.buf_len = self.sparse_budget + gen_len + (self.outlier_chunk + local_chunk + 7) * chunk_size
        self.k_cache_buffer = torch.zeros(L, B, H, self.buf_len, D, dtype=dtype, device=self.device)
        self.v_cache_buffer = torch.zeros(L, B, H, self.buf_len, D, dtype=dtype, device=self.device)
        self.kv_offset = 0
        self.prefill = 0
        self.gen_offset = 0
        self.prefilled_batch = 0
        self.k_landmark = None
        self.k_landmark_idx = None
        self.U = None
        self.SV = None
        # reuse-cache state of the reference path (shadow.py:387-392)
        nblk = B * H
        self.offsets = torch.zeros(nblk * self.select_sets, dtype=torch.int32, device=self.device)
        self.cnts = torch.zeros(nblk, dtype=torch.int32, device=self.device)
        self.signals = torch.zeros(nblk, dtype=torch.int32, device=self.device)
        self.position_ids = torch.full((L, B, H, self.select_sets), -1, dtype=torch.int64, device=self.device)
        self.temp = torch.zeros(B, H, self.select_sets, chunk_size * D, dtype=dtype, device=self.device)
        self.output = torch.zeros(B, H, self.sparse_budget, D, dtype=dtype, device=self.device)
        # slot table of the fused path
        self.slots = torch.full((L, B, H, self.select_sets), -1, dtype=torch.int32, device=self.device)
        self.copy_stream = torch.cuda.Stream(device=self.device)
        self._fused_geom = None
        self._fused_ws = None

    # ------------------------------------------------------------------ info
    def print_stats(self):
        print(f"ShadowKV_CPU(B200) | sparse budget {self.sparse_budget} | chunk size {self.chunk_size} | "
              f"rank {self.rank} | cached {self.kv_offset} | local_chunk {self.local_chunk} | "
              f"outlier_chunk {self.outlier_chunk}")

    def get_kv_len(self):
        return self.kv_offset

    # --------------------------------------------------------------- prefill
    def get_svd(self, new_k_cache: torch.Tensor, layer_idx: int, heads: tuple[int, int] | None = None):
        """Rank-r factors of the pre-RoPE keys (shadow.py:411-444): U [B,T,r], SV^T [B,H,D,r].

        ``heads=(h0, hn)``: ``new_k_cache`` holds the keys of every kv head of the model and this
        cache keeps kv heads h0 .. h0+hn-1 (the heads of one rank when the heads are sharded over
        GPUs): the factorisation runs over all heads, as the reference's (U shared by every head),
        and this cache keeps U and its heads' rows of SV."""
        if new_k_cache.dim() == 4 and new_k_cache.shape[1] <= 32:
            k = new_k_cache.transpose(1, 2).reshape(new_k_cache.shape[0], -1, new_k_cache.shape[1] * self.head_dim)
        else:
            k = new_k_cache
        h_all = k.shape[-1] // self.head_dim
        h0, hn = heads if heads is not None else (0, h_all)
        if hn != self.num_key_value_heads or h0 < 0 or h0 + hn > h_all:
            raise RuntimeError(f"keys of {h_all} kv heads, heads {h0}..{h0 + hn - 1} for a cache of "
                               f"{self.num_key_value_heads}")
        bsz, T, _ = k.shape
        if layer_idx == 0 and self.prefilled_batch == 0:
            self.U = torch.zeros(self.num_layers, self.batch_size, T, self.rank, dtype=self.dtype, device=self.device)
            self.SV = torch.zeros(self.num_layers, self.batch_size, self.num_key_value_heads, self.head_dim, self.rank,
                                  dtype=self.dtype, device=self.device)
        if self.svd_method == "gram":
            # the same leading subspace from the Gram matrix: K^T K on the tensor cores
            # (skv_gram, float64 result), its leading eigenvectors V (float64 eigensolve),
            # then U = K V / s
            kb = k.to(self.device).to(torch.bfloat16)
            G = torch.stack([fused.gram(kb[i]) for i in range(bsz)])
            evals, evecs = torch.linalg.eigh(G)
            order = torch.argsort(evals, dim=-1, descending=True)[:, : self.rank]
            v = torch.gather(evecs, 2, order.unsqueeze(1).expand(-1, evecs.shape[1], -1))  # [b, HD, r]
            s = torch.sqrt(torch.clamp(torch.gather(evals, 1, order), min=0))
            u = (kb.float() @ v.float()) / torch.clamp(s, min=1e-30).float().unsqueeze(1)
            s, vt = s.float(), v.transpose(1, 2).float()
        else:
            kf = k.to(self.device).float()
            u, s, v = torch.svd(kf)
            u, s, vt = u[:, :, : self.rank], s[:, : self.rank], v.transpose(1, 2)[:, : self.rank]
        pb = self.prefilled_batch
        self.U[layer_idx][pb:pb + bsz].copy_(u.to(self.dtype))
        sv = torch.matmul(torch.diag_embed(s), vt).to(self.dtype)  # [b, r, H*D]
        sv = sv.view(bsz, self.rank, h_all, self.head_dim)[:, :, h0:h0 + hn].permute(0, 2, 3, 1)  # [b, H, D, r]
        self.SV[layer_idx][pb:pb + bsz].copy_(sv)

    def register_k_landmark(self, k_landmark, k_landmark_idx, layer_idx):
        num_landmarks = k_landmark.shape[-2]
        bsz = k_landmark.shape[0]
        if layer_idx == 0 and self.prefilled_batch == 0:
            H, G = self.num_key_value_heads, self.num_key_value_groups
            self.k_landmark = torch.zeros(self.num_layers, self.batch_size, H, num_landmarks, self.head_dim,
                                          dtype=self.dtype, device=self.device)
            self.k_landmark_idx = torch.zeros(self.num_layers, self.batch_size, H, num_landmarks, dtype=torch.long,
                                              device=self.device)
            nblk = (num_landmarks + 255) // 256
            self.gemm_o = torch.zeros(self.batch_size, H, G, num_landmarks, dtype=torch.bfloat16, device=self.device)
            self.softmax_o = torch.zeros_like(self.gemm_o)
            self.norm = torch.zeros(self.batch_size * H, G, nblk, dtype=torch.float32, device=self.device)
            self.sum = torch.zeros_like(self.norm)
        pb = self.prefilled_batch
        self.k_landmark[layer_idx][pb:pb + bsz].copy_(k_landmark)
        self.k_landmark_idx[layer_idx][pb:pb + bsz].copy_(k_landmark_idx)

    def prefill_kv_cache(self, new_v_cache: torch.Tensor, layer_idx: int, key_states_roped: torch.Tensor,
                         last_query_states: torch.Tensor = None):
        """Landmarks, outliers, host V and the first selection (shadow.py:463-544)."""
        bsz, H, incoming, D = new_v_cache.shape
        c = self.chunk_size
        self.prefill = incoming
        max_ctx_chunks = incoming // c
        self.max_ctx_chunks_len = max_ctx_chunks * c
        if max_ctx_chunks > self.host_chunks:
            raise RuntimeError(f"prompt of {incoming} tokens exceeds max_length {self.max_length}")
        pb = self.prefilled_batch
        self.v_cache_cpu[layer_idx][pb:pb + bsz, :, :max_ctx_chunks].copy_(
            new_v_cache[:, :, : self.max_ctx_chunks_len].reshape(bsz, H, max_ctx_chunks, c * D))
        self.chunks = incoming // c - self.local_chunk
        if self.geometry == "cpu":
            self.chunks = self.chunks - self.chunks % 8
        self.prefill_local = incoming - self.chunks * c
        kb, vb = self.k_cache_buffer[layer_idx], self.v_cache_buffer[layer_idx]
        kb[pb:pb + bsz, :, : self.prefill_local].copy_(key_states_roped[:, :, -self.prefill_local:])
        vb[pb:pb + bsz, :, : self.prefill_local].copy_(new_v_cache[:, :, -self.prefill_local:])

        ctx = key_states_roped[:, :, : self.chunks * c].reshape(bsz, H, self.chunks, c, D)
        landmark_candidates = ctx.mean(dim=-2)
        cos_sim = F.cosine_similarity(landmark_candidates.unsqueeze(3).expand(-1, -1, -1, c, -1), ctx, dim=-1)
        outlier_idx = cos_sim.min(dim=-1).values.topk(self.outlier_chunk, largest=False).indices
        gidx = outlier_idx.unsqueeze(-1).unsqueeze(-1).expand(-1, -1, -1, c, D)
        outlier_k = ctx.gather(dim=2, index=gidx).reshape(bsz, H, self.outlier_chunk * c, D)
        outlier_v = new_v_cache[:, :, : self.chunks * c].reshape(bsz, H, self.chunks, c, D).gather(
            dim=2, index=gidx).reshape(bsz, H, self.outlier_chunk * c, D)
        self.sparse_start = self.prefill_local + self.outlier_chunk * c
        self.sparse_end = self.sparse_start + self.sparse_budget
        if self.sparse_end + self.gen_len > self.buf_len:
            raise RuntimeError("K/V buffer too small for the prefill geometry")
        self.kernel_offset = self.sparse_start * D
        self.kernel_stride = self.buf_len * D
        kb[pb:pb + bsz, :, self.prefill_local:self.sparse_start].copy_(outlier_k)
        vb[pb:pb + bsz, :, self.prefill_local:self.sparse_start].copy_(outlier_v)

        all_idx = torch.arange(self.chunks, device=key_states_roped.device).expand(bsz, H, -1)
        mask = torch.ones_like(all_idx, dtype=torch.bool)
        mask.scatter_(dim=-1, index=outlier_idx, value=False)
        rest_idx = all_idx.masked_select(mask).view(bsz, H, -1)
        self.register_k_landmark(
            landmark_candidates.gather(dim=2, index=rest_idx.unsqueeze(-1).expand(-1, -1, -1, D)), rest_idx, layer_idx)

        # first selection with the last prompt query (shadow.py:521-534)
        G = self.num_key_value_groups
        lm = self.k_landmark[layer_idx][pb:pb + bsz]
        chunk_attn = torch.einsum("bhgd,bhcd->bhgc", last_query_states.reshape(bsz, H, G, D).to(lm.dtype), lm)
        chunk_attn = F.softmax(chunk_attn / math.sqrt(128), dim=-1, dtype=torch.float32).to(self.dtype)
        chunk_attn, _ = torch.max(chunk_attn, dim=-2)
        merged = torch.topk(chunk_attn, k=self.select_sets, dim=-1).indices
        selected = self.k_landmark_idx[layer_idx][pb:pb + bsz].gather(dim=-1, index=merged)
        self.position_ids[layer_idx][pb:pb + bsz].copy_(selected)
        self.slots[layer_idx][pb:pb + bsz].copy_(selected.to(torch.int32))
        tok = (selected.unsqueeze(-1) * c + torch.arange(c, device=selected.device)).view(bsz, H, -1)
        vb[pb:pb + bsz, :, self.sparse_start:self.sparse_end].copy_(
            new_v_cache.gather(dim=-2, index=tok.unsqueeze(-1).expand(-1, -1, -1, D)))
        kb[pb:pb + bsz, :, self.sparse_start:self.sparse_end].copy_(
            key_states_roped.gather(dim=-2, index=tok.unsqueeze(-1).expand(-1, -1, -1, D)))
        if layer_idx == self.num_layers - 1:
            self.prefilled_batch += bsz
            if self.prefilled_batch == self.batch_size:
                self.kv_offset += incoming

    def prefill_kv_cache_native(self, new_v_cache: torch.Tensor, layer_idx: int, key_states_roped: torch.Tensor,
                                last_query_states: torch.Tensor, build_events=None):
        """``prefill_kv_cache`` as GPU kernels (``skv_prefill_build``): host value store,
        landmarks and outliers (bf16 op by op like the torch ops), first selection with
        fp32 scores, buffer rows.  Same state layout; outliers listed by (similarity,
        chunk id), the first selection in ascending chunk id per slot.  ``build_events``
        (two CUDA events) bracket the device-state kernels on the current stream, the
        host-store copy running beside them on the copy stream."""
        import ctypes
        from ._lib import PrefillGeom, check, lib
        bsz, H, incoming, D = new_v_cache.shape
        c = self.chunk_size
        if incoming // c > self.host_chunks:
            raise RuntimeError(f"prompt of {incoming} tokens exceeds max_length {self.max_length}")
        chunks = incoming // c - self.local_chunk
        if self.geometry == "cpu":
            chunks = chunks - chunks % 8
        prefill_local = incoming - chunks * c
        sparse_start = prefill_local + self.outlier_chunk * c
        if sparse_start + self.sparse_budget + self.gen_len > self.buf_len:
            raise RuntimeError("K/V buffer too small for the prefill geometry")
        num_landmarks = chunks - self.outlier_chunk
        if self.k_landmark is None:
            G = self.num_key_value_groups
            self.k_landmark = torch.zeros(self.num_layers, self.batch_size, H, num_landmarks, D, dtype=self.dtype,
                                          device=self.device)
            self.k_landmark_idx = torch.zeros(self.num_layers, self.batch_size, H, num_landmarks, dtype=torch.long,
                                              device=self.device)
            nblk = (num_landmarks + 255) // 256
            self.gemm_o = torch.zeros(self.batch_size, H, G, num_landmarks, dtype=torch.bfloat16, device=self.device)
            self.softmax_o = torch.zeros_like(self.gemm_o)
            self.norm = torch.zeros(self.batch_size * H, G, nblk, dtype=torch.float32, device=self.device)
            self.sum = torch.zeros_like(self.norm)
        if self.k_landmark.shape[-2] != num_landmarks:
            raise RuntimeError("every layer and sequence of one cache must have the same prompt geometry")
        pb = self.prefilled_batch
        pg = PrefillGeom(batch=bsz, kv_heads=H, q_heads=self.num_attention_heads, tokens=incoming, chunks=chunks,
                         outlier_chunk=self.outlier_chunk, select_sets=self.select_sets, buf_len=self.buf_len,
                         host_chunks=self.host_chunks)
        nbytes = int(lib.skv_prefill_workspace(ctypes.byref(pg)))
        if nbytes == 0:
            raise RuntimeError("prefill geometry rejected: " + (lib.skv_last_error() or b"").decode())
        ws = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        k = key_states_roped.contiguous()
        v = new_v_cache.contiguous()
        q = last_query_states.reshape(bsz, self.num_attention_heads, D).to(self.dtype).contiguous()
        for t in (k, v, q):
            if not t.is_cuda or t.dtype != self.dtype:
                raise RuntimeError("prefill inputs must be bf16 CUDA tensors")
        cur = torch.cuda.current_stream(self.device)
        # the 8 MB-per-head copy into the host store runs on the copy stream, beside the kernels
        self.copy_stream.wait_stream(cur)
        check(lib.skv_prefill_store_values(ctypes.byref(pg), v.data_ptr(),
                                           self.v_cache_cpu[layer_idx][pb:pb + bsz].data_ptr(),
                                           self.copy_stream.cuda_stream), "skv_prefill_store_values")
        if build_events is not None:
            build_events[0].record(cur)
        check(lib.skv_prefill_build(
            ctypes.byref(pg), k.data_ptr(), v.data_ptr(), q.data_ptr(),
            self.k_cache_buffer[layer_idx][pb:pb + bsz].data_ptr(), self.v_cache_buffer[layer_idx][pb:pb + bsz].data_ptr(),
            self.k_landmark[layer_idx][pb:pb + bsz].data_ptr(), self.k_landmark_idx[layer_idx][pb:pb + bsz].data_ptr(),
            self.slots[layer_idx][pb:pb + bsz].data_ptr(), self.position_ids[layer_idx][pb:pb + bsz].data_ptr(),
            ws.data_ptr(), nbytes, cur.cuda_stream), "skv_prefill_build")
        if build_events is not None:
            build_events[1].record(cur)
        cur.wait_stream(self.copy_stream)
        v.record_stream(self.copy_stream)
        self.prefill = incoming
        self.max_ctx_chunks_len = (incoming // c) * c
        self.chunks = chunks
        self.prefill_local = prefill_local
        self.sparse_start = sparse_start
        self.sparse_end = sparse_start + self.sparse_budget
        self.kernel_offset = self.sparse_start * D
        self.kernel_stride = self.buf_len * D
        if layer_idx == self.num_layers - 1:
            self.prefilled_batch += bsz
            if self.prefilled_batch == self.batch_size:
                self.kv_offset += incoming
        return ws  # keep the scratch alive until the stream is past the launch

    def H2D(self):
        """The state already lives on the device; kept for API parity (shadow.py:599-619)."""
        torch.cuda.synchronize(self.device)

    # ------------------------------------------------ decode: reference path
    def get_retrieval_position_ids(self, layer_idx, query_states):
        """shadow.py:547-576 with the B200 bindings."""
        self.incoming_q_len = query_states.shape[-2]
        B, H, G = self.batch_size, self.num_key_value_heads, self.num_key_value_groups
        lm = self.k_landmark[layer_idx]
        shadowkv.batch_gemm_softmax(query_states.contiguous(), lm, self.gemm_o, self.norm, self.sum,
                                    self.softmax_o, B * H, G * self.incoming_q_len, lm.shape[-2], self.head_dim,
                                    1 / math.sqrt(128), 0)
        if G > 1:
            chunk_attn, _ = torch.max(self.softmax_o.view(B, H, G, -1), dim=-2)
        else:
            chunk_attn = self.softmax_o.view(B, H, -1)
        merged = torch.topk(chunk_attn.view(B, H, -1), k=self.select_sets, dim=-1).indices
        selected = self.k_landmark_idx[layer_idx].gather(dim=-1, index=merged)
        shadowkv.reorder_keys_and_compute_offsets(self.position_ids[layer_idx], selected, self.offsets, self.cnts,
                                                  B, H, self.select_sets)
        return self.position_ids[layer_idx]

    def _gen_offset(self, layer_idx):
        return self.gen_offset if layer_idx == self.num_layers - 1 else self.gen_offset + self.incoming_q_len

    def get_value_cache(self, layer_idx, position_ids):
        """shadow.py:578-584."""
        host = self.v_cache_cpu[layer_idx]
        shadowkv.gather_copy_with_offsets(host, self.v_cache_buffer[layer_idx], self.temp, self.offsets, self.cnts,
                                          self.signals, self.batch_size, self.num_key_value_heads,
                                          int(host.stride(1)), int(self.sparse_budget * self.head_dim),
                                          self.kernel_offset, self.kernel_stride, self.select_sets)
        return self.v_cache_buffer[layer_idx][:, :, : self.sparse_end + self._gen_offset(layer_idx)]

    def get_key_cache(self, layer_idx, position_ids, rope_func, cos_sin_cache):
        """shadow.py:586-597 (``rope_func`` is unused, as in the reference)."""
        kb = self.k_cache_buffer[layer_idx]
        shadowkv.gather_copy_d2d_with_offsets(kb, self.offsets, self.cnts, self.batch_size, self.num_key_value_heads,
                                              int(self.sparse_budget * self.head_dim), self.kernel_offset,
                                              self.kernel_stride, self.select_sets)
        batch_gather_gemm_rotary_pos_emb_cuda(self.U[layer_idx], self.SV[layer_idx], cos_sin_cache, position_ids,
                                              self.output, self.chunk_size, kb, self.sparse_start, self.sparse_end,
                                              self.cnts)
        return kb[:, :, : self.sparse_end + self._gen_offset(layer_idx)]

    def update_kv_cache(self, new_k_cache, new_v_cache, layer_idx):
        """shadow.py:621-633: append the new token's post-RoPE K and V."""
        incoming = new_k_cache.shape[-2]
        s0 = self.sparse_end + self.gen_offset
        if s0 + incoming > self.buf_len:
            raise RuntimeError("generated-token region of the K/V buffer is full")
        self.v_cache_buffer[layer_idx][:, :, s0:s0 + incoming].copy_(new_v_cache, non_blocking=True)
        self.k_cache_buffer[layer_idx][:, :, s0:s0 + incoming].copy_(new_k_cache, non_blocking=True)
        if layer_idx == self.num_layers - 1:
            self.kv_offset += incoming
            self.gen_offset += incoming

    def clear(self):
        self.k_cache_buffer.zero_()
        self.v_cache_buffer.zero_()
        self.k_landmark = None
        self.k_landmark_idx = None
        self.U = None
        self.SV = None
        self.kv_offset = 0
        self.prefill = 0
        self.gen_offset = 0
        self.prefill_local = 0
        self.prefilled_batch = 0
        self.position_ids.fill_(-1)
        self.slots.fill_(-1)

    # ---------------------------------------------------- decode: fused path
    def fused_geometry(self, cos_sin_cache: torch.Tensor) -> fused.Geometry:
        if self._fused_geom is None:
            glm = cos_sin_cache.shape[-1] == 64
            self._fused_geom = fused.Geometry(
                batch=self.batch_size, kv_heads=self.num_key_value_heads, q_heads=self.num_attention_heads,
                rank=self.rank, select_sets=self.select_sets, num_landmarks=self.k_landmark.shape[-2],
                num_chunks=self.host_chunks, ctx_len=self.U.shape[2], buf_len=self.buf_len,
                sparse_start=self.sparse_start, rope_mode=1 if glm else 0,
                cos_sin_stride=cos_sin_cache.stride(0), cos_sin_rows=cos_sin_cache.shape[0],
                head_dim=self.head_dim, chunk_size=self.chunk_size)
            self._fused_ws = fused.DecodeWorkspace(self._fused_geom, self.device)
        return self._fused_geom

    def append_fused(self, layer_idx, query_states, key_states, value_states, positions, cos_sin_cache,
                     q_out=None):
        """RoPE of the new token's q/k and append of k/v at ``sparse_end + gen_offset`` (one kernel).

        query_states [B, Hq, 1, D], key/value_states [B, Hkv, 1, D] (pre-RoPE),
        positions [B] or [B, 1] int64.  Returns the rotated query [B, Hq, 1, D].
        Same effect as RoPE + ``update_kv_cache`` (shadow.py:621-633).
        """
        g = self.fused_geometry(cos_sin_cache)
        row = self.sparse_end + self.gen_offset
        if row >= self.buf_len:
            raise RuntimeError("generated-token region of the K/V buffer is full")
        B, Hq, Hk, D = self.batch_size, self.num_attention_heads, self.num_key_value_heads, self.head_dim
        if q_out is None:
            q_out = torch.empty(B, Hq, 1, D, dtype=self.dtype, device=self.device)
        fused.append(g, query_states.reshape(B, Hq, D), key_states.reshape(B, Hk, D),
                     value_states.reshape(B, Hk, D), positions.reshape(B), cos_sin_cache, q_out,
                     self.k_cache_buffer[layer_idx], self.v_cache_buffer[layer_idx], row)
        if layer_idx == self.num_layers - 1:
            self.kv_offset += 1
            self.gen_offset += 1
        return q_out

    def append_select_fused(self, layer_idx, query_states, key_states, value_states, positions, cos_sin_cache,
                            q_out=None):
        """``append_fused`` + ``select_fused`` in one scoring pass; returns the rotated query."""
        g = self.fused_geometry(cos_sin_cache)
        row = self.sparse_end + self.gen_offset
        if row >= self.buf_len:
            raise RuntimeError("generated-token region of the K/V buffer is full")
        B, Hq, Hk, D = self.batch_size, self.num_attention_heads, self.num_key_value_heads, self.head_dim
        if q_out is None:
            q_out = torch.empty(B, Hq, 1, D, dtype=self.dtype, device=self.device)
        self.incoming_q_len = 1
        fused.append_select(g, self._fused_ws, query_states.reshape(B, Hq, D), key_states.reshape(B, Hk, D),
                            value_states.reshape(B, Hk, D), positions.reshape(B), cos_sin_cache, q_out,
                            self.k_cache_buffer[layer_idx], self.v_cache_buffer[layer_idx], row,
                            self.k_landmark[layer_idx], self.k_landmark_idx[layer_idx], self.slots[layer_idx])
        if layer_idx == self.num_layers - 1:
            self.kv_offset += 1
            self.gen_offset += 1
        return q_out

    def select_fused(self, layer_idx, query_states, cos_sin_cache):
        """Scoring + top-k + slot-stable reuse diff of one layer (fused kernels)."""
        self.incoming_q_len = query_states.shape[-2]
        g = self.fused_geometry(cos_sin_cache)
        q = query_states.reshape(self.batch_size, self.num_attention_heads, self.head_dim)
        fused.select(g, self._fused_ws, q.contiguous(), self.k_landmark[layer_idx], self.k_landmark_idx[layer_idx],
                     self.slots[layer_idx])

    def fetch_values_fused(self, layer_idx, stream=None):
        fused.gather_values(self._fused_geom, self._fused_ws, self.v_cache_cpu[layer_idx],
                            self.v_cache_buffer[layer_idx], stream)

    def reconstruct_keys_fused(self, layer_idx, cos_sin_cache, stream=None):
        fused.reconstruct_keys(self._fused_geom, self._fused_ws, self.U[layer_idx], self.SV[layer_idx], cos_sin_cache,
                               self.k_cache_buffer[layer_idx], stream)

    def sparse_attention_fused(self, layer_idx, query_states, seq_len, cos_sin_cache, out=None):
        """Fetch of the missed values + reconstruction of the missed keys + attention, one launch."""
        q = query_states.reshape(self.batch_size, self.num_attention_heads, self.head_dim)
        if out is None:
            out = torch.empty_like(q)
        return fused.sparse_attention(self._fused_geom, self._fused_ws, q, self.U[layer_idx], self.SV[layer_idx],
                                      cos_sin_cache, self.v_cache_cpu[layer_idx], self.k_cache_buffer[layer_idx],
                                      self.v_cache_buffer[layer_idx], seq_len, out)

    def decode_step_fused(self, layer_idx, query_states, key_states, value_states, positions, cos_sin_cache,
                          out=None, head_groups: int | None = None, q_out=None, row_dev=None):
        """One whole decode step of a layer in one library call (``skv_decode_step``): RoPE of the
        new token's q/k and append at ``sparse_end + gen_offset``, scoring, top-k, slot-stable reuse
        diff, fetch of the missed values, reconstruction of the missed keys, attention over
        ``[0, sparse_end + gen_offset + 1)``.  Same results as ``append_select_fused`` +
        ``sparse_attention_fused``.  ``head_groups`` > 1 (batch 1) pipelines the step over groups
        of kv heads so the first group's value fetch starts after a fraction of the landmark scan
        (default ``auto_head_groups``).  ``row_dev`` (one int32 on the device, = sparse_end +
        gen_offset): the append position read at run time (``graph.DecodeGraph`` replays a captured
        step at later positions with it); the launches are then sized for the whole buffer.
        Returns ``out`` [B, Hq, D]."""
        B, Hq, Hk, D = self.batch_size, self.num_attention_heads, self.num_key_value_heads, self.head_dim
        if head_groups is None:
            head_groups = auto_head_groups(B, Hk)
        g = self.fused_geometry(cos_sin_cache)
        row = self.sparse_end + self.gen_offset
        if row >= self.buf_len:
            raise RuntimeError("generated-token region of the K/V buffer is full")
        sws = getattr(self, "_step_ws", None)
        if sws is None or sws.head_groups != head_groups:
            sws = self._step_ws = fused.StepWorkspace(g, head_groups, self.device)
        if q_out is None:
            q_out = torch.empty(B, Hq, 1, D, dtype=self.dtype, device=self.device)
        if out is None:
            out = torch.empty(B, Hq, D, dtype=self.dtype, device=self.device)
        if row_dev is not None:  # launches sized for the last row of the buffer
            row = self.buf_len - 1
        fused.step(g, sws, query_states.reshape(B, Hq, D), key_states.reshape(B, Hk, D),
                   value_states.reshape(B, Hk, D), positions.reshape(B), cos_sin_cache, q_out,
                   self.k_cache_buffer[layer_idx], self.v_cache_buffer[layer_idx], row, self.k_landmark[layer_idx],
                   self.k_landmark_idx[layer_idx], self.slots[layer_idx], self.U[layer_idx], self.SV[layer_idx],
                   self.v_cache_cpu[layer_idx], row + 1, out, row_dev=row_dev)
        self.incoming_q_len = 1
        if layer_idx == self.num_layers - 1:
            self.kv_offset += 1
            self.gen_offset += 1
        return out

    def decode_step_microbatched(self, layer_idx, query_states, key_states, value_states, positions, cos_sin_cache,
                                 out, parts: int, q_out=None, max_ctas: int = 64):
        """The fused step (``append_select_fused`` + ``sparse_attention_fused``) in ``parts`` slices of
        the batch: slice i's scoring and selection run on a high-priority stream while slice i-1's
        value fetch, capped at ``max_ctas`` CTAs (plenty to keep the host link busy), holds the
        others -- the link no longer waits for the whole batch's selection.  The fetches of
        consecutive slices alternate between two streams, so one's tail overlaps the next one's
        start.  ``out`` [B, Hq, D]."""
        B, Hq, Hk, D = self.batch_size, self.num_attention_heads, self.num_key_value_heads, self.head_dim
        if parts < 1 or B % parts:
            raise RuntimeError(f"batch {B} does not split into {parts} equal parts")
        g = self.fused_geometry(cos_sin_cache)
        row = self.sparse_end + self.gen_offset
        if row >= self.buf_len:
            raise RuntimeError("generated-token region of the K/V buffer is full")
        mb = B // parts
        key = (parts, mb)
        if getattr(self, "_mb_state", None) is None or self._mb_state[0] != key:
            import dataclasses
            gp = dataclasses.replace(g, batch=mb)
            self._mb_state = (key, gp, [fused.DecodeWorkspace(gp, self.device) for _ in range(parts)],
                              torch.cuda.Stream(device=self.device, priority=-1),
                              [torch.cuda.Stream(device=self.device, priority=0) for _ in range(2)])
        _, gp, wss, hi, los = self._mb_state
        if q_out is None:
            q_out = torch.empty(B, Hq, 1, D, dtype=self.dtype, device=self.device)
        q = query_states.reshape(B, Hq, D)
        k = key_states.reshape(B, Hk, D)
        v = value_states.reshape(B, Hk, D)
        pos = positions.reshape(B)
        qo = q_out.reshape(B, Hq, D)
        last = layer_idx == self.num_layers - 1
        seq_len = self.sparse_end + (self.gen_offset + 1)
        cur = torch.cuda.current_stream(self.device)
        hi.wait_stream(cur)
        for lo in los:
            lo.wait_stream(cur)
        for i in range(parts):
            sl = slice(i * mb, (i + 1) * mb)
            lo = los[i % 2]  # consecutive slices' fetches may overlap: the link never waits for a tail
            with torch.cuda.stream(hi):
                fused.append_select(gp, wss[i], q[sl], k[sl], v[sl], pos[sl], cos_sin_cache, qo[sl],
                                    self.k_cache_buffer[layer_idx][sl], self.v_cache_buffer[layer_idx][sl], row,
                                    self.k_landmark[layer_idx][sl], self.k_landmark_idx[layer_idx][sl],
                                    self.slots[layer_idx][sl], stream=hi)
                ev = torch.cuda.Event()
                ev.record(hi)
            with torch.cuda.stream(lo):
                lo.wait_event(ev)
                fused.sparse_attention(gp, wss[i], qo[sl], self.U[layer_idx][sl], self.SV[layer_idx][sl],
                                       cos_sin_cache, self.v_cache_cpu[layer_idx][sl],
                                       self.k_cache_buffer[layer_idx][sl], self.v_cache_buffer[layer_idx][sl],
                                       seq_len, out[sl], stream=lo, max_ctas=max_ctas)
        cur.wait_stream(hi)
        for lo in los:
            cur.wait_stream(lo)
        self.incoming_q_len = 1
        if last:
            self.kv_offset += 1
            self.gen_offset += 1
        return out

    def sparse_attention_gather(self, layer_idx, query_states, seq_len, cos_sin_cache, peer):
        """``sparse_attention_fused`` with the output rows sent to every rank's landing buffer
        (kv heads split over ranks; ``peer`` is a ``peer.PeerOutput``, ``peer.finish`` ends the step)."""
        q = query_states.reshape(self.batch_size, self.num_attention_heads, self.head_dim)
        peer.attention(self._fused_geom, self._fused_ws, q, self.U[layer_idx], self.SV[layer_idx], cos_sin_cache,
                       self.v_cache_cpu[layer_idx], self.k_cache_buffer[layer_idx], self.v_cache_buffer[layer_idx],
                       seq_len)

    def attention(self, layer_idx, query_states, seq_len, out=None):
        """GQA decode attention over buffer rows [0, seq_len) -> [B, Hq, D]."""
        g = self._fused_geom if self._fused_geom is not None else fused.Geometry(
            batch=self.batch_size, kv_heads=self.num_key_value_heads, q_heads=self.num_attention_heads,
            rank=self.rank, select_sets=self.select_sets, num_landmarks=self.select_sets,
            num_chunks=self.host_chunks, ctx_len=self.max_length, buf_len=self.buf_len, sparse_start=0)
        if self._fused_ws is None or self._fused_geom is None:
            self._attn_ws = getattr(self, "_attn_ws", None) or fused.DecodeWorkspace(g, self.device)
            ws = self._attn_ws
        else:
            ws = self._fused_ws
        q = query_states.reshape(self.batch_size, self.num_attention_heads, self.head_dim).contiguous()
        if out is None:
            out = torch.empty_like(q)
        return fused.attention(g, ws, q, self.k_cache_buffer[layer_idx], self.v_cache_buffer[layer_idx], seq_len, out)

    def hit_rate(self, step: bool = False) -> float:
        """Fraction of selected chunks served from the reuse cache in the last fused selection
        (``step``: in the last ``decode_step_fused``)."""
        ws = getattr(self, "_step_ws", None) if step else self._fused_ws
        if ws is None:
            return float("nan")
        miss = ws.miss_count.sum().item()
        return 1.0 - miss / (self.batch_size * self.num_key_value_heads * self.select_sets)

    def sync_slots_from_position_ids(self, layer_idx=None):
        layers = range(self.num_layers) if layer_idx is None else [layer_idx]
        for l in layers:
            self.slots[l].copy_(self.position_ids[l].to(torch.int32))

    def sync_position_ids_from_slots(self, layer_idx=None):
        layers = range(self.num_layers) if layer_idx is None else [layer_idx]
        for l in layers:
            self.position_ids[l].copy_(self.slots[l].to(torch.int64))
