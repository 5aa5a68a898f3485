"""``ShadowAttention`` for B200 (reference models/attention/shadow.py:6-49).

``decode`` follows the reference step for step: RoPE of the new q/k, append
to the K/V buffers, chunk selection, value fetch on the cache's copy stream
overlapped with key reconstruction on the current stream, join, attention.
The attention is the library's split-K GQA kernel instead of
``flash_attn_with_kvcache``; the q/k RoPE uses the library's RoPE binding
instead of vllm's ``rotary_embedding`` custom op (llama.py:149-154).
``decode_fused`` runs the same step on the fused slot-stable kernels.

``prefill`` builds the cache state (SVD in torch; landmarks, outliers, host
store and first selection in torch or, with ``native=True``, with the
library's prefill kernels) and returns no attention output.
"""
from __future__ import annotations

import torch

from .kvcache import ShadowKVCache_CPU, auto_microbatch
from .tensor_op import apply_rotary_pos_emb_cuda


class ShadowAttention:
    def __init__(self, kv_cache: ShadowKVCache_CPU, num_key_value_groups, head_dim, hidden_size,
                 cos_sin_cache: torch.Tensor):
        self.kv_cache = kv_cache
        self.num_key_value_groups = num_key_value_groups
        self.head_dim = head_dim
        self.hidden_size = hidden_size
        self.cos_sin_cache = cos_sin_cache

    def apply_rotary_pos_emb(self, q: torch.Tensor, k: torch.Tensor, position_ids: torch.Tensor):
        """RoPE of q [B, Hq, S, D] and k [B, Hkv, S, D] at token positions [B, S] (int64)."""
        B, Hq, S, D = q.shape
        Hk = k.shape[1]
        pq = position_ids.view(B, 1, S).expand(B, Hq, S)
        pk = position_ids.view(B, 1, S).expand(B, Hk, S)
        return apply_rotary_pos_emb_cuda(q, self.cos_sin_cache, pq), apply_rotary_pos_emb_cuda(k, self.cos_sin_cache, pk)

    def prefill(self, query_states, key_states, value_states, position_ids, layer_idx, native=False):
        """Build the cache state of one layer (pre-RoPE k -> SVD; post-RoPE k -> landmarks).

        ``native=True`` builds the landmarks, outliers, host store, first selection and
        buffer rows with the library's prefill kernels instead of the torch ops."""
        kv = self.kv_cache
        kv.get_svd(key_states, layer_idx=layer_idx)
        q, k = self.apply_rotary_pos_emb(query_states, key_states, position_ids)
        if native:
            kv.prefill_kv_cache_native(value_states, layer_idx, k, q[:, :, -1:])
        else:
            kv.prefill_kv_cache(value_states, layer_idx, k, q[:, :, -1:])

    def decode(self, query_states, key_states, value_states, position_ids, layer_idx):
        """models/attention/shadow.py:22-48 -> attention output [B, 1, Hq, D]."""
        kv = self.kv_cache
        query_states, key_states = self.apply_rotary_pos_emb(query_states, key_states, position_ids)
        kv.update_kv_cache(key_states, value_states, layer_idx)
        pos = kv.get_retrieval_position_ids(layer_idx=layer_idx, query_states=query_states)
        curr = torch.cuda.current_stream()
        copy_stream = kv.copy_stream
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_stream(curr)
            value_states = kv.get_value_cache(layer_idx, pos)
        key_states = kv.get_key_cache(layer_idx=layer_idx, position_ids=pos, rope_func=None,
                                      cos_sin_cache=self.cos_sin_cache)
        curr.wait_stream(copy_stream)
        out = kv.attention(layer_idx, query_states, key_states.shape[2])
        return out.view(out.shape[0], 1, out.shape[1], out.shape[2])

    def decode_fused(self, query_states, key_states, value_states, position_ids, layer_idx, microbatch=None):
        """Same step on the fused kernels (slot-stable reuse cache): scoring +
        selection, then one launch for value fetch, key reconstruction and attention.

        ``microbatch``: batch slices whose selection overlaps the previous slice's
        fetch (``decode_step_microbatched``); ``None`` picks min(8, B // 2) slices
        from 8 sequences up and one slice below."""
        kv = self.kv_cache
        B = kv.batch_size
        parts = microbatch if microbatch is not None else auto_microbatch(B)
        while parts > 1 and B % parts:
            parts -= 1
        if parts > 1:
            out = torch.empty(B, kv.num_attention_heads, kv.head_dim, dtype=kv.dtype, device=kv.device)
            kv.decode_step_microbatched(layer_idx, query_states.contiguous(), key_states.contiguous(),
                                        value_states.contiguous(), position_ids.contiguous(), self.cos_sin_cache,
                                        out, parts)
            return out.view(B, 1, out.shape[1], out.shape[2])
        query_states = kv.append_select_fused(layer_idx, query_states.contiguous(), key_states.contiguous(),
                                              value_states.contiguous(), position_ids.contiguous(),
                                              self.cos_sin_cache)
        seq_len = kv.sparse_end + kv._gen_offset(layer_idx)
        out = kv.sparse_attention_fused(layer_idx, query_states, seq_len, self.cos_sin_cache)
        return out.view(out.shape[0], 1, out.shape[1], out.shape[2])

    def decode_graph(self, head_groups: int | None = None, chain: bool = False):
        """A ``graph.DecodeGraph`` over this attention's cache: the decode step of every layer
        captured once as a CUDA graph and replayed for the following tokens."""
        from .graph import DecodeGraph
        return DecodeGraph(self, head_groups=head_groups, chain=chain)

    def decode_fused_split(self, query_states, key_states, value_states, position_ids, layer_idx):
        """decode_fused with fetch, reconstruction and attention as three launches
        (fetch on the copy stream, overlapping the reconstruction)."""
        kv = self.kv_cache
        query_states = kv.append_select_fused(layer_idx, query_states.contiguous(), key_states.contiguous(),
                                              value_states.contiguous(), position_ids.contiguous(),
                                              self.cos_sin_cache)
        curr = torch.cuda.current_stream()
        copy_stream = kv.copy_stream
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_stream(curr)
            kv.fetch_values_fused(layer_idx, copy_stream)
        kv.reconstruct_keys_fused(layer_idx, self.cos_sin_cache)
        curr.wait_stream(copy_stream)
        seq_len = kv.sparse_end + kv._gen_offset(layer_idx)
        out = kv.attention(layer_idx, query_states, seq_len)
        return out.view(out.shape[0], 1, out.shape[1], out.shape[2])
