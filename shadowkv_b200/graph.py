"""The decode step of every layer captured once as a CUDA graph and replayed.

The reference runs the decode step layer by layer, eagerly: models/base.py:85-100
calls each layer in turn, and the attention of a layer (models/attention/
shadow.py:22-48) launches the RoPE, the selection, the value fetch on the
cache's copy stream (a fork and a join per layer) and the attention one
kernel at a time.  ``DecodeGraph`` records the attention part of all layers of
a step -- one ``skv_decode_step`` per layer, each forking onto the library's
streams for its kv-head groups and joining back -- as one CUDA graph, and
replays it for every later token.

The token position advances on the device: the step reads the row it
appends at (``sparse_end + gen_offset``) from a device int that the graph
itself increments after the last layer, so one capture serves every step
until the generated-token region of the buffers is full.

Usage::

    g = DecodeGraph(attn)                 # attn: ShadowAttention over a prefilled cache
    out = g.step(q, k, v, positions)      # q [L,B,Hq,1,D], k/v [L,B,Hkv,1,D] pre-RoPE, positions [B]
                                          # out [L,B,Hq,D]; the first call runs eagerly and captures

With ``chain=True`` layer l+1's query is layer l's attention output (q[0]
alone is read), a data dependency between the layers inside the graph, as
between the layers of a model.
"""
from __future__ import annotations

import torch

from .attention import ShadowAttention
from .kvcache import auto_head_groups


class DecodeGraph:
    def __init__(self, attn: ShadowAttention, head_groups: int | None = None, chain: bool = False):
        kv = attn.kv_cache
        self.attn, self.kv, self.chain = attn, kv, chain
        self.layers = kv.num_layers
        B, Hq, Hk, D = kv.batch_size, kv.num_attention_heads, kv.num_key_value_heads, kv.head_dim
        self.head_groups = head_groups if head_groups is not None else auto_head_groups(B, Hk)
        dev, dt = kv.device, kv.dtype
        L = self.layers
        self.q = torch.zeros(L, B, Hq, 1, D, dtype=dt, device=dev)
        self.k = torch.zeros(L, B, Hk, 1, D, dtype=dt, device=dev)
        self.v = torch.zeros(L, B, Hk, 1, D, dtype=dt, device=dev)
        self.positions = torch.zeros(B, dtype=torch.int64, device=dev)
        self.q_rot = torch.empty(L, B, Hq, 1, D, dtype=dt, device=dev)
        self.out = torch.empty(L, B, Hq, D, dtype=dt, device=dev)
        self.row = torch.zeros(1, dtype=torch.int32, device=dev)  # the append row of the next step
        self.graph = None

    def _body(self):
        kv = self.kv
        B, Hq, D = kv.batch_size, kv.num_attention_heads, kv.head_dim
        for l in range(self.layers):
            q_in = self.q[l] if (l == 0 or not self.chain) else self.out[l - 1].view(B, Hq, 1, D)
            kv.decode_step_fused(l, q_in, self.k[l], self.v[l], self.positions, self.attn.cos_sin_cache,
                                 out=self.out[l], head_groups=self.head_groups, q_out=self.q_rot[l],
                                 row_dev=self.row)
        self.row.add_(1)  # the next step appends one row further

    def step(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        """One decode step of every layer.  q [L, B, Hq, 1, D] (with ``chain``: [B, Hq, 1, D] or the
        same [L, ...] of which layer 0 is read), k and v [L, B, Hkv, 1, D], all pre-RoPE;
        positions [B] int64.  Returns the attention outputs [L, B, Hq, D] (a buffer the next call
        overwrites).  The first call runs the step eagerly and captures the graph; every later
        call replays it."""
        kv = self.kv
        if kv.sparse_end + kv.gen_offset >= kv.buf_len:
            raise RuntimeError("generated-token region of the K/V buffer is full")
        if self.chain and q.dim() == 4:
            self.q[0].copy_(q)
        else:
            self.q.copy_(q)
        self.k.copy_(k)
        self.v.copy_(v)
        self.positions.copy_(positions.reshape(-1))
        if self.graph is None:
            # the first step runs eagerly: it creates the workspaces and the library's streams and
            # sets the kernels' shared-memory limits outside stream capture
            self.row.fill_(kv.sparse_end + kv.gen_offset)
            self._body()
            torch.cuda.synchronize(kv.device)
            saved = (kv.gen_offset, kv.kv_offset)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._body()  # recorded only: the cache's host counters are restored below
            kv.gen_offset, kv.kv_offset = saved
            return self.out
        self.graph.replay()
        kv.gen_offset += 1
        kv.kv_offset += 1
        return self.out

    def close(self):
        """Release the graph (before the cache or the process group goes away)."""
        self.graph = None
