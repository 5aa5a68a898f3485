"""Attention output of kv-head-sharded ranks, gathered over peer memory.

With the kv heads of a sequence split over the GPUs of one node (one process
per GPU; ``sharding.head_range``), o_proj needs every rank's attention rows.
The reference would all-gather them after the attention (one NCCL
collective per layer, ``models/attention/shadow.py:48`` -> o_proj).  Here the
fused attention kernel's merge writes its rows straight into every rank's
landing buffer over NVLink and bumps every rank's arrival counter
(``skv_decode_sparse_attention_gather``); ``finish`` waits for the counter
(bounded) and copies the full ``[batch, q_heads_total, 128]`` output out of
the landing buffer (``skv_peer_gather_finish``).

Each rank owns one peer block (``cudaMalloc``), shared through CUDA IPC
handles exchanged with ``torch.distributed.all_gather_object``.  The
landing buffer is double-buffered by step parity, so a rank one step ahead
never overwrites rows a slower rank is still copying.  Every rank must call
``attention`` and ``finish`` once per step, in that order, on one stream.

A ``finish`` whose bounded wait runs out (a rank died or stopped stepping)
sets its block's sticky status and copies nothing; every later ``finish`` on
the block does nothing.  ``check`` (between steps) raises ``ShadowKVError``
once that happened; the ranks must then re-create their peer blocks.
"""
from __future__ import annotations

import ctypes

import torch

from . import decode
from ._lib import SKV_MAX_PEERS, PeerGather, ShadowKVError, check, lib


class PeerOutput:
    def __init__(self, batch: int, q_heads_total: int, q_head0: int, merges_per_step: int, rank: int,
                 blocks, own_block: int, imported=()):
        if not 1 <= len(blocks) <= SKV_MAX_PEERS:
            raise RuntimeError(f"peer gather supports 1..{SKV_MAX_PEERS} ranks")
        self.batch, self.q_heads_total = batch, q_heads_total
        self.pg = PeerGather()
        self.pg.world, self.pg.rank = len(blocks), rank
        self.pg.q_head0, self.pg.q_heads_total, self.pg.merges_per_step = q_head0, q_heads_total, merges_per_step
        self.pg.batch = batch
        for r, b in enumerate(blocks):
            self.pg.block[r] = b
        self._own = own_block
        self._imported = list(imported)

    @staticmethod
    def block_bytes(batch: int, q_heads_total: int) -> int:
        return int(lib.skv_peer_block_bytes(batch, q_heads_total))

    @staticmethod
    def alloc_block(nbytes: int) -> int:
        p = ctypes.c_void_p()
        check(lib.skv_peer_alloc(nbytes, ctypes.byref(p)), "skv_peer_alloc")
        return p.value

    @classmethod
    def create(cls, batch: int, q_heads_total: int, q_head0: int, merges_per_step: int, group=None):
        """Collective over ``group``: every rank allocates its block and maps everyone else's."""
        import torch.distributed as dist
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        own = cls.alloc_block(cls.block_bytes(batch, q_heads_total))
        h = (ctypes.c_ubyte * 64)()
        check(lib.skv_peer_export(own, h), "skv_peer_export")
        handles = [None] * world
        dist.all_gather_object(handles, bytes(h), group=group)
        blocks, imported = [], []
        for r, hb in enumerate(handles):
            if r == rank:
                blocks.append(own)
                continue
            p = ctypes.c_void_p()
            check(lib.skv_peer_import((ctypes.c_ubyte * 64).from_buffer_copy(hb), ctypes.byref(p)), "skv_peer_import")
            blocks.append(p.value)
            imported.append(p.value)
        return cls(batch, q_heads_total, q_head0, merges_per_step, rank, blocks, own, imported)

    @classmethod
    def in_process(cls, batch: int, q_heads_total: int, q_head0s, merges_per_step: int):
        """Ranks emulated in one process on one GPU (tests): one block per rank, no IPC."""
        nbytes = cls.block_bytes(batch, q_heads_total)
        blocks = [cls.alloc_block(nbytes) for _ in q_head0s]
        outs = [cls(batch, q_heads_total, q0, merges_per_step, r, blocks, blocks[r]) for r, q0 in enumerate(q_head0s)]
        return outs

    def attention(self, geom: decode.Geometry, ws: decode.DecodeWorkspace, q, U, SVt, cos_sin, v_host, k_buf, v_buf,
                  seq_len: int, stream=None):
        """``decode.sparse_attention`` with the output sent to every rank's landing buffer."""
        if v_host.is_cuda or not v_host.is_pinned() or v_host.dtype != torch.bfloat16 or not v_host.is_contiguous():
            raise RuntimeError("v_host must be a contiguous pinned CPU bf16 tensor")
        g = geom.c()
        req = decode._req
        check(lib.skv_decode_sparse_attention_gather(
            ctypes.byref(g), req(q, "q", torch.bfloat16), req(U, "U", torch.bfloat16), req(SVt, "SVt", torch.bfloat16),
            req(cos_sin, "cos_sin", torch.bfloat16), v_host.data_ptr(), req(k_buf, "k_buf", torch.bfloat16),
            req(v_buf, "v_buf", torch.bfloat16), ws.miss_slot.data_ptr(), ws.miss_chunk.data_ptr(),
            ws.miss_count.data_ptr(), int(seq_len), ctypes.byref(self.pg), ws.sparse_ws.data_ptr(), ws.sparse_bytes,
            decode._stream(stream)), "skv_decode_sparse_attention_gather")

    def finish(self, out: torch.Tensor, stream=None) -> torch.Tensor:
        """Wait for every rank's rows of this step; ``out`` = the full [batch, q_heads_total, 128] output."""
        decode._req(out, "out", torch.bfloat16, (self.batch, self.q_heads_total, 128))
        check(lib.skv_peer_gather_finish(ctypes.byref(self.pg), self.batch, out.data_ptr(), decode._stream(stream)),
              "skv_peer_gather_finish")
        return out

    def status(self) -> int:
        """This rank's block status (0: fine; 4: a finish timed out).  Synchronises the device."""
        st = ctypes.c_uint32(0)
        check(lib.skv_peer_status(ctypes.byref(self.pg), ctypes.byref(st)), "skv_peer_status")
        return int(st.value)

    def check(self) -> None:
        """Raise if a finish of this rank timed out (the peer blocks must then be re-created)."""
        st = self.status()
        if st:
            raise ShadowKVError(f"peer gather of rank {self.pg.rank}: a finish timed out waiting for the other "
                                f"ranks' rows (status {st}); re-create the peer blocks on every rank")

    def close(self, free_own: bool = True):
        """Unmap the peers' blocks and free this rank's (after every rank is done with it)."""
        for p in self._imported:
            check(lib.skv_peer_close(p), "skv_peer_close")
        self._imported = []
        if free_own and self._own:
            check(lib.skv_peer_free(self._own), "skv_peer_free")
            self._own = 0
