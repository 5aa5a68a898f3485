"""Two-GPU check of the peer-memory gather (run by tests/test_gpu_multi.py under torchrun).

Every rank owns half of the kv heads of one sequence (tiny workload).  For a
few decode steps it runs the fused attention with its rows written to both
ranks' landing buffers (``PeerOutput``) and, on a twin of its state, the
plain fused attention whose outputs NCCL all-gathers; the two full outputs
must be identical on every rank.  Exit status 0 = equal.
"""
import copy
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device(f"cuda:{local}"))
    from shadowkv_b200 import sharding, workload
    from shadowkv_b200.peer import PeerOutput
    from shadowkv_b200._lib import device_errors
    base = copy.deepcopy(workload.CONFIGS["tiny"])
    k0, kn, q0, qn = sharding.head_range(base.kv_heads, base.q_heads, world, rank)
    cfg = copy.deepcopy(base)
    cfg.kv_heads, cfg.q_heads = kn, qn
    dev = f"cuda:{local}"
    lay, twin = workload.Layer(cfg, device=dev, seed=30 + rank), workload.Layer(cfg, device=dev, seed=30 + rank)
    B = cfg.batch
    peer = PeerOutput.create(B, base.q_heads, q0, B * base.kv_heads)
    full = torch.empty(B, base.q_heads, 128, dtype=torch.bfloat16, device=dev)
    ref = torch.empty(world * B * qn, 128, dtype=torch.bfloat16, device=dev)
    device_errors()
    ok = True
    for step in range(6):
        torch.manual_seed(1000 * step + rank)
        q, k, v = lay.next_inputs()
        pos = torch.full((B, 1), lay.cache.sparse_end + 200 + step, dtype=torch.int64, device=dev)
        for L, gather in ((lay, True), (twin, False)):
            c, attn = L.cache, L.attn
            c.fused_geometry(attn.cos_sin_cache)
            c.gen_offset = 0
            qr = c.append_select_fused(0, q, k, v, pos, attn.cos_sin_cache)
            sl = c.sparse_end + c._gen_offset(0)
            if gather:
                c.sparse_attention_gather(0, qr, sl, attn.cos_sin_cache, peer)
                peer.finish(full)
            else:
                o = c.sparse_attention_fused(0, qr, sl, attn.cos_sin_cache)
                dist.all_gather_into_tensor(ref, o.reshape(B * qn, 128))
            c.gen_offset = 0
        torch.cuda.synchronize()
        got = full.view(torch.int16).cpu()
        exp = ref.view(world, B, qn, 128).permute(1, 0, 2, 3).reshape(B, world * qn, 128).view(torch.int16).cpu()
        if not torch.equal(got, exp):
            print(f"rank {rank} step {step}: peer gather differs from the NCCL all-gather", flush=True)
            ok = False
    errs = device_errors()[0]
    if errs:
        print(f"rank {rank}: {errs} device errors", flush=True)
        ok = False
    torch.cuda.synchronize()
    dist.barrier()
    peer.close()
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    if rank == 0:
        print("peer gather check:", "ok" if flag.item() else "FAILED", flush=True)
    sys.exit(0 if flag.item() else 1)


if __name__ == "__main__":
    main()
