"""Benchmark of the ShadowKV sparse decode step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config config1]

One step = one decode step of one layer through ``ShadowAttention.decode_fused``:
RoPE of the new q/k, append, landmark scoring + top-k + reuse diff (two
launches), then one launch that fetches the missed value chunks from pinned
host memory (zero-copy), reconstructs the missed keys on the tensor cores
with RoPE and computes the GQA attention (``--split``: the last three stages
as separate launches, the fetch on a copy stream).
The workload is BASELINE configs[1] (Llama-3-8B shape, 122880 context, budget
2048, rank 160) with seeded synthetic inputs; every rank runs its own
sequence (batch-sharded weak scaling, no collective on the data path).

Printed: one JSON line (rank 0).  ``value`` = tokens/s of the whole job with
inputs resident (device-timed, CUDA events, max over ranks); ``e2e`` = the
same through the host API with the query/new-token inputs copied from pinned
host memory and the attention output brought back every step (the fused
step writes it straight into pinned host memory; the split and head-sharded
steps copy it back).
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HBM_FALLBACK_GBS = 6650.0


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d.get("hbm_gbs", HBM_FALLBACK_GBS)), "measured"
    return HBM_FALLBACK_GBS, "fallback"


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons read through NVML every 10 ms
    while the timed region runs (read-only queries; no setting is changed)."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap"}

    def __init__(self, index: int):
        self.index = index
        self.sm, self.reasons, self.max_sm = [], set(), None
        self._stop = threading.Event()
        self.ok = False

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            bus = torch.cuda.get_device_properties(self.index)
            self.h = pynvml.nvmlDeviceGetHandleByPciBusId(
                f"{bus.pci_domain_id:08x}:{bus.pci_bus_id:02x}:{bus.pci_device_id:02x}.0")
            self.max_sm = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.nv = pynvml
            self.ok = True
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception as e:  # pragma: no cover - reported in the JSON line
            self.err = repr(e)
        return self

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.sm.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                try:
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                except AttributeError:
                    r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.01)

    def __exit__(self, *a):
        self._stop.set()
        if self.ok:
            self.t.join(timeout=2)

    def summary(self):
        if not self.ok or not self.sm:
            return {"sm_mhz": None, "sm_max_mhz": self.max_sm, "reasons": ["unsampled"],
                    "error": getattr(self, "err", "no samples")}
        return {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": self.max_sm, "reasons": sorted(self.reasons),
                "samples": len(self.sm), "source": "NVML, 10 ms"}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()


def link_bandwidth_gbs(sizes=(64 << 20, 256 << 20), reps=8) -> float:
    """Measured host->device bandwidth (copy engine, page-locked source allocated after the
    NUMA binding, like the value store): best of ``reps`` copies at each size."""
    best = 0.0
    for nbytes in sizes:
        src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        dst = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        for _ in range(reps + 1):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            dst.copy_(src, non_blocking=True)
            e.record()
            e.synchronize()
            best = max(best, nbytes / (s.elapsed_time(e) * 1e-3) / 1e9)
        del src, dst
    return best


def sm_read_link(flush, heads=8, chunks=4096, misses_per_head=(2048, 256), reps=5) -> dict:
    """Host-link rate of reads issued by the SMs: a zero-copy pinned-read microbenchmark run
    in-run with the library's own fetch kernel (``skv_decode_gather_values`` ->
    ``fetch_misses_kernel``, 16 chunks of 2 KiB per CTA).  The source is a 64 MB page-locked
    buffer allocated after the NUMA binding, like the value store, viewed as ``heads`` heads of
    ``chunks`` chunks; each launch reads random distinct chunks of every head into a device
    buffer, with the L2 flushed before it and CUDA events on the launching stream.  For each
    entry of ``misses_per_head``: the median duration of a launch and its rate; the first
    entry (32 MB) gives the sustained rate, the second (4 MB, one config-1 step's misses) the
    rate of one step-sized burst, ramp-up and drain included."""
    import ctypes
    from shadowkv_b200._lib import DecodeGeom, check, lib
    host = torch.empty(1, heads, chunks, 1024, dtype=torch.bfloat16).pin_memory()
    gen = torch.Generator().manual_seed(7)
    out = {}
    for M in misses_per_head:
        geom = DecodeGeom(1, heads, heads, 128, 8, 8, M, 0, chunks, chunks * 8, 8 * M, 0, 0, 128, 0, 1.0)
        v_buf = torch.empty(heads, 8 * M, 128, dtype=torch.bfloat16, device="cuda")
        slot = torch.arange(M, dtype=torch.int32).repeat(heads, 1).cuda()
        count = torch.full((heads,), M, dtype=torch.int32, device="cuda")
        times = []
        for r in range(reps + 1):
            chunk = torch.stack([torch.randperm(chunks, generator=gen)[:M] for _ in range(heads)]).to(torch.int32).cuda()
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            st = torch.cuda.current_stream()
            a.record(st)
            check(lib.skv_decode_gather_values(ctypes.byref(geom), host.data_ptr(), v_buf.data_ptr(),
                                               slot.data_ptr(), chunk.data_ptr(), count.data_ptr(),
                                               st.cuda_stream), "skv_decode_gather_values")
            b.record(st)
            b.synchronize()
            if r:  # the first launch warms the kernel up
                times.append(a.elapsed_time(b) * 1e3)
        us = statistics.median(times)
        nbytes = heads * M * 2048
        out[M] = {"bytes": nbytes, "us": us, "gbs": nbytes / (us * 1e-6) / 1e9}
        del v_buf
    del host
    return out


def zero_copy_peak(sm_link: dict) -> tuple[float, str, dict]:
    """The host-link peak of the roofline from ``sm_read_link``: the sustained rate of the
    zero-copy pinned-read microbenchmark (its largest size), how it was measured, and the
    step-sized burst beside it."""
    big, burst = (sm_link[k] for k in sorted(sm_link, reverse=True)[:2])
    kind = (f"measured in-run: zero-copy pinned-read microbenchmark, the library's fetch_misses_kernel "
            f"(16 chunks of 2 KiB per CTA) over {big['bytes'] / 1e6:.1f} MB of random 2 KiB chunks of a "
            f"64 MB page-locked buffer, L2 flushed, median of 5 launches")
    return big["gbs"], kind, {"bytes": burst["bytes"], "us": burst["us"], "gbs": burst["gbs"]}


def algorithmic_bytes(cache, misses: int, seq_len: int):
    """HBM and host-link bytes of one layer of a step (per-unit figures of the roofline model)."""
    B, H, D = cache.batch_size, cache.num_key_value_heads, cache.head_dim
    L = cache.k_landmark.shape[-2]
    r = cache.rank
    hbm = (B * H * L * D * 2               # landmark scan
           + misses * 8 * r * 2            # gathered U rows
           + B * H * D * r * 2             # SV^T
           + misses * 2048 * 2             # K and V slot writes
           + B * H * seq_len * D * 2 * 2)  # attention K + V read
    host = misses * 2048
    return hbm, host


def graph_kernel_times(cache, step_body, flush, load_inputs, stream, groups, steps, seq_len):
    """Kernel times of the graph-replayed one-call step (skv_decode_step).

    The step is captured once more with ``skv_decode_step_timing`` on: the same launches
    (programmatic dependent launch included), whose CTAs stamp the GPU's global timer at their
    start (after the wait for the kernel before them) and end into a span pair per (kv-head
    group, kernel), stamped by every replay.  Each replay follows an L2 flush; its step is timed
    with CUDA events on the caller's stream, its spans read after it.  Returns ``(kernel_us,
    (host bytes, attention-phase us) per step, per-launch figures of the attention kernel)``;
    the attention phase runs from the first attention CTA past its wait (the first group's
    selection complete) to the last attention CTA's end."""
    from shadowkv_b200 import decode as fz
    torch.cuda.synchronize()
    prev = fz.step_timing(True)
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step_body()
        torch.cuda.synchronize()
    finally:
        fz.step_timing(prev)
    score, sel, att, phase, first_att, step, host, launch_bytes = [], [], [], [], [], [], [], []
    for i in steps:
        flush.zero_()
        load_inputs(i)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        g.replay()
        b.record(stream)
        b.synchronize()
        step.append(1e3 * a.elapsed_time(b))
        t = fz.step_kernel_times(groups)
        mc = cache._step_ws.miss_count.view(-1).tolist()  # per (sequence, kv head)
        per = len(mc) // groups  # the heads of a group (batch 1 when groups > 1)
        for gi, (s0, e0, s1, e1, s2, e2) in enumerate(t):
            score.append(e0 - s0)
            sel.append(e1 - s1)
            if s2 is not None:
                att.append(e2 - s2)
                launch_bytes.append(algorithmic_bytes(cache, sum(mc[gi * per:(gi + 1) * per]), seq_len)[1])
        if all(x[4] is not None for x in t):
            phase.append(max(x[5] for x in t) - min(x[4] for x in t))
            first_att.append(min(x[4] for x in t))
        host.append(algorithmic_bytes(cache, sum(mc), seq_len)[1])
    del g
    mean = statistics.mean
    kernel_us = {"scoring": mean(score), "selection": mean(sel), "step_with_stamps": mean(step), "groups": groups}
    per_launch = None
    if att and phase:
        kernel_us.update({"sparse_attention": mean(att), "attention_phase": mean(phase),
                          "attention_phase_start": mean(first_att)})
        per_launch = {"host_bytes": mean(launch_bytes), "us": mean(att),
                      "gbs": mean(launch_bytes) / (mean(att) * 1e-6) / 1e9}
    return kernel_us, (mean(host), mean(phase) if phase else None), per_launch


def select_kernels(cache):
    """Kernels of one fused append+select call (2, or 3 with the keys kernel of long contexts)."""
    import ctypes
    from shadowkv_b200._lib import lib
    return int(lib.skv_decode_select_kernels(ctypes.byref(cache._fused_geom.c())))


def run_b200(args, world, rank, local):
    from shadowkv_b200 import workload
    from shadowkv_b200._lib import device_errors

    if os.environ.get("SKV_NUMA_BIND", "1") == "1":
        from shadowkv_b200 import numa
        numa.bind_to_gpu_numa(local)
    cfg = workload.CONFIGS[args.config]
    NL = args.layers
    if NL > 1:
        cfg = dataclasses.replace(cfg, layers=NL)
    if args.batch:
        cfg = dataclasses.replace(cfg, batch=args.batch)
    heads_sharded = args.shard == "heads" and world > 1
    if heads_sharded and NL > 1:
        raise SystemExit("--layers > 1 runs with --shard batch")
    if args.microbatch is None:
        from shadowkv_b200.kvcache import auto_microbatch
        args.microbatch = 1 if heads_sharded or args.split else auto_microbatch(cfg.batch)
    full_cfg = cfg
    if heads_sharded:
        # rank r owns kv heads [r*Hkv/N, (r+1)*Hkv/N) and their GQA groups; inside the step
        # every rank ends with the attention rows of all heads (o_proj's input): written to
        # every rank's memory over NVLink by the attention kernel itself (--gather peer),
        # or all-gathered by NCCL after it (--gather nccl)
        from shadowkv_b200 import sharding
        k0, kn, q0, qn = sharding.head_range(cfg.kv_heads, cfg.q_heads, world, rank)
        cfg = dataclasses.replace(cfg, kv_heads=kn, q_heads=qn)
    peer_out = None
    torch.manual_seed(0)
    # kv heads sharded: every rank factorises the keys of all heads (one key seed), as one model
    layer = workload.Layer(cfg, device=f"cuda:{local}", seed=1000 + rank,
                           kv_heads_of=(k0, kn, full_cfg.kv_heads) if heads_sharded else None, key_seed=1000)
    cache, attn = layer.cache, layer.attn
    B, Hq, Hkv = cfg.batch, cfg.q_heads, cfg.kv_heads
    n = args.steps + args.warmup
    inputs = [layer.next_inputs() for _ in range(min(n, 256))]
    pos0 = cfg.ctx
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")  # > 126 MB L2

    hbm_peak, peak_kind = measured_peaks()
    link_peak = link_bandwidth_gbs()
    main = torch.cuda.current_stream()
    copy_stream = cache.copy_stream

    # static inputs of the captured step
    # static inputs of the captured step: views of one device staging buffer, so the
    # end-to-end run brings a step's inputs over with a single host->device copy
    shapes = [(inputs[0][0].shape, torch.bfloat16), (inputs[0][1].shape, torch.bfloat16),
              (inputs[0][2].shape, torch.bfloat16), ((B, 1), torch.int64)]
    offs, nbytes = [], 0
    for shp, dt in shapes:
        offs.append(nbytes)
        nbytes += (math.prod(shp) * torch.empty((), dtype=dt).element_size() + 255) // 256 * 256
    d_in = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")

    def staged(buf):
        return [buf[o:o + math.prod(shp) * torch.empty((), dtype=dt).element_size()].view(dt).view(shp)
                for o, (shp, dt) in zip(offs, shapes)]

    s_q, s_k, s_v, s_pos = staged(d_in)
    s_pos.fill_(pos0)
    s_out = torch.empty(B, Hq, 128, dtype=torch.bfloat16, device="cuda")
    # heads sharded: every rank ends the step with the attention output of all heads
    s_full = None
    if heads_sharded and args.gather == "peer" and not args.split:
        from shadowkv_b200.peer import PeerOutput
        peer_out = PeerOutput.create(B, full_cfg.q_heads, q0, B * full_cfg.kv_heads)
        s_full = torch.empty(B, full_cfg.q_heads, 128, dtype=torch.bfloat16, device="cuda")
    elif heads_sharded:
        s_full = torch.empty(world * B * Hq, 128, dtype=torch.bfloat16, device="cuda")
    s_qr = torch.empty(B, Hq, 1, 128, dtype=torch.bfloat16, device="cuda")
    # several layers: layer l + 1 takes layer l's attention output as its query
    # (a real data dependency between the layers, as in the model)
    s_mid = [torch.empty(B, Hq, 128, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    cache.fused_geometry(attn.cos_sin_cache)
    # the one-call step (skv_decode_step), pipelined over kv-head groups at batch 1
    use_step = not (args.split or args.two_calls or heads_sharded or args.microbatch > 1)
    from shadowkv_b200 import decode as fz
    fz.early_fetch(args.early_fetch)
    from shadowkv_b200.kvcache import auto_head_groups
    head_groups = (args.head_groups or auto_head_groups(B, Hkv)) if use_step else 1

    def step_misses():
        ws = cache._step_ws if use_step else cache._fused_ws
        return int(ws.miss_count.sum().item())

    def load_inputs(i):
        q, k, v = inputs[i % len(inputs)]
        s_q.copy_(q)
        s_k.copy_(k)
        s_v.copy_(v)
        s_pos.fill_(pos0 + i)

    def step_body(final_out=None, ins=None):
        """One decode step of NL layers on the static inputs (appends at row sparse_end); ``ins``:
        other (q, k, v, position) tensors of the step (page-locked host ones for the e2e run)."""
        cache.gen_offset = 0
        x_q, x_k, x_v, x_pos = ins if ins is not None else (s_q, s_k, s_v, s_pos)
        for li in range(NL):
            q_in = x_q if li == 0 else s_mid[(li - 1) % 2]
            out = (s_out if final_out is None else final_out) if li == NL - 1 else s_mid[li % 2]
            if args.microbatch > 1 and not args.split and not heads_sharded:
                seq_len = cache.sparse_end + cache.gen_offset + 1
                cache.decode_step_microbatched(li, q_in, s_k, s_v, s_pos, attn.cos_sin_cache, out,
                                               args.microbatch, q_out=s_qr, max_ctas=args.fetch_ctas)
                continue
            if use_step:
                cache.decode_step_fused(li, q_in, x_k, x_v, x_pos, attn.cos_sin_cache, out=out,
                                        head_groups=head_groups, q_out=s_qr)
                seq_len = cache.sparse_end + cache._gen_offset(li)
                continue
            qr = cache.append_select_fused(li, q_in, s_k, s_v, s_pos, attn.cos_sin_cache, q_out=s_qr)
            seq_len = cache.sparse_end + cache._gen_offset(li)
            if args.split:
                cur = torch.cuda.current_stream()
                with torch.cuda.stream(copy_stream):
                    copy_stream.wait_stream(cur)
                    cache.fetch_values_fused(li, copy_stream)
                cache.reconstruct_keys_fused(li, attn.cos_sin_cache)
                cur.wait_stream(copy_stream)
                cache.attention(li, qr, seq_len, out=out)
            elif peer_out is not None:
                cache.sparse_attention_gather(li, qr, seq_len, attn.cos_sin_cache, peer_out)
                peer_out.finish(s_full)
            else:
                cache.sparse_attention_fused(li, qr, seq_len, attn.cos_sin_cache, out=out)
        if heads_sharded and peer_out is None:
            torch.distributed.all_gather_into_tensor(s_full, s_out.view(B * Hq, 128))
        cache.gen_offset = 0
        return seq_len

    # warm-up (eager), then capture one step as a CUDA graph
    for i in range(args.warmup):
        load_inputs(i)
        seq_len = step_body()
    torch.cuda.synchronize()
    graph = None
    if not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            seq_len = step_body()
        torch.cuda.synchronize()

    def run_step(i):
        load_inputs(i)
        if graph is not None:
            graph.replay()
        else:
            step_body()

    for i in range(2):  # replay warm-up
        run_step(i)
    barrier(world)

    per_step, fetch_ms, misses_all, seqlens = [], [], [], []
    with ClockSampler(local) as clk:
        barrier(world)
        t_wall = time.perf_counter()
        for i in range(args.warmup, n):
            flush.zero_()
            load_inputs(i)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(main)
            if graph is not None:
                graph.replay()
            else:
                step_body()
            e.record(main)
            e.synchronize()
            per_step.append(s.elapsed_time(e))
            misses_all.append(step_misses())
            seqlens.append(seq_len)
        barrier(world)
        t_wall = time.perf_counter() - t_wall
    errs = device_errors()[0]
    if errs:
        raise RuntimeError(f"{errs} device-side index errors during the benchmark")
    # the copy-engine figure varies from one measurement to the next on a shared host: the
    # link peak is the best of the measurements before and after the timed steps
    link_samples = [link_peak, link_bandwidth_gbs()]
    link_peak = max(link_samples)
    # the link as the step's kernels read it: the zero-copy pinned-read microbenchmark (the
    # library's own fetch kernel), sustained and as one step-sized burst.  Its sustained rate
    # is the host-link peak of the roofline (the step's reads are issued by the SMs: the
    # missed chunks are known only on the device); the copy-engine figure is reported beside it
    link_ce = link_peak
    link_zc, link_zc_kind, link_burst = zero_copy_peak(sm_read_link(flush))

    # ---- per-kernel times.  The one-call step: the same step captured once more with CUDA
    # events around each kv-head group's kernels (skv_decode_step_timing: event nodes on the
    # groups' own streams, recorded by every replay), replayed after an L2 flush.  Other
    # launch modes: the kernels launched eagerly, one group at a time.
    graph_timed = use_step and graph is not None and NL == 1
    per_launch = None
    if graph_timed:
        kernel_us, link_bytes_us, per_launch = graph_kernel_times(
            cache, step_body, flush, load_inputs, main, head_groups, range(args.warmup, min(n, args.warmup + 50)),
            statistics.mean(seqlens))
    else:
        # each kernel group bracketed by CUDA events on the stream it runs on (L2 flushed
        # before each step)
        names = (["append_select", "fetch_values", "reconstruct_keys", "attention"] if args.split
                 else ["append_select", "sparse_attention"])
        parts = {k: [] for k in names}
        for i in range(args.warmup, min(n, args.warmup + 100)):
            flush.zero_()
            load_inputs(i)
            cache.gen_offset = 0
            torch.cuda.synchronize()

            def timed(name, fn, stream):
                # a GPU-side sleep keeps the stream busy until the launch is enqueued, so the
                # events bracket device execution only, not host launch latency
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(stream):
                    torch.cuda._sleep(400_000)
                    a.record(stream)
                    r = fn()
                    b.record(stream)
                b.synchronize()
                parts[name].append(a.elapsed_time(b))
                return r

            qr = timed("append_select", lambda: cache.append_select_fused(0, s_q, s_k, s_v, s_pos, attn.cos_sin_cache,
                                                                          q_out=s_qr), main)
            sl = cache.sparse_end + cache._gen_offset(0)
            if args.split:
                timed("fetch_values", lambda: cache.fetch_values_fused(0, copy_stream), copy_stream)
                timed("reconstruct_keys", lambda: cache.reconstruct_keys_fused(0, attn.cos_sin_cache), main)
                timed("attention", lambda: cache.attention(0, qr, sl, out=s_out), main)
            else:
                timed("sparse_attention", lambda: cache.sparse_attention_fused(0, qr, sl, attn.cos_sin_cache, out=s_out),
                      main)
            misses_all.append(int(cache._fused_ws.miss_count.sum().item()))
            cache.gen_offset = 0
        fetch_ms = parts["fetch_values" if args.split else "sparse_attention"]
        kernel_us = {k: 1e3 * statistics.mean(v) for k, v in parts.items() if v}

    ms_step = sum(per_step) / len(per_step)
    ms_step_max = max_over_ranks(ms_step, world)
    tokens = B if heads_sharded else B * world
    value = tokens / (ms_step_max / 1e3)
    misses = statistics.mean(misses_all)
    hit_rate = 1.0 - misses / (B * Hkv * cache.select_sets)
    hbm_1, host_1 = algorithmic_bytes(cache, misses, statistics.mean(seqlens))  # one layer, one launch
    hbm_b, host_b = hbm_1 * NL, host_1 * NL  # the misses of layer 0 stand for every layer of the step
    t_roof = max(hbm_b / (hbm_peak * 1e9), host_b / (link_zc * 1e9))
    t_roof_ce = max(hbm_b / (hbm_peak * 1e9), host_b / (link_ce * 1e9))
    if graph_timed and link_bytes_us[1]:
        # host bytes of the step over the attention phase of the graph-replayed step
        link_achieved = link_bytes_us[0] / (link_bytes_us[1] * 1e-6) / 1e9
    elif graph_timed:  # early fetch: the values come in during the selection kernels
        link_achieved = link_bytes_us[0] / (kernel_us["step_with_stamps"] * 1e-6) / 1e9
    else:
        fetch_avg = statistics.mean(fetch_ms)  # one launch of the fetching kernel on layer 0
        link_achieved = host_1 / (fetch_avg * 1e-3) / 1e9 if fetch_avg > 0 else 0.0

    # ---- e2e: inputs copied from pinned host memory, the output brought back, every step
    # per step: the inputs packed in one pinned host buffer (q, k, v, position)
    h_in = []
    for j, inp in enumerate(inputs):
        hb = torch.zeros(nbytes, dtype=torch.uint8).pin_memory()
        for dst, src in zip(staged(hb)[:3], inp):
            dst.copy_(src.cpu())
        h_in.append(hb)
    h_out = torch.empty(*(s_full.shape if heads_sharded else (B, Hq, 128)), dtype=torch.bfloat16).pin_memory()
    # the fused step writes its output straight into the page-locked host buffer
    # (the merge stores it over the link: no separate device-to-host copy)
    out_direct = not heads_sharded and not args.split
    # the one-call step of one layer reads its inputs from page-locked host memory itself (a
    # staging kernel at its start, inside the timed region): the e2e graph is captured on the
    # inputs' views of one page-locked buffer, into which each step's inputs are put
    host_in = out_direct and use_step and graph is not None and NL == 1
    h_stage = torch.zeros(nbytes, dtype=torch.uint8).pin_memory() if host_in else None
    graph_e2e = None
    if out_direct and graph is not None:
        torch.cuda.synchronize()
        graph_e2e = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_e2e):
            step_body(h_out, staged(h_stage) if host_in else None)
        torch.cuda.synchronize()
    nin = len(inputs)
    e2e_ms = []
    for i in range(args.warmup, n):
        flush.zero_()
        hb = h_in[i % nin]
        staged(hb)[3].fill_(pos0 + i)
        if host_in:
            h_stage.copy_(hb)  # this step's inputs, where the step reads them
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(main)
        if not host_in:
            d_in.copy_(hb, non_blocking=True)  # the step's packed inputs, pinned host -> device
        if out_direct:
            if graph_e2e is not None:
                graph_e2e.replay()
            else:
                step_body(h_out)
        else:
            if graph is not None:
                graph.replay()
            else:
                step_body()
            h_out.copy_(s_full if heads_sharded else s_out, non_blocking=True)
        e.record(main)
        e.synchronize()
        e2e_ms.append(s.elapsed_time(e))
    e2e_step = max_over_ranks(sum(e2e_ms) / len(e2e_ms), world)
    # every rank's own figures (the slowest rank sets the step; the links are per GPU)
    mine = [rank, ms_step * 1e3, link_zc, link_achieved, hit_rate, link_ce]
    per_rank = [mine]
    if world > 1:
        t = torch.tensor(mine, dtype=torch.float64, device="cuda")
        allt = [torch.empty_like(t) for _ in range(world)]
        torch.distributed.all_gather(allt, t)
        per_rank = [x.tolist() for x in allt]
    # host -> device bytes of a step: the inputs the staging kernel reads, or the packed buffer
    h2d = sum(math.prod(shp) * torch.empty((), dtype=dt).element_size() for shp, dt in shapes) if host_in else nbytes
    d2h = h_out.numel() * h_out.element_size()
    used_graph = graph is not None
    del graph, graph_e2e

    res = {
        "metric": ("sparse-attn decode tokens/s (Llama-3-8B shape, 122k ctx)" if NL == 1 else
                   f"sparse-attn decode tokens/s ({NL} attention layers, Llama-3-8B shape, 122k ctx)"),
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step_max,
        "higher_is_better": True,
        "scaling": "strong" if heads_sharded else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded; BASELINE configs[1] shapes and distributions)",
        # the same workload string as the reference arm (oracle/cpu_reference.py) for the same run
        "config": {"workload": f"{cfg.name}: {'one decode layer' if NL == 1 else f'{NL} chained decode layers'}"
                               f", B={B}, {Hq}q/{Hkv}kv heads"
                               f"{' per GPU' if heads_sharded else ''}, ctx {cfg.ctx}, "
                               f"budget {cfg.budget}, rank {cfg.rank}",
                   "placement": "V in page-locked host memory, B sequences per GPU",
                   "global_batch": tokens, "seq_len": cfg.ctx,
                   "parallelism": ((f"kv-head-sharded x{world} (attention rows written to every rank over "
                                    f"NVLink peer memory by the attention kernel)" if peer_out is not None else
                                    f"kv-head-sharded x{world} (NCCL all-gather of the attention output)")
                                   if heads_sharded else f"batch-sharded x{world}"),
                   "l2": "flushed between timed steps (256 MB write)", "hit_rate": hit_rate,
                   "microbatch": args.microbatch, "fetch_ctas": args.fetch_ctas if args.microbatch > 1 else None,
                   "step": (f"skv_decode_step, {head_groups} kv-head group(s), early fetch "
                            f"{'on' if args.early_fetch else 'off'}" if use_step else
                            "append_select + fetch/reconstruct/attend launches")},
        "roofline": {"kernel": ("fetch_misses_kernel (zero-copy V gather)" if args.split else
                                "sparse_attend_kernel (zero-copy V gather + key reconstruction + attention)"),
                     "bound": "host_link",
                     "achieved": link_achieved, "peak": link_zc, "unit": "GB/s",
                     "frac": link_achieved / link_zc if link_zc else None,
                     # host-link bytes per launch: the missed chunks of this run (2048 B each);
                     # the ncu capture of this workload read exactly the missed bytes over the link
                     "traffic": host_1,
                     "traffic_kind": ("computed: missed chunks x 2048 B per "
                                      + ("step (every kv-head group's launch)" if graph_timed else "launch")
                                      + " (equal to the ncu sysmem read bytes of the capture in profiles/)"),
                     "peak_kind": link_zc_kind,
                     "peak_copy_engine": link_ce,
                     "frac_copy_engine": link_achieved / link_ce if link_ce else None,
                     "peak_copy_engine_kind": "measured in-run: pinned H2D copy-engine bandwidth, 64 and "
                                              "256 MB copies (best of the measurements before and after "
                                              "the timed steps)",
                     "peak_copy_engine_samples": link_samples,
                     "achieved_kind": ("host bytes of the step / attention phase of the graph-replayed step "
                                       "(first attention CTA past its wait to the last attention CTA's end: "
                                       "global-timer stamps of skv_decode_step_timing)" if graph_timed else
                                       "host bytes of one launch / its eager duration (CUDA events on its stream)"),
                     "per_launch": per_launch},
        "step_roofline": {"t_roof_us": t_roof * 1e6, "t_step_us": ms_step * 1e3,
                          "frac": t_roof / (ms_step * 1e-3), "hbm_bytes": hbm_b, "host_bytes": host_b,
                          "hbm_peak_gbs": hbm_peak, "hbm_peak_kind": peak_kind,
                          "link_peak_gbs": link_zc, "link_peak_kind": link_zc_kind,
                          "link_burst": link_burst,
                          "t_roof_copy_engine_us": t_roof_ce * 1e6, "frac_copy_engine": t_roof_ce / (ms_step * 1e-3),
                          "link_copy_engine_gbs": link_ce},
        "e2e": {"value": tokens / (e2e_step / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "inputs": ("read from page-locked host memory by the step (staging kernel in the timed region)"
                           if host_in else "copied from page-locked host memory by cudaMemcpyAsync in the timed region"),
                "output": ("written to page-locked host memory by the step's attention merge" if out_direct else
                           "copied to page-locked host memory in the timed region")},
        "kernel_us": kernel_us,
        "kernel_us_kind": ("graph-replayed step, the kernels' own global-timer spans per kv-head group "
                           "(skv_decode_step_timing: first CTA start after its wait to last CTA end), "
                           "L2 flushed before each replay" if graph_timed else
                           "eager launches, one kernel group at a time, L2 flushed before each step"),
        "per_rank": [{"rank": int(r), "step_us": round(st, 2), "link_peak_gbs": round(lp, 2),
                      "link_achieved_gbs": round(la, 2), "hit_rate": round(hr, 4),
                      "link_copy_engine_gbs": round(lc, 2)}
                     for r, st, lp, la, hr, lc in per_rank],
        "graph": used_graph,
        "gpu_launches": (select_kernels(cache) + (3 if args.split else 1)) * NL * args.steps
                        * (args.microbatch if args.microbatch > 1 and not args.split and not heads_sharded else 1)
                        * head_groups,
        "clocks": clk.summary(),
        "wall_s": t_wall,
    }
    if peer_out is not None:
        torch.cuda.synchronize()
        torch.distributed.barrier()  # every rank is done writing into the others' blocks
        peer_out.close()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(layer, inputs, seconds=args.cpu_seconds, layers=NL)
    return res


def run_kat(args):
    """The reference's own benchmark of the reuse-cache copy, on the drop-in bindings.

    kernels/test_cached_gather_copy.cu:50-61,224-300,356-362,479-525: 192 (sequence,
    head) blocks of 256 chunk slots over a 128K-token page-locked value store per
    block, 154 of the 256 chunks kept from the previous selection; the reorder runs
    before each copy, CUDA events bracket the copy alone (3 warm-up + 10 timed
    iterations), and the reported bandwidth counts all 256 chunks of every block
    (GiB/s), as the reference prints it.  The link figure counts the missed
    chunks only."""
    import numpy as np
    from shadowkv_b200 import shadowkv as skv
    nb, m, hits, cpu_chunks = 24 * 8, 256, 154, 128 * 1024 // 8
    rng = np.random.default_rng(12345)
    keys = np.empty((nb, m), np.int64)
    query = np.empty((nb, m), np.int64)
    for b in range(nb):
        k = np.sort(rng.choice(cpu_chunks, m, replace=False))
        fresh = rng.choice(np.setdiff1d(np.arange(cpu_chunks), k), m - hits, replace=False)
        keys[b], query[b] = k, np.concatenate([k[rng.choice(m, hits, replace=False)], fresh])
    values = torch.empty(nb * cpu_chunks * 1024, dtype=torch.bfloat16, pin_memory=True)  # 6.4 GB
    stride = m * 8 * 128
    buf = torch.zeros(nb * stride, dtype=torch.bfloat16, device="cuda")
    temp = torch.zeros(1, dtype=torch.bfloat16, device="cuda")  # unused by this library
    keys_d = torch.from_numpy(keys).cuda()
    query_d = torch.from_numpy(query).cuda()
    cached = torch.empty_like(keys_d)
    offsets = torch.empty(nb * m, dtype=torch.int32, device="cuda")
    cnts = torch.empty(nb, dtype=torch.int32, device="cuda")
    signals = torch.zeros(nb, dtype=torch.int32, device="cuda")
    copy_ms, reorder_ms = [], []
    warmup, iters = max(3, args.warmup), 10
    for i in range(warmup + iters):
        cached.copy_(keys_d)
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        evs[0].record()
        skv.reorder_keys_and_compute_offsets(cached, query_d, offsets, cnts, 24, 8, m)
        evs[1].record()
        skv.gather_copy_with_offsets(values, buf, temp, offsets, cnts, signals, 24, 8, cpu_chunks * 1024,
                                     m * 1024, 0, stride, m)
        evs[2].record()
        evs[2].synchronize()
        if i >= warmup:
            reorder_ms.append(evs[0].elapsed_time(evs[1]))
            copy_ms.append(evs[1].elapsed_time(evs[2]))
    assert int(cnts.sum().item()) == nb * hits
    t = statistics.mean(copy_ms) * 1e-3
    return {"metric": "reuse-cache copy bandwidth (reference test_cached_gather_copy.cu)",
            "value": m * 2048 * nb / t / 2 ** 30, "unit": "GiB/s (all 256 chunks per block, as the reference counts)",
            "link_gbs": (m - hits) * 2048 * nb / t / 1e9, "copy_us": t * 1e6,
            "reorder_us": statistics.mean(reorder_ms) * 1e3, "iterations": iters, "warmup": warmup,
            "config": {"blocks": nb, "map_size": m, "hits": hits, "host_chunks_per_block": cpu_chunks},
            "higher_is_better": True, "n_gpus": 1}


def run_prefill(args):
    """Prefill state build of one layer (config1 shapes, B=1): torch restatement vs skv_prefill_build.

    Both include the 252 MB device-to-host copy of the values into the page-locked
    chunk store (the reference's prefill does it too); the SVD is not part of either."""
    import types
    from shadowkv_b200 import workload
    from shadowkv_b200.kvcache import ShadowKVCache_CPU
    cfg = workload.CONFIGS[args.config]
    T, Hk, Hq, D = cfg.ctx, cfg.kv_heads, cfg.q_heads, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    k_roped = torch.randn(1, Hk, T, D, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(1, Hk, T, D, generator=g, device="cuda").to(torch.bfloat16)
    q_last = torch.randn(1, Hq, 1, D, generator=g, device="cuda").to(torch.bfloat16)
    conf = types.SimpleNamespace(num_attention_heads=Hq, num_key_value_heads=Hk, hidden_size=Hq * D,
                                 num_hidden_layers=1)
    cache = ShadowKVCache_CPU(conf, batch_size=1, max_length=T, device="cuda", sparse_budget=cfg.budget,
                              rank=cfg.rank, local_chunk=cfg.local_chunk, outlier_chunk=cfg.outliers,
                              gen_len=cfg.gen_len, geometry=cfg.geometry)
    times = {"torch": [], "native": [], "build": []}
    for i in range(args.warmup + args.steps):
        for kind in ("torch", "native"):
            cache.prefilled_batch, cache.kv_offset = 0, 0
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            if kind == "torch":
                cache.prefill_kv_cache(v, 0, k_roped, q_last)
            else:
                cache.prefill_kv_cache_native(v, 0, k_roped, q_last, build_events=(b0, b1))
            e.record()
            e.synchronize()
            if i >= args.warmup:
                times[kind].append(s.elapsed_time(e))
                if kind == "native":
                    times["build"].append(b0.elapsed_time(b1))
    tn, tt, tb = (statistics.median(times[k]) for k in ("native", "torch", "build"))
    host_bytes = (T // 8) * 8 * D * 2 * Hk
    # the rank-r factorisation of the pre-RoPE keys (get_svd): the tensor-core Gram kernel alone,
    # the whole Gram path (Gram + float64 eigensolve of the D x D matrix + U = K V / s), and the
    # reference's method, torch.svd of K in fp32 (skipped past 131072 rows: minutes, not ms)
    from shadowkv_b200 import decode
    k_pre = torch.randn(1, T, Hk * D, generator=g, device="cuda").to(torch.bfloat16)
    svd = {"gram_kernel": [], "gram_path": [], "torch_svd": []}
    methods = ["gram", "exact"] if T <= 131072 else ["gram"]
    for i in range(args.warmup + max(3, args.steps // 4)):
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        decode.gram(k_pre[0])
        e.record()
        e.synchronize()
        if i >= args.warmup:
            svd["gram_kernel"].append(s.elapsed_time(e))
        for m in methods:
            cache.svd_method = m
            cache.prefilled_batch = 0
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            cache.get_svd(k_pre, 0)
            e.record()
            e.synchronize()
            if i >= args.warmup:
                svd["gram_path" if m == "gram" else "torch_svd"].append(s.elapsed_time(e))
    svd_ms = {k: statistics.median(v) for k, v in svd.items() if v}
    gram_flops = 2.0 * T * (Hk * D) ** 2 / 2  # upper triangle (and diagonal blocks) of K^T K
    return {"metric": f"prefill state build ms ({cfg.name} shapes, one layer)", "value": tn, "unit": "ms",
            "higher_is_better": False, "steps": args.steps, "warmup": args.warmup,
            "torch_path_ms": tt, "speedup_vs_torch_path": tt / tn,
            "device_state_kernels_ms": tb, "host_store_bytes": host_bytes,
            "host_store_gbs": host_bytes / (tn * 1e-3) / 1e9,
            "factorisation_ms": svd_ms,
            "gram_kernel_tflops": gram_flops / (svd_ms["gram_kernel"] * 1e-3) / 1e12,
            "gram_kernel_gbs": (T * Hk * D * 2 * ((Hk * D // 128) + 1) / 2) / (svd_ms["gram_kernel"] * 1e-3) / 1e9,
            "config": {"workload": f"{cfg.name}: B=1, {Hq}q/{Hk}kv heads, T {T}, {cfg.outliers} outliers, "
                                   f"budget {cfg.budget}; includes the device-to-host copy of the values"},
            "data": "synthetic (seeded normal keys/values)"}


def cpu_baseline(layer, inputs, seconds=15.0, layers=1):
    """The oracle port of the reference's torch-eager decode step, timed on the host cores."""
    import numpy as np
    from oracle import shadowkv_oracle as o
    st = export_state(layer)
    cores = len(os.sched_getaffinity(0))
    times = []
    t_end = time.perf_counter() + seconds
    i = 0
    while time.perf_counter() < t_end and i < len(inputs):
        q = inputs[i][0].float().cpu().numpy()[:, :, 0, :]
        t0 = time.perf_counter()
        o.torch_path_decode_step(st, q, st.sparse_end)
        times.append(time.perf_counter() - t0)
        i += 1
    med = statistics.median(times)
    return {"value": layer.cfg.batch / (med * layers), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{len(times)} full config1 decode steps of the numpy port (median)"
                      + (f", one layer's time x {layers} layers" if layers > 1 else "")}


def export_state(layer):
    import numpy as np
    from oracle import shadowkv_oracle as o
    c = layer.cache
    f = lambda t: t.float().cpu().numpy()
    H, D = c.num_key_value_heads, c.head_dim
    v_full = f(c.v_cache_cpu[0]).reshape(c.batch_size, H, -1, D)
    st = o.TorchPathDecodeState(
        k_landmark=f(c.k_landmark[0]), k_landmark_idx=c.k_landmark_idx[0].cpu().numpy(), U=f(c.U[0]),
        SV=np.ascontiguousarray(f(c.SV[0]).transpose(0, 1, 3, 2)), v_full=v_full, k_buf=f(c.k_cache_buffer[0]),
        v_buf=f(c.v_cache_buffer[0]), cos_sin=f(layer.cos_sin), sparse_start=c.sparse_start,
        sparse_end=c.sparse_end, select_sets=c.select_sets)
    return st


def other_partitions(args, world, rank, local):
    """At N > 1, beside the batch-sharded line: the same step sharded by kv head (B=1, each rank
    Hkv/N heads, attention rows exchanged over NVLink peer memory), and BASELINE config 4's shape
    (B=32 per box, sharded by kv head).  Each is measured like the main line (warm-up, L2 flush,
    device events, max over ranks) and summarised here."""
    import copy
    import gc
    out = {}
    for name, over in (("shard_heads", dict(shard="heads", batch=0)),
                       ("config4_shape", dict(shard="heads", batch=32))):
        a = copy.copy(args)
        for k, v in over.items():
            setattr(a, k, v)
        a.no_cpu_baseline = True
        a.microbatch = None
        gc.collect()
        torch.cuda.empty_cache()
        r = run_b200(a, world, rank, local)
        out[name] = {k: r[k] for k in ("value", "unit", "ms_per_step", "scaling", "e2e", "per_rank", "kernel_us",
                                       "gpu_launches")}
        out[name]["config"] = {k: r["config"][k] for k in ("workload", "global_batch", "parallelism")}
        out[name]["link_gbs"] = r["roofline"]["achieved"]
        out[name]["step_roofline_frac"] = r["step_roofline"]["frac"]
        out[name]["step_roofline_frac_copy_engine"] = r["step_roofline"]["frac_copy_engine"]
        out[name]["clocks"] = r["clocks"]
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="config1")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch eagerly instead of replaying a CUDA graph")
    ap.add_argument("--kat", action="store_true",
                    help="the reference's reuse-cache copy benchmark (test_cached_gather_copy.cu) on the drop-in bindings")
    ap.add_argument("--prefill", action="store_true",
                    help="time the prefill state build of one layer (torch path vs skv_prefill_build)")
    ap.add_argument("--gather", default="peer", choices=["peer", "nccl"],
                    help="--shard heads: how every rank gets all heads' attention rows")
    ap.add_argument("--batch", type=int, default=0, help="sequences per GPU (default: the config's, 1)")
    ap.add_argument("--microbatch", type=int, default=None,
                    help="batch slices whose selection overlaps the previous slice's value fetch "
                         "(default: as ShadowAttention.decode_fused picks, 1 below 8 sequences per GPU)")
    ap.add_argument("--fetch-ctas", type=int, default=64,
                    help="--microbatch: CTAs of each slice's fetch + attention (the rest run the next selection)")
    ap.add_argument("--layers", type=int, default=1,
                    help="decode layers per step (chained: each layer's output is the next one's query)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--shard", default="batch", choices=["batch", "heads"],
                    help="multi-GPU partition: one sequence per rank (weak scaling) or the kv heads of one "
                         "sequence split over the ranks with an NCCL all-gather of the outputs (strong scaling)")
    ap.add_argument("--head-groups", type=int, default=None,
                    help="kv-head groups of the pipelined one-call step at batch 1 (default: auto, 4 for 8 kv heads)")
    ap.add_argument("--early-fetch", action="store_true",
                    help="the one-call step with the early value fetch (the selection kernel fetches the misses "
                         "and computes the attention)")
    ap.add_argument("--two-calls", action="store_true",
                    help="run the step as append_select + sparse_attention (all heads in one chain)")
    ap.add_argument("--no-extra-shards", action="store_true",
                    help="at N > 1, skip the kv-head-sharded and config-4-shape measurements beside the main line")
    ap.add_argument("--split", action="store_true",
                    help="fetch / reconstruction / attention as three launches instead of the fused kernel")
    args = ap.parse_args()
    if args.impl == "reference":
        # the CPU reference arm runs on rank 0 only; other ranks exit without work
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        from oracle import cpu_reference
        res = cpu_reference.run(args, world, rank)
        print(json.dumps(res), flush=True)
        return
    if args.prefill:
        print(json.dumps(run_prefill(args)), flush=True)
        return
    if args.kat:
        print(json.dumps(run_kat(args)), flush=True)
        return
    world, rank, local = dist_setup()
    res = run_b200(args, world, rank, local)
    if world > 1 and args.shard == "batch" and not args.no_extra_shards:
        res["other_partitions"] = other_partitions(args, world, rank, local)
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
