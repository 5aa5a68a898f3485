"""Timeline of one graph-replayed decode step, from the trace build.

    python -m shadowkv_b200.timeline config1 --groups 4

Builds the trace library (``-DSKV_TRACE``, ``libshadowkv_b200_trace.so``; the
product library is left as it is), re-runs itself with ``SKV_LIB`` pointing
at it, captures ``decode_step_fused`` of one prefilled layer in a CUDA graph
and replays it ``--steps`` times, each after an L2 flush, between two stamp
kernels on the caller's stream.  The replay with the median step is reported:

* the first and last stamp of every phase event (scoring, selection,
  attention), in microseconds after the first stamp kernel;
* per work item of the attention kernel (one 128-row block of one kv head):
  when its value loads were issued, when its keys were reconstructed (RoPE
  included), when its values were in, and when the head's merge ended -- the
  evidence of whether the reconstruction ever waits for, or holds up, the host
  link.

Record layout of the attention kernel (``sparse_attend_kernel``): word 0 = SM
id | kv head << 8 | block << 20, word 1 = the group's K buffer address, words
2..7 = global-timer stamps (item start, loads issued, keys done, values in,
ticket, merge end or 0).  Selection records carry 0x5E1 / 0x5E2 in word 1,
early-fetch tail records 0xF0F0 in word 7; they are not attention items.  Scan
records (``score_tma_kernel``, one per CTA) carry 0x5C0 in word 1: word 0 =
kv head | split << 16, words 2.. = start, first tile in, ns waiting for tiles,
tile loop done, tiles, end.
"""
from __future__ import annotations

import argparse
import ctypes
import os
import sys

EVENTS = ["score_start", "score_tile0", "score_end", "sel_start", "sel_waited", "sel_keys", "sel_cand", "sel_end",
          "sa_start", "sa_waited", "sa_issued", "sa_keys", "sa_values", "sa_ticket", "sa_merged", "mark_before",
          "mark_after", "sel_C", "sel_tile", "sel_hist", "sel_sync1", "sel_scan", "sel_marked", "sel_ranked",
          "sel_diff", "sa_lists", "fx_tail", "fx_keys", "fx_values", "fx_end"]
MARK_BEFORE, MARK_AFTER = 15, 16
SCAN_W1 = 0x5C0
NOT_ATTENTION_W1 = (0x5E1, 0x5E2, 0xF1F1, SCAN_W1)
FX_TAIL_W7 = 0xF0F0


def _pct(a, fs=(0, .25, .5, .75, .9, 1)):
    a = sorted(a)
    return [round(a[int(f * (len(a) - 1))], 1) for f in fs]


def attention_items(recs, t0):
    """Attention work-item records of one replay (stamps after t0)."""
    return [r for r in recs if r[1] not in NOT_ATTENTION_W1 and r[7] != FX_TAIL_W7 and r[2] > t0]


def scan_items(recs, t0):
    """Landmark-scan CTA records (``score_tma_kernel``) of one replay."""
    return [r for r in recs if r[1] == SCAN_W1 and r[2] > t0]


def summarise_scan(items, t0):
    """Lines of the landmark-scan summary: per CTA start, first tile in, end, and the share of
    its tile loop spent waiting for tiles."""
    T = lambda x: (x - t0) / 1e3
    first = [(r[3] - r[2]) / 1e3 for r in items if r[3]]
    loop = [(r[5] - r[2]) / 1e3 for r in items if r[5]]
    wait = [r[4] / 1e3 for r in items]
    share = [r[4] / max(1, r[5] - r[2]) for r in items if r[5]]
    return [f"  scan CTAs: {len(items)}, tiles per CTA {min(r[6] for r in items)}-{max(r[6] for r in items)}",
            f"  scan CTA start (us) p0/p50/p100: {_pct([T(r[2]) for r in items], (0, .5, 1))}",
            f"  scan CTA end   (us) p0/p50/p100: {_pct([T(r[7]) for r in items if r[7]], (0, .5, 1))}",
            f"  start -> first tile in (us) p0/p50/p100: {_pct(first, (0, .5, 1))}",
            f"  start -> tile loop done (us) p0/p50/p100: {_pct(loop, (0, .5, 1))}",
            f"  waiting for tiles (us) p50/p100: {_pct(wait, (.5, 1))}, share of the loop p50: "
            f"{sorted(share)[len(share) // 2]:.2f}"]


def summarise(items, t0):
    """Lines of the keys-versus-values summary of the attention items."""
    T = lambda x: (x - t0) / 1e3
    keys = [T(r[4]) for r in items]
    vals = [T(r[5]) for r in items]
    out = [f"  attention items: {len(items)}",
           f"  keys done  (us) p0/p25/p50/p75/p90/p100: {_pct(keys)}",
           f"  values in  (us) p0/p25/p50/p75/p90/p100: {_pct(vals)}",
           f"  items whose keys were done after their values were in: {sum(r[4] > r[5] for r in items)}"]
    work = [(r[4] - r[3]) / 1e3 for r in items]
    out.append(f"  loads issued -> keys done (us) p0/p50/p90/p100: {_pct(work, (0, .5, .9, 1))}")
    slack = [(r[5] - r[4]) / 1e3 for r in items]
    out.append(f"  keys done -> values in (us) p0/p10/p50: {_pct(slack, (0, .1, .5))}")
    crit = max(items, key=lambda r: r[5])
    out.append(f"  last values in: kv head {(crit[0] >> 8) & 0xfff} block {crit[0] >> 20}: start {T(crit[2]):.1f}"
               f" issued {T(crit[3]):.1f} keys {T(crit[4]):.1f} values {T(crit[5]):.1f} ticket {T(crit[6]):.1f}")
    tight = [r for r in items if (r[5] - r[4]) / 1e3 < 1.5]
    if tight:
        out.append(f"  items with values in when keys were done (< 1.5 us apart): {len(tight)}, "
                   f"the last at {max(T(r[5]) for r in tight):.1f} us")
    merged = [T(r[7]) for r in items if r[7] > t0]
    if merged:
        out.append(f"  merges ended: first {min(merged):.1f} last {max(merged):.1f} us "
                   f"(last ticket {max(T(r[6]) for r in items):.1f} us)")
    return out


def run(config: str, groups: int, steps: int, early: bool) -> None:
    import torch
    from . import decode as fz
    from . import workload
    from ._lib import lib
    for name, args in (("skv_trace_read", [ctypes.c_void_p, ctypes.c_int]),
                       ("skv_trace_mark", [ctypes.c_int, ctypes.c_void_p]),
                       ("skv_trace_records", [ctypes.c_void_p, ctypes.c_int])):
        getattr(lib, name).argtypes = args  # AttributeError: not a trace build
    fz.early_fetch(early)
    nrec = 4096
    buf = (ctypes.c_ulonglong * 64)()
    rec = (ctypes.c_ulonglong * (nrec * 8))()
    layer = workload.Layer(workload.CONFIGS[config], device="cuda:0", seed=1000)
    cache, attn, cfg = layer.cache, layer.attn, layer.cfg
    inputs = [layer.next_inputs() for _ in range(steps + 1)]
    s_q, s_k, s_v = [t.clone() for t in inputs[0]]
    pos = torch.full((cfg.batch,), cfg.ctx, dtype=torch.int64, device="cuda")
    s_qr = torch.empty(cfg.batch, cfg.q_heads, 1, 128, dtype=torch.bfloat16, device="cuda")
    s_out = torch.empty(cfg.batch, cfg.q_heads, 128, dtype=torch.bfloat16, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def body():
        cache.gen_offset = 0  # every replay appends at the same row
        cache.decode_step_fused(0, s_q, s_k, s_v, pos, attn.cos_sin_cache, out=s_out, head_groups=groups, q_out=s_qr)
        cache.gen_offset = 0

    for _ in range(3):
        body()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        body()
    torch.cuda.synchronize()
    runs = []
    for i in range(steps):
        q, k, v = inputs[1 + i]
        s_q.copy_(q), s_k.copy_(k), s_v.copy_(v), flush.zero_()
        torch.cuda.synchronize()
        lib.skv_trace_read(buf, 32)
        lib.skv_trace_records(None, 0)
        st = torch.cuda.current_stream().cuda_stream
        lib.skv_trace_mark(MARK_BEFORE, st)
        g.replay()
        lib.skv_trace_mark(MARK_AFTER, st)
        torch.cuda.synchronize()
        lib.skv_trace_read(buf, 32)
        n = min(lib.skv_trace_records(rec, nrec), nrec)
        t0 = buf[2 * MARK_BEFORE]
        ev = {nm: ((buf[2 * j] - t0) / 1e3, (buf[2 * j + 1] - t0) / 1e3)
              for j, nm in enumerate(EVENTS) if buf[2 * j + 1] and j not in (MARK_BEFORE, MARK_AFTER)}
        recs = [list(rec[8 * j: 8 * j + 8]) for j in range(n)]
        runs.append(((buf[2 * MARK_AFTER] - t0) / 1e3, ev, recs, t0))
    runs.sort(key=lambda r: r[0])
    tot, ev, recs, t0 = runs[len(runs) // 2]
    print(f"{config}, {groups} kv-head group(s), early fetch {'on' if early else 'off'}: median of {steps} replays, "
          f"stamp kernel to stamp kernel {tot:.1f} us (trace build)")
    for nm in EVENTS:
        if nm in ev:
            print(f"  {nm:12s} first {ev[nm][0]:7.1f} last {ev[nm][1]:7.1f}")
    scans = scan_items(recs, t0)
    if scans:
        print("\n".join(summarise_scan(scans, t0)))
    items = attention_items(recs, t0)
    if items:
        print("\n".join(summarise(items, t0)))


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("config", nargs="?", default="config1")
    p.add_argument("--groups", type=int, default=4, help="kv-head groups of the step (1..8)")
    p.add_argument("--steps", type=int, default=7, help="graph replays; the median one is reported")
    p.add_argument("--early-fetch", action="store_true")
    args = p.parse_args(argv)
    from .build import TRACE_LIB, build_trace
    if os.environ.get("SKV_LIB") != TRACE_LIB:
        build_trace()
        os.environ["SKV_LIB"] = TRACE_LIB
        os.execv(sys.executable, [sys.executable, "-m", "shadowkv_b200.timeline", *(argv or sys.argv[1:])])
    run(args.config, args.groups, args.steps, args.early_fetch)
    return 0


if __name__ == "__main__":
    sys.exit(main())
