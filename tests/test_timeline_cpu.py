"""The trace-timeline summary (``shadowkv_b200.timeline``) on hand-made records.

No GPU: the records are built here in the layout the attention kernel writes in trace builds
(word 0 = SM | kv head << 8 | block << 20, word 1 = K buffer address, words 2..7 = stamps).
"""
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def _timeline():
    # imported by path: the package's __init__ does not load the library, the module itself
    # imports it only inside run()
    spec = importlib.util.spec_from_file_location(
        "shadowkv_b200.timeline", os.path.join(HERE, "..", "shadowkv_b200", "timeline.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules.setdefault("shadowkv_b200.timeline", mod)
    spec.loader.exec_module(mod)
    return mod


def _rec(head, blk, start, issued, keys, values, ticket, merged, t0=1_000_000):
    us = lambda x: t0 + int(x * 1000) if x else 0
    return [head << 8 | blk << 20, 0x7F0000000000, us(start), us(issued), us(keys), us(values), us(ticket),
            us(merged)]


def test_attention_items_skip_selection_and_tail_records():
    tl = _timeline()
    t0 = 1_000_000
    recs = [_rec(0, 1, 30, 31, 40, 60, 61, 0),
            [0, 0x5E1, t0 + 5, 0, 0, 0, 0, 0],            # selection record
            [0, 0x7F00, t0 + 5, 0, 0, 0, 0, tl.FX_TAIL_W7],  # early-fetch tail record
            _rec(1, 2, 30, 31, 40, 60, 61, 0, t0=t0 - 10_000_000)]  # stale: before the mark
    items = tl.attention_items(recs, t0)
    assert len(items) == 1 and items[0][0] == 1 << 20


def test_summary_reports_the_critical_item_and_late_keys():
    tl = _timeline()
    t0 = 1_000_000
    items = [_rec(0, 0, 30, 31, 35, 36, 37, 0),     # values in when its keys were done
             _rec(0, 1, 30, 32, 45, 90, 91, 95),    # last values in: merges the head
             _rec(1, 0, 31, 33, 70, 65, 71, 80)]    # keys after values
    lines = "\n".join(tl.summarise(items, t0))
    assert "attention items: 3" in lines
    assert "keys were done after their values were in: 1" in lines
    assert "last values in: kv head 0 block 1: start 30.0 issued 32.0 keys 45.0 values 90.0 ticket 91.0" in lines
    assert "(< 1.5 us apart): 2, the last at 65.0 us" in lines  # keys after values counts too
    assert "merges ended: first 80.0 last 95.0 us (last ticket 91.0 us)" in lines
