"""CPU: the C-ABI library loads, exports every declared symbol, validates arguments."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "shadowkv_b200.h")).read()
    return sorted(set(re.findall(r"SKV_API\s+[\w\s\*]*?\b(skv_\w+)\s*\(", src)))


def test_header_declares_the_reference_bindings_and_decode_api():
    names = declared_symbols()
    for n in ["skv_gather_copy", "skv_gather_copy_d2d_with_offsets", "skv_reorder_keys_and_compute_offsets",
              "skv_gather_copy_with_offsets", "skv_apply_rotary_pos_emb", "skv_apply_rotary_pos_emb_new",
              "skv_apply_rotary_pos_emb_new_v2", "skv_apply_rotary_pos_emb_push_cache",
              "skv_apply_rotary_pos_emb_push_cache_opt", "skv_apply_rotary_pos_emb_push_cache_opt_glm",
              "skv_batch_gather_gemm", "skv_batch_gemm_softmax", "skv_decode_select", "skv_decode_gather_values",
              "skv_decode_reconstruct_keys", "skv_decode_attention"]:
        assert n in names


def test_library_exports_every_declared_symbol():
    from shadowkv_b200 import _lib
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for n in declared_symbols():
        assert hasattr(lib, n), n
    assert set(_lib.SIGNATURES) >= set(declared_symbols())


def test_version_and_empty_error():
    from shadowkv_b200._lib import lib
    assert lib.skv_version() >= 10000
    assert isinstance(lib.skv_last_error(), bytes)


def test_argument_errors_are_reported_without_launching():
    from shadowkv_b200._lib import lib, ShadowKVError, check
    rc = lib.skv_reorder_keys_and_compute_offsets(None, None, None, None, 1, 8, 256, None)
    assert rc == 1
    assert b"null" in lib.skv_last_error()
    rc = lib.skv_reorder_keys_and_compute_offsets(8, 8, 8, 8, 1, 8, 2048, None)
    assert rc == 2 and b"map_size" in lib.skv_last_error()
    with pytest.raises(ShadowKVError):
        check(rc, "reorder")
    rc = lib.skv_batch_gather_gemm(16, 16, None, None, 16, 16, 1, 8, 1024, 128, 100, 2048, 1024, 8, 16, None)
    assert rc == 2 and b"rank" in lib.skv_last_error()
    rc = lib.skv_batch_gemm_softmax(16, 16, 16, 16, 16, 16, 8, 4, 1000, 64, 1.0, 0.0, None)
    assert rc == 2 and b"k must be 128" in lib.skv_last_error()


def test_decode_workspace_sizes_are_pure_host():
    from shadowkv_b200.decode import Geometry
    from shadowkv_b200._lib import lib
    g = Geometry(batch=1, kv_heads=8, q_heads=32, rank=160, select_sets=256, num_landmarks=15308,
                 num_chunks=15360, ctx_len=122880, buf_len=2720, sparse_start=416).c()
    sel = lib.skv_decode_select_workspace(ctypes.byref(g))
    # logits (8 heads x 15308 x 4 fp32) + partials
    assert sel >= 8 * 15308 * 4 * 4
    # the attention keeps its split partials in shared memory (cluster reduction)
    assert lib.skv_decode_attention_workspace(ctypes.byref(g), 2464) == 0
    bad = Geometry(batch=1, kv_heads=8, q_heads=30, rank=160, select_sets=256, num_landmarks=15308,
                   num_chunks=15360, ctx_len=122880, buf_len=2720, sparse_start=416).c()
    assert lib.skv_decode_select_workspace(ctypes.byref(bad)) == 0


def test_ctypes_signatures_match_header_parameter_counts():
    """Every ctypes argtypes list has as many entries as the C declaration has parameters."""
    from shadowkv_b200 import _lib
    src = open(os.path.join(ROOT, "include", "shadowkv_b200.h")).read()
    decls = dict(re.findall(r"SKV_API\s+[\w\s\*]*?\b(skv_\w+)\s*\(([^)]*)\)", src, flags=re.S))
    for name, params in decls.items():
        params = params.strip()
        n = 0 if params in ("", "void") else params.count(",") + 1
        assert len(_lib.SIGNATURES[name]) == n, f"{name}: header {n} params, ctypes {len(_lib.SIGNATURES[name])}"


def test_peer_gather_struct_and_block_size_match_the_header():
    from shadowkv_b200 import _lib
    # int world, rank, q_head0, q_heads_total, merges_per_step, batch; void *block[8]
    assert ctypes.sizeof(_lib.PeerGather) == 24 + 8 * _lib.SKV_MAX_PEERS
    assert _lib.PeerGather.block.offset == 24 and _lib.PeerGather.batch.offset == 20
    src = open(os.path.join(ROOT, "include", "shadowkv_b200.h")).read()
    assert re.search(r"#define SKV_MAX_PEERS\s+%d\b" % _lib.SKV_MAX_PEERS, src)
    # counter | status | epoch | landing [2][batch][q_heads_total][128] bf16
    assert _lib.lib.skv_peer_block_bytes(1, 32) == 256 + 2 * 32 * 128 * 2
    assert _lib.lib.skv_peer_block_bytes(0, 32) == 0 and _lib.lib.skv_peer_block_bytes(2, 0) == 0


def test_prefill_geometry_checks_are_pure_host():
    from shadowkv_b200 import _lib
    ok = dict(batch=1, kv_heads=2, q_heads=8, tokens=2048, chunks=252, outlier_chunk=8, select_sets=32,
              buf_len=2048, host_chunks=256)
    assert _lib.lib.skv_prefill_workspace(ctypes.byref(_lib.PrefillGeom(**ok))) > 0
    for bad in (dict(chunks=300),            # chunks exceed the prompt
                dict(outlier_chunk=300),     # more outliers than supported
                dict(select_sets=250),       # fewer landmarks than selected chunks
                dict(buf_len=100),           # buffer too small for local + outlier + selected rows
                dict(host_chunks=10),        # host store smaller than the prompt
                dict(q_heads=7)):            # q heads not a multiple of kv heads
        g = dict(ok, **bad)
        assert _lib.lib.skv_prefill_workspace(ctypes.byref(_lib.PrefillGeom(**g))) == 0, bad


def test_peer_output_description_is_built_on_the_host():
    from shadowkv_b200.peer import PeerOutput
    p = PeerOutput(batch=2, q_heads_total=32, q_head0=16, merges_per_step=16, rank=1, blocks=[0x1000, 0x2000],
                   own_block=0)  # own_block 0: nothing to free
    assert (p.pg.world, p.pg.rank, p.pg.q_head0, p.pg.q_heads_total, p.pg.merges_per_step, p.pg.batch) == \
        (2, 1, 16, 32, 16, 2)
    assert list(p.pg.block[:2]) == [0x1000, 0x2000] and not any(p.pg.block[2:])
    with pytest.raises(RuntimeError):
        PeerOutput(1, 8, 0, 2, 0, [0x1000] * 9, 0)  # more ranks than the library supports
    with pytest.raises(RuntimeError):
        PeerOutput(1, 8, 0, 2, 0, [], 0)


def test_auto_head_groups_keeps_two_heads_per_group():
    from shadowkv_b200.kvcache import auto_head_groups
    assert [auto_head_groups(1, h) for h in (1, 2, 3, 4, 6, 8, 16)] == [1, 1, 1, 2, 2, 4, 4]
    assert auto_head_groups(2, 8) == 1  # a batch is sliced by sequence instead


def test_auto_microbatch_divides_the_batch():
    from shadowkv_b200.kvcache import auto_microbatch
    assert [auto_microbatch(b) for b in (1, 2, 7)] == [1, 1, 1]  # short selections: one slice
    assert [auto_microbatch(b) for b in (8, 12, 16, 32, 48)] == [4, 6, 8, 8, 8]
    for b in range(1, 130):
        assert b % auto_microbatch(b) == 0 and 1 <= auto_microbatch(b) <= 8


def test_every_entry_point_rejects_null_arguments_before_launching():
    """All-null / all-zero arguments give a non-zero status and a message, never a crash."""
    from shadowkv_b200 import _lib
    lib = _lib.lib
    special = {"skv_last_error", "skv_version",
               "skv_device_errors",          # null outputs are allowed (the counts are only reset)
               "skv_peer_free",              # freeing null is a no-op, as free()
               "skv_decode_step_early_fetch",  # process settings: return the previous value
               "skv_decode_step_timing"}
    checked = 0
    for name, args in _lib.SIGNATURES.items():
        if name in special or name in _lib._RET or not args:
            continue
        vals = [0 if a in (ctypes.c_int, ctypes.c_size_t) else 0.0 if a is ctypes.c_float else None for a in args]
        rc = getattr(lib, name)(*vals)
        if name == "skv_decode_select_kernels":
            assert rc == 0  # a kernel count: 0 = not a valid geometry
        else:
            assert rc == 1, (name, rc, lib.skv_last_error())
            assert lib.skv_last_error(), name
        checked += 1
    assert checked >= 30
    assert lib.skv_peer_free(None) == 0


def test_last_error_is_per_host_thread():
    """Calls from several host threads: each thread reads its own last error."""
    import threading
    from shadowkv_b200._lib import lib
    gate = threading.Barrier(2)
    seen = {}

    def caller(tag):
        if tag == "null":
            rc = lib.skv_reorder_keys_and_compute_offsets(None, None, None, None, 1, 8, 256, None)
        else:
            rc = lib.skv_reorder_keys_and_compute_offsets(8, 8, 8, 8, 1, 8, 2048, None)
        gate.wait()  # both errors are set before either thread reads
        seen[tag] = (rc, lib.skv_last_error())

    ts = [threading.Thread(target=caller, args=(t,)) for t in ("null", "map")]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert seen["null"][0] == 1 and b"null" in seen["null"][1]
    assert seen["map"][0] == 2 and b"map_size" in seen["map"][1]


C_HOST = r"""
#include <stdio.h>
#include <string.h>
#include "shadowkv_b200.h"
int main(void) {
    skv_decode_geom g;
    skv_prefill_geom p;
    memset(&g, 0, sizeof g);
    g.batch = 1; g.kv_heads = 8; g.q_heads = 32; g.head_dim = 128; g.rank = 160; g.chunk_size = 8;
    g.select_sets = 256; g.num_landmarks = 15308; g.num_chunks = 15360; g.ctx_len = 122880;
    g.buf_len = 2720; g.sparse_start = 416; g.rope_mode = 0; g.cos_sin_stride = 128;
    g.cos_sin_rows = 124928; g.scale = 0.08838834764831845f;
    memset(&p, 0, sizeof p);
    p.batch = 1; p.kv_heads = 8; p.q_heads = 32; p.tokens = 122880; p.chunks = 15356;
    p.outlier_chunk = 48; p.select_sets = 256; p.buf_len = 2720; p.host_chunks = 15360;
    int st = skv_reorder_keys_and_compute_offsets(NULL, NULL, NULL, NULL, 1, 8, 256, NULL);
    printf("%d %zu %zu %zu %zu %d %s\n", skv_version(), skv_decode_select_workspace(&g),
           skv_decode_sparse_attention_workspace(&g, 2465), skv_prefill_workspace(&p),
           skv_peer_block_bytes(32, 32), st, skv_last_error());
    return 0;
}
"""


def test_c_host_program_uses_the_header_and_library(tmp_path):
    """The boundary from plain C: the header compiles as C99 (-pedantic, no warnings), the
    program links against the library, and its host-side answers equal the ctypes binding's."""
    import shutil
    import subprocess
    from shadowkv_b200 import _lib
    from shadowkv_b200.decode import Geometry
    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    src = tmp_path / "host.c"
    src.write_text(C_HOST)
    exe = tmp_path / "host"
    libdir = os.path.dirname(_lib.LIB_PATH)
    build = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror",
                            "-I", os.path.join(ROOT, "include"), str(src), "-L", libdir, "-lshadowkv_b200",
                            f"-Wl,-rpath,{libdir}", "-o", str(exe)], capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stderr
    f = run.stdout.split(maxsplit=6)
    g = Geometry(batch=1, kv_heads=8, q_heads=32, rank=160, select_sets=256, num_landmarks=15308,
                 num_chunks=15360, ctx_len=122880, buf_len=2720, sparse_start=416, cos_sin_rows=124928).c()
    pg = _lib.PrefillGeom(batch=1, kv_heads=8, q_heads=32, tokens=122880, chunks=15356, outlier_chunk=48,
                          select_sets=256, buf_len=2720, host_chunks=15360)
    lib = _lib.lib
    assert int(f[0]) == lib.skv_version()
    assert int(f[1]) == lib.skv_decode_select_workspace(ctypes.byref(g)) > 0
    assert int(f[2]) == lib.skv_decode_sparse_attention_workspace(ctypes.byref(g), 2465) > 0
    assert int(f[3]) == lib.skv_prefill_workspace(ctypes.byref(pg)) > 0
    assert int(f[4]) == lib.skv_peer_block_bytes(32, 32) > 0
    assert int(f[5]) == 1 and "null" in f[6]


def test_peer_finish_refuses_a_batch_the_blocks_do_not_hold():
    """Checked on the host before any launch: a finish for another batch than the blocks were
    sized for, or a merge count above batch * q_heads_total, is an invalid argument."""
    from shadowkv_b200 import _lib
    from shadowkv_b200.peer import PeerOutput
    p = PeerOutput(batch=2, q_heads_total=32, q_head0=0, merges_per_step=16, rank=0, blocks=[0x1000], own_block=0)
    st = _lib.lib.skv_peer_gather_finish(ctypes.byref(p.pg), 3, ctypes.c_void_p(0x2000), None)
    assert st == 1 and b"batch" in _lib.lib.skv_last_error()
    p.pg.merges_per_step = 2 * 32 + 1
    st = _lib.lib.skv_peer_gather_finish(ctypes.byref(p.pg), 2, ctypes.c_void_p(0x2000), None)
    assert st == 1
