"""GPU: the allocation-free selection entry point against the regular one.

skv_decode_select_noalloc exists for callers that cannot hand the library a
scratch buffer -- a host that drives the library through an FFI without a
CUDA allocator of its own, or a runtime that forbids device allocation on the
token path.  Its scratch is a fixed array inside the library.  This test calls
it through the C ABI and checks that two consecutive calls produce exactly the
slots and miss lists of skv_decode_select with a caller workspace (integer
outputs: bit-exact), and that an oversized geometry is refused.

The file name keeps it last in collection order; it does not depend on state
left by other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import shadowkv_oracle as o

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _bf16(x):
    return torch.from_numpy(o.f32_to_bf16_bits(np.asarray(x, np.float32)).view(np.int16)).view(torch.bfloat16).to(DEV)


def test_noalloc_select_matches_workspace_select_on_two_calls():
    from shadowkv_b200 import decode as fz
    from shadowkv_b200._lib import check, lib

    rng = np.random.default_rng(2024)
    B, H, G, L, K = 1, 8, 4, 15308, 256
    chunks = L + 48
    geom = fz.Geometry(batch=B, kv_heads=H, q_heads=H * G, rank=160, select_sets=K, num_landmarks=L,
                       num_chunks=chunks, ctx_len=chunks * 8, buf_len=K * 8 + 600, sparse_start=416)
    g = geom.c()
    lm = _bf16(rng.standard_normal((B, H, L, 128)))
    lidx = torch.from_numpy(np.stack([np.sort(rng.permutation(chunks)[:L]) for _ in range(H)])[None]).to(DEV)
    start = np.stack([rng.permutation(lidx[0, h].cpu().numpy())[:K] for h in range(H)])[None].astype(np.int32)
    slots_ref = torch.from_numpy(start.copy()).to(DEV)
    slots_na = torch.from_numpy(start.copy()).to(DEV)
    ws = fz.DecodeWorkspace(geom, DEV)
    mk = lambda: (torch.zeros(B * H, K, dtype=torch.int32, device=DEV), torch.zeros(B * H, K, dtype=torch.int32, device=DEV),
                  torch.zeros(B * H, dtype=torch.int32, device=DEV))
    ms, mc, mn = mk()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        q = _bf16(rng.standard_normal((B, H * G, 128)))
        fz.select(geom, ws, q, lm, lidx, slots_ref)
        check(lib.skv_decode_select_noalloc(ctypes.byref(g), q.data_ptr(), lm.data_ptr(), lidx.data_ptr(),
                                            slots_na.data_ptr(), ms.data_ptr(), mc.data_ptr(), mn.data_ptr(),
                                            stream), "skv_decode_select_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(slots_na, slots_ref), f"slots differ on call {call}"
        assert torch.equal(mn, ws.miss_count), f"miss counts differ on call {call}"
        for i in range(B * H):
            n = int(mn[i])
            assert torch.equal(ms[i, :n], ws.miss_slot[i, :n])
            assert torch.equal(mc[i, :n], ws.miss_chunk[i, :n])


def test_noalloc_select_refuses_a_geometry_beyond_its_scratch():
    from shadowkv_b200 import decode as fz
    from shadowkv_b200._lib import lib
    geom = fz.Geometry(batch=64, kv_heads=8, q_heads=32, rank=160, select_sets=256, num_landmarks=15308,
                       num_chunks=15360, ctx_len=122880, buf_len=2720, sparse_start=416)
    g = geom.c()
    assert lib.skv_decode_select_workspace(ctypes.byref(g)) > 32 << 20
    null = ctypes.c_void_p(0)
    dummy = torch.zeros(16, dtype=torch.int32, device=DEV)
    rc = lib.skv_decode_select_noalloc(ctypes.byref(g), dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(),
                                       dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), null)
    assert rc == 2
    assert b"allocation-free" in lib.skv_last_error()
