"""The binding calls of the reference's ``ShadowKVCache_CPU`` decode step: recorded, then replayed.

TEST INFRASTRUCTURE.  The reference's offload cache (models/kvcache/shadow.py:301-651) reaches
its CUDA library through six functions of ``kernels.shadowkv``:

* ``batch_gemm_softmax``                      models/kvcache/shadow.py:553-566
* ``reorder_keys_and_compute_offsets``        models/kvcache/shadow.py:574
* ``gather_copy_with_offsets``                models/kvcache/shadow.py:580
* ``gather_copy_d2d_with_offsets``            models/kvcache/shadow.py:592
* ``batch_gather_gemm``                       models/tensor_op.py:225-241
* ``apply_rotary_pos_emb_push_cache_opt``     models/tensor_op.py:180-189

``Recorder`` stands in for that module while the UNMODIFIED reference class (and the two
wrappers of models/tensor_op.py:176-243, taken from the source file) runs on the CPU in
``make_golden.py``.  It records each call -- the binding's name and its positional arguments,
ints and floats as given, tensors as the cache attribute they view (storage offset, shape,
strides) or, for temporaries, as a value -- and computes the outputs with the oracle, written
into the class's own tensors so that its state evolves step by step as on the GPU.  The decode
step also appends the new token's K/V with plain tensor copies (``update_kv_cache``,
models/kvcache/shadow.py:621-633); those are recorded as ``append`` events.

``oracle_outputs`` is the oracle side of one call, used by the recorder and by the replay
tests, which call the same binding of ``shadowkv_b200.shadowkv`` with the same arguments.
"""
from __future__ import annotations

import hashlib
import json

import numpy as np
import torch

from oracle import shadowkv_oracle as o

BINDINGS = ("batch_gemm_softmax", "reorder_keys_and_compute_offsets", "gather_copy_with_offsets",
            "gather_copy_d2d_with_offsets", "batch_gather_gemm", "apply_rotary_pos_emb_push_cache_opt")

# the positional arguments each binding writes
OUTPUTS = {
    "batch_gemm_softmax": (2, 3, 4, 5),                      # D, Norm, Sum, Softmax
    "reorder_keys_and_compute_offsets": (0, 2, 3),           # cached ids (reordered), offsets, cnts
    "gather_copy_with_offsets": (1,),                        # the V buffer of the layer
    "gather_copy_d2d_with_offsets": (0,),                    # the K buffer of the layer
    "batch_gather_gemm": (5,),                               # the reconstruction buffer
    "apply_rotary_pos_emb_push_cache_opt": (3,),             # the K buffer of the layer
}

_DT = {"bfloat16": torch.bfloat16, "float32": torch.float32, "int64": torch.int64, "int32": torch.int32}


def _dtname(t: torch.Tensor) -> str:
    return str(t.dtype).replace("torch.", "")


def to_np(t: torch.Tensor) -> np.ndarray:
    """Host copy: bf16 as float32 values, the rest in their own type."""
    t = t.detach().cpu()
    return t.float().numpy() if t.dtype == torch.bfloat16 else t.numpy().copy()


def bits(t: torch.Tensor) -> np.ndarray:
    """The bytes of a tensor as an integer array (bf16 -> int16), for bit-exact comparison."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy()
    if t.dtype == torch.float32:
        return t.view(torch.int32).numpy()
    return t.numpy()


def digest(t: torch.Tensor) -> str:
    return hashlib.sha256(np.ascontiguousarray(bits(t)).tobytes()).hexdigest()


def _bf16_of(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)


def oracle_outputs(name: str, a: list) -> dict:
    """The oracle's result of one binding call.

    ``a`` holds the resolved positional arguments: tensors as host torch tensors (any device
    copied to the CPU), scalars as given.  Returns {argument index: host tensor} with the full
    new contents of every argument the binding writes, in that argument's shape and dtype.
    """
    if name == "batch_gemm_softmax":
        A, B, D, N, S, P, batch, m, n, k, alpha, beta = a
        eD, eN, eS, eP = o.batch_gemm_softmax(to_np(A), to_np(B), batch, m, n, k, alpha, beta)
        return {2: _bf16_of(eD).reshape(D.shape), 3: torch.from_numpy(eN.reshape(N.shape).copy()),
                4: torch.from_numpy(eS.reshape(S.shape).copy()), 5: _bf16_of(eP).reshape(P.shape)}
    if name == "reorder_keys_and_compute_offsets":
        cached, cur, off, cnts, batch, heads, map_size = a
        keys, eoff, ecnt = o.reorder_keys_and_compute_offsets(to_np(cached).reshape(-1, map_size),
                                                              to_np(cur).reshape(-1, map_size))
        return {0: torch.from_numpy(keys).reshape(cached.shape).to(cached.dtype),
                2: torch.from_numpy(eoff).reshape(off.shape), 3: torch.from_numpy(ecnt).reshape(cnts.shape)}
    if name == "gather_copy_with_offsets":
        values, vbuf, temp, off, cnts, signals, batch, heads, cpu_len, gpu_len, gpu_off, gpu_stride, map_size = a
        new = o.gather_copy_with_offsets(bits(values), bits(vbuf), to_np(off), to_np(cnts), cpu_len, gpu_len,
                                         gpu_off, gpu_stride, map_size)
        return {1: torch.from_numpy(new).view(torch.bfloat16).reshape(vbuf.shape)}
    if name == "gather_copy_d2d_with_offsets":
        keys, off, cnts, batch, heads, gpu_len, gpu_off, gpu_stride, map_size = a
        new = o.gather_copy_d2d_with_offsets(bits(keys), to_np(off), to_np(cnts), gpu_off, gpu_stride, map_size)
        return {0: torch.from_numpy(new).view(torch.bfloat16).reshape(keys.shape)}
    if name == "batch_gather_gemm":
        (U, SVt, cos, sin, pid, out, batch, heads, seq_len, dim, rank, budget, max_seq_len, chunk,
         cnts) = a
        e = o.batch_gather_gemm(to_np(U).reshape(batch, seq_len, rank), to_np(SVt).reshape(batch, heads, dim, rank),
                                to_np(pid).reshape(batch, heads, -1), to_np(cnts), chunk)
        new = to_np(out).reshape(batch, heads, budget, dim)
        keep = np.isnan(e)  # rows of hit chunks: the binding leaves them as they were
        new = np.where(keep, new, e)
        return {5: _bf16_of(new).reshape(out.shape)}
    if name == "apply_rotary_pos_emb_push_cache_opt":
        x, cs, pid, cache, cnts = a[:5]
        sparse_start, sparse_end, half_dim, chunk = a[-4:]
        new = o.apply_rotary_pos_emb_push_cache_opt(to_np(x), to_np(cs), to_np(pid), to_np(cache), to_np(cnts),
                                                    sparse_start, sparse_end, chunk)
        return {3: _bf16_of(new).reshape(cache.shape)}
    raise KeyError(name)


class Recorder:
    """Stands in for ``kernels.shadowkv``: records each call and runs the oracle in its place.

    ``named()`` returns the tensors an argument may view, by name (the cache's attributes and
    the attention's RoPE table); any other tensor argument is recorded as a value.
    """

    def __init__(self, named):
        self.named = named
        self.events = []   # json-able descriptions
        self.values = {}   # name -> np array (values of temporaries)
        self.digests = []  # per event: {arg index: sha256 of the written tensor after the call}

    def _describe(self, t):
        if isinstance(t, torch.Tensor):
            ptr = t.untyped_storage().data_ptr()
            for name, base in self.named().items():
                if isinstance(base, torch.Tensor) and base.untyped_storage().data_ptr() == ptr:
                    assert base.storage_offset() == 0
                    return {"t": name, "off": t.storage_offset(), "shape": list(t.shape),
                            "stride": list(t.stride()), "dtype": _dtname(t)}
            key = f"val{len(self.values)}"
            self.values[key] = bits(t)
            return {"v": key, "shape": list(t.shape), "dtype": _dtname(t)}
        if isinstance(t, bool) or not isinstance(t, (int, float)):
            raise TypeError(f"unexpected argument {type(t)}")
        return {"i": int(t)} if isinstance(t, int) else {"f": float(t)}

    def append(self, layer, row, k, v):
        """The class's K/V append of one token (models/kvcache/shadow.py:626-628)."""
        self.events.append({"name": "append", "layer": layer, "row": row,
                            "k": self._describe(k.clone()), "v": self._describe(v.clone())})
        self.digests.append({})

    def _call(self, name, *args):
        self.events.append({"name": name, "args": [self._describe(x) for x in args]})
        res = oracle_outputs(name, list(args))
        for i, t in res.items():
            args[i].copy_(t)
        self.digests.append({i: digest(args[i]) for i in res})

    def __getattr__(self, name):
        if name in BINDINGS:
            return lambda *args: self._call(name, *args)
        raise AttributeError(name)


def pack(recorder: Recorder) -> dict:
    """npz fields of a recorded trace."""
    meta = {"events": recorder.events, "digests": recorder.digests}
    out = {"trace_json": np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)}
    for k, v in recorder.values.items():
        out[k] = v
    return out


def unpack(d) -> tuple:
    meta = json.loads(bytes(d["trace_json"]).decode())
    return meta["events"], [{int(k): v for k, v in dg.items()} for dg in meta["digests"]]


def value_tensor(d, desc) -> torch.Tensor:
    """A recorded temporary as a host tensor of its dtype."""
    arr = np.asarray(d[desc["v"]])
    dt = _DT[desc["dtype"]]
    t = torch.from_numpy(arr.copy())
    if dt == torch.bfloat16:
        t = t.view(torch.bfloat16)
    elif dt == torch.float32:
        t = t.view(torch.float32)
    return t.reshape(desc["shape"])


def resolve(d, desc, state, device):
    """One recorded argument over ``state`` (name -> tensor, wherever it lives): a view of a
    named tensor with the recorded geometry, a temporary moved to ``device``, or a scalar."""
    if "i" in desc:
        return desc["i"]
    if "f" in desc:
        return desc["f"]
    if "t" in desc:
        base = state[desc["t"]]
        assert _dtname(base) == desc["dtype"], (desc, base.dtype)
        return base.as_strided(desc["shape"], desc["stride"], desc["off"])
    return value_tensor(d, desc).to(device)


def meta_of(d) -> dict:
    return json.loads(bytes(d["meta_json"]).decode())


def build_state(d, device, pin: bool = True) -> dict:
    """The offload class's tensors after prefill and ``H2D``, rebuilt from the regenerated inputs
    and the stored parts, each checked against the digest the recording took; on ``device``
    except ``v_cache_cpu`` (page-locked host memory when ``pin``), plus the RoPE table
    ``cos_sin``.  The K/V buffers hold the prompt's last ``prefill_local`` rows, then the outlier
    chunks in the recorded order, then the first selection's chunks
    (models/kvcache/shadow.py:477-481, 497-502, 532-535)."""
    from tests.golden.make_golden import trace_inputs
    meta = meta_of(d)
    cfg = meta["config"]
    x = trace_inputs(**cfg)
    L, B, H, T = cfg["L"], cfg["B"], cfg["Hkv"], cfg["T"]
    ps, ss, se, chunks = meta["prefill_local"], meta["sparse_start"], meta["sparse_end"], meta["chunks"]
    st = {n: torch.zeros(info["shape"], dtype=_DT[info["dtype"]]) for n, info in meta["state"].items()}
    c, D = 8, 128
    st["v_cache_cpu"].copy_(torch.from_numpy(x["v"].reshape(st["v_cache_cpu"].shape)))
    oidx = np.asarray(d["outlier_idx"]).astype(np.int64)
    pid = np.asarray(d["init_position_ids"]).astype(np.int64)
    for name, src in (("k_cache_buffer", x["k_rot"]), ("v_cache_buffer", x["v"])):
        buf = np.zeros(st[name].shape, dtype=np.float32)
        ch = src[:, :, :, : chunks * c].reshape(L, B, H, chunks, c * D)
        buf[..., :ps, :] = src[..., T - ps:, :]
        buf[..., ps:ss, :] = np.take_along_axis(ch, oidx[..., None], axis=3).reshape(L, B, H, ss - ps, D)
        buf[..., ss:se, :] = np.take_along_axis(ch, pid[..., None], axis=3).reshape(L, B, H, se - ss, D)
        st[name].copy_(torch.from_numpy(buf))
    for n in ("U", "SV", "k_landmark"):
        st[n].copy_(torch.from_numpy(np.asarray(d["init_" + n])).view(torch.bfloat16).reshape(st[n].shape))
    st["k_landmark_idx"].copy_(torch.from_numpy(np.asarray(d["init_k_landmark_idx"]).astype(np.int64)))
    st["position_ids"].copy_(torch.from_numpy(pid))
    for n, info in meta["state"].items():
        assert digest(st[n]) == info["digest"], f"rebuilt {n} differs from the recorded state"
    out = {}
    for n, t in st.items():
        out[n] = (t.pin_memory() if pin else t) if n == "v_cache_cpu" else t.to(device)
    out["cos_sin"] = torch.from_numpy(np.asarray(x["cos_sin_bits"])).view(torch.bfloat16).to(device)
    return out


def replay(d, state, device, call) -> None:
    """Walk the recorded events over ``state``: the token appends are done here with tensor
    copies (models/kvcache/shadow.py:626-628); each binding call is handed to
    ``call(index, name, resolved args, recorded digests of its outputs)``."""
    events, digests = unpack(d)
    for i, e in enumerate(events):
        if e["name"] == "append":
            l, row = e["layer"], e["row"]
            state["k_cache_buffer"][l][:, :, row:row + 1].copy_(value_tensor(d, e["k"]).to(device))
            state["v_cache_buffer"][l][:, :, row:row + 1].copy_(value_tensor(d, e["v"]).to(device))
            continue
        call(i, e["name"], [resolve(d, a, state, device) for a in e["args"]], digests[i])
