"""Seeded synthetic ShadowKV decode workloads (stand-ins for the RULER prompts).

The reference measures on RULER / LongBench prompts with real model weights
(test/e2e.py:34-136), which are not available offline.  These generators
produce inputs with the reference's shapes and the value distributions named
by the benchmark configurations:

* pre-RoPE keys ``K = U0 @ W0 + 0.05 * N(0, 1)`` with ``U0 [T, r_true] ~
  N(0, 1)`` and ``W0 [r_true, Hkv*128] ~ N(0, 1/sqrt(r_true))``;
* values and queries ``~ N(0, 1)``; RoPE theta 500000 (Llama-3) or the GLM
  partial rotary table;
* optional query correlation ``q_t = rho * q_{t-1} + sqrt(1 - rho^2) * N``.

``build_layer`` runs the (torch) prefill of ``ShadowKVCache_CPU`` so that the
decode state -- U, SV, landmarks, pinned host V, K/V buffers, slots -- is
exactly what the reference's prefill would build from these keys.
"""
from __future__ import annotations

import math
import types
from dataclasses import dataclass

import torch

from .attention import ShadowAttention
from .kvcache import ShadowKVCache_CPU


@dataclass
class WorkloadConfig:
    name: str
    ctx: int
    q_heads: int
    kv_heads: int
    r_true: int
    rank: int
    budget: int
    outliers: int
    batch: int = 1
    layers: int = 1
    local_chunk: int = 4
    geometry: str = "torch"     # "torch": 32-token local window; "cpu": chunks rounded to 8
    rope: str = "llama"         # "llama" (theta 500000) or "glm"
    rho: float = 0.0            # step-to-step query correlation
    gen_len: int = 128
    svd: str = "gram"


CONFIGS = {
    # CPU plumbing case (fp32 in the reference); bf16 on the GPU here
    "config0": WorkloadConfig("config0", ctx=8192, q_heads=8, kv_heads=2, r_true=32, rank=64, budget=512,
                              outliers=8, svd="exact"),
    # Llama-3-8B-shaped single-layer decode at 122880 context
    "config1": WorkloadConfig("config1", ctx=122880, q_heads=32, kv_heads=8, r_true=96, rank=160, budget=2048,
                              outliers=48),
    # BASELINE configs[3] shape, one layer: GLM-4-9B-1M (32/2 heads, partial rotary), correlated queries
    "config3": WorkloadConfig("config3", ctx=1048576, q_heads=32, kv_heads=2, r_true=96, rank=160, budget=2048,
                              outliers=48, rope="glm", rho=0.9),
    # small case for tests and smoke
    "tiny": WorkloadConfig("tiny", ctx=2048, q_heads=8, kv_heads=2, r_true=16, rank=64, budget=256, outliers=8,
                           svd="exact"),
}


def llama_cos_sin(n: int, theta: float = 500000.0, dim: int = 128, device=None) -> torch.Tensor:
    """``cat(cos[:, :64], sin[:, :64])`` as the reference builds it (models/llama.py:137-141,167), bf16."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float32, device=device) / dim))
    t = torch.arange(n, dtype=torch.float32, device=device)
    freqs = torch.outer(t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).to(torch.bfloat16).contiguous()


def glm_cos_sin(n: int, rot_dim: int = 64, base: float = 10000.0, device=None) -> torch.Tensor:
    """GLM rotary table, row = cos(32) | sin(32) (models/glm.py:132-133), bf16."""
    inv = 1.0 / (base ** (torch.arange(0, rot_dim, 2, dtype=torch.float32, device=device) / rot_dim))
    ang = torch.outer(torch.arange(n, dtype=torch.float32, device=device), inv)
    return torch.cat((ang.cos(), ang.sin()), dim=-1).to(torch.bfloat16).contiguous()


def rope_glm_torch(x: torch.Tensor, cos_sin: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """GLM partial interleaved RoPE (models/glm.py:207-230) in torch, for prefill keys/queries."""
    cs = cos_sin[positions]
    xr, xp = x[..., :64], x[..., 64:]
    c, s = cs[..., :32], cs[..., 32:64]
    out = torch.stack([xr[..., 0::2] * c - xr[..., 1::2] * s, xr[..., 1::2] * c + xr[..., 0::2] * s], dim=-1)
    return torch.cat((out.flatten(-2), xp), dim=-1)


class Layer:
    """One prefilled decode layer plus a seeded stream of decode inputs."""

    def __init__(self, cfg: WorkloadConfig, device="cuda", seed: int = 0, kv_heads_of=None, key_seed=None):
        """``kv_heads_of=(k0, kn, Hkv_total)``: this layer holds kv heads k0 .. k0+kn-1 of a model of
        Hkv_total (``cfg`` has kn kv heads and their q heads): every rank generates the keys of all
        heads from ``key_seed`` (the same on every rank) and factorises them together, as the
        reference does, then keeps its heads; values and queries come from ``seed``."""
        self.cfg = cfg
        self.kv_heads_of = kv_heads_of
        self.key_gen = None
        if kv_heads_of is not None:
            self.key_gen = torch.Generator(device=torch.device(device)).manual_seed(
                key_seed if key_seed is not None else seed)
        self.device = torch.device(device)
        D = 128
        g = torch.Generator(device=self.device).manual_seed(seed)
        self.gen = g
        T, Hq, Hk = cfg.ctx, cfg.q_heads, cfg.kv_heads
        self.config = types.SimpleNamespace(num_attention_heads=Hq, num_key_value_heads=Hk, hidden_size=Hq * D,
                                            num_hidden_layers=cfg.layers)
        rows = T + cfg.gen_len + 1024
        self.cos_sin = (llama_cos_sin(rows, device=self.device) if cfg.rope == "llama"
                        else glm_cos_sin(rows, device=self.device))
        self.cache = ShadowKVCache_CPU(self.config, batch_size=cfg.batch, max_length=T, device=self.device,
                                       sparse_budget=cfg.budget, rank=cfg.rank, local_chunk=cfg.local_chunk,
                                       outlier_chunk=cfg.outliers, gen_len=cfg.gen_len, geometry=cfg.geometry,
                                       svd=cfg.svd)
        self.attn = ShadowAttention(self.cache, Hq // Hk, D, Hq * D, self.cos_sin)
        for layer in range(cfg.layers):
            self._prefill_layer(layer, g)
        self.step = 0
        self.q_prev = None

    def _prefill_layer(self, layer, g):
        cfg, D, dev = self.cfg, 128, self.device
        B, T, Hq, Hk = cfg.batch, cfg.ctx, cfg.q_heads, cfg.kv_heads
        k0, Hk_all = (self.kv_heads_of[0], self.kv_heads_of[2]) if self.kv_heads_of else (0, Hk)
        gk = self.key_gen if self.key_gen is not None else g
        for b in range(B):
            U0 = torch.randn(T, cfg.r_true, generator=gk, device=dev)
            W0 = torch.randn(cfg.r_true, Hk_all * D, generator=gk, device=dev) / math.sqrt(math.sqrt(cfg.r_true))
            k_all = (U0 @ W0).add_(torch.randn(T, Hk_all * D, generator=gk, device=dev), alpha=0.05)
            k_all = k_all.to(torch.bfloat16).view(1, T, Hk_all, D).transpose(1, 2).contiguous()  # [1, Hk_all, T, D]
            del U0
            k_pre = k_all[:, k0:k0 + Hk].contiguous()
            v = torch.randn(1, Hk, T, D, generator=g, device=dev).to(torch.bfloat16)
            q_last = torch.randn(1, Hq, 1, D, generator=g, device=dev).to(torch.bfloat16)
            pos = torch.arange(T, device=dev)
            # every kv head's keys are factorised together (U shared by all heads)
            svd_keys, svd_heads = (k_all, (k0, Hk)) if self.kv_heads_of else (k_pre, None)
            if cfg.rope == "llama":
                self.cache.get_svd(svd_keys, layer, heads=svd_heads)
                cs = self.cos_sin[:T].float()
                cos = torch.cat((cs[:, :64], cs[:, :64]), -1)
                sin = torch.cat((cs[:, 64:], cs[:, 64:]), -1)
                kf = k_pre.float()
                k_roped = (kf * cos + torch.cat((-kf[..., 64:], kf[..., :64]), -1) * sin).to(torch.bfloat16)
            else:
                self.cache.get_svd(svd_keys, layer, heads=svd_heads)
                k_roped = rope_glm_torch(k_pre.float(), self.cos_sin.float(), pos).to(torch.bfloat16)
            self.cache.prefill_kv_cache(v, layer, k_roped, q_last)
            del k_pre, k_all, svd_keys, k_roped, v
        torch.cuda.synchronize(self.device)

    def next_inputs(self):
        """Post-RoPE query [B, Hq, 1, D] and the new token's k, v [B, Hkv, 1, D] for the next step."""
        cfg, D, dev, g = self.cfg, 128, self.device, self.gen
        B, Hq, Hk = cfg.batch, cfg.q_heads, cfg.kv_heads
        z = torch.randn(B, Hq, 1, D, generator=g, device=dev)
        if cfg.rho > 0 and self.q_prev is not None:
            z = cfg.rho * self.q_prev + math.sqrt(1 - cfg.rho ** 2) * z
        self.q_prev = z
        k = torch.randn(B, Hk, 1, D, generator=g, device=dev).to(torch.bfloat16)
        v = torch.randn(B, Hk, 1, D, generator=g, device=dev).to(torch.bfloat16)
        return z.to(torch.bfloat16), k, v
