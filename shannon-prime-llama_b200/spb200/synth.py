"""Seeded synthetic K/V/Q with the shapes and value distributions of the
benchmark configurations (no public dataset is involved):

  K = RoPE(z * s),  z ~ N(0,1) per element, s ~ LogNormal(0, sigma) per
      dimension drawn once per (layer, head) slot, RoPE theta 10000 in the
      llama.cpp "normal" adjacent-pair convention (pairs (2i, 2i+1),
      frequency theta^(-2i/d)) at positions pos0 .. pos0+T-1;
  V = N(0,1);
  Q = N(0, sigma_q) in fp16.

numpy versions (PCG64, per-slot seeds) feed the CPU parity tests; the torch
versions generate the same distributions on the GPU for full-size runs
(their values differ from numpy's; only the distribution is shared).
"""
from __future__ import annotations

import numpy as np


def slot_seed(cfg_seed: int, layer: int, head: int) -> int:
    """splitmix64(cfg_seed ^ (layer << 20 ^ head))."""
    z = (cfg_seed ^ ((layer << 20) ^ head)) & 0xFFFFFFFFFFFFFFFF
    z = (z + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
    return z ^ (z >> 31)


def rope_np(x: np.ndarray, pos0: int, theta: float = 10000.0) -> np.ndarray:
    """x [T][d] float32 -> RoPE'd (float64 angles, float32 result)."""
    T, d = x.shape
    i = np.arange(d // 2, dtype=np.float64)
    freq = theta ** (-2.0 * i / d)
    ang = (pos0 + np.arange(T, dtype=np.float64))[:, None] * freq[None, :]
    c, s = np.cos(ang), np.sin(ang)
    a, b = x[:, 0::2].astype(np.float64), x[:, 1::2].astype(np.float64)
    out = np.empty_like(x, dtype=np.float32)
    out[:, 0::2] = a * c - b * s
    out[:, 1::2] = a * s + b * c
    return out


def kv_slot_np(cfg_seed: int, layer: int, head: int, n_pos: int, head_dim: int,
               sigma: float = 0.5, pos0: int = 0):
    """K, V [n_pos][head_dim] float32 for one (layer, head) slot."""
    rng = np.random.Generator(np.random.PCG64(slot_seed(cfg_seed, layer, head)))
    s = rng.lognormal(0.0, sigma, size=head_dim).astype(np.float32)
    z = rng.standard_normal((n_pos, head_dim), dtype=np.float32)
    k = rope_np(z * s[None, :], pos0)
    v = rng.standard_normal((n_pos, head_dim), dtype=np.float32)
    return k, v


def q_np(cfg_seed: int, n_layers: int, n_q_heads: int, head_dim: int, sigma_q: float):
    rng = np.random.Generator(np.random.PCG64(slot_seed(cfg_seed, 0xFFFFF, 0xABC)))
    return (rng.standard_normal((n_layers, n_q_heads, head_dim)) * sigma_q).astype(np.float16)


def kv_layer_torch(gen, n_pos: int, n_heads: int, head_dim: int, sigma: float = 0.5,
                   pos0: int = 0, device="cuda", dtype=None):
    """K, V [n_pos][n_heads][head_dim] on the GPU (torch.Generator gen)."""
    import torch
    dtype = dtype or torch.float32
    s = torch.empty(n_heads, head_dim, device=device).log_normal_(0.0, sigma, generator=gen)
    z = torch.randn(n_pos, n_heads, head_dim, device=device, generator=gen)
    k = z * s[None]
    i = torch.arange(head_dim // 2, device=device, dtype=torch.float64)
    freq = 10000.0 ** (-2.0 * i / head_dim)
    ang = (pos0 + torch.arange(n_pos, device=device, dtype=torch.float64))[:, None] * freq[None]
    c = torch.cos(ang).float()[:, None, :]
    sn = torch.sin(ang).float()[:, None, :]
    a, b = k[..., 0::2].clone(), k[..., 1::2].clone()
    k[..., 0::2] = a * c - b * sn
    k[..., 1::2] = a * sn + b * c
    v = torch.randn(n_pos, n_heads, head_dim, device=device, generator=gen)
    return k.to(dtype), v.to(dtype)
