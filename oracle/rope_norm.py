"""RoPE and RMSNorm oracle (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

Restates nanoslg/models.py:
  RMSNorm.forward               25-34  fp32 statistics, normalised value cast to x.dtype,
                                       then weight * (an op in the weight's dtype)
  precompute_rope_frequencies   37-66  inv_freq = theta^(-2i/D), optional Llama-3
                                       frequency scaling, cos/sin of cat(f, f)
  apply_rotary_emb              69-83  x*cos + cat(-x2, x1)*sin, cos/sin cast to x.dtype
"""
import math

import torch


def rope_table(dim, max_pos, theta, rope_scaling=None):
    """(cos, sin), each fp32 [max_pos, dim] (models.py:37-66)."""
    freqs = 1.0 / (theta ** (torch.arange(0, dim, 2)[: dim // 2].float() / dim))
    if rope_scaling and rope_scaling.get("rope_type") == "llama3":
        factor = rope_scaling.get("factor", 8.0)
        lo = rope_scaling.get("low_freq_factor", 1.0)
        hi = rope_scaling.get("high_freq_factor", 4.0)
        old_ctx = rope_scaling.get("original_max_position_embeddings", 8192)
        lo_wl, hi_wl = old_ctx / lo, old_ctx / hi
        new = []
        for f in freqs:
            wl = 2 * math.pi / f
            if wl < hi_wl:
                new.append(f)
            elif wl > lo_wl:
                new.append(f / factor)
            else:
                s = (old_ctx / wl - lo) / (hi - lo)
                new.append((1 - s) * f / factor + s * f)
        freqs = torch.tensor(new, dtype=freqs.dtype)
    t = torch.arange(max_pos, dtype=torch.float32)
    f = torch.outer(t, freqs)
    f = torch.cat((f, f), dim=-1)
    return f.cos(), f.sin()


def apply_rotary(x, cos, sin):
    """x [B,S,H,D], cos/sin [B,S,D] rows already gathered (models.py:69-83)."""
    cos = cos[:, :, None, :].to(x.dtype)
    sin = sin[:, :, None, :].to(x.dtype)
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return x * cos + torch.cat((-x2, x1), dim=-1) * sin


def rmsnorm(x, weight, eps):
    """models.py:31-34."""
    x32 = x.float()
    return weight * (x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)
