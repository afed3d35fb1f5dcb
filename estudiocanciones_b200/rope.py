"""Llama-3 scaled RoPE table, bit-identical to the reference's.

The table is an input of the RoPE kernels, computed once per cache size on the
host in fp32 and copied to the device, as the reference does.  The fp32 values
must match the reference exactly, so the arithmetic follows the same sequence
as ``rope_cache`` (``app/engine.py:28-43``): fp32 ``1/base**(2i/hd)``, the
wavelength rule in Python floats (base 5e5, factor 32, low/high factors 1/4,
original context 8192), an fp32 outer product with the positions, cos and sin.
"""
from __future__ import annotations

import math

import torch


def rope_table(head_dim: int, max_seq: int, base=500_000, factor=32, low=1, high=4, ctx=8192) -> torch.Tensor:
    """``[max_seq, head_dim/2, 2]`` fp32 table of (cos, sin) for interleaved pairs."""
    half = torch.arange(0, head_dim, 2)[: head_dim // 2].float()
    freq = 1.0 / (base ** (half / head_dim))
    short_wave, long_wave = ctx / high, ctx / low
    scaled = []
    for f in freq.tolist():
        wave = 2 * math.pi / f
        if wave < short_wave:
            scaled.append(f)
        elif wave > long_wave:
            scaled.append(f / factor)
        else:
            w = (ctx / wave - low) / (high - low)
            scaled.append((1 - w) * f / factor + w * f)
    theta = torch.tensor(scaled, dtype=torch.float32)
    angle = torch.outer(torch.arange(max_seq, dtype=torch.float32), theta)
    return torch.stack([angle.cos(), angle.sin()], -1)
