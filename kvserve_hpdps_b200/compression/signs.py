"""Rademacher signs and Hadamard matrices of the randomized Hadamard transform.

The transform of a head vector x (length D, a power of two) is
``y = H (s * x) / sqrt(D)`` with H the Sylvester Hadamard matrix and s a
vector of +-1 signs; the inverse is ``x = s * (H y) / sqrt(D)``.

Signs must match the reference bit for bit, so they are drawn exactly as it
draws them (kvserve_v1/compression/transformer/hadamard_func.py:105-159,
kv_hadamard_quant.py:32-54): a CPU ``torch.Generator`` seeded with
``base_seed ^ (layer << 16) ^ head`` produces ``randint(0, 2, (D,), int8)``,
mapped to ``2*b - 1``.
"""

from __future__ import annotations

import math
from functools import lru_cache

import torch


def rademacher_signs(layer_id: int, num_heads: int, head_dim: int,
                     base_seed: int, head_offset: int = 0) -> torch.Tensor:
    """float32 [num_heads, head_dim] of +-1.  ``head_offset`` selects global
    heads ``head_offset .. head_offset+num_heads-1`` (the reference seeds with
    the local head index; callers pass 0 to keep that behaviour)."""
    gen = torch.Generator(device="cpu")
    rows = []
    for h in range(num_heads):
        gen.manual_seed(int(base_seed) ^ (int(layer_id) << 16) ^ (h + head_offset))
        b = torch.randint(0, 2, (head_dim,), generator=gen, dtype=torch.int8)
        rows.append(b.float().mul_(2).sub_(1))
    return torch.stack(rows)


@lru_cache(maxsize=8)
def _sylvester(n: int) -> torch.Tensor:
    if n & (n - 1) or n <= 0:
        raise ValueError(f"Hadamard size must be a power of two, got {n}")
    h = torch.ones((1, 1), dtype=torch.float32)
    while h.shape[0] < n:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return h


def hadamard_matrix(n: int) -> torch.Tensor:
    """Unnormalised Sylvester Hadamard matrix (+-1 entries), float32 [n, n]."""
    return _sylvester(n).clone()


def pow2_chunks(dim: int) -> list[int]:
    """Descending powers of two summing to ``dim`` (96 -> [64, 32]); the
    transform of a non-power-of-two head_dim is applied per chunk
    (reference hadamard_func.py:50-73)."""
    out, rem = [], dim
    while rem > 0:
        c = 1 << (rem.bit_length() - 1)
        out.append(c)
        rem -= c
    return out


def fwht_fp32(x: torch.Tensor) -> torch.Tensor:
    """Orthonormal FWHT over the last dim in float32 (chunked when the size is
    not a power of two).  CPU oracle of the device transform."""
    xf = x.to(torch.float32)
    parts, start = [], 0
    for size in pow2_chunks(xf.shape[-1]):
        part = xf.narrow(-1, start, size)
        parts.append((part @ _sylvester(size).to(part.device)) / math.sqrt(size))
        start += size
    return torch.cat(parts, dim=-1) if len(parts) > 1 else parts[0]
