"""Synthetic KV workloads (no datasets or checkpoints are needed).

KV values are N(0, 1) from a seeded generator; a fraction of key channels
per head is scaled by ``outlier_scale`` to mimic the outlier channels of
real key caches.  Requests are stored in a paged cache in the NHD layout
``[2, num_blocks, block_size, H, D]`` at shuffled physical blocks, like a
serving engine's cache after some churn.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence

import torch


def outlier_channels(num_heads: int, head_dim: int, fraction: float = 0.03,
                     count: Optional[int] = None, seed: int = 1) -> torch.Tensor:
    """Bool [H, D]: channels scaled as outliers (``count`` per head, or
    round(fraction * D))."""
    g = torch.Generator().manual_seed(seed)
    k = count if count is not None else max(1, round(fraction * head_dim))
    mask = torch.zeros(num_heads, head_dim, dtype=torch.bool)
    for h in range(num_heads):
        mask[h, torch.randperm(head_dim, generator=g)[:k]] = True
    return mask


def synthetic_kv(num_tokens: int, num_heads: int, head_dim: int = 128, seed: int = 0,
                 outlier_fraction: float = 0.03, outlier_count: Optional[int] = None,
                 outlier_scale: float = 12.0, device="cpu",
                 dtype=torch.bfloat16) -> torch.Tensor:
    """[2, tokens, H, D] KV for one layer of one request."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    kv = torch.randn((2, num_tokens, num_heads, head_dim), generator=g, dtype=torch.float32)
    if outlier_scale != 1.0 and (outlier_fraction > 0 or outlier_count):
        m = outlier_channels(num_heads, head_dim, outlier_fraction, outlier_count, seed + 7)
        kv[0][:, m] *= outlier_scale
    return kv.to(device=device, dtype=dtype)


@dataclass
class PagedWorkload:
    cache: torch.Tensor                 # [L, 2, num_blocks, bs, H, D]
    block_ids: list[list[int]]          # per request
    n_tokens: list[int]

    @property
    def block_size(self) -> int:
        return self.cache.shape[3]


def paged_workload(num_layers: int, token_counts: Sequence[int], num_heads: int,
                   block_size: int = 16, head_dim: int = 128, seed: int = 0,
                   extra_blocks: int = 3, device="cpu", outlier_fraction: float = 0.03,
                   outlier_scale: float = 12.0, fill: bool = True) -> PagedWorkload:
    """A paged cache holding every request's KV at shuffled blocks.

    With ``fill=False`` the cache is allocated (zeros) but not populated;
    useful for large benchmark caches that are filled on the device.
    """
    nblk = [(t + block_size - 1) // block_size for t in token_counts]
    total = sum(nblk) + extra_blocks
    g = torch.Generator().manual_seed(seed + 1000)
    perm = torch.randperm(total, generator=g).tolist()
    cache = torch.zeros((num_layers, 2, total, block_size, num_heads, head_dim),
                        dtype=torch.bfloat16, device=device)
    block_ids, pos = [], 0
    for n in nblk:
        block_ids.append(perm[pos:pos + n])
        pos += n
    if fill:
        for r, (t, ids) in enumerate(zip(token_counts, block_ids)):
            rows = len(ids) * block_size
            for layer in range(num_layers):
                kv = synthetic_kv(rows, num_heads, head_dim, seed=seed * 7919 + r * 131 + layer,
                                  outlier_fraction=outlier_fraction, outlier_scale=outlier_scale,
                                  device=device)
                kv[:, t:] = 0  # unused slots of the last block
                idx = torch.tensor(ids, device=device)
                cache[layer, :, idx] = kv.view(2, len(ids), block_size, num_heads, head_dim)
    return PagedWorkload(cache, block_ids, list(map(int, token_counts)))


def gather_request(cache_layer: torch.Tensor, block_ids: Sequence[int]) -> torch.Tensor:
    """[2, nb, bs, H, D] dense copy of one request's blocks of one layer."""
    idx = torch.tensor(list(block_ids), device=cache_layer.device, dtype=torch.long)
    return cache_layer[:, idx].clone()
