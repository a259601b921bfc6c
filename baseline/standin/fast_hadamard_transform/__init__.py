"""Plain-PyTorch stand-in for the ``fast_hadamard_transform`` package.

The reference's ``decompress_v3`` (kvserve_v1/tilelang_ops/kv_hadamard_quant.py:1410-1486)
imports ``fast_hadamard_transform.hadamard_transform`` for its inverse
transform.  That CUDA extension is not installed in this image and cannot be
built offline, so the benchmark's reference arm puts this directory on
``sys.path`` instead.  It computes the same function -- the unnormalised
Walsh-Hadamard transform (Sylvester order) along the last dimension, in
fp32, multiplied by ``scale`` and returned in the input dtype -- as one
matrix product against the Hadamard matrix (cuBLAS on a GPU).  Nothing of
this repository's package, kernels or engine is used.
"""

from __future__ import annotations

import torch

_MATS: dict = {}


def _hadamard(n: int, device) -> torch.Tensor:
    key = (n, str(device))
    h = _MATS.get(key)
    if h is None:
        if n < 1 or n & (n - 1):
            raise ValueError(f"hadamard_transform needs a power-of-two size, got {n}")
        h = torch.ones(1, 1, dtype=torch.float32)
        while h.shape[0] < n:
            h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
        h = h.to(device)
        _MATS[key] = h
    return h


def hadamard_transform(x: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
    """``(x @ H_n) * scale`` over the last dimension n (a power of two)."""
    n = x.shape[-1]
    y = torch.matmul(x.reshape(-1, n).float(), _hadamard(n, x.device))
    return (y * scale).to(x.dtype).reshape(x.shape)


__all__ = ["hadamard_transform"]
