"""Per-layer KV transforms of the offline caches, on ``[batch, heads,
tokens, head_dim]`` states.

* ``NoneTransform``: identity.
* ``HeadHadamard``: randomized Hadamard per (layer, head): Rademacher signs
  seeded ``base_seed ^ (layer << 16) ^ head`` on a CPU generator, forward
  ``FWHT(x * s) / sqrt(D)``, inverse ``FWHT(y) / sqrt(D) * s``, power-of-two
  chunks for other head sizes (reference cache_utils.py:22-155).
* ``AffineTransform``: per-layer learned affine map, ``diag`` (x * exp(log
  scale), log scale clamped to [-5, 5]) or ``full`` (x @ W^T), followed by an
  optional clip to +-softplus(c) with separate key/value clip vectors
  (reference cache_utils.py:157-285).  Parameters load from a ``torch.save``
  file ``{layer: {"state_dict": {...}}}`` (keys ``log_scale`` or
  ``linear.weight``, ``clip_k``, ``clip_v``); missing layers use the identity
  map with the default clip.
"""

from __future__ import annotations

import math
import os
from typing import Optional

import torch

from kvserve_hpdps_b200.compression.signs import fwht_fp32, rademacher_signs


class NoneTransform:
    def transform(self, x: torch.Tensor, layer_idx: int, kind: str = "k") -> torch.Tensor:
        return x

    def inverse(self, y: torch.Tensor, layer_idx: int, kind: str = "k") -> torch.Tensor:
        return y


class HeadHadamard:
    def __init__(self, base_seed: int = 0x3333):
        self.base_seed = int(base_seed)
        self._signs: dict[tuple, torch.Tensor] = {}

    def signs(self, layer_idx: int, num_heads: int, head_dim: int, device, dtype) -> torch.Tensor:
        key = (layer_idx, num_heads, head_dim, str(device), dtype)
        s = self._signs.get(key)
        if s is None:
            s = rademacher_signs(layer_idx, num_heads, head_dim, self.base_seed)
            s = s.to(device=device, dtype=dtype).view(1, num_heads, 1, head_dim)
            self._signs[key] = s
        return s

    def transform(self, x: torch.Tensor, layer_idx: int, kind: str = "k") -> torch.Tensor:
        s = self.signs(layer_idx, x.shape[1], x.shape[3], x.device, x.dtype)
        return fwht_fp32(x * s).to(x.dtype)

    def inverse(self, y: torch.Tensor, layer_idx: int, kind: str = "k") -> torch.Tensor:
        s = self.signs(layer_idx, y.shape[1], y.shape[3], y.device, y.dtype)
        return fwht_fp32(y).to(y.dtype) * s


def _inv_softplus(y: float) -> float:
    return math.log(math.expm1(y))


class AffineTransform:
    def __init__(self, head_dim: int, mode: str = "diag", learnable_clip: bool = True,
                 clip_init: float = 4.0, params_path: Optional[str] = None, device="cpu"):
        if mode not in ("diag", "full"):
            raise ValueError("affine mode must be 'diag' or 'full'")
        self.head_dim = int(head_dim)
        self.mode = mode
        self.learnable_clip = learnable_clip
        self.clip_init = float(clip_init)
        self.device = torch.device(device)
        self.params: dict[int, dict[str, torch.Tensor]] = {}
        self._inv_cache: dict[int, torch.Tensor] = {}
        if params_path:
            self.load(params_path)

    def load(self, path: str) -> None:
        if not os.path.exists(path):
            raise FileNotFoundError(f"affine parameter file {path} not found")
        raw = torch.load(path, map_location=self.device)
        for k, v in raw.items():
            try:
                idx = int(k)
            except (TypeError, ValueError):
                continue
            self.params[idx] = dict(v["state_dict"] if isinstance(v, dict) and "state_dict" in v
                                    else v)

    def _layer(self, layer_idx: int) -> dict[str, torch.Tensor]:
        p = self.params.get(int(layer_idx))
        if p is None:
            p = {}
            if self.mode == "diag":
                p["log_scale"] = torch.zeros(self.head_dim, device=self.device)
            else:
                p["linear.weight"] = torch.eye(self.head_dim, device=self.device)
            if self.learnable_clip:
                c = torch.full((self.head_dim,), _inv_softplus(self.clip_init), device=self.device)
                p["clip_k"], p["clip_v"] = c, c.clone()
            self.params[int(layer_idx)] = p
        return p

    def transform(self, x: torch.Tensor, layer_idx: int, kind: str = "k") -> torch.Tensor:
        p = self._layer(layer_idx)
        if self.mode == "diag":
            y = x * torch.exp(p["log_scale"].clamp(-5.0, 5.0)).to(x)
        else:
            y = x @ p["linear.weight"].to(x).t()
        if self.learnable_clip:
            a = torch.nn.functional.softplus(p["clip_k" if kind == "k" else "clip_v"].float()).to(y)
            y = torch.maximum(torch.minimum(y, a), -a)
        return torch.nan_to_num(y)

    def inverse(self, y: torch.Tensor, layer_idx: int, kind: str = "k") -> torch.Tensor:
        p = self._layer(layer_idx)
        if self.mode == "diag":
            return torch.nan_to_num(y * torch.exp(-p["log_scale"].clamp(-5.0, 5.0)).to(y))
        inv = self._inv_cache.get(int(layer_idx))
        if inv is None:
            inv = torch.linalg.inv(p["linear.weight"].to(torch.float64))
            self._inv_cache[int(layer_idx)] = inv
        return y @ inv.to(y).t()

    # the reference's older names (cache_utils.py AffineTransform); its
    # forward_transform hands ``kind`` to transform's layer slot, here each
    # argument goes where its name says
    def forward_transform(self, x: torch.Tensor, kind: str, layer_idx: int) -> torch.Tensor:
        return self.transform(x, layer_idx, kind)

    def inverse_transform(self, x: torch.Tensor, layer_idx: int) -> torch.Tensor:
        return self.inverse(x, layer_idx)


def make_transform(kind: str, base_seed: int = 0x3333, head_dim: int = 128,
                   params_path: Optional[str] = None, device="cpu"):
    if kind == "none":
        return NoneTransform()
    if kind == "hadamard":
        return HeadHadamard(base_seed)
    if kind == "affine":
        return AffineTransform(head_dim, "diag", params_path=params_path, device=device)
    raise ValueError(f"transform_type must be none, hadamard or affine, got {kind!r}")
