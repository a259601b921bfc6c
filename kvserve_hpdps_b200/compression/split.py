"""Hybrid-precision split helpers of the generic quantizer, with the
reference's call signatures (kvserve_v1/compression/quantizer/split_func.py:
9-194): every function takes the layer id, the tensor(s) of one layer
(``[blocks, block_size, heads, head_dim]``) and a boolean mask whose row
``layer_id`` (head masks, ``[layers, heads]``) or entry ``layer_id`` (layer
masks, ``[layers]``) is True for LOW precision.

* ``head_split`` -> (LOW heads, HIGH heads) in head order;
  ``head_restore`` cuts a packed tensor (LOW heads first, then HIGH, the
  quantizer's layout) back into the two parts; ``head_reconstruct`` puts
  the parts back at their heads' positions.
* ``layer_split`` / ``layer_restore`` -> (tensor, empty) for a LOW layer,
  (empty, tensor) for a HIGH one; ``layer_reconstruct`` returns whichever
  part is non-empty.

The LOW head count is read from the mask on the host (masks are small CPU
tensors), so ``head_restore`` makes no device round trip for a CPU mask.
"""

from __future__ import annotations

from typing import Any, Optional

import torch

__all__ = ["head_split", "head_restore", "head_reconstruct", "layer_split", "layer_restore",
           "layer_reconstruct"]


def _mask_row(mask: Optional[torch.Tensor], layer_id: int, name: str) -> torch.Tensor:
    if mask is None or mask.dtype != torch.bool:
        raise ValueError(f"{name} must be a bool tensor (True = low precision)")
    return mask[layer_id]


def _empty_like(t: torch.Tensor) -> torch.Tensor:
    return torch.zeros(0, dtype=t.dtype, device=t.device)


def head_split(layer_id: int, tensor: torch.Tensor, head_scores: Optional[torch.Tensor] = None,
               **kwargs: Any) -> tuple[torch.Tensor, torch.Tensor]:
    m = _mask_row(head_scores, layer_id, "head_scores").to(tensor.device)
    return tensor[:, :, m, :], tensor[:, :, ~m, :]


def head_restore(layer_id: int, tensor: torch.Tensor, head_scores: Optional[torch.Tensor] = None,
                 **kwargs: Any) -> tuple[torch.Tensor, torch.Tensor]:
    n_low = int(_mask_row(head_scores, layer_id, "head_scores").cpu().sum())
    return tensor[:, :, :n_low, :], tensor[:, :, n_low:, :]


def head_reconstruct(layer_id: int, low_tensor: torch.Tensor, high_tensor: torch.Tensor,
                     head_scores: Optional[torch.Tensor] = None, **kwargs: Any) -> torch.Tensor:
    row = _mask_row(head_scores, layer_id, "head_scores")
    ref = low_tensor if low_tensor.numel() else high_tensor
    m = row.to(ref.device)
    out = torch.empty((*ref.shape[:2], m.numel(), *ref.shape[3:]), dtype=ref.dtype,
                      device=ref.device)
    if low_tensor.numel():
        out[:, :, m] = low_tensor.to(ref.dtype)
    if high_tensor.numel():
        out[:, :, ~m] = high_tensor.to(ref.dtype)
    return out


def layer_split(layer_id: int, tensor: torch.Tensor, layer_scores: Optional[torch.Tensor] = None,
                **kwargs: Any) -> tuple[torch.Tensor, torch.Tensor]:
    low = bool(_mask_row(layer_scores, layer_id, "layer_scores"))
    return (tensor, _empty_like(tensor)) if low else (_empty_like(tensor), tensor)


def layer_restore(layer_id: int, tensor: torch.Tensor,
                  layer_scores: Optional[torch.Tensor] = None,
                  **kwargs: Any) -> tuple[torch.Tensor, torch.Tensor]:
    return layer_split(layer_id, tensor, layer_scores)


def layer_reconstruct(layer_id: int, low_tensor: torch.Tensor, high_tensor: torch.Tensor,
                      layer_scores: Optional[torch.Tensor] = None,
                      **kwargs: Any) -> torch.Tensor:
    return low_tensor if low_tensor.numel() else high_tensor
