"""Paged KV block helpers (reference: kvserve_v1/utils/kv_utils.py).

Layouts: FlashAttention ``[2, num_blocks, block_size, H, D]`` and
MLA/FlashInfer ``[num_blocks, 2, ...]``.  ``extract``/``inject`` by block ids
move whole blocks (the reference's semantics, including injecting only the
overlap when the two sides' block counts differ).  On CUDA bf16 caches with
the FlashAttention layout the copies run on this framework's block-copy
kernel; other cases use PyTorch indexing.
"""

from __future__ import annotations

from typing import Sequence

import torch


def make_slot_mapping(token_ids: Sequence[int], block_ids: Sequence[int],
                      block_size: int) -> torch.Tensor:
    """Absolute slot of each token: block_ids[t // bs] * bs + t % bs (CPU int64)."""
    n = len(token_ids)
    b = torch.tensor(list(block_ids), dtype=torch.long)
    slots = (b.unsqueeze(1) * block_size + torch.arange(block_size)).flatten()
    return slots[:n]


def extract_kv_from_layer(kv_layer: torch.Tensor, slot_mapping: torch.Tensor) -> torch.Tensor:
    """[2, tokens, kv_dim] copy of the given slots of a [2, nb, bs, ...] layer."""
    flat = kv_layer.reshape(2, kv_layer.shape[1] * kv_layer.shape[2], -1)
    return flat[:, slot_mapping.to(flat.device), :].clone()


def inject_kv_into_layer(kv_layer: torch.Tensor, kv_data: torch.Tensor,
                         slot_mapping: torch.Tensor) -> None:
    flat = kv_layer.reshape(2, kv_layer.shape[1] * kv_layer.shape[2], -1)
    flat[:, slot_mapping.to(flat.device), :] = kv_data.to(flat.device)


def _fast_path(t: torch.Tensor) -> bool:
    return (t.is_cuda and t.dtype == torch.bfloat16 and t.dim() == 5 and t.shape[0] == 2
            and t.shape[-1] == 128 and t.shape[2] % 16 == 0 and t.is_contiguous())


def extract_kv_from_layer_by_blocks(kv_layer: torch.Tensor, block_ids: Sequence[int]) -> torch.Tensor:
    """Copy one request's blocks out of a paged layer."""
    ids = list(map(int, block_ids))
    if not ids:
        return kv_layer[:, :0].clone() if kv_layer.shape[0] == 2 else kv_layer[:0].clone()
    if _fast_path(kv_layer):
        from kvserve_hpdps_b200.ops import kernels as K
        out = torch.empty((2, len(ids), *kv_layer.shape[2:]), dtype=kv_layer.dtype,
                          device=kv_layer.device)
        idx = torch.tensor(ids, dtype=torch.int32).to(kv_layer.device, non_blocking=True)
        K.block_copy(kv_layer, idx, out.data_ptr(), gather=True)
        return out
    idx = torch.tensor(ids, device=kv_layer.device, dtype=torch.long)
    if kv_layer.shape[0] == 2:
        return kv_layer[:, idx].clone()
    if kv_layer.shape[1] == 2:
        return kv_layer[idx].clone()
    raise RuntimeError(f"unsupported KV layout {tuple(kv_layer.shape)}")


def inject_kv_into_layer_by_blocks(kv_layer: torch.Tensor, kv_data: torch.Tensor,
                                   block_ids: Sequence[int], request_id: str = "") -> None:
    """Write one request's blocks back; when the payload has fewer blocks than
    ``block_ids``, only the overlap is written."""
    ids = list(map(int, block_ids))
    if not ids:
        return
    payload = kv_data.to(kv_layer.device)
    if kv_layer.shape[0] == 2:
        n = payload.shape[1]
        ids = ids[:n]
        if _fast_path(kv_layer) and payload.is_contiguous() and payload.shape[1] == len(ids):
            from kvserve_hpdps_b200.ops import kernels as K
            idx = torch.tensor(ids, dtype=torch.int32).to(kv_layer.device, non_blocking=True)
            K.block_copy(kv_layer, idx, payload.data_ptr(), gather=False)
            return
        kv_layer[:, torch.tensor(ids, device=kv_layer.device)] = payload[:, :len(ids)]
        return
    if kv_layer.shape[1] == 2:
        n = payload.shape[0]
        ids = ids[:n]
        kv_layer[torch.tensor(ids, device=kv_layer.device)] = payload[:len(ids)]
        return
    raise RuntimeError(f"unsupported KV layout for request {request_id}: {tuple(kv_layer.shape)}")
