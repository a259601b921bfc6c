"""Optional NVTX ranges around the connector's stages.

With ``KVSERVE_NVTX=1`` the producer's compress-and-send, the consumer's load
and decode, and the fused manager's paged compress/decompress appear as named
ranges on an Nsight Systems timeline; otherwise the context manager costs one
branch.  Per-kernel timing inside the fused stages comes from the device
trace (``kvserve_hpdps_b200.ops.kernels.set_trace``).
"""

from __future__ import annotations

import contextlib
import os

_ENABLED = os.environ.get("KVSERVE_NVTX", "0") == "1"


def enabled() -> bool:
    return _ENABLED


@contextlib.contextmanager
def nvtx(name: str):
    if not _ENABLED:
        yield
        return
    import torch
    if not torch.cuda.is_available():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
