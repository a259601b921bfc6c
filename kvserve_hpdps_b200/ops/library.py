"""The lossless codecs as PyTorch operators (``torch.ops.kvserve.*``).

Importing this module registers, with ``torch.library.custom_op``:

* ``kvserve::rans_encode(Tensor data) -> Tensor``: interleaved rANS stream of
  the bytes of ``data`` (exact size);
* ``kvserve::rans_decode(Tensor stream, int n) -> Tensor``: ``n`` bytes;
* ``kvserve::lc_encode(Tensor data) -> Tensor``: BIT_2 + RZE_1 stream;
* ``kvserve::lc_decode(Tensor stream, int n) -> Tensor``: ``n`` bytes.

CUDA tensors run this package's kernels (an encode reads the stream size
back, one synchronisation); CPU tensors run the native CPU rANS coder and the
reference LC coder, which write the same streams.  Each op has a fake
(meta) implementation, so it can appear in traced programs: an encoded
stream's length is data dependent and is declared as an unbacked size.
"""

from __future__ import annotations

import torch

from kvserve_hpdps_b200.ops import kernels as K

__all__ = ["rans_encode", "rans_decode", "lc_encode", "lc_decode"]


def _bytes(data: torch.Tensor) -> torch.Tensor:
    return data.contiguous().view(torch.uint8).reshape(-1)


@torch.library.custom_op("kvserve::rans_encode", mutates_args=())
def rans_encode(data: torch.Tensor) -> torch.Tensor:
    return K.rans_encode(_bytes(data), trim=True)


@rans_encode.register_fake
def _(data):
    n = torch.library.get_ctx().new_dynamic_size()
    return data.new_empty((n,), dtype=torch.uint8)


@torch.library.custom_op("kvserve::rans_decode", mutates_args=())
def rans_decode(stream: torch.Tensor, n: int) -> torch.Tensor:
    return K.rans_decode(stream.contiguous(), int(n))


@rans_decode.register_fake
def _(stream, n):
    return stream.new_empty((n,), dtype=torch.uint8)


@torch.library.custom_op("kvserve::lc_encode", mutates_args=())
def lc_encode(data: torch.Tensor) -> torch.Tensor:
    return K.lc_encode(_bytes(data), trim=True)


@lc_encode.register_fake
def _(data):
    n = torch.library.get_ctx().new_dynamic_size()
    return data.new_empty((n,), dtype=torch.uint8)


@torch.library.custom_op("kvserve::lc_decode", mutates_args=())
def lc_decode(stream: torch.Tensor, n: int) -> torch.Tensor:
    return K.lc_decode(stream.contiguous(), int(n))


@lc_decode.register_fake
def _(stream, n):
    return stream.new_empty((n,), dtype=torch.uint8)
