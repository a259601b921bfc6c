"""Lossless codecs of the pipeline's last stage.

``KVServeCodec`` keeps the reference's constructor and ``encode/decode``
signatures (kvserve_v1/compression/codec/kvserve_codec.py:18-151) so custom
pipelines written for it run unchanged; the coding itself is this
framework's own:

* ``"rans"``: interleaved rANS with per-chunk frequency tables, on the GPU
  (sm_100a kernels) or the CPU (same byte stream);
* ``"bitpack"``: fixed-width packing at ceil(log2(max+1)) bits of the byte
  stream (lossless for any input);
* ``"lc"``: LC-style BIT_2 (16-bit bit-plane shuffle) + RZE_1 (zero-byte
  elimination) after the published LC stages, this framework's own device
  kernels and threaded CPU coder (same byte stream as the numpy reference
  in ``compression/lc.py``; the reference calls a closed external library
  for ``codec_type: "lc"``);
* ``"none"``: raw bytes.

The reference's closed nvCOMP algorithms are not used.  Their names map to
the nearest own codec: ``nvcomp``/``ANS``, ``Cascaded``, ``Deflate``,
``GDeflate``, ``LZ4``, ``Zstd`` -> ``rans``; ``nvcomp``/``Bitcomp`` ->
``bitpack``.  The resolved codec is recorded in the stream header, so
decoding never depends on the configured name.

Encoded stream = 16-byte header ``[magic u32 'KVC1', codec u32, n u64]``
followed by the codec payload (for ``bitpack`` one more 16-byte block
``[bits u32, pad]``).
"""

from __future__ import annotations

import math
from typing import Any, Optional

import numpy as np
import torch

from kvserve_hpdps_b200.compression.components import Codec

MAGIC = 0x3143564B  # "KVC1"
CODEC_IDS = {"none": 0, "rans": 1, "bitpack": 2, "lc": 3}
CODEC_NAMES = {v: k for k, v in CODEC_IDS.items()}

_NVCOMP_ALGOS = ("ANS", "Bitcomp", "Cascaded", "Deflate", "GDeflate", "LZ4", "Zstd")


_NVCOMP_MAPPING = ("nvcomp algorithms map to this framework's own lossless coders (nvCOMP is "
                   "not used): Bitcomp -> bitpack; ANS, Cascaded, Deflate, GDeflate, LZ4, "
                   "Zstd -> rans (an entropy coder: the dictionary/LZ algorithms are not "
                   "reproduced)")
_mapped_logged: set = set()


def resolve_codec(codec_type: Optional[str], algorithm: Optional[str] = None) -> str:
    """Map a reference or own codec name to one of none | rans | bitpack | lc.

    The reference's ``nvcomp`` codec names an nvCOMP algorithm; here each
    maps to an own coder: ``Bitcomp`` -> bit-packing, every other one
    (``ANS``, ``Cascaded``, ``Deflate``, ``GDeflate``, ``LZ4``, ``Zstd``) ->
    the rANS entropy coder.  A name other than ``ANS``/``Bitcomp`` is logged
    once with that mapping, since the dictionary coders are not reproduced."""
    ct = (codec_type or "nvcomp").lower()
    if ct in ("rans", "bitpack", "none", "lc"):
        return ct
    if ct == "nvcomp":
        algo = algorithm or "ANS"
        if algo not in _NVCOMP_ALGOS:
            raise ValueError(f"invalid nvcomp algorithm {algo!r}; expected one of "
                             f"{', '.join(_NVCOMP_ALGOS)} ({_NVCOMP_MAPPING})")
        if algo not in ("ANS", "Bitcomp") and algo not in _mapped_logged:
            _mapped_logged.add(algo)
            from kvserve_hpdps_b200.utils.logger import get_logger
            get_logger(__name__).warning("nvcomp algorithm %s runs as the rans coder (%s)",
                                         algo, _NVCOMP_MAPPING)
        return "bitpack" if algo == "Bitcomp" else "rans"
    raise ValueError(f"invalid codec type {codec_type!r}; expected rans, bitpack, none, "
                     f"nvcomp or lc ({_NVCOMP_MAPPING})")


def _header(codec: str, n: int, device) -> torch.Tensor:
    """16-byte container header.  On a CUDA device it is written by two fill
    kernels (a copy from pageable host memory would synchronise the stream)."""
    if torch.device(device).type == "cuda":
        h = torch.empty(2, dtype=torch.int64, device=device)
        h[0] = MAGIC | (CODEC_IDS[codec] << 32)  # little-endian [magic u32, codec u32]
        h[1] = int(n)
        return h.view(torch.uint8)
    h = np.zeros(2, dtype="<u8")
    h.view("<u4")[0] = MAGIC
    h.view("<u4")[1] = CODEC_IDS[codec]
    h[1] = n
    return torch.from_numpy(h.view(np.uint8).copy())


def parse_header(stream: torch.Tensor) -> tuple[str, int]:
    h = stream[:16].cpu().numpy().view("<u8")
    if stream.is_cuda:
        from kvserve_hpdps_b200.ops import kernels as K
        K._xfer["d2h"] += 16
    if int(h.view("<u4")[0]) != MAGIC:
        raise ValueError("not a KVC1 stream")
    return CODEC_NAMES[int(h.view("<u4")[1])], int(h[1])


def encode_bytes(data: torch.Tensor, codec: str) -> torch.Tensor:
    """Encode the bytes of ``data`` (any dtype) on its device."""
    from kvserve_hpdps_b200.ops import kernels as K
    src = data.contiguous().view(torch.uint8).reshape(-1)
    n = src.numel()
    hdr = _header(codec, n, src.device)
    if n == 0 or codec == "none":
        return torch.cat([hdr, src])
    if codec == "rans":
        return torch.cat([hdr, K.rans_encode(src)])
    if codec == "lc":
        return torch.cat([hdr, K.lc_encode(src)])
    if codec == "bitpack":
        mx = int(src.max().item())
        bits = max(1, math.ceil(math.log2(mx + 1))) if mx > 0 else 1
        rows = (n + 127) // 128
        pad = torch.zeros(rows * 128, dtype=torch.uint8, device=src.device)
        pad[:n] = src
        packed = _bitpack_rows(pad.view(rows, 128), bits)
        ext = torch.zeros(16, dtype=torch.uint8, device=src.device)
        ext[0] = bits
        return torch.cat([hdr, ext, packed.reshape(-1)])
    raise ValueError(codec)


def decode_bytes(stream: torch.Tensor, device=None) -> torch.Tensor:
    """Decode a stream produced by :func:`encode_bytes` into uint8 [n]."""
    from kvserve_hpdps_b200.ops import kernels as K
    codec, n = parse_header(stream)
    body = stream[16:]
    if device is not None and body.device != torch.device(device):
        body = body.to(device)
    if n == 0 or codec == "none":
        return body[:n].contiguous()
    if codec == "rans":
        return K.rans_decode(body.contiguous(), n)
    if codec == "lc":
        return K.lc_decode(body, n)
    if codec == "bitpack":
        bits = int(body[0].item())
        rows = (n + 127) // 128
        packed = body[16:16 + rows * 16 * bits].contiguous()
        return _bitunpack_rows(packed.view(rows, 16 * bits), bits).reshape(-1)[:n].contiguous()
    raise ValueError(codec)


def _bitpack_rows(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """[rows, 128] -> [rows, 16*bits] in the kernels' packing layout
    (vectorised torch on any device)."""
    rows = codes.shape[0]
    c = codes.to(torch.int64).view(rows, 4, 32) & ((1 << bits) - 1)
    pos = torch.arange(32, device=codes.device) * bits
    words = torch.zeros((rows, 4, bits), dtype=torch.int64, device=codes.device)
    wi, bo = pos // 32, pos % 32
    for j in range(32):
        words[:, :, wi[j]] |= (c[:, :, j] << bo[j]) & 0xFFFFFFFF
        if bo[j] + bits > 32:
            words[:, :, wi[j] + 1] |= c[:, :, j] >> (32 - bo[j])
    return words.to(torch.int32).contiguous().view(torch.uint8).view(rows, 16 * bits)


def _bitunpack_rows(packed: torch.Tensor, bits: int) -> torch.Tensor:
    rows = packed.shape[0]
    w = packed.contiguous().view(torch.int32).to(torch.int64).view(rows, 4, bits) & 0xFFFFFFFF
    out = torch.empty((rows, 4, 32), dtype=torch.int64, device=packed.device)
    mask = (1 << bits) - 1
    for j in range(32):
        bit = j * bits
        wi, bo = bit // 32, bit % 32
        v = w[:, :, wi] >> bo
        if bo + bits > 32:
            v = v | (w[:, :, wi + 1] << (32 - bo))
        out[:, :, j] = v & mask
    return out.to(torch.uint8).view(rows, 128)


class KVServeCodec(Codec):
    """Pipeline codec stage (reference-compatible signatures)."""

    def __init__(self, **kwargs: Any):
        self.codec_type = kwargs.get("codec_type", "nvcomp")
        self.nvcomp_algorithm = kwargs.get("nvcomp_algorithm", "ANS")
        self.resolved = resolve_codec(self.codec_type, self.nvcomp_algorithm)

    def validate(self) -> None:
        resolve_codec(self.codec_type, self.nvcomp_algorithm)

    def update_params(self, **kwargs: Any) -> None:
        super().update_params(**kwargs)
        self.resolved = resolve_codec(self.codec_type, self.nvcomp_algorithm)

    def encode(self, layer_id: int, tensor: torch.Tensor, **kwargs: Any) -> torch.Tensor:
        return encode_bytes(tensor, self.resolved)

    def decode(self, layer_id: int, compressed_data: torch.Tensor, original_dtype: str,
               original_shape: list[int], device: str, **kwargs: Any) -> torch.Tensor:
        raw = decode_bytes(compressed_data, device)
        dtype = getattr(torch, str(original_dtype).replace("torch.", ""))
        return raw.view(dtype).reshape([int(s) for s in original_shape])


# Reference-compatible class for the LC codec slot.
class LCCodec(KVServeCodec):
    """``codec_type: "lc"``: BIT_2 + RZE_1 (see :mod:`compression.lc`)."""

    def __init__(self, **kwargs: Any):
        kwargs = dict(kwargs)
        kwargs["codec_type"] = "lc"
        super().__init__(**kwargs)


class nvCOMPCodec:  # noqa: N801 - the reference's class name
    """The reference's standalone nvCOMP wrapper interface
    (kvserve_v1/compression/codec/nvcomp_func.py:10-121): ``encode(tensor)``
    returns the uint8 stream of the tensor's bytes, ``decode(stream,
    original_dtype, original_shape, device)`` rebuilds the tensor.  The
    algorithm name selects this package's codec as in
    :func:`resolve_codec` (``Bitcomp`` -> bit-packing, the others -> rANS);
    no nvCOMP library is involved."""

    def __init__(self, algorithm: str = "ANS", **kwargs: Any):
        self.algorithm = algorithm
        self.codec = resolve_codec("nvcomp", algorithm)

    def encode(self, tensor: torch.Tensor) -> torch.Tensor:
        if tensor.numel() == 0:
            return torch.empty(0, dtype=torch.uint8, device=tensor.device)
        return encode_bytes(tensor, self.codec)

    def decode(self, compressed_tensor: torch.Tensor, original_dtype: str,
               original_shape: list, device: str, **kwargs: Any) -> torch.Tensor:
        dtype = getattr(torch, str(original_dtype).replace("torch.", ""))
        if compressed_tensor.numel() == 0:
            return torch.empty([int(s) for s in original_shape], dtype=dtype, device=device)
        raw = decode_bytes(compressed_tensor, device)
        return raw.view(dtype).reshape([int(s) for s in original_shape])
