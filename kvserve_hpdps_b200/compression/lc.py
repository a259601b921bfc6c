"""LC-style codec (BIT_2 then RZE_1): host reference of the device codec.

The stream format and both stages are described in ``ops/csrc/lc_codec.cu``;
this module writes and reads the identical byte stream with numpy, for CPU
tensors and as the oracle of the device kernels.
"""

from __future__ import annotations

import numpy as np

MAGIC = 0x3242434C  # "LCB2"
CHUNK = 16384


def _pad16(x: int) -> int:
    return (x + 15) & ~15


def max_bytes(n: int) -> int:
    nc = (n + CHUNK - 1) // CHUNK
    return _pad16(24 + 4 * (nc + 1)) + nc * (16 + _pad16(CHUNK))


def _shuffle(chunk: np.ndarray) -> np.ndarray:
    """BIT_2 of one chunk: plane-major [16][G] little-endian u32 as bytes."""
    cb = chunk.size
    words = (cb + 1) // 2
    groups = (words + 31) // 32
    buf = np.zeros(groups * 64, dtype=np.uint8)
    buf[:cb] = chunk
    w = buf.view("<u2").reshape(groups, 32).astype(np.uint32)
    shifts = np.arange(32, dtype=np.uint32)
    planes = np.empty((16, groups), dtype="<u4")
    for b in range(16):
        planes[b] = (((w >> b) & 1) << shifts).sum(axis=1, dtype=np.uint64).astype(np.uint32)
    return planes.view(np.uint8).reshape(-1)


def _unshuffle(sb: np.ndarray, cb: int) -> np.ndarray:
    groups = sb.size // 64
    planes = sb.view("<u4").reshape(16, groups).astype(np.uint32)
    lanes = np.arange(32, dtype=np.uint32)
    words = np.zeros((groups, 32), dtype=np.uint32)
    for b in range(16):
        words |= ((planes[b][:, None] >> lanes[None, :]) & 1) << b
    return words.astype("<u2").view(np.uint8).reshape(-1)[:cb]


def encode(data: np.ndarray) -> np.ndarray:
    """uint8 [n] (n > 0) -> stream bytes."""
    src = np.ascontiguousarray(data, dtype=np.uint8).reshape(-1)
    n = src.size
    nc = (n + CHUNK - 1) // CHUNK
    recs = []
    for c in range(nc):
        chunk = src[c * CHUNK:(c + 1) * CHUNK]
        cb = chunk.size
        sb = _shuffle(chunk)
        nzmask = sb != 0
        nz = int(nzmask.sum())
        coded = 16 + sb.size // 8 + nz
        if coded >= 16 + _pad16(cb):
            rec = np.zeros(16 + _pad16(cb), dtype=np.uint8)
            rec[:16].view("<u4")[:] = [0, cb, 0, 0]
            rec[16:16 + cb] = chunk
        else:
            rec = np.zeros(_pad16(coded), dtype=np.uint8)
            rec[:16].view("<u4")[:] = [1, nz, 0, 0]
            rec[16:16 + sb.size // 8] = np.packbits(nzmask, bitorder="little")
            rec[16 + sb.size // 8:coded] = sb[nzmask]
        recs.append(rec)
    lens = np.array([r.size for r in recs], dtype=np.uint64)
    offs = np.concatenate([[0], np.cumsum(lens)]).astype("<u4")
    head = _pad16(24 + 4 * (nc + 1))
    out = np.zeros(head, dtype=np.uint8)
    out[:8].view("<u4")[:] = [MAGIC, CHUNK]
    out[8:16].view("<u8")[0] = n
    out[16:24].view("<u4")[:] = [nc, 0]
    out[24:24 + 4 * (nc + 1)] = offs.view(np.uint8)
    return np.concatenate([out] + recs)


def decode(stream: np.ndarray, n: int) -> np.ndarray:
    s = np.ascontiguousarray(stream, dtype=np.uint8).reshape(-1)
    nc = (n + CHUNK - 1) // CHUNK
    head = _pad16(24 + 4 * (nc + 1))
    h = s[:8].view("<u4")
    if s.size < head or int(h[0]) != MAGIC or int(s[8:16].view("<u8")[0]) != n \
            or int(s[16:20].view("<u4")[0]) != nc:
        raise ValueError("not an LCB2 stream of this size")
    offs = s[24:24 + 4 * (nc + 1)].view("<u4").astype(np.int64)
    out = np.empty(n, dtype=np.uint8)
    for c in range(nc):
        rec = s[head + offs[c]:head + offs[c + 1]]
        cb = min(CHUNK, n - c * CHUNK)
        kind, cnt = (int(x) for x in rec[:8].view("<u4"))
        if kind == 0:
            out[c * CHUNK:c * CHUNK + cb] = rec[16:16 + cb]
            continue
        groups = ((cb + 1) // 2 + 31) // 32
        S = groups * 64
        mask = np.unpackbits(rec[16:16 + S // 8], bitorder="little").astype(bool)
        if int(mask.sum()) != cnt:
            raise ValueError(f"corrupt LC record {c}")
        sb = np.zeros(S, dtype=np.uint8)
        sb[mask] = rec[16 + S // 8:16 + S // 8 + cnt]
        out[c * CHUNK:c * CHUNK + cb] = _unshuffle(sb, cb)
    return out
