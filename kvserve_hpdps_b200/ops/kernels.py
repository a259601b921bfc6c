"""Python entry points of the native kernels (torch tensors in, tensors out).

Three groups:

* fused layer ops (:func:`quantize_layer`, :func:`dequantize_layer`): the
  producer's Hadamard + hybrid quantization of every request of one layer,
  read straight from the paged KV cache through a block table, and the
  consumer's dequantization + inverse transform + scatter into its own paged
  cache;
* the lossless codec (:func:`rans_encode`, :func:`rans_decode`,
  :func:`bitpack`, :func:`bitunpack`), on CUDA or CPU tensors with the same
  byte format;
* transfer helpers (block gather/scatter, copies with a release flag,
  bounded flag waits, the NVLink probe) and error metrics.

All device ops run on the current CUDA stream and never synchronise the
host, except where a function documents that it returns a host value.
"""

from __future__ import annotations

import ctypes
import math
import threading
from dataclasses import dataclass, field
from functools import lru_cache
from typing import Optional, Sequence

import numpy as np
import torch

from kvserve_hpdps_b200.compression.signs import hadamard_matrix, rademacher_signs
from kvserve_hpdps_b200.ops import _lib
from kvserve_hpdps_b200.ops._lib import LayerLaunch, PagedKV, check, lib

HEAD_DIM = 128
TILE_ROWS = 128
RANS_CHUNK = 32768
ENGINE_TCGEN05 = 0       # warp-specialized persistent tcgen05 kernels (default)
ENGINE_SIMT = 1          # SIMT butterfly
ENGINE_TCGEN05_TILE = 2  # tcgen05, one CTA per tile
ENGINE_TCGEN05_PERSISTENT = 3  # persistent tcgen05 without warp specialization

ERR_NAMES = {0: "none", 1: "mbarrier timeout", 2: "ready-flag timeout", 3: "bounds",
             4: "corrupt stream", 5: "overflow"}


_xfer = {"h2d": 0, "d2h": 0}


def reset_transfer_counters() -> None:
    """Reset the host<->device byte counters (benchmark accounting)."""
    _xfer["h2d"] = 0
    _xfer["d2h"] = 0


def transfer_counters() -> dict:
    """Bytes copied host->device (descriptor tables) and device->host (sizes,
    headers, error words) by this module since the last reset."""
    return dict(_xfer)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# ----------------------------------------------------------------- workspace
class _Workspace:
    """Scratch of one (device, stream) reused across launches (grown on
    demand): kernels queued on different streams may run at the same time,
    so each stream has its own buffers and completion counters; the device
    error word is shared by every stream of the device."""

    def __init__(self, device: torch.device, err: torch.Tensor):
        self.device = device
        self.err = err
        self.counters = torch.zeros(64, dtype=torch.int32, device=device)
        self._bufs: dict[str, torch.Tensor] = {}
        self._lock = threading.Lock()

    def buf(self, name: str, nbytes: int, dtype=torch.uint8) -> torch.Tensor:
        esz = torch.empty((), dtype=dtype).element_size()
        n = max(1, (nbytes + esz - 1) // esz)
        with self._lock:
            t = self._bufs.get(name)
            if t is None or t.numel() < n:
                t = torch.empty(int(n * 1.25) + 16, dtype=dtype, device=self.device)
                self._bufs[name] = t
        return t[:n]


_ws: dict[tuple, _Workspace] = {}
_err_words: dict[int, torch.Tensor] = {}
_ws_lock = threading.Lock()


def workspace(device: torch.device) -> _Workspace:
    """The scratch of ``device``'s current stream."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    stream = torch.cuda.current_stream(idx).cuda_stream
    key = (device.type, idx, stream)
    with _ws_lock:
        ws = _ws.get(key)
        if ws is None:
            dev = torch.device("cuda", idx)
            err = _err_words.get(idx)
            if err is None:
                err = _err_words[idx] = torch.zeros(4, dtype=torch.int32, device=dev)
            ws = _ws[key] = _Workspace(dev, err)
        return ws


def read_device_error(device: torch.device, reset: bool = True) -> int:
    """Host read (synchronising) of the device error word; 0 = no error."""
    ws = workspace(device)
    code = int(ws.err[0].item())
    _xfer["d2h"] += 4
    if reset and code:
        ws.err.zero_()
    return code


class ErrorMonitor:
    """Non-blocking watch of a device's error word for serving loops.

    ``poll()`` returns the code seen by the previous poll once that poll's
    asynchronous copy has landed (0 while it is in flight or when no error
    was recorded), then schedules a new copy of the word into pinned host
    memory on the current stream followed by clearing the word, so kernels
    that fail between two polls are reported at the second one without the
    host ever waiting on the device."""

    def __init__(self, device: torch.device):
        self.device = device
        self._host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._event: Optional[torch.cuda.Event] = None

    def poll(self) -> int:
        code = 0
        if self._event is not None:
            if not self._event.query():
                return 0
            code = int(self._host[0])
        ws = workspace(self.device)
        self._host.copy_(ws.err[:1], non_blocking=True)
        ws.err.zero_()
        self._event = torch.cuda.current_stream(self.device).record_event()
        _xfer["d2h"] += 4
        return code


class StepErrors:
    """Every step's device error word, read one step late: ``push()`` (after
    the step's work is enqueued) copies the word into pinned host memory on
    the current stream and clears it; ``check(keep)`` waits for all but the
    newest ``keep`` copies and raises on an error.  With ``keep=1`` the host
    enqueues step s+1 while step s still runs, and still reads every step's
    result; ``check(0)`` at the end reads the last one."""

    def __init__(self, device: torch.device, depth: int = 4):
        self.device = device
        self._free = [torch.zeros(1, dtype=torch.int32).pin_memory() for _ in range(depth)]
        self._pending: list = []

    def push(self) -> None:
        if not self._free:
            self.check(0)
        host = self._free.pop()
        ws = workspace(self.device)
        host.copy_(ws.err[:1], non_blocking=True)
        ws.err.zero_()
        self._pending.append((host, torch.cuda.current_stream(self.device).record_event()))
        _xfer["d2h"] += 4

    def check(self, keep: int = 0) -> None:
        while len(self._pending) > keep:
            host, ev = self._pending.pop(0)
            ev.synchronize()
            code = int(host[0])
            self._free.append(host)
            if code:
                raise RuntimeError(f"device error {code} ({ERR_NAMES.get(code, '?')})")


def check_device_error(device: torch.device, what: str = "kernel") -> None:
    code = read_device_error(device)
    if code:
        raise RuntimeError(f"{what}: device error {code} ({ERR_NAMES.get(code, '?')})")


# ---------------------------------------------------------- transform images
def _sw128_offsets() -> torch.Tensor:
    """Byte offset of element (a, b) of a 128x128 bf16 matrix in the K-major
    128-byte-swizzled UMMA layout (two 16 KB halves, b = reduction index)."""
    a = torch.arange(128).view(128, 1).expand(128, 128)
    b = torch.arange(128).view(1, 128).expand(128, 128)
    hb = b // 64
    byte = (b % 64) * 2
    chunk = (byte // 16) ^ (a % 8)
    return hb * 16384 + (a // 8) * 1024 + (a % 8) * 128 + chunk * 16 + byte % 16


@lru_cache(maxsize=1)
def _offsets_cached() -> torch.Tensor:
    return _sw128_offsets()


def swizzle_image(mat: torch.Tensor) -> torch.Tensor:
    """uint8[32768] image of a 128x128 matrix (bf16) in the SW128 K-major layout."""
    bf = mat.to(torch.bfloat16).contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
    img = torch.zeros(32768, dtype=torch.uint8)
    off = _offsets_cached().flatten()
    img[off] = (bf.flatten() & 0xFF).to(torch.uint8)
    img[off + 1] = (bf.flatten() >> 8).to(torch.uint8)
    return img


def transform_images(signs: Optional[torch.Tensor], num_heads: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Forward and inverse operand images, uint8 [H*32768] each.

    Forward: Bf[a][b] = s[b] H[a][b] (consumes the signed input).
    Inverse: Bi[a][b] = s[a] H[a][b] (signs on the output channel).
    ``signs=None`` gives identity images (no transform).
    """
    H = hadamard_matrix(HEAD_DIM)
    fwd, inv = [], []
    for h in range(num_heads):
        if signs is None:
            eye = torch.eye(HEAD_DIM)
            fwd.append(swizzle_image(eye))
            inv.append(swizzle_image(eye))
        else:
            s = signs[h].to(torch.float32)
            fwd.append(swizzle_image(H * s.view(1, -1)))
            inv.append(swizzle_image(H * s.view(-1, 1)))
    return torch.cat(fwd), torch.cat(inv)


def sign_bits(signs: Optional[torch.Tensor], num_heads: int) -> list[list[int]]:
    out = []
    for h in range(num_heads):
        words = [0, 0, 0, 0]
        if signs is not None:
            for d in range(HEAD_DIM):
                if float(signs[h, d]) < 0:
                    words[d >> 5] |= 1 << (d & 31)
        out.append(words)
    return out


# --------------------------------------------------------------- layer plan
def code_bits(levels: float, packed: bool) -> int:
    """Bits per code: 8 for byte codes, ceil(log2(levels)) when bit-packed."""
    if not packed:
        return 8
    return max(1, min(8, math.ceil(math.log2(max(2.0, float(levels))))))


@dataclass
class LayerPlan:
    """Quantization description of one layer on one rank."""
    num_heads: int
    key_levels: list[float]
    value_levels: list[float]
    signs: Optional[torch.Tensor]            # [H, 128] +-1, or None (identity)
    packed: bool = False                     # fixed-width bit packing of codes
    clamp_top: bool = True
    # Uniform code width in bits (e.g. 4: two codes per byte, the symbols an
    # entropy coder sees); heads whose codes do not fit keep 8.  Overrides
    # ``packed``'s per-head minimal widths.
    code_width: Optional[int] = None
    group_of_head: list[int] = field(default_factory=list)
    groups: list[list[int]] = field(default_factory=list)
    key_bits: list[int] = field(default_factory=list)
    value_bits: list[int] = field(default_factory=list)
    seg_prefix: list[int] = field(default_factory=list)
    _images: dict = field(default_factory=dict)
    _params: Optional[_lib.LayerParams] = None

    def __post_init__(self):
        H = self.num_heads
        if H > _lib.MAX_HEADS:
            raise ValueError(f"at most {_lib.MAX_HEADS} KV heads per rank, got {H}")
        if not self.group_of_head:
            gid: dict[float, int] = {}
            self.groups = []
            for h, v in enumerate(self.value_levels):
                v = float(v)
                if v not in gid:
                    gid[v] = len(gid)
                    self.groups.append([])
                self.group_of_head.append(gid[v])
                self.groups[gid[v]].append(h)
        else:
            G = max(self.group_of_head) + 1
            self.groups = [[h for h in range(H) if self.group_of_head[h] == g] for g in range(G)]
        if self.code_width:
            top = 0 if self.clamp_top else 1  # largest code is levels-1 (+1 unclamped)

            def width(levels: float) -> int:
                return self.code_width if float(levels) - 1 + top < 2 ** self.code_width else 8
            if not self.key_bits:
                self.key_bits = [width(v) for v in self.key_levels]
            if not self.value_bits:
                self.value_bits = [width(v) for v in self.value_levels]
            self.packed = any(b != 8 for b in self.key_bits + self.value_bits)
        if not self.key_bits:
            self.key_bits = [code_bits(v, self.packed) for v in self.key_levels]
        if not self.value_bits:
            self.value_bits = [code_bits(v, self.packed) for v in self.value_levels]
        pref = [0]
        for b in self.key_bits + self.value_bits:
            pref.append(pref[-1] + 16 * b)
        self.seg_prefix = pref

    @property
    def n_groups(self) -> int:
        return len(self.groups)

    def row_bytes(self) -> int:
        """Code bytes per token row over every (kv, head) segment."""
        return self.seg_prefix[-1]

    def meta_bytes(self, rows: int) -> int:
        return 2 * (2 * self.num_heads * HEAD_DIM + 2 * self.n_groups * rows)

    def images(self, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
        key = str(device)
        if key not in self._images:
            f, i = transform_images(self.signs, self.num_heads)
            self._images[key] = (f.to(device), i.to(device))
        return self._images[key]

    def params(self) -> _lib.LayerParams:
        if self._params is None:
            p = _lib.LayerParams()
            H = self.num_heads
            p.H = H
            p.n_groups = self.n_groups
            for h in range(H):
                p.key_levels[h] = float(self.key_levels[h])
                p.value_levels[h] = float(self.value_levels[h])
                p.key_bits[h] = self.key_bits[h]
                p.value_bits[h] = self.value_bits[h]
                p.group_of_head[h] = self.group_of_head[h]
            for i, v in enumerate(self.seg_prefix):
                p.seg_prefix[i] = v
            for h, words in enumerate(sign_bits(self.signs, H)):
                for j in range(4):
                    p.sign_bits[h][j] = words[j]
            p.clamp_top = 1 if self.clamp_top else 0
            p.transform = 1 if self.signs is not None else 0
            p.out_scale = 1.0 / math.sqrt(HEAD_DIM) if self.signs is not None else 1.0
            self._params = p
        return self._params


@lru_cache(maxsize=512)
def _signs_cached(layer_id: int, num_heads: int, seed: int) -> torch.Tensor:
    return rademacher_signs(layer_id, num_heads, HEAD_DIM, seed)


def make_layer_plan(num_heads: int, key_levels, value_levels, seed: Optional[int], layer_id: int,
                    packed: bool = False, clamp_top: bool = True,
                    code_width: Optional[int] = None) -> LayerPlan:
    signs = None if seed is None else _signs_cached(int(layer_id), int(num_heads), int(seed))
    return LayerPlan(num_heads, [float(x) for x in key_levels], [float(x) for x in value_levels],
                     signs, packed=packed, clamp_top=clamp_top, code_width=code_width)


def decode_plan(num_heads: int, group_of_head: Sequence[int], key_bits: Sequence[int],
                value_bits: Sequence[int], seed: Optional[int], layer_id: int) -> LayerPlan:
    """Plan for the consumer side, rebuilt from wire metadata (levels are
    not needed to dequantize: only groups, bits and the transform)."""
    signs = None if seed is None else _signs_cached(int(layer_id), int(num_heads), int(seed))
    packed = any(b != 8 for b in list(key_bits) + list(value_bits))
    return LayerPlan(num_heads, [2.0] * num_heads, [2.0] * num_heads, signs, packed=packed,
                     group_of_head=list(group_of_head), key_bits=list(key_bits),
                     value_bits=list(value_bits))


# ------------------------------------------------------------ launch tables
def _align16(x: int) -> int:
    return (x + 15) & ~15


def _num_blocks(kv_layer: torch.Tensor) -> int:
    """Blocks of a [2, nb, ...] (FlashAttention) or [nb, 2, ...] (FlashInfer) layer."""
    if kv_layer.shape[1] == 2 and kv_layer.shape[0] != 2:
        return kv_layer.shape[0]
    return kv_layer.shape[1]


def paged_kv(kv_layer: torch.Tensor) -> PagedKV:
    """Describe a paged KV layer tensor for the kernels.

    Accepts logical [2, nb, bs, H, D] (FlashAttention) and [nb, 2, bs, H, D]
    (FlashInfer) bf16 tensors whose (slot, head, d) block is either
    token-major (NHD: strides H*D, D, 1) or head-major (HND: strides D,
    bs*D, 1), as vLLM's attention backends allocate them.
    """
    if kv_layer.dtype != torch.bfloat16:
        raise TypeError(f"KV cache must be bf16, got {kv_layer.dtype}")
    if kv_layer.dim() != 5 or kv_layer.shape[-1] != HEAD_DIM:
        raise ValueError(f"expected a [2, nb, bs, H, {HEAD_DIM}] layer, got {tuple(kv_layer.shape)}")
    st = kv_layer.stride()
    bs, H, D = kv_layer.shape[2], kv_layer.shape[3], kv_layer.shape[4]
    if st[4] != 1:
        raise ValueError("KV layer head_dim must be contiguous")
    if st[3] == D and st[2] == H * D:
        hnd = 0
    elif st[2] == D and st[3] == bs * D:
        hnd = 1
    else:
        raise ValueError(f"unsupported KV block layout with strides {st}")
    if bs % 16:
        raise ValueError("block_size must be a multiple of 16")
    p = PagedKV()
    p.base = kv_layer.data_ptr()
    if kv_layer.shape[1] == 2 and kv_layer.shape[0] != 2:
        p.block_stride, p.kv_stride = st[0], st[1]
    else:
        p.kv_stride, p.block_stride = st[0], st[1]
    p.num_blocks = _num_blocks(kv_layer)
    p.slot_stride, p.head_stride = st[2], st[3]
    p.block_size = bs
    p.hnd = hnd
    return p


class LayerSlots:
    """Device-side description of the layers one launch can address.

    Slot i pairs a paged KV tensor with its LayerPlan.  Holds the device
    arrays of PagedKV records, TMA tensor maps (K and V plane per slot),
    LayerParams and the forward/inverse transform images.  All plans must
    have the same number of heads.
    """

    def __init__(self, kv_layers: Sequence[torch.Tensor], plans: Sequence[LayerPlan]):
        if len(kv_layers) != len(plans) or not plans:
            raise ValueError("one plan per KV layer tensor is required")
        self.kv_layers = list(kv_layers)
        self.plans = list(plans)
        self.device = kv_layers[0].device
        self.num_heads = plans[0].num_heads
        if any(p.num_heads != self.num_heads for p in plans):
            raise ValueError("all slots of a launch must have the same number of heads")
        for t in kv_layers:
            if t.shape[3] != self.num_heads:
                raise ValueError(f"KV tensor has {t.shape[3]} heads, plan has {self.num_heads}")
        n = len(plans)
        kvs = (PagedKV * n)(*[paged_kv(t) for t in kv_layers])
        lps = (_lib.LayerParams * n)(*[p.params() for p in plans])
        maps = (ctypes.c_uint8 * (256 * n))()
        if self.device.type == "cuda":
            for i in range(n):
                rc = lib().kvs_make_plane_maps(ctypes.byref(kvs[i]), self.num_heads,
                                               ctypes.addressof(maps) + 256 * i)
                check(rc, "make_plane_maps")
        self._kvs = self._to_dev(bytes(kvs))
        self._lps = self._to_dev(bytes(lps))
        self._maps = self._to_dev(bytes(maps))
        fwd, inv = zip(*[p.images(torch.device("cpu")) for p in plans])
        self.bmat_stride = self.num_heads * 32768
        self.bmat_fwd = torch.cat(fwd).to(self.device)
        self.bmat_inv = torch.cat(inv).to(self.device)

    def _to_dev(self, raw: bytes) -> torch.Tensor:
        t = torch.frombuffer(bytearray(raw), dtype=torch.uint8).clone()
        return t.to(self.device) if self.device.type == "cuda" else t

    def item_constants(self) -> tuple[np.ndarray, ...]:
        """Per slot (cached): number of blocks, block size, code bytes per
        token row, value groups; WorkItems indexes them by item slot."""
        c = self.__dict__.get("_item_consts")
        if c is None:
            c = tuple(np.asarray(v, dtype=np.int64) for v in (
                [_num_blocks(t) for t in self.kv_layers],
                [t.shape[2] for t in self.kv_layers],
                [p.row_bytes() for p in self.plans],
                [p.n_groups for p in self.plans]))
            self._item_consts = c
        return c

    @classmethod
    def single(cls, kv_layer: torch.Tensor, plan: LayerPlan) -> "LayerSlots":
        return cls([kv_layer], [plan])


class WorkItems:
    """Work items of a launch: (slot, block ids, valid tokens) triples.

    Codes of item r start at ``code_off[r]`` (segments ``[kv][head][row]``
    of ``16*bits`` bytes), its fp16 metadata at ``meta_off[r]``.
    """

    def __init__(self, slots: LayerSlots, items: Sequence[tuple[int, Sequence[int], int]],
                 code_offsets: Optional[Sequence[int]] = None,
                 meta_offsets: Optional[Sequence[int]] = None):
        """``code_offsets`` / ``meta_offsets`` override where each item's
        codes / metadata start (used to decode a subset of the items of a
        larger message in place).

        Items that pass the same block-id sequence object (e.g. one request
        at every layer) share one copy of it in the device block table."""
        self.slots = slots
        dev = slots.device
        self.device = dev
        uniq: dict[int, int] = {}  # id(block sequence) -> index into arrs
        arrs: list[np.ndarray] = []
        s_l, li_l, n_l = [], [], []
        for s, b, n in items:
            k = id(b)
            li = uniq.get(k)
            if li is None:
                li = uniq[k] = len(arrs)
                src = b.detach().cpu() if isinstance(b, torch.Tensor) else b
                arrs.append(np.asarray(src, dtype=np.int64).reshape(-1))
            s_l.append(int(s))
            li_l.append(li)
            n_l.append(int(n))
        lists = [a.tolist() for a in arrs]
        self.items = [(s, lists[li], n) for s, li, n in zip(s_l, li_l, n_l)]
        R = len(s_l)
        s_a = np.asarray(s_l, dtype=np.int64)
        li_a = np.asarray(li_l, dtype=np.int64)
        n_a = np.asarray(n_l, dtype=np.int64)
        consts = slots.item_constants()  # per slot: blocks, block size, row bytes, groups
        nb_s, bs_s, rb_s, g_s = (c[s_a] for c in consts)
        lens = np.asarray([a.size for a in arrs], dtype=np.int64)
        lo = np.asarray([a.min() if a.size else 0 for a in arrs], dtype=np.int64)
        hi = np.asarray([a.max() if a.size else -1 for a in arrs], dtype=np.int64)
        bad = np.nonzero((lo[li_a] < 0) | (hi[li_a] >= nb_s))[0]
        if bad.size:
            r = int(bad[0])
            v = int(lo[li_a[r]]) if lo[li_a[r]] < 0 else int(hi[li_a[r]])
            raise ValueError(f"block id {v} outside the {int(nb_s[r])} blocks "
                             f"of layer slot {int(s_a[r])}")
        rows = lens[li_a] * bs_s
        tiles = (rows + TILE_ROWS - 1) // TILE_ROWS
        prefix = np.concatenate([[0], np.cumsum(tiles)])
        list_off = np.concatenate([[0], np.cumsum(lens)[:-1]]) if arrs else np.zeros(0, np.int64)
        csz = (rows * rb_s + 15) & ~15
        msz = (2 * (2 * slots.num_heads * HEAD_DIM + 2 * g_s * rows) + 15) & ~15
        code_off = np.concatenate([[0], np.cumsum(csz)])
        meta_off = np.concatenate([[0], np.cumsum(msz)])
        row_off = np.concatenate([[0], np.cumsum(rows)])
        self.n_rows = rows.tolist()
        self.n_tokens = n_l
        self.tiles = tiles.tolist()
        self.total_tiles = int(prefix[-1])
        self.code_off = code_off[:-1].tolist()
        self.meta_off = meta_off[:-1].tolist()
        self.row_off = row_off[:-1].tolist()
        self.code_bytes, self.meta_bytes = int(code_off[-1]), int(meta_off[-1])
        self.total_rows = int(row_off[-1])
        for offs in (code_offsets, meta_offsets):
            if offs is not None and any(int(o) % 16 for o in offs):
                raise ValueError("item code / metadata offsets must be multiples of 16 bytes")
        if code_offsets is not None:
            if len(code_offsets) != R:
                raise ValueError("one code offset per item is required")
            self.code_off = [int(x) for x in code_offsets]
            self.code_bytes = int(max((o + r * b for o, r, b in
                                       zip(self.code_off, rows.tolist(), rb_s.tolist())),
                                      default=0))
        if meta_offsets is not None:
            if len(meta_offsets) != R:
                raise ValueError("one metadata offset per item is required")
            self.meta_off = [int(x) for x in meta_offsets]
            self.meta_bytes = int(max((o + 2 * (2 * slots.num_heads * HEAD_DIM + 2 * g * r)
                                       for o, r, g in
                                       zip(self.meta_off, rows.tolist(), g_s.tolist())),
                                      default=0))
        bt = np.concatenate(arrs) if arrs else np.zeros(0, np.int64)
        nbt = int(bt.size)
        ints = np.concatenate([bt, list_off[li_a] if R else np.zeros(0, np.int64), n_a, rows,
                               prefix, s_a]).astype(np.int32)
        longs = np.asarray(self.code_off + self.meta_off + self.row_off, dtype=np.int64)
        hi_t = torch.from_numpy(ints if ints.size else np.zeros(1, np.int32))
        hl_t = torch.from_numpy(longs if longs.size else np.zeros(1, np.int64))
        if dev.type == "cuda":
            hi_t, hl_t = hi_t.pin_memory(), hl_t.pin_memory()
            self._ints = hi_t.to(dev, non_blocking=True)
            self._longs = hl_t.to(dev, non_blocking=True)
            _xfer["h2d"] += hi_t.numel() * 4 + hl_t.numel() * 8
        else:
            self._ints, self._longs = hi_t.clone(), hl_t.clone()
        self._o = {"bt": 0, "off": nbt, "ntok": nbt + R, "rows": nbt + 2 * R,
                   "prefix": nbt + 3 * R, "slot": nbt + 4 * R + 1}

    @property
    def num_items(self) -> int:
        return len(self.items)

    def req_table(self) -> _lib.ReqTable:
        R = self.num_items
        base = self._ints.data_ptr()
        lb = self._longs.data_ptr()
        rt = _lib.ReqTable()
        rt.block_table = base + 4 * self._o["bt"]
        rt.bt_off = base + 4 * self._o["off"]
        rt.n_tokens = base + 4 * self._o["ntok"]
        rt.n_rows = base + 4 * self._o["rows"]
        rt.tile_prefix = base + 4 * self._o["prefix"]
        rt.slot = base + 4 * self._o["slot"]
        rt.code_off = lb
        rt.meta_off = lb + 8 * R
        rt.row_off = lb + 16 * R
        rt.num_req = R
        return rt

    def item_codes(self, codes: torch.Tensor, r: int) -> torch.Tensor:
        plan = self.slots.plans[self.items[r][0]]
        return codes[self.code_off[r]:self.code_off[r] + self.n_rows[r] * plan.row_bytes()]

    def item_meta(self, meta: torch.Tensor, r: int) -> torch.Tensor:
        plan = self.slots.plans[self.items[r][0]]
        return meta[self.meta_off[r]:self.meta_off[r] + plan.meta_bytes(self.n_rows[r])]


class RequestBatch:
    """Single-layer convenience: requests of one layer (slot 0)."""

    def __init__(self, block_ids: Sequence[Sequence[int]], n_tokens: Sequence[int],
                 block_size: int, device: torch.device):
        self.block_ids = [list(map(int, b)) for b in block_ids]
        self.n_tokens = [int(n) for n in n_tokens]
        self.block_size = int(block_size)
        self.device = device
        self.n_rows = [len(b) * self.block_size for b in self.block_ids]
        self._items: dict[int, WorkItems] = {}

    def items_for(self, slots: LayerSlots) -> WorkItems:
        key = id(slots)
        if key not in self._items:
            self._items[key] = WorkItems(slots, [(0, b, n) for b, n in zip(self.block_ids, self.n_tokens)])
        return self._items[key]

    def layout(self, plan: LayerPlan) -> tuple[list[int], list[int], int, int]:
        code_off, meta_off = [], []
        c = m = 0
        for rows in self.n_rows:
            code_off.append(c)
            meta_off.append(m)
            c += _align16(rows * plan.row_bytes())
            m += _align16(plan.meta_bytes(rows))
        return code_off, meta_off, c, m


# ---------------------------------------------------------------- fused ops
# Device trace of the warp-specialized kernels (diagnostics; off by default).
TRACE_CTAS = 8
TRACE_EVENTS = ("tile_ready", "mma_issued", "refill_issued", "epi_mma_seen", "epi_done",
                "acc_free_seen", "epi_quantized", "epi_staged")
# the dequantize kernel's events, same slots
TRACE_EVENTS_DEQUANT = ("unpack_start", "unpack_done", "mma_issued", "epi_mma_seen",
                        "epi_stores_issued", "a_full_seen", "codes_ready", "codes_issued")
_trace = {"buf": None, "jobs": 0}


@lru_cache(maxsize=None)
def _sm_count(index: int) -> int:
    return torch.cuda.get_device_properties(index).multi_processor_count


def _raw_block_layout(kv_layer: torch.Tensor) -> tuple[PagedKV, str]:
    """Descriptor of a paged layer for whole-block raw copies (any dtype and
    head size) and its block order ("nhd" or "hnd").  Each (plane, block)
    must be one dense run of ``bs * H * D`` elements."""
    if kv_layer.dim() != 5:
        raise ValueError(f"expected a [2, nb, bs, H, D] layer, got {tuple(kv_layer.shape)}")
    st, sh = kv_layer.stride(), kv_layer.shape
    bs, H, D = sh[2], sh[3], sh[4]
    if st[4] == 1 and st[3] == D and st[2] == H * D:
        order = "nhd"
    elif st[4] == 1 and st[2] == D and st[3] == bs * D:
        order = "hnd"
    else:
        raise ValueError(f"KV blocks are not dense (strides {st})")
    p = PagedKV()
    p.base = kv_layer.data_ptr()
    if sh[1] == 2 and sh[0] != 2:
        p.block_stride, p.kv_stride = st[0], st[1]
    else:
        p.kv_stride, p.block_stride = st[0], st[1]
    p.num_blocks = _num_blocks(kv_layer)
    p.slot_stride, p.head_stride = st[2], st[3]
    p.block_size = bs
    p.hnd = 1 if order == "hnd" else 0
    return p, order


class RawItems:
    """Uncompressed whole-block transfer of (layer, block ids) items between
    paged KV layers and one flat buffer, in one launch per direction.

    The flat buffer holds the items back to back, each as
    ``[2, len(blocks), block_size, H, D]`` (the reference's per-layer raw
    layout, kvserve_v1/utils/kv_utils.py:59-80); items (0, b), (1, b), ...
    (L-1, b) therefore form the stacked ``[L, 2, nb, bs, H, D]`` request
    tensor.  Block ids are checked here against each layer's cache and
    again on the device.  Descriptors reach the device in one copy.
    """

    def __init__(self, kv_layers: Sequence[torch.Tensor],
                 items: Sequence[tuple[int, Sequence[int]]]):
        if not kv_layers or not items:
            raise ValueError("at least one layer and one item are required")
        self.device = kv_layers[0].device
        descs = [_raw_block_layout(t) for t in kv_layers]
        orders = {o for _, o in descs}
        if len(orders) != 1:
            raise ValueError("all layers of a raw transfer must share one block order")
        self.block_order = orders.pop()
        shapes = {tuple(t.shape[2:]) for t in kv_layers}
        dtypes = {t.dtype for t in kv_layers}
        if len(shapes) != 1 or len(dtypes) != 1:
            raise ValueError("all layers of a raw transfer must share block shape and dtype")
        self.block_shape = shapes.pop()
        self.dtype = dtypes.pop()
        self.elem_bytes = torch.empty((), dtype=self.dtype).element_size()
        bs, H, D = self.block_shape
        self.block_bytes = bs * H * D * self.elem_bytes
        if self.block_bytes % 16:
            raise ValueError("a KV block must be a multiple of 16 bytes")
        uniq: dict[int, int] = {}
        lists: list[list[int]] = []
        norm = []
        for s, b in items:
            k = id(b)
            if k not in uniq:
                uniq[k] = len(lists)
                lists.append(b.tolist() if isinstance(b, torch.Tensor) else [int(x) for x in b])
            norm.append((int(s), uniq[k]))
        span = [(min(b), max(b)) if b else (0, -1) for b in lists]
        for s, li in norm:
            if not 0 <= s < len(kv_layers):
                raise ValueError(f"item layer {s} outside the {len(kv_layers)} layers")
            lo, hi = span[li]
            nb = descs[s][0].num_blocks
            if lo < 0 or hi >= nb:
                raise ValueError(f"block id {lo if lo < 0 else hi} outside the {nb} blocks "
                                 f"of layer slot {s}")
        bt, list_off = [], []
        for b in lists:
            list_off.append(len(bt))
            bt.extend(b)
        ritems = (_lib.RawItem * len(norm))()
        prefix = [0]
        flat = 0
        self.item_offsets, self.item_blocks = [], []
        for i, (s, li) in enumerate(norm):
            nb = len(lists[li])
            ritems[i].bt_off, ritems[i].flat_off = list_off[li], flat
            ritems[i].slot, ritems[i].nblocks = s, nb
            self.item_offsets.append(flat)
            self.item_blocks.append(nb)
            flat += 2 * nb * self.block_bytes
            prefix.append(prefix[-1] + 2 * nb)
        self.flat_bytes = flat
        self.n_units = prefix[-1]
        self.n_items = len(norm)
        kvs = (PagedKV * len(descs))(*[d for d, _ in descs])
        parts = [bytes(kvs), bytes(ritems),
                 torch.tensor(prefix, dtype=torch.int64).numpy().tobytes(),
                 torch.tensor(bt or [0], dtype=torch.int32).numpy().tobytes()]
        offs, raw = [], bytearray()
        for p in parts:
            offs.append(len(raw))
            raw += p
            raw += bytes((-len(raw)) % 16)
        host = torch.frombuffer(raw, dtype=torch.uint8).clone()
        if self.device.type == "cuda":
            host = host.pin_memory()
            _xfer["h2d"] += host.numel()
        self._desc = host.to(self.device, non_blocking=True)
        base = self._desc.data_ptr()
        self._ptrs = [base + o for o in offs]  # kvs, items, prefix, block table

    def flat_shape(self, r: int = 0) -> tuple[int, ...]:
        return (2, self.item_blocks[r]) + tuple(self.block_shape)


def paged_raw(raw: RawItems, flat_ptr: int, gather: bool, flag_ptr: Optional[int] = None,
              flag_value: int = 0, trailer_ptr: Optional[int] = None,
              checksum: Optional[torch.Tensor] = None, max_ctas: Optional[int] = None) -> None:
    """Gather (paged -> flat) or scatter (flat -> paged) every item of ``raw``
    in one launch on the current stream.  ``flat_ptr`` may be a peer GPU's
    memory for the gather.  With ``checksum`` (int64[2] on the device) the
    gather also computes the message checksum of the flat bytes (as
    :func:`checksum` would); ``trailer_ptr`` receives it and ``flag_ptr``
    receives ``flag_value`` (release, system scope) once everything landed."""
    dev = raw.device
    ws = workspace(dev)
    a = _lib.RawLaunch()
    a.kvs, a.items, a.unit_prefix, a.block_table = raw._ptrs
    a.flat = flat_ptr
    a.err = ws.err.data_ptr()
    a.ck = checksum.data_ptr() if checksum is not None else None
    a.trailer = trailer_ptr if (checksum is not None and trailer_ptr is not None) else None
    a.counter = ws.counters[6:7].data_ptr() if flag_ptr is not None else None
    a.flag = flag_ptr
    a.n_units, a.n_items = raw.n_units, raw.n_items
    a.dir = 0 if gather else 1
    a.block_bytes, a.elem_bytes = raw.block_bytes, raw.elem_bytes
    a.flag_value = flag_value & 0xFFFFFFFF
    if max_ctas is None:
        max_ctas = 8 * _sm_count(dev.index if dev.index is not None else torch.cuda.current_device())
    check(lib().kvs_paged_raw(ctypes.byref(a), int(max_ctas), _stream(dev)), "paged_raw")


def set_trace(device: Optional[torch.device], jobs_per_cta: int = 256) -> Optional[torch.Tensor]:
    """Enable (device given) or disable (None) globaltimer tracing of the
    warp-specialized kernels for the first TRACE_CTAS CTAs of each launch;
    returns the trace buffer [TRACE_CTAS, jobs_per_cta, 8] (int64 ns, 0 =
    no event).  Every traced launch overwrites it."""
    if device is None:
        _trace["buf"], _trace["jobs"] = None, 0
        return None
    _trace["buf"] = torch.zeros((TRACE_CTAS, jobs_per_cta, 8), dtype=torch.int64, device=device)
    _trace["jobs"] = int(jobs_per_cta)
    return _trace["buf"]


def _check_extents(codes: torch.Tensor, meta: torch.Tensor, items: WorkItems) -> None:
    """The kernels address codes and metadata at the items' offsets: buffers
    shorter than the items' extents (a message whose layout does not match
    the consumer's requests) are refused before a launch could read or
    write past them."""
    cb = codes.numel() * codes.element_size()
    mb = meta.numel() * meta.element_size()
    if cb < items.code_bytes or mb < items.meta_bytes:
        raise ValueError(f"code/metadata buffers of {cb}/{mb} bytes are shorter than the "
                         f"{items.code_bytes}/{items.meta_bytes} bytes the work items address")


def _launch(slots: LayerSlots, items: WorkItems, bmat: torch.Tensor, codes, meta, kstat, vstat,
            engine: int, ck: Optional[torch.Tensor] = None, ck_off: int = 0) -> LayerLaunch:
    dev = slots.device
    L = LayerLaunch()
    L.kvs = slots._kvs.data_ptr()
    L.maps = slots._maps.data_ptr()
    L.lps = slots._lps.data_ptr()
    L.rt = items.req_table()
    L.bmat = bmat.data_ptr()
    L.bmat_stride = slots.bmat_stride
    L.codes = codes.data_ptr()
    L.meta = meta.data_ptr()
    L.kstat = 0 if kstat is None else kstat.data_ptr()
    L.vstat = 0 if vstat is None else vstat.data_ptr()
    L.err = workspace(dev).err.data_ptr()
    L.total_tiles = items.total_tiles
    L.num_heads = slots.num_heads
    L.engine = engine
    L.stream = _stream(dev)
    if _trace["buf"] is not None:
        L.trace = _trace["buf"].data_ptr()
        L.trace_jobs = _trace["jobs"]
    if ck is not None:
        L.ck = ck.data_ptr()
        L.ck_off = int(ck_off)
    return L


def quantize(slots: LayerSlots, items: WorkItems, codes: Optional[torch.Tensor] = None,
             meta: Optional[torch.Tensor] = None, engine: int = ENGINE_TCGEN05,
             ck: Optional[torch.Tensor] = None,
             ck_off: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize every work item (layer, request) in four launches; returns
    (codes u8, meta u8) laid out as described by ``items``.  ``codes`` may
    be a view of a peer GPU's receive ring (the quantize kernel's own 16-byte
    stores write it over NVLink); with ``ck`` (int64[2] on the device, engine
    0) the kernel adds the message checksum of the code bytes it stores,
    ``ck_off`` being the message offset of ``codes[0]``."""
    dev = slots.device
    ws = workspace(dev)
    if codes is None:
        codes = torch.empty(max(items.code_bytes, 16), dtype=torch.uint8, device=dev)
    if meta is None:
        meta = torch.empty(max(items.meta_bytes, 16), dtype=torch.uint8, device=dev)
    _check_extents(codes, meta, items)
    n_pairs = items.num_items * slots.num_heads * HEAD_DIM
    kstat = ws.buf("kstat", 8 * n_pairs, torch.int32)
    vstat = ws.buf("vstat", 8 * items.total_rows * slots.num_heads, torch.float32)
    L = _launch(slots, items, slots.bmat_fwd, codes, meta, kstat, vstat, engine, ck, ck_off)
    lb = lib()
    check(lb.kvs_init_key_stats(kstat.data_ptr(), n_pairs, L.stream), "init_key_stats")
    check(lb.kvs_stats(ctypes.byref(L)), "stats")
    if engine == ENGINE_TCGEN05:  # value (min, 1/scale) per row and group, once
        vparam = ws.buf("vparam", 2 * items.total_rows * slots.num_heads * 4, torch.float32)
        L.vparam = vparam.data_ptr()
        check(lb.kvs_value_params(ctypes.byref(L), max(items.n_rows, default=0)),
              "value_params")
    check(lb.kvs_quant(ctypes.byref(L)), "quant")
    return codes, meta


def dequantize(codes: torch.Tensor, meta: torch.Tensor, dst_slots: LayerSlots, items: WorkItems,
               engine: int = ENGINE_TCGEN05) -> None:
    """Dequantize + inverse transform every item into its destination slot
    (paged cache) at the item's block ids (one launch)."""
    _check_extents(codes, meta, items)
    L = _launch(dst_slots, items, dst_slots.bmat_inv, codes, meta, None, None, engine)
    check(lib().kvs_dequant_inverse(ctypes.byref(L)), "dequant_inverse")


def quantize_layer(kv_layer: torch.Tensor, batch: RequestBatch, plan: LayerPlan,
                   codes: Optional[torch.Tensor] = None, meta: Optional[torch.Tensor] = None,
                   engine: int = ENGINE_TCGEN05,
                   slots: Optional[LayerSlots] = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Single-layer form of :func:`quantize` (codes at batch.layout(plan))."""
    slots = slots or LayerSlots.single(kv_layer, plan)
    return quantize(slots, batch.items_for(slots), codes, meta, engine)


def dequantize_layer(codes: torch.Tensor, meta: torch.Tensor, dst_layer: torch.Tensor,
                     batch: RequestBatch, plan: LayerPlan, engine: int = ENGINE_TCGEN05,
                     slots: Optional[LayerSlots] = None) -> None:
    slots = slots or LayerSlots.single(dst_layer, plan)
    dequantize(codes, meta, slots, batch.items_for(slots), engine)


# ------------------------------------------------------------------- codec
def rans_max_bytes(n: int, chunk: int = RANS_CHUNK) -> int:
    return int(lib().kvs_rans_max_bytes(n, chunk))


def lc_encode(data: torch.Tensor, trim: bool = True) -> torch.Tensor:
    """LC-style (BIT_2 + RZE_1) stream of the bytes of ``data`` (format in
    ``csrc/lc_codec.cu``).  CUDA: three launches; with ``trim`` the host
    reads the stream size (one synchronisation).  CPU: the native coder
    (chunks on host threads), which writes the identical stream; the numpy
    module ``compression.lc`` is the reference of both."""
    from kvserve_hpdps_b200.compression import lc as lc_ref
    src = data.contiguous().view(torch.uint8).reshape(-1)
    n = src.numel()
    if n == 0:
        raise ValueError("empty input")
    if src.device.type == "cpu":
        lb = lib()
        cap = int(lb.kvs_cpu_lc_max_bytes(n))
        buf = torch.empty(cap, dtype=torch.uint8)
        size = int(lb.kvs_cpu_lc_encode(src.data_ptr(), n, buf.data_ptr(), cap))
        if size == 0:
            raise RuntimeError("CPU LC encode failed")
        return buf[:size].clone()
    dev = src.device
    lb = lib()
    ws = workspace(dev)
    out = torch.empty(int(lb.kvs_lc_max_bytes(n)), dtype=torch.uint8, device=dev)
    staging = ws.buf("lc_staging", int(lb.kvs_lc_staging_bytes(n)))
    nchunks = (n + lc_ref.CHUNK - 1) // lc_ref.CHUNK
    rec_len = ws.buf("lc_len", 4 * nchunks, torch.int32)
    total = ws.buf("lc_total", 8, torch.int64)
    check(lb.kvs_lc_encode(src.data_ptr(), n, staging.data_ptr(), rec_len.data_ptr(),
                           out.data_ptr(), total.data_ptr(), _stream(dev)), "lc_encode")
    if trim:
        _xfer["d2h"] += 8
        return out[:int(total[0].item())]
    return out


def lc_decode(stream: torch.Tensor, n: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Bytes of an LC stream; a corrupt stream records ERR_CORRUPT in the
    device error word (CUDA) or raises ValueError (CPU)."""
    if stream.device.type == "cpu":
        s = stream.contiguous()
        res = torch.empty(int(n), dtype=torch.uint8) if out is None else out
        rc = lib().kvs_cpu_lc_decode(s.data_ptr(), s.numel(), res.data_ptr(), int(n))
        if rc != 0:
            raise ValueError(f"corrupt LC stream ({rc})")
        return res
    dev = stream.device
    if out is None:
        out = torch.empty(int(n), dtype=torch.uint8, device=dev)
    s = stream.contiguous()
    check(lib().kvs_lc_decode(s.data_ptr(), s.numel(), out.data_ptr(), int(n),
                              workspace(dev).err.data_ptr(), _stream(dev)), "lc_decode")
    return out


def rans_encode(data: torch.Tensor, out: Optional[torch.Tensor] = None, chunk: int = RANS_CHUNK,
                flag: Optional[torch.Tensor] = None, flag_value: int = 0,
                trim: bool = True) -> torch.Tensor:
    """Entropy-code the bytes of ``data``.

    CUDA: returns the stream buffer; with ``trim`` (default) the host reads
    the stream size (one synchronisation) and the result is trimmed to it,
    otherwise the full worst-case buffer is returned (the size is in the
    stream header).  CPU: always exact size.
    """
    src = data.contiguous().view(torch.uint8).reshape(-1)
    n = src.numel()
    lb = lib()
    if src.device.type == "cpu":
        cap = int(lb.kvs_cpu_rans_max_bytes(n, chunk))
        buf = torch.empty(cap, dtype=torch.uint8)
        size = int(lb.kvs_cpu_rans_encode(src.data_ptr(), n, chunk, buf.data_ptr(), cap))
        if size == 0:
            raise RuntimeError("CPU rANS encode failed")
        return buf[:size].clone()
    dev = src.device
    ws = workspace(dev)
    cap = int(lb.kvs_rans_max_bytes(n, chunk))
    if out is None:
        out = torch.empty(cap, dtype=torch.uint8, device=dev)
    elif out.numel() < cap:
        raise ValueError(f"output buffer too small ({out.numel()} < {cap})")
    staging = ws.buf("rans_staging", int(lb.kvs_rans_staging_bytes(n, chunk)))
    sizes = ws.buf("rans_sizes", 4 * int(lb.kvs_rans_sizes_words(n, chunk)), torch.int32)
    total = ws.buf("rans_total", 8, torch.int64)
    msg = None
    if flag is not None:
        msg = _lib.RansMsg()
        msg.counter = ws.counters[0:1].data_ptr()
        msg.flag, msg.flag_value = flag.data_ptr(), flag_value & 0xFFFFFFFF
    check(lb.kvs_rans_encode(src.data_ptr(), n, chunk, staging.data_ptr(), sizes.data_ptr(),
                             out.data_ptr(), total.data_ptr(),
                             ctypes.byref(msg) if msg is not None else None, _stream(dev)),
          "rans_encode")
    if trim:
        _xfer["d2h"] += 8
        return out[:int(total[0].item())]
    return out


def rans_stream_size(stream: torch.Tensor) -> int:
    """Total bytes of a stream from its header (host read)."""
    hdr = stream[:32].cpu().numpy().view("<u8")
    return int(hdr[3])


def rans_decode(stream: torch.Tensor, n: int, out: Optional[torch.Tensor] = None,
                chunk: int = RANS_CHUNK) -> torch.Tensor:
    """Decode ``n`` bytes (uint8 tensor on the stream's device)."""
    lb = lib()
    if stream.device.type == "cpu":
        s = stream.contiguous()
        res = torch.empty(n, dtype=torch.uint8) if out is None else out
        rc = lb.kvs_cpu_rans_decode(s.data_ptr(), s.numel(), res.data_ptr(), n)
        if rc != 0:
            raise RuntimeError(f"CPU rANS decode failed ({rc})")
        return res
    dev = stream.device
    res = torch.empty(n, dtype=torch.uint8, device=dev) if out is None else out
    s = stream.contiguous()
    check(lb.kvs_rans_decode(s.data_ptr(), s.numel(), res.data_ptr(), n, chunk,
                             workspace(dev).err.data_ptr(), _stream(dev)), "rans_decode")
    return res


def rans_encode_ptr(src_ptr: int, n: int, out_ptr: int, device: torch.device,
                    flag_ptr: Optional[int] = None, flag_value: int = 0,
                    chunk: int = RANS_CHUNK) -> None:
    """Encode ``n`` device bytes at ``src_ptr`` into ``out_ptr`` (capacity
    :func:`rans_max_bytes`; may be a peer GPU's buffer).  With ``flag_ptr``
    the last CTA publishes ``flag_value`` there after a system-scope fence.
    No host synchronisation."""
    rans_encode_message(src_ptr, n, out_ptr, device, flag_ptr=flag_ptr, flag_value=flag_value,
                        chunk=chunk)


def rans_encode_message(src_ptr: int, n: int, out_ptr: int, device: torch.device,
                        total: Optional[torch.Tensor] = None,
                        prefix: Optional[Sequence[int]] = None, msg_off: int = 0,
                        ck: Optional[torch.Tensor] = None, trailer_ptr: Optional[int] = None,
                        flag_ptr: Optional[int] = None, flag_value: int = 0,
                        chunk: int = RANS_CHUNK) -> None:
    """Encode ``n`` device bytes at ``src_ptr`` straight into a transfer
    message: the stream is written at ``out_ptr`` (capacity
    :func:`rans_max_bytes`; may be a peer GPU's receive ring, reached by this
    framework's own stores), ``prefix`` (four uint32) is stored in the 16
    bytes before it (the container header), ``total`` (int64[1] on the
    device) receives the stream size, ``ck`` (int64[2], zeroed) accumulates
    the message checksum of everything written (``msg_off`` = message
    offset of ``out_ptr``, a multiple of 16), and the last CTA stores the
    finished checksum to ``trailer_ptr`` and publishes ``flag_value`` at
    ``flag_ptr`` (release, system scope).  Three launches, no host
    synchronisation."""
    lb = lib()
    ws = workspace(device)
    staging = ws.buf("rans_staging", int(lb.kvs_rans_staging_bytes(n, chunk)))
    sizes = ws.buf("rans_sizes", 4 * int(lb.kvs_rans_sizes_words(n, chunk)), torch.int32)
    if total is None:
        total = ws.buf("rans_total", 8, torch.int64)
    m = _lib.RansMsg()
    if prefix is not None:
        for i, w in enumerate(prefix):
            m.prefix[i] = int(w) & 0xFFFFFFFF
        m.has_prefix = 1
    m.msg_off = int(msg_off)
    m.ck = _ptr(ck)
    m.trailer = trailer_ptr if ck is not None else None
    if flag_ptr is not None:
        m.counter = ws.counters[3:4].data_ptr()
        m.flag, m.flag_value = flag_ptr, flag_value & 0xFFFFFFFF
    check(lb.kvs_rans_encode(src_ptr, n, chunk, staging.data_ptr(), sizes.data_ptr(), out_ptr,
                             total.data_ptr(), ctypes.byref(m), _stream(device)), "rans_encode")


def rans_decode_ptr(stream_ptr: int, n: int, out_ptr: int, device: torch.device,
                    chunk: int = RANS_CHUNK, stream_bytes: Optional[int] = None) -> None:
    """Decode from a raw device pointer; ``stream_bytes`` (the buffer's size,
    when known) bounds every read of a corrupt stream."""
    length = (1 << 64) - 1 if stream_bytes is None else int(stream_bytes)
    check(lib().kvs_rans_decode(stream_ptr, length, out_ptr, n, chunk,
                                workspace(device).err.data_ptr(), _stream(device)), "rans_decode")


def bitpack(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """Pack rows of 128 codes to ``bits`` bits each (CPU reference of the
    device layout): [rows, 128] u8 -> [rows, 16*bits] u8."""
    c = codes.contiguous().to("cpu").view(-1, HEAD_DIM)
    out = torch.empty((c.shape[0], 16 * bits), dtype=torch.uint8)
    lib().kvs_cpu_bitpack(c.data_ptr(), c.shape[0], bits, out.data_ptr())
    return out


def bitunpack(packed: torch.Tensor, bits: int) -> torch.Tensor:
    p = packed.contiguous().to("cpu").view(-1, 16 * bits)
    out = torch.empty((p.shape[0], HEAD_DIM), dtype=torch.uint8)
    lib().kvs_cpu_bitunpack(p.data_ptr(), p.shape[0], bits, out.data_ptr())
    return out


# ------------------------------------------------------------ data movement
def block_copy(kv_layer: torch.Tensor, blocks: torch.Tensor, flat_ptr: int, gather: bool,
               flag: Optional[torch.Tensor] = None, flag_value: int = 0) -> None:
    """Gather (paged -> flat) or scatter (flat -> paged) whole blocks of both
    planes.  ``flat_ptr`` may point into a peer GPU's memory."""
    p = paged_kv(kv_layer)
    nb = blocks.numel()
    block_elems = kv_layer.shape[2] * kv_layer.shape[3] * kv_layer.shape[4]
    ws = workspace(kv_layer.device)
    counter = ws.counters[1:2] if flag is not None else None
    check(lib().kvs_block_copy(ctypes.byref(p), blocks.data_ptr(), nb, block_elems, flat_ptr,
                               0 if gather else 1, _ptr(counter), _ptr(flag), flag_value,
                               ws.err.data_ptr(), _stream(kv_layer.device)), "block_copy")


def copy_bytes(src_ptr: int, dst_ptr: int, nbytes: int, device: torch.device,
               flag_ptr: Optional[int] = None, flag_value: int = 0, max_blocks: int = 592) -> None:
    """Vectorised copy (16-byte multiple) on ``device``'s current stream."""
    ws = workspace(device)
    counter = ws.counters[2:3].data_ptr() if flag_ptr is not None else None
    check(lib().kvs_copy16(src_ptr, dst_ptr, nbytes, counter, flag_ptr, flag_value, max_blocks,
                           _stream(device)), "copy16")


def _grid_per_seg(segs: Sequence[tuple[int, int, int]], floor: int) -> int:
    """CTAs per segment: enough for the largest segment to use the whole GPU
    (one CTA per 256 KB, up to 8 per SM), at least ``floor``."""
    big = max((int(s[2]) for s in segs), default=0)
    return int(max(floor, min(1184, big >> 18)))


def copy_segments(segments: Sequence[Sequence[int]], device: torch.device,
                  flag_ptr: Optional[int] = None, flag_value: int = 0,
                  blocks_per_seg: Optional[int] = None, ck: Optional[torch.Tensor] = None,
                  trailer_ptr: Optional[int] = None) -> None:
    """Copy several (src_ptr, dst_ptr, nbytes[, msg_off]) ranges in one launch
    on the current stream; destinations may be peer memory.  With ``ck``
    (int64[2] on the device, zeroed by the caller or added to by earlier
    kernels of the same message) the copy adds the message checksum of the
    bytes it writes at message offset ``msg_off``; with ``flag_ptr``, the
    last CTA stores the finished checksum to ``trailer_ptr`` (when both are
    given) and publishes ``flag_value`` (release, system scope) after every
    segment is written."""
    segs = [tuple(s) + (0,) * (4 - len(s)) for s in segments if s[2] > 0]
    if not segs:
        if flag_ptr is not None:
            set_flag(flag_ptr, flag_value, device)
        return
    host = torch.tensor([v for s in segs for v in s], dtype=torch.int64)
    if device.type == "cuda":
        host = host.pin_memory()
        _xfer["h2d"] += host.numel() * 8
    dev_segs = host.to(device, non_blocking=True)
    ws = workspace(device)
    counter = ws.counters[4:5].data_ptr() if flag_ptr is not None else None
    if blocks_per_seg is None:
        blocks_per_seg = _grid_per_seg(segs, 32)
    check(lib().kvs_copy_segments(dev_segs.data_ptr(), len(segs), blocks_per_seg, counter,
                                  flag_ptr, flag_value, _ptr(ck),
                                  trailer_ptr if ck is not None else None, _stream(device)),
          "copy_segments")
    # dev_segs may be freed now: the caching allocator only reuses its block
    # for work ordered after this launch on the same stream.


def zero_checksum(ck: torch.Tensor) -> None:
    """Zero the int64[2] checksum accumulators on the current stream."""
    check(lib().kvs_zero2(ck.data_ptr(), _stream(ck.device)), "zero2")


def _ck_segments(segments: Sequence[Sequence[int]], device: torch.device) -> torch.Tensor:
    rows = [tuple(s) + (0,) * (5 - len(s)) for s in segments] or [(0, 0, 0, 0, 0)]
    host = torch.tensor([v for s in rows for v in s], dtype=torch.int64)
    if device.type == "cuda":
        host = host.pin_memory()
        _xfer["h2d"] += host.numel() * 8
    return host.to(device, non_blocking=True)


def checksum(segments: Sequence[Sequence[int]], out: torch.Tensor,
             blocks_per_seg: Optional[int] = None) -> None:
    """Message checksum of (src_ptr, message_offset, nbytes[, len_ptr,
    len_add]) segments into ``out`` (int64[2] on the device): the plain and
    the position-weighted sums of the message's little-endian 32-bit words,
    mod 2^64.  A segment with ``len_ptr`` (device address of a uint64) is
    ``min(nbytes, *len_ptr + len_add)`` bytes long, read on the device."""
    segs = [s for s in segments if s[2] > 0]
    dev = out.device
    d = _ck_segments(segs, dev)
    if blocks_per_seg is None:
        blocks_per_seg = _grid_per_seg(segs, 16)
    check(lib().kvs_checksum(d.data_ptr(), len(segs), out.data_ptr(), blocks_per_seg,
                             _stream(dev)), "checksum")


def verify_checksum(segments: Sequence[Sequence[int]], expected_ptr: int,
                    device: torch.device, blocks_per_seg: Optional[int] = None) -> None:
    """Recompute the checksum of ``segments`` (as :func:`checksum`) on
    ``device`` and record ERR_CORRUPT in the device error word when it
    differs from the int64[2] at ``expected_ptr`` (device memory).  Nothing
    waits on the host."""
    segs = [s for s in segments if s[2] > 0]
    d = _ck_segments(segs, device)
    ws = workspace(device)
    scratch = torch.empty(2, dtype=torch.int64, device=device)  # stream-ordered reuse
    if blocks_per_seg is None:
        blocks_per_seg = _grid_per_seg(segs, 16)
    check(lib().kvs_checksum_verify(d.data_ptr(), len(segs), expected_ptr, scratch.data_ptr(),
                                    ws.err.data_ptr(), blocks_per_seg, _stream(device)),
          "checksum_verify")


def wait_flag(flag_ptr: int, expected: int, device: torch.device, timeout_s: float = 2.0,
              waited_ns: Optional[torch.Tensor] = None) -> None:
    """Launch a bounded device wait until *flag == expected (ERR_FLAG_TIMEOUT
    in the device error word when it expires)."""
    check(lib().kvs_wait_flag(flag_ptr, expected, int(timeout_s * 1e9),
                              workspace(device).err.data_ptr(), _ptr(waited_ns),
                              _stream(device)), "wait_flag")


def set_flag(flag_ptr: int, value: int, device: torch.device) -> None:
    check(lib().kvs_set_flag(flag_ptr, value, _stream(device)), "set_flag")


def probe_push(src: torch.Tensor, dst_ptr: int, nbytes: int, stamps: torch.Tensor,
               blocks: int = 296) -> None:
    """Timed push of ``nbytes`` from ``src`` to ``dst_ptr`` (peer memory);
    ``stamps`` (int64[2], reset by the caller to (max, 0)) receives the
    [first start, last end] globaltimer stamps in ns."""
    check(lib().kvs_probe_push(src.data_ptr(), dst_ptr, nbytes, stamps.data_ptr(), blocks,
                               _stream(src.device)), "probe_push")


# ----------------------------------------------------------------- metrics
def kv_error(ref: torch.Tensor, approx: torch.Tensor) -> dict:
    """rel-MSE, MSE, cosine and max |a-r| between two bf16 tensors of the
    same size, from one fused device reduction (one host read)."""
    if ref.numel() != approx.numel():
        raise ValueError("size mismatch")
    r = ref.contiguous().view(-1)
    a = approx.contiguous().view(-1)
    if r.device.type != "cuda":
        from kvserve_hpdps_b200.compression.oracle import error_metrics
        return error_metrics(r, a)
    acc = torch.zeros(4, dtype=torch.float64, device=r.device)
    mx = torch.zeros(1, dtype=torch.int32, device=r.device)
    check(lib().kvs_kv_error(r.data_ptr(), a.data_ptr(), r.numel(), acc.data_ptr(),
                             mx.data_ptr(), _stream(r.device)), "kv_error")
    sd, sr, sa, sx = acc.tolist()
    maxabs = float(mx.view(torch.float32).item())
    n = r.numel()
    return {"rel_mse": sd / max(sr, 1e-300), "mse": sd / max(n, 1),
            "cosine": sx / max(math.sqrt(sr * sa), 1e-300), "max_abs": maxabs}


def logit_agreement(ref_logits: torch.Tensor, approx_logits: torch.Tensor) -> dict:
    """Top-1 agreement and mean KL(ref || approx) of two [rows, vocab] fp32
    logit matrices (one device pass, one host read)."""
    r = ref_logits.float().contiguous()
    a = approx_logits.float().contiguous()
    rows, vocab = r.shape
    out = torch.empty((rows, 3), dtype=torch.float32, device=r.device)
    check(lib().kvs_logit_agreement(r.data_ptr(), a.data_ptr(), rows, vocab, out.data_ptr(),
                                    _stream(r.device)), "logit_agreement")
    o = out.cpu()
    agree = float((o[:, 0] == o[:, 1]).float().mean())
    return {"top1_agreement": agree, "kl_mean": float(o[:, 2].mean()), "rows": rows}
