"""Default-mode compression manager on the fused sm_100a kernels.

This is the default backend (reference: the TileLang manager,
kvserve_v1/compression/tilelang_manager.py).  It offers the same surface:

* whole-request: :meth:`compress_all_layers` / :meth:`decompress_all_layers`;
* per-layer overlap API: :meth:`compress_quant_layer`, :meth:`finalize_codec`,
  :meth:`compress_layer_full`, :meth:`finalize_chunked`,
  :meth:`finalize_layer_group`, :meth:`decompress_layer_group`;

and adds the paged fast path used by this framework's connector and
benchmark: :meth:`quantize_paged` reads every (layer, request) item straight
from the paged caches through block tables in one set of launches, and
:meth:`dequantize_paged` scatters into the consumer's paged caches.

Wire form (unchanged from the reference so envelopes interoperate):
codes are ``uint8 [L, 2, H, B, bs, D]`` heads-outer; each layer's
``quantization_params`` entry is ``{"key_meta": {"min_val": fp16[H, D],
"quant_scale": fp16[H, D], "axis": "channel"}, "value_meta":
{"per_group_list": [{"head_idx": int64[n], "min_val": fp16[rows, 1, 1],
"quant_scale": fp16[rows, 1, 1]}, ...]}}``.  The code buffer is then
entropy-coded by this framework's codec (``codec.py``); when the codec is
``bitpack`` the kernels write bit-packed codes directly and the per-segment
bit widths travel as ``code_bits``.
"""

from __future__ import annotations

import math
import os
import time
from dataclasses import dataclass
from typing import Any, Optional, Sequence

import torch

from kvserve_hpdps_b200.compression.codec import decode_bytes, encode_bytes, resolve_codec
from kvserve_hpdps_b200.compression.config import (DEFAULT_HADAMARD_SEED, FUSED_QUANTIZER_DEFAULTS,
                                                   CompressedKVData)
from kvserve_hpdps_b200.compression.head_scores import HybridPrecisionPlan
from kvserve_hpdps_b200.utils.logger import get_logger

from kvserve_hpdps_b200.utils.tracing import nvtx  # noqa: E402

logger = get_logger(__name__)

BACKEND = "kvs_fused"


def _engine_from_env() -> int:
    v = os.environ.get("KVSERVE_ENGINE", "tcgen05").lower()
    return {"simt": 1, "1": 1, "tile": 2, "2": 2, "persistent": 3, "3": 3}.get(v, 0)


@dataclass
class PagedBatch:
    """Result of :meth:`FusedCompressionManager.quantize_paged`."""
    codes: torch.Tensor          # uint8 code buffer (items in order)
    meta: torch.Tensor           # uint8 view of the fp16 metadata buffer
    items: Any                   # ops.kernels.WorkItems
    layer_ids: list[int]         # layer id of each slot
    plans: list[Any]             # LayerPlan of each slot

    def item_nbytes(self, r: int) -> int:
        plan = self.plans[self.items.items[r][0]]
        return self.items.n_rows[r] * plan.row_bytes() + plan.meta_bytes(self.items.n_rows[r])


class FusedCompressionManager:
    """Hadamard + hybrid quantization + codec on the fused kernels."""

    backend = BACKEND

    def __init__(self, num_kv_heads: int, head_size: int, quantizer_config: Optional[dict],
                 codec_config: Optional[dict], base_seed: int = DEFAULT_HADAMARD_SEED,
                 tp_rank: int = 0, tp_size: int = 1, transform: bool = True,
                 engine: Optional[int] = None, num_layers: Optional[int] = None):
        if head_size != 128:
            raise ValueError(f"the fused path needs head_size 128, got {head_size}")
        qc = dict(FUSED_QUANTIZER_DEFAULTS)
        qc.update(quantizer_config or {})
        self.quantizer_config = qc
        self.codec_config = dict(codec_config or {})
        self.codec = resolve_codec(self.codec_config.get("codec_type", "nvcomp"),
                                   self.codec_config.get("nvcomp_algorithm", "ANS"))
        self.packed = self.codec == "bitpack"
        self.stream_codec = self.codec if self.codec in ("rans", "lc") else "none"
        # With the entropy coder, codes are stored as 4-bit nibbles (two codes
        # per coded byte): half the symbols for the coder at the same
        # compression ratio.  codec_config["symbol_bits"] = 8 keeps byte codes.
        self.code_width = 4 if (self.stream_codec == "rans" and
                                int(self.codec_config.get("symbol_bits", 4)) == 4) else None
        self.num_kv_heads = int(num_kv_heads)
        self.head_size = int(head_size)
        self.base_seed = int(base_seed) if transform else None
        self.tp_rank, self.tp_size = int(tp_rank), int(tp_size)
        self.engine = _engine_from_env() if engine is None else int(engine)
        self.hybrid = HybridPrecisionPlan(
            num_layers, self.num_kv_heads, qc.get("model_name"), qc["hybrid_ratio"],
            qc["high_key_max_value"], qc["high_value_max_value"], qc["low_key_max_value"],
            qc["low_value_max_value"], qc.get("split_type", "head"), self.tp_rank, self.tp_size)
        self._plans: dict[int, Any] = {}
        self._slot_cache: dict[tuple, Any] = {}
        self._last_decompress_timing: Optional[dict] = None
        logger.info("fused manager: heads=%d codec=%s packed=%s engine=%d seed=%s",
                    self.num_kv_heads, self.codec, self.packed, self.engine, self.base_seed)

    # ----------------------------------------------------------- plans
    def plan(self, layer_id: int):
        from kvserve_hpdps_b200.ops import kernels as K
        layer_id = int(layer_id)
        if layer_id not in self._plans:
            self._plans[layer_id] = K.make_layer_plan(
                self.num_kv_heads, self.hybrid.key_levels_for(layer_id).tolist(),
                self.hybrid.value_levels_for(layer_id).tolist(), self.base_seed, layer_id,
                packed=self.packed, code_width=self.code_width)
        return self._plans[layer_id]

    def _slots(self, tensors: Sequence[torch.Tensor], plans: Sequence[Any]):
        from kvserve_hpdps_b200.ops import kernels as K
        key = tuple((t.data_ptr(), tuple(t.shape), tuple(t.stride())) for t in tensors) + \
            tuple(id(p) for p in plans)
        sl = self._slot_cache.get(key)
        if sl is None:
            if len(self._slot_cache) > 64:
                self._slot_cache.clear()
            sl = K.LayerSlots(list(tensors), list(plans))
            self._slot_cache[key] = sl
        return sl

    def supports_overlap(self) -> bool:
        return True

    # --------------------------------------------------- paged fast path
    def quantize_paged(self, kv_layers: Sequence[torch.Tensor], layer_ids: Sequence[int],
                       requests: Sequence[tuple[Sequence[int], int]],
                       codes: Optional[torch.Tensor] = None,
                       meta: Optional[torch.Tensor] = None) -> PagedBatch:
        """Quantize every (layer, request) item: ``kv_layers[i]`` is the paged
        cache of layer ``layer_ids[i]``; ``requests`` are (block ids, valid
        tokens).  Items are ordered layer-major, so for one request the code
        buffer is the reference's ``[L, 2, H, B, bs, D]`` layout."""
        from kvserve_hpdps_b200.ops import kernels as K
        plans = [self.plan(l) for l in layer_ids]
        slots = self._slots(kv_layers, plans)
        items = K.WorkItems(slots, [(i, b, n) for i in range(len(kv_layers)) for b, n in requests])
        codes, meta = K.quantize(slots, items, codes, meta, engine=self.engine)
        return PagedBatch(codes, meta, items, list(layer_ids), plans)

    def dequantize_paged(self, batch: PagedBatch, dst_layers: Sequence[torch.Tensor],
                         dst_requests: Optional[Sequence[tuple[Sequence[int], int]]] = None,
                         codes: Optional[torch.Tensor] = None,
                         meta: Optional[torch.Tensor] = None) -> None:
        """Dequantize ``batch`` into the destination paged caches (one per
        layer of the batch) at ``dst_requests`` block ids (default: the
        producer's)."""
        from kvserve_hpdps_b200.ops import kernels as K
        slots = self._slots(dst_layers, batch.plans)
        if dst_requests is None:
            items = K.WorkItems(slots, batch.items.items)
        else:
            items = K.WorkItems(slots, [(i, b, n) for i in range(len(dst_layers))
                                        for b, n in dst_requests])
        K.dequantize(batch.codes if codes is None else codes,
                     batch.meta if meta is None else meta, slots, items, engine=self.engine)

    def compress_paged_requests(self, kv_layers: Sequence[torch.Tensor], layer_ids: Sequence[int],
                                requests: Sequence[tuple[Sequence[int], int]],
                                member_tids: Optional[Sequence[str]] = None,
                                trim: bool = True, deferred: bool = False,
                                extra_meta: Optional[dict] = None) -> CompressedKVData:
        """Compress the given layers of several requests into ONE message:
        one codec stream over every (layer, request) item, layer-major.

        Metadata: ``grouped=True, layout="items_packed"``, ``member_tids``,
        ``member_tokens``, ``member_blocks``, ``layer_ids``, ``layer_plans``
        (per layer: value group of each head and code bits, plain ints) and
        ``quantization_params = [meta]``: the fp16 metadata of every item in
        the kernels' device layout as ONE aux tensor (item offsets follow from
        the plans and block counts).  Decoders also accept the per-item
        ``layout="items"`` form.

        ``trim=False`` returns the codec's worst-case stream buffer instead of
        reading the stream size back (which synchronises the host with the
        device); the stream records its own length and the decoder takes the
        code byte count from the metadata.  ``deferred=True`` (entropy coder
        only) returns the codes themselves with ``deferred_codec`` set in the
        metadata: a transport encodes them on its way out and sends only the
        stream's bytes (the NCCL transport on its send thread), and a
        consumer that receives them unencoded decodes them as plain codes.
        Without an entropy coder the body is always the code buffer itself
        (``container=False``: no header, no copy)."""
        with nvtx("kvs.quantize"):
            batch = self.quantize_paged(kv_layers, layer_ids, requests)
        codes = batch.codes[:batch.items.code_bytes]
        container = True
        with nvtx("kvs.encode"):
            if self.stream_codec == "none":
                body, container = codes, False
            elif deferred and self.stream_codec == "rans":
                body, container = codes, False
            elif trim:
                body = encode_bytes(codes, self.stream_codec)
            else:
                body = self._encode_untrimmed(codes)
        items = batch.items
        H = self.num_kv_heads
        meta = {"grouped": True, "layout": "items_packed", "layer_ids": [int(l) for l in layer_ids],
                "member_tids": list(member_tids) if member_tids else
                [str(i) for i in range(len(requests))],
                "member_tokens": [int(n) for _, n in requests],
                "member_blocks": [len(b) for b, _ in requests],
                "block_size": int(kv_layers[0].shape[2]), "num_heads": H,
                "device": str(batch.codes.device),
                "layer_plans": [{"group_of_head": list(p.group_of_head),
                                 "code_bits": list(p.key_bits) + list(p.value_bits)}
                                for p in batch.plans],
                "meta_bytes": int(items.meta_bytes),
                "quantization_params": [batch.meta[:max(items.meta_bytes, 16)]],
                "code_bytes": int(items.code_bytes), "backend": BACKEND, "codec": self.codec,
                "stream_codec": self.stream_codec, "transform_seed": self.base_seed}
        if not container:
            meta["container"] = False
            if self.stream_codec != "none":
                meta["deferred_codec"] = self.stream_codec
        meta.update(extra_meta or {})
        orig = sum(len(kv_layers) * 2 * n * H * self.head_size * 2 for _, n in requests)
        self._last_batch = batch
        return CompressedKVData(request_id="grp", layer_id=int(layer_ids[-1]),
                                compressed_tensor=body, metadata=meta, original_size=orig,
                                compressed_size=int(body.numel()))

    def send_paged_requests(self, transport, request_id: str, layer_names: Sequence[str],
                            kv_layers: Sequence[torch.Tensor], layer_ids: Sequence[int],
                            requests: Sequence[tuple[Sequence[int], int]],
                            member_tids: Optional[Sequence[str]] = None,
                            extra_meta: Optional[dict] = None) -> dict:
        """Compress the requests and hand them to ``transport`` as ONE
        message, written by the producer kernels straight into the
        consumer's receive ring when the transport offers it (NVLink ring
        transport: ``open_message``), else through ``send_bundle``.

        Direct path, on the current stream, no host synchronisation:
        statistics and quantization read the paged caches; without an
        entropy coder the quantize kernel stores the codes into the ring over
        NVLink and sums their message checksum on the way; with rANS the
        codes stay local and the encoder's compaction kernel stores only the
        coded stream (its worst case is reserved, only its own bytes cross
        the link); a final copy brings the fp16 metadata and its last CTA
        stores the checksum and publishes the ready flag.

        ``extra_meta`` joins the message's metadata (controller mode: the
        profile the consumer decodes with).  Returns ``{"original_size",
        "wire_nbytes", "direct"}`` where ``wire_nbytes`` is the reserved
        (upper-bound) size on the direct path; the exact size reaches the
        transport's sent listeners."""
        from kvserve_hpdps_b200.compression.wire import build_wire
        from kvserve_hpdps_b200.ops import kernels as K
        direct = (hasattr(transport, "open_message") and self.engine == 0
                  and self.stream_codec in ("none", "rans") and kv_layers[0].is_cuda)
        if not direct:
            cd = self.compress_paged_requests(kv_layers, layer_ids, requests, member_tids,
                                              trim=False, deferred=True, extra_meta=extra_meta)
            wire = build_wire(cd)
            transport.send_bundle(request_id, list(layer_names), wire.meta, wire.body_chunks,
                                  wire.aux_tensors, member_tids=list(member_tids or []) or None)
            return {"original_size": cd.original_size, "wire_nbytes": wire.nbytes,
                    "direct": False}
        plans = [self.plan(l) for l in layer_ids]
        slots = self._slots(kv_layers, plans)
        items = K.WorkItems(slots, [(i, b, n) for i in range(len(kv_layers)) for b, n in requests])
        code_bytes, meta_bytes = max(items.code_bytes, 16), max(items.meta_bytes, 16)
        body_cap = 16 + K.rans_max_bytes(code_bytes) if self.stream_codec == "rans" else code_bytes
        try:
            msg = transport.open_message([body_cap, meta_bytes])
        except RuntimeError as e:
            transport.record_unsent(request_id, list(member_tids or []) or None, e)
            return {"original_size": 0, "wire_nbytes": 0, "direct": True}
        try:
            return self._send_direct(transport, msg, request_id, layer_names, kv_layers,
                                     layer_ids, requests, member_tids, plans, slots, items,
                                     code_bytes, meta_bytes, body_cap, extra_meta)
        except Exception as e:
            # nothing committed: the space comes back once queued work is done
            transport.abort_message(msg, request_id, list(member_tids or []) or None, e)
            raise

    def _send_direct(self, transport, msg, request_id, layer_names, kv_layers, layer_ids,
                     requests, member_tids, plans, slots, items, code_bytes, meta_bytes,
                     body_cap, extra_meta: Optional[dict] = None) -> dict:
        """Kernels and header of :meth:`send_paged_requests`' direct path."""
        from kvserve_hpdps_b200.compression.codec import CODEC_IDS, MAGIC
        from kvserve_hpdps_b200.compression.wire import build_wire
        from kvserve_hpdps_b200.ops import kernels as K
        dev = kv_layers[0].device
        rans = self.stream_codec == "rans"
        meta_local = torch.empty(meta_bytes, dtype=torch.uint8, device=dev)
        total = None
        with nvtx("kvs.quantize_to_ring"):
            if rans:
                codes = torch.empty(code_bytes, dtype=torch.uint8, device=dev)
                K.quantize(slots, items, codes, meta_local, engine=self.engine)
            else:  # codes straight into the peer ring, checksummed as they are stored
                K.quantize(slots, items, transport.view(msg, 0), meta_local, engine=self.engine,
                           ck=msg.ck, ck_off=0)
        with nvtx("kvs.encode_to_ring"):
            if rans:
                K.copy_segments([(meta_local.data_ptr(), msg.ptrs[1], meta_bytes, msg.offsets[1])],
                                dev, ck=msg.ck)
                total = torch.empty(1, dtype=torch.int64, device=dev)
                K.rans_encode_message(codes.data_ptr(), code_bytes, msg.ptrs[0] + 16, dev,
                                      total=total,
                                      prefix=[MAGIC, CODEC_IDS["rans"], code_bytes & 0xFFFFFFFF,
                                              code_bytes >> 32],
                                      msg_off=16, ck=msg.ck, trailer_ptr=msg.trailer_ptr,
                                      flag_ptr=msg.flag_ptr, flag_value=msg.flag_value)
            else:
                K.copy_segments([(meta_local.data_ptr(), msg.ptrs[1], meta_bytes, msg.offsets[1])],
                                dev, flag_ptr=msg.flag_ptr, flag_value=msg.flag_value,
                                ck=msg.ck, trailer_ptr=msg.trailer_ptr)
        H = self.num_kv_heads
        body_view = transport.view(msg, 0)
        meta_view = transport.view(msg, 1)
        info = {"grouped": True, "layout": "items_packed", "layer_ids": [int(l) for l in layer_ids],
                "member_tids": list(member_tids) if member_tids else
                [str(i) for i in range(len(requests))],
                "member_tokens": [int(n) for _, n in requests],
                "member_blocks": [len(b) for b, _ in requests],
                "block_size": int(kv_layers[0].shape[2]), "num_heads": H, "device": str(dev),
                "layer_plans": [{"group_of_head": list(p.group_of_head),
                                 "code_bits": list(p.key_bits) + list(p.value_bits)}
                                for p in plans],
                "meta_bytes": int(items.meta_bytes), "quantization_params": [meta_view],
                "code_bytes": int(items.code_bytes), "backend": BACKEND, "codec": self.codec,
                "stream_codec": self.stream_codec, "transform_seed": self.base_seed}
        if not rans:
            info["container"] = False
        info.update(extra_meta or {})
        orig = sum(len(kv_layers) * 2 * n * H * self.head_size * 2 for _, n in requests)
        cd = CompressedKVData(request_id="grp", layer_id=int(layer_ids[-1]),
                              compressed_tensor=body_view, metadata=info, original_size=orig,
                              compressed_size=int(body_cap))
        wire = build_wire(cd, max_chunk_bytes=1 << 62)
        specs = [{"shape": [body_cap], "dtype": "uint8"}, {"shape": [meta_bytes], "dtype": "uint8"}]
        # the stream's length sits at byte 24 of its header, 16 bytes into the body
        dyn = {"seg": 0, "len_off": 16 + 24, "len_add": 16} if rans else None
        sent = (total, 16 + meta_bytes) if rans else None
        transport.commit_message(msg, request_id, list(layer_names), wire.meta, specs, 1,
                                 member_tids=list(member_tids or []) or None, dyn_len=dyn,
                                 sent_bytes=sent)
        return {"original_size": orig, "wire_nbytes": body_cap + meta_bytes, "direct": True}

    def _message_plans(self, meta: dict) -> list:
        """Consumer-side plans of a grouped message, one per layer."""
        from kvserve_hpdps_b200.ops import kernels as K
        seed = meta.get("transform_seed", self.base_seed)
        layer_ids = meta["layer_ids"]
        if meta.get("layout") == "items_packed":
            cache = self.__dict__.setdefault("_decode_plans", {})
            out = []
            for lid, lp in zip(layer_ids, meta["layer_plans"]):
                goh, bits = tuple(lp["group_of_head"]), tuple(lp["code_bits"])
                H = len(goh)
                key = (H, goh, bits, seed, int(lid))
                if key not in cache:
                    cache[key] = K.decode_plan(H, list(goh), list(bits[:H]), list(bits[H:]),
                                               seed, int(lid))
                out.append(cache[key])
            return out
        R = len(meta["member_tids"])
        qp = meta["quantization_params"]
        return [self.plan_from_canon(qp[i * R], layer_ids[i], seed) for i in range(len(layer_ids))]

    @staticmethod
    def _message_offsets(meta: dict, plans: Sequence[Any]) -> tuple[list[int], list[int]]:
        """Code and metadata offsets of every (layer, member) item of the
        producer's message (layer-major; same rule as the kernels' layout)."""
        bs = int(meta["block_size"])
        co, mo, c, m = [], [], 0, 0
        for plan in plans:
            for nb in meta["member_blocks"]:
                rows = nb * bs
                co.append(c)
                mo.append(m)
                c += (rows * plan.row_bytes() + 15) & ~15
                m += (plan.meta_bytes(rows) + 15) & ~15
        return co, mo

    def _encode_untrimmed(self, codes: torch.Tensor) -> torch.Tensor:
        """Container header + the worst-case stream buffer (no host read of the
        stream size); the stream records its own length."""
        from kvserve_hpdps_b200.compression.codec import _header
        from kvserve_hpdps_b200.ops import kernels as K
        if self.stream_codec == "lc" and codes.is_cuda:
            return torch.cat([_header("lc", codes.numel(), codes.device),
                              K.lc_encode(codes, trim=False)])
        if self.stream_codec != "rans":
            return encode_bytes(codes, self.stream_codec)
        hdr = _header("rans", codes.numel(), codes.device)
        out = torch.empty(16 + K.rans_max_bytes(codes.numel()), dtype=torch.uint8,
                          device=codes.device)
        out[:16] = hdr
        K.rans_encode(codes, out=out[16:], trim=False)
        return out

    @staticmethod
    def _decode_body(body: torch.Tensor, meta: dict, device) -> torch.Tensor:
        """Codes of a message body.  The codec and the code byte count come
        from the message metadata, so nothing is read back to the host (the
        body may be an untrimmed stream buffer); other bodies go through the
        self-describing container."""
        from kvserve_hpdps_b200.ops import kernels as K
        sc, n = meta.get("stream_codec"), meta.get("code_bytes")
        if meta.get("container") is False:  # the codes themselves (no codec or not yet encoded)
            data = body.view(torch.uint8).reshape(-1)
            if data.device != torch.device(device):
                data = data.to(device)
            return data[:int(n)]
        if sc is None or n is None or body.device.type != "cuda":
            return decode_bytes(body, device)
        if body.device != torch.device(device):
            body = body.to(device)
        data = body.view(torch.uint8).reshape(-1)[16:]
        if sc == "rans":
            return K.rans_decode(data, int(n))
        if sc == "lc":
            return K.lc_decode(data, int(n))
        return data[:int(n)]

    def decompress_paged_requests(self, compressed: CompressedKVData,
                                  dst_layers: Sequence[torch.Tensor],
                                  dst_requests: Sequence[tuple[Sequence[int], int]]) -> None:
        """Inverse of :meth:`compress_paged_requests` into the consumer's
        paged caches (``dst_layers[i]`` for the message's i-th layer) at the
        consumer's block ids."""
        from kvserve_hpdps_b200.ops import kernels as K
        meta = compressed.metadata
        device = dst_layers[0].device
        codes = self._decode_body(compressed.compressed_tensor, meta, device)
        plans = self._message_plans(meta)
        slots = self._slots(dst_layers, plans)
        items = K.WorkItems(slots, [(i, b, n) for i in range(len(dst_layers)) for b, n in dst_requests])
        if meta.get("layout") == "items_packed":
            if items.meta_bytes != int(meta["meta_bytes"]):
                raise ValueError("consumer block counts do not match the message's")
            meta_buf = meta["quantization_params"][0]
            if meta_buf.device != device:
                meta_buf = meta_buf.to(device)
        else:
            qp = meta["quantization_params"]
            meta_buf = torch.zeros(max(items.meta_bytes, 16), dtype=torch.uint8, device=device)
            for r in range(items.num_items):
                m = self.meta_from_canon(qp[r])
                meta_buf[items.meta_off[r]:items.meta_off[r] + m.numel()] = m.to(device)
        K.dequantize(codes, meta_buf, slots, items, engine=self.engine)

    def decompress_members(self, compressed: CompressedKVData, dst_layers: Sequence[torch.Tensor],
                           member_blocks: dict[int, Sequence[int]]) -> None:
        """Decode a multi-request message once (cached) and dequantize only
        the members in ``member_blocks`` (member index -> consumer block ids)
        into ``dst_layers`` (one per layer of the message)."""
        from kvserve_hpdps_b200.ops import kernels as K
        meta = compressed.metadata
        device = dst_layers[0].device
        key = id(compressed.compressed_tensor)
        cache = self.__dict__.setdefault("_decoded", {})
        if key not in cache:
            if len(cache) > 8:
                cache.pop(next(iter(cache)))
            cache[key] = self._decode_body(compressed.compressed_tensor, meta, device)
        codes = cache[key]
        layer_ids = meta["layer_ids"]
        R = len(meta["member_tids"])
        plans = self._message_plans(meta)
        code_offs, meta_offs = self._message_offsets(meta, plans)
        slots = self._slots(dst_layers, plans)
        sel = [(l, r) for l in range(len(layer_ids)) for r in sorted(member_blocks)]
        packed = meta.get("layout") == "items_packed"
        items = K.WorkItems(slots, [(l, member_blocks[r], meta["member_tokens"][r]) for l, r in sel],
                            code_offsets=[code_offs[l * R + r] for l, r in sel],
                            meta_offsets=[meta_offs[l * R + r] for l, r in sel] if packed else None)
        if packed:
            meta_buf = meta["quantization_params"][0]
            if meta_buf.device != device:
                meta_buf = meta_buf.to(device)
        else:
            qp = meta["quantization_params"]
            meta_buf = torch.zeros(max(items.meta_bytes, 16), dtype=torch.uint8, device=device)
            for i, (l, r) in enumerate(sel):
                m = self.meta_from_canon(qp[l * R + r])
                meta_buf[items.meta_off[i]:items.meta_off[i] + m.numel()] = m.to(device)
        K.dequantize(codes, meta_buf, slots, items, engine=self.engine)

    # ------------------------------------------------------ canon metadata
    def canon_meta(self, meta: torch.Tensor, off: int, plan, rows: int) -> dict:
        """Wire-form metadata of one item (views into ``meta``)."""
        H, G = plan.num_heads, plan.n_groups
        f = meta[off:off + plan.meta_bytes(rows)].view(torch.float16)
        kmin = f[:H * 128].view(H, 128)
        ksc = f[H * 128:2 * H * 128].view(H, 128)
        vmin = f[2 * H * 128:2 * H * 128 + G * rows].view(G, rows)
        vsc = f[2 * H * 128 + G * rows:2 * H * 128 + 2 * G * rows].view(G, rows)
        groups = [{"head_idx": torch.tensor(plan.groups[g], dtype=torch.int64, device=meta.device),
                   "min_val": vmin[g].view(rows, 1, 1), "quant_scale": vsc[g].view(rows, 1, 1)}
                  for g in range(G)]
        out = {"key_meta": {"min_val": kmin, "quant_scale": ksc, "axis": "channel"},
               "value_meta": {"per_group_list": groups}}
        if plan.packed:
            out["code_bits"] = list(plan.key_bits) + list(plan.value_bits)
        return out

    def plan_from_canon(self, canon: dict, layer_id: int, seed: Optional[int]):
        """Consumer-side plan rebuilt from one item's wire metadata."""
        from kvserve_hpdps_b200.ops import kernels as K
        H = int(canon["key_meta"]["min_val"].shape[0])
        goh = [0] * H
        for g, grp in enumerate(canon["value_meta"]["per_group_list"]):
            for h in grp["head_idx"].tolist():
                goh[int(h)] = g
        bits = list(canon.get("code_bits") or [8] * (2 * H))
        key = (H, tuple(goh), tuple(bits), seed, int(layer_id))
        cache = self.__dict__.setdefault("_decode_plans", {})
        if key not in cache:
            cache[key] = K.decode_plan(H, goh, bits[:H], bits[H:], seed, layer_id)
        return cache[key]

    @staticmethod
    def meta_from_canon(canon: dict) -> torch.Tensor:
        """Device-layout fp16 metadata (uint8 view) of one item."""
        km = canon["key_meta"]
        parts = [km["min_val"].reshape(-1), km["quant_scale"].reshape(-1)]
        groups = canon["value_meta"]["per_group_list"]
        parts += [g["min_val"].reshape(-1) for g in groups]
        parts += [g["quant_scale"].reshape(-1) for g in groups]
        return torch.cat([p.to(torch.float16) for p in parts]).view(torch.uint8)

    # ------------------------------------------------------- whole request
    def compress_all_layers(self, all_layers_data: torch.Tensor, request_id: str,
                            config: Any = None, metadata: Optional[dict] = None
                            ) -> Optional[CompressedKVData]:
        """Compress a dense ``[L, 2, B, bs, H, D]`` request."""
        if not isinstance(all_layers_data, torch.Tensor) or all_layers_data.dim() != 6:
            logger.error("expected a 6-D tensor, got %s", getattr(all_layers_data, "shape", None))
            return None
        x = all_layers_data.contiguous()
        L, _, B, bs, H, D = x.shape
        t0 = time.monotonic()
        batch = self.quantize_paged([x[l] for l in range(L)], list(range(L)),
                                    [(list(range(B)), B * bs)])
        body = encode_bytes(batch.codes[:batch.items.code_bytes], self.stream_codec)
        if body.is_cuda:
            torch.cuda.synchronize(body.device)
        t_ms = (time.monotonic() - t0) * 1e3
        qparams = [self.canon_meta(batch.meta, batch.items.meta_off[l], batch.plans[l],
                                   batch.items.n_rows[l]) for l in range(L)]
        meta = {
            "request_id": request_id, "num_layers": L, "codec_applied": True,
            "codec_shape": [L, 2, H, B, bs, D], "codec_dtype": "uint8",
            "device": str(x.device), "original_dtype": str(x.dtype).replace("torch.", ""),
            "original_shape": list(x.shape), "quantization_params": qparams,
            "backend": BACKEND, "codec": self.codec, "transform_seed": self.base_seed,
            "t_quant_ms": t_ms, "t_codec_ms": 0.0,
        }
        meta.update(metadata or {})
        return CompressedKVData(request_id=request_id, layer_id=L - 1, compressed_tensor=body,
                                metadata=meta, original_size=x.numel() * x.element_size(),
                                compressed_size=body.numel())

    def decompress_all_layers(self, compressed: CompressedKVData, config: Any = None
                              ) -> Optional[torch.Tensor]:
        if compressed.is_chunked:
            return self._decompress_chunked(compressed)
        meta = compressed.metadata
        L = int(meta["num_layers"])
        _, _, H, B, bs, D = [int(s) for s in meta["codec_shape"]]
        device = torch.device(meta.get("device", "cuda"))
        t0 = time.monotonic()
        codes = decode_bytes(compressed.compressed_tensor, device)
        t_codec = (time.monotonic() - t0) * 1e3
        out = torch.empty((L, 2, B, bs, H, D), dtype=torch.bfloat16, device=device)
        self._dequant_dense(codes, meta["quantization_params"], list(range(L)), out,
                            meta.get("transform_seed", self.base_seed))
        if out.is_cuda:
            torch.cuda.synchronize(device)
        self._last_decompress_timing = {"t_codec_decode_ms": t_codec,
                                        "t_dequant_ms": (time.monotonic() - t0) * 1e3 - t_codec}
        return out

    def _dequant_dense(self, codes: torch.Tensor, qparams: Sequence[dict],
                       layer_ids: Sequence[int], out: torch.Tensor, seed) -> None:
        """Dequantize per-layer items of one request into dense ``out``
        ``[L, 2, B, bs, H, D]`` (codes concatenated layer-major)."""
        from kvserve_hpdps_b200.ops import kernels as K
        L, _, B, bs = out.shape[:4]
        plans = [self.plan_from_canon(qparams[i], layer_ids[i], seed) for i in range(L)]
        metas = [self.meta_from_canon(q) for q in qparams]
        slots = K.LayerSlots([out[i] for i in range(L)], plans)
        items = K.WorkItems(slots, [(i, list(range(B)), B * bs) for i in range(L)])
        meta_buf = torch.zeros(max(items.meta_bytes, 16), dtype=torch.uint8, device=out.device)
        for i, m in enumerate(metas):
            meta_buf[items.meta_off[i]:items.meta_off[i] + m.numel()] = m.to(out.device)
        codes = codes.to(out.device)
        if codes.numel() < items.code_bytes:
            raise ValueError("code buffer shorter than the layout requires")
        K.dequantize(codes, meta_buf, slots, items, engine=self.engine)

    # ----------------------------------------------- per-layer overlap API
    def compress_quant_layer(self, kv_layer: torch.Tensor, layer_id: int):
        """Quantize one dense layer ``[2, B, bs, H, D]``; returns
        (codes ``[2, H, B, bs, 16*bits]`` bytes when every segment has the same
        code width, else flat bytes; canon meta)."""
        x = kv_layer.contiguous()
        _, B, bs, H, D = x.shape
        batch = self.quantize_paged([x], [layer_id], [(list(range(B)), B * bs)])
        codes = batch.codes[:batch.items.code_bytes]
        widths = set(batch.plans[0].key_bits + batch.plans[0].value_bits)
        if len(widths) == 1:  # one code width: [2, H, B, bs, 16 * width] bytes
            codes = codes.view(2, H, B, bs, 16 * widths.pop())
        canon = self.canon_meta(batch.meta, 0, batch.plans[0], B * bs)
        return codes, canon

    def finalize_codec(self, q_perm_layers, canon_metas, request_id, original_dtype,
                       original_shape) -> CompressedKVData:
        buf = torch.cat([q.reshape(-1) for q in q_perm_layers])
        body = encode_bytes(buf, self.stream_codec)
        L = len(q_perm_layers)
        _, _, B, bs, H, D = [int(s) for s in original_shape]
        meta = {"request_id": request_id, "num_layers": L, "codec_applied": True,
                "codec_shape": [L, 2, H, B, bs, D], "codec_dtype": "uint8",
                "device": str(buf.device), "original_dtype": original_dtype,
                "original_shape": list(original_shape), "quantization_params": list(canon_metas),
                "backend": BACKEND, "codec": self.codec, "transform_seed": self.base_seed}
        return CompressedKVData(request_id=request_id, layer_id=L - 1, compressed_tensor=body,
                                metadata=meta, original_size=int(math.prod(original_shape)) * 2,
                                compressed_size=body.numel())

    def finalize_layer_group(self, q_perms, cmetas, member_tids, member_blocks,
                             layer_id) -> CompressedKVData:
        """One codec call over the independently quantized requests of a
        layer (lossless merge; each member keeps its own scales)."""
        buf = torch.cat([q.reshape(-1) for q in q_perms])
        body = encode_bytes(buf, self.stream_codec)
        H = self.num_kv_heads
        bs = int(q_perms[0].shape[3]) if q_perms[0].dim() == 5 else None
        meta = {"grouped": True, "num_members": len(q_perms), "member_tids": list(member_tids),
                "member_blocks": [int(b) for b in member_blocks],
                "member_bytes": [int(q.numel()) for q in q_perms],
                "block_size": bs, "num_heads": H, "codec_dtype": "uint8",
                "device": str(buf.device), "layer_id": int(layer_id),
                "quantization_params": list(cmetas), "backend": BACKEND, "codec": self.codec,
                "transform_seed": self.base_seed}
        return CompressedKVData(request_id="grp", layer_id=int(layer_id), compressed_tensor=body,
                                metadata=meta, original_size=sum(int(b) for b in member_blocks),
                                compressed_size=body.numel())

    def decompress_layer_group(self, compressed: CompressedKVData):
        """Decode a grouped layer once and dequantize each member; returns
        [(transfer_id, kv [2, blocks, bs, H, D])]."""
        meta = compressed.metadata
        device = torch.device(meta.get("device", "cuda"))
        codes = decode_bytes(compressed.compressed_tensor, device)
        layer_id = int(meta["layer_id"])
        bs = int(meta["block_size"])
        H = int(meta["num_heads"])
        out, off = [], 0
        for i, (tid, nb) in enumerate(zip(meta["member_tids"], meta["member_blocks"])):
            n = int(meta["member_bytes"][i])
            dense = torch.empty((1, 2, nb, bs, H, self.head_size), dtype=torch.bfloat16,
                                device=device)
            self._dequant_dense(codes[off:off + n], [meta["quantization_params"][i]], [layer_id],
                                dense, meta.get("transform_seed", self.base_seed))
            off += n
            out.append((tid, dense[0]))
        return out

    def compress_layer_full(self, kv_layer: torch.Tensor, layer_id: int):
        """One layer through quantization and codec; returns (bytes, chunk meta)."""
        codes, canon = self.compress_quant_layer(kv_layer, layer_id)
        body = encode_bytes(codes, self.stream_codec)
        _, B, bs, H, D = kv_layer.shape
        chunk_meta = {"codec_applied": True, "codec_shape": [2, H, B, bs, D],
                      "codec_dtype": "uint8", "quantization_params": [canon],
                      "layer_id": int(layer_id)}
        return body, chunk_meta

    def finalize_chunked(self, chunks, chunk_metas, request_id, original_dtype, original_shape):
        return CompressedKVData(
            request_id=request_id, layer_id=len(chunks) - 1, compressed_tensor=None,
            metadata={"request_id": request_id, "num_layers": len(chunks),
                      "device": str(chunks[0].device), "original_dtype": original_dtype,
                      "original_shape": list(original_shape), "backend": BACKEND,
                      "codec": self.codec, "transform_seed": self.base_seed},
            original_size=int(math.prod(original_shape)) * 2,
            compressed_size=sum(int(c.numel()) for c in chunks), is_chunked=True,
            chunks=list(chunks), chunk_metadata=list(chunk_metas))

    def _decompress_chunked(self, compressed: CompressedKVData) -> torch.Tensor:
        meta = compressed.metadata
        device = torch.device(meta.get("device", "cuda"))
        seed = meta.get("transform_seed", self.base_seed)
        outs = []
        t0 = time.monotonic()
        for chunk, cm in zip(compressed.chunks, compressed.chunk_metadata):
            _, H, B, bs, D = [int(s) for s in cm["codec_shape"]]
            codes = decode_bytes(chunk, device)
            dense = torch.empty((1, 2, B, bs, H, D), dtype=torch.bfloat16, device=device)
            self._dequant_dense(codes, cm["quantization_params"], [int(cm.get("layer_id", 0))],
                                dense, seed)
            outs.append(dense[0])
        result = torch.stack(outs, 0)
        if result.is_cuda:
            torch.cuda.synchronize(device)
        self._last_decompress_timing = {"t_codec_decode_ms": 0.0,
                                        "t_dequant_ms": (time.monotonic() - t0) * 1e3}
        return result

    def warmup(self, block_size: int = 16) -> None:
        """Run every kernel once on a dummy layer so lazy initialisation
        (module load, tensor-map encoder lookup) is off the request path."""
        if not torch.cuda.is_available():
            return
        try:
            dummy = torch.randn(2, 1, block_size, self.num_kv_heads, self.head_size,
                                dtype=torch.bfloat16, device="cuda")
            cd = self.compress_all_layers(dummy.unsqueeze(0), "warmup")
            self.decompress_all_layers(cd)
            torch.cuda.synchronize()
        except Exception as e:  # noqa: BLE001
            logger.warning("fused warmup failed: %s", e)
