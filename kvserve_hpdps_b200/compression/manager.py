"""KVCompressionAdapter: the connector-facing compression API and mode switch.

Modes (``kv_connector_extra_config["compression"]``, reference
kvserve_v1/compression/manager.py:54-389):

* ``"default"``: fused sm_100a path with ``DEFAULT_COMPRESSION_CONFIG``; the
  quantizer's ``model_name`` is replaced by the served model's name so the
  matching head-score table is used;
* custom dict: fused path when the quantizer uses channel keys and token
  values (``backend: "generic"`` forces the PyTorch pipeline), otherwise the
  generic Transform -> Quantizer -> Codec pipeline;
* controller dict: per request, the online controller picks a profile from
  the profile library given the request size, the measured link bandwidth,
  the model time, the SLO and the accuracy requirement; ``None`` means "send
  raw".  The chosen profile's config travels in the metadata
  (``ctrl_profile_cfg``) so the consumer needs no controller state.

Shapes: the connector's stacked KV is ``[L, 2, B, bs, H, D]`` (a 4-D
``[L, 2, tokens, H*D]`` input is viewed as one block).  Compressed messages
are marked by the layer-name sentinel ``"__compressed__"``.
"""

from __future__ import annotations

import copy
import json
import time
from typing import Any, Optional

import torch

from kvserve_hpdps_b200.compression.config import (DEFAULT_HADAMARD_SEED, CompressedKVData,
                                                   CompressionConfig,
                                                   get_default_compression_config, validate_spec)
from kvserve_hpdps_b200.utils.logger import get_logger

logger = get_logger(__name__)

COMPRESSED_SENTINEL = "__compressed__"


def is_compressed_layer_names(layer_names: list[str]) -> bool:
    return bool(layer_names) and layer_names[0] == COMPRESSED_SENTINEL


def strip_sentinel(layer_names: list[str]) -> list[str]:
    return layer_names[1:] if is_compressed_layer_names(layer_names) else layer_names


def add_sentinel(layer_names: list[str]) -> list[str]:
    return [COMPRESSED_SENTINEL] + list(layer_names)


def _cfg_key(cfg: dict) -> str:
    return json.dumps(cfg, sort_keys=True, default=str)


def use_fused(cfg: dict) -> bool:
    """Whether a custom pipeline config runs on the fused kernels."""
    from kvserve_hpdps_b200.compression.components import custom_impls
    from kvserve_hpdps_b200.compression.quantizer import fused_compatible
    if cfg.get("backend") == "generic" or custom_impls(cfg):
        return False  # user components run in the generic pipeline
    if cfg.get("backend") in ("fused", "tilelang"):
        return True
    pipeline = cfg.get("pipeline") or []
    return "quantizer" in pipeline and fused_compatible(cfg.get("quantizer_config"))


class KVCompressionAdapter:
    _CONTEXT_TTL_S = 300.0

    def __init__(self, compression_spec: Any, num_kv_heads: int, head_size: int,
                 model_name: Optional[str] = None, tp_rank: int = 0, tp_size: int = 1,
                 num_layers: Optional[int] = None, bandwidth_fn=None):
        validate_spec(compression_spec)
        self._num_kv_heads = int(num_kv_heads)
        self._head_size = int(head_size)
        self._model_name = model_name
        self._tp_rank, self._tp_size = int(tp_rank), int(tp_size)
        self._num_layers = num_layers
        self._controller = None
        self._service_cfg: dict = {}
        self._bandwidth_fn = bandwidth_fn
        self._last_contexts: dict[str, tuple[float, dict]] = {}
        self._manager_cache: dict[str, tuple[Any, Optional[CompressionConfig]]] = {}
        self._last_decompress_timing: Optional[dict] = None
        self._cpu_fallback_mgr = None
        self._paged_ctl: Optional[bool] = None  # controller mode: every profile fused
        self.spec = compression_spec
        if compression_spec == "default":
            cfg = get_default_compression_config()
            self._patch_model_name(cfg)
            self._manager, self._config = self._build(cfg)
        elif isinstance(compression_spec, dict) and compression_spec.get("mode") == "controller":
            self._init_controller(compression_spec)
            self._manager, self._config = None, None
        else:
            cfg = copy.deepcopy(compression_spec)
            if self._model_name and "quantizer_config" in cfg and \
                    not cfg["quantizer_config"].get("model_name"):
                cfg["quantizer_config"]["model_name"] = self._model_name
            self._manager, self._config = self._build(cfg)

    # ---------------------------------------------------------- builders
    def _patch_model_name(self, cfg: dict) -> None:
        if self._model_name and "quantizer_config" in cfg:
            cfg["quantizer_config"]["model_name"] = self._model_name

    def _init_controller(self, spec: dict) -> None:
        from kvserve_hpdps_b200.controller.online_controller import OnlineController
        from kvserve_hpdps_b200.controller.profile_library import ProfileLibrary
        library = ProfileLibrary(spec["library_path"])
        self._controller = OnlineController(library, epsilon=spec.get("epsilon", 0.1),
                                            alpha=spec.get("alpha", 0.2),
                                            seed=spec.get("seed"))
        state = spec.get("bandit_state_path")
        if state:
            self._controller.try_load_state(state)
        self._bandit_state_path = state
        self._service_cfg = dict(spec.get("service_config", {}))

    def _make_config(self, cfg: dict, custom: frozenset = frozenset()) -> CompressionConfig:
        qc = cfg.get("quantizer_config")
        if qc is not None and "quantizer" not in custom:  # a user quantizer gets its own dict
            qc = dict(qc)
            qc["tp_rank"] = self._tp_rank
            qc["tensor_parallel_size"] = self._tp_size
            if self._num_layers:
                qc.setdefault("num_layers", self._num_layers)
        return CompressionConfig(enabled=cfg.get("enabled", True), pipeline=cfg.get("pipeline", []),
                                 transformer_config=cfg.get("transformer_config"),
                                 quantizer_config=qc, codec_config=cfg.get("codec_config"),
                                 min_compress_size=cfg.get("min_compress_size", 0))

    def _build(self, cfg: dict):
        if use_fused(cfg):
            from kvserve_hpdps_b200.compression.fused_manager import FusedCompressionManager
            pipeline = cfg.get("pipeline") or ["transformer", "quantizer", "codec"]
            transform = "transformer" in pipeline or cfg is not None and cfg.get("backend") in (
                "fused", "tilelang") or self.spec == "default"
            seed = (cfg.get("transformer_config") or {}).get("seed", DEFAULT_HADAMARD_SEED)
            codec_cfg = cfg.get("codec_config") if "codec" in pipeline else {"codec_type": "none"}
            mgr = FusedCompressionManager(self._num_kv_heads, self._head_size,
                                          cfg.get("quantizer_config"), codec_cfg, base_seed=seed,
                                          tp_rank=self._tp_rank, tp_size=self._tp_size,
                                          transform=transform, num_layers=self._num_layers)
            mgr.min_compress_size = int(cfg.get("min_compress_size", 0))
            return mgr, None
        from kvserve_hpdps_b200.compression.codec import KVServeCodec
        from kvserve_hpdps_b200.compression.components import custom_impls, resolve_component
        from kvserve_hpdps_b200.compression.pipeline_manager import CompressionManager
        from kvserve_hpdps_b200.compression.quantizer import KVServeQuantizer
        from kvserve_hpdps_b200.compression.transformer import KVServeTransformer
        pipeline = cfg.get("pipeline", [])
        config = self._make_config(cfg, custom=set(custom_impls(cfg)))
        built_in = {"transformer": KVServeTransformer, "quantizer": KVServeQuantizer,
                    "codec": KVServeCodec}
        classes = [(resolve_component(k, cfg.get(f"{k}_impl")) or built_in[k])
                   if k in pipeline else None for k in ("transformer", "quantizer", "codec")]
        mgr = CompressionManager(config, *classes)
        return mgr, config

    def _get_cached_manager(self, cfg: dict):
        key = _cfg_key(cfg)
        if key not in self._manager_cache:
            c = copy.deepcopy(cfg)
            # profiles from a library name no model: use the served model's
            # head-score table, as custom specs do
            if self._model_name and "quantizer_config" in c and \
                    not c["quantizer_config"].get("model_name"):
                c["quantizer_config"]["model_name"] = self._model_name
            self._manager_cache[key] = self._build(c)
        return self._manager_cache[key]

    @property
    def manager(self):
        return self._manager

    @property
    def controller_mode(self) -> bool:
        return self._controller is not None

    def _fused(self) -> bool:
        return getattr(self._manager, "backend", None) == "kvs_fused"

    def _cpu_fallback(self):
        """Generic-pipeline twin of the fused manager for tensors off the GPU
        (the fused kernels need CUDA), as the reference falls back to its
        quantizer + codec manager when its fused op is unavailable: the same
        quantizer settings (fused defaults filled in), the Hadamard with the
        same seed when the fused path applies it, and the same codec.  Its
        messages carry ``backend: generic`` and decode on any device."""
        if self._cpu_fallback_mgr is None:
            m = self._manager
            pipeline = (["transformer"] if m.base_seed is not None else []) + ["quantizer"]
            if m.codec != "none":
                pipeline.append("codec")
            spec = {"enabled": True, "pipeline": pipeline, "backend": "generic",
                    "transformer_config": {"transform_type": "hadamard",
                                           "seed": m.base_seed if m.base_seed is not None
                                           else DEFAULT_HADAMARD_SEED},
                    "quantizer_config": dict(m.quantizer_config),
                    "codec_config": dict(m.codec_config),
                    "min_compress_size": int(getattr(m, "min_compress_size", 0))}
            self._cpu_fallback_mgr = self._build(spec)
        return self._cpu_fallback_mgr

    # ------------------------------------------------------------ public
    def _to_6d(self, stacked: torch.Tensor) -> torch.Tensor:
        if stacked.dim() == 6:
            return stacked.contiguous()
        if stacked.dim() == 4:
            L, _, T, _ = stacked.shape
            return stacked.contiguous().view(L, 2, 1, T, self._num_kv_heads, self._head_size)
        raise ValueError(f"unsupported KV rank {stacked.dim()} (shape {tuple(stacked.shape)})")

    def compress(self, stacked_kv: torch.Tensor, request_id: str) -> Optional[CompressedKVData]:
        meta = {"original_dtype": str(stacked_kv.dtype).replace("torch.", ""),
                "original_shape": list(stacked_kv.shape)}
        x = self._to_6d(stacked_kv)
        if self._controller is not None:
            return self._compress_controller(x, request_id, meta)
        if x.numel() * x.element_size() < getattr(self._manager, "min_compress_size", 0):
            return None
        if self._fused() and not x.is_cuda:
            mgr, conf = self._cpu_fallback()
            return mgr.compress_all_layers(x, request_id, conf, meta)
        return self._manager.compress_all_layers(x, request_id, self._config, meta)

    def decompress(self, compressed: CompressedKVData) -> Optional[torch.Tensor]:
        if self._controller is not None:
            cfg = compressed.metadata.get("ctrl_profile_cfg")
            if cfg is None:
                logger.error("controller mode: ctrl_profile_cfg missing from metadata")
                return None
            mgr, conf = self._get_cached_manager(cfg)
        elif self._fused() and (compressed.metadata or {}).get("backend") == "generic":
            mgr, conf = self._cpu_fallback()  # a message of the CPU fallback
        else:
            mgr, conf = self._manager, self._config
        res = mgr.decompress_all_layers(compressed, conf)
        self._last_decompress_timing = getattr(mgr, "_last_decompress_timing", None)
        if res is None:
            return None
        if isinstance(res, list):
            res = torch.cat(res, 0)
        shape = compressed.metadata.get("original_shape")
        if shape is not None:
            return res.contiguous().view(*[int(s) for s in shape])
        return res.contiguous().view(res.shape[0], 2, -1, self._num_kv_heads * self._head_size)

    def get_last_decompress_timing(self) -> Optional[dict]:
        return self._last_decompress_timing

    # per-layer overlap API (fused backend)
    def supports_overlap(self) -> bool:
        return self._manager is not None and hasattr(self._manager, "compress_quant_layer")

    def supports_paged(self) -> bool:
        """Paged multi-request compression (the fused kernels: CUDA tensors).
        In controller mode: when every profile of the library runs on the
        fused kernels; each message then names the profile it was coded
        with (``ctrl_profile_cfg``), as the whole-tensor path does."""
        if self._controller is not None:
            if self._paged_ctl is None:
                self._paged_ctl = all(use_fused(dict(p.compression_config or {}))
                                      for p in self._controller.library.get_all_profiles())
            return self._paged_ctl
        return self._manager is not None and hasattr(self._manager, "compress_paged_requests")

    def _paged_manager(self, kv_layers, requests, request_id: str):
        """(manager, extra metadata) for a paged message; (None, None) when
        the controller picks no compression for it."""
        if self._controller is None:
            return self._manager, None
        volume = float(sum(len(kv_layers) * 2 * int(n) * self._num_kv_heads * self._head_size
                           * kv_layers[0].element_size() for _, n in requests))
        profile, ctx = self.select_profile(volume, request_id)
        if profile is None:
            logger.debug("controller: no compression for %s (%s)", request_id, ctx.get("reason"))
            return None, None
        mgr, _ = self._get_cached_manager(profile.compression_config)
        return mgr, {"ctrl_profile_cfg": profile.compression_config,
                     "ctrl_profile_id": profile.profile_id}

    def _decode_manager(self, compressed: CompressedKVData):
        cfg = (compressed.metadata or {}).get("ctrl_profile_cfg") \
            if self._controller is not None else None
        if cfg is not None:
            return self._get_cached_manager(cfg)[0]
        if self._manager is None:
            raise RuntimeError("controller mode: ctrl_profile_cfg missing from metadata")
        return self._manager

    def compress_quant_layer(self, kv_layer, layer_id):
        return self._manager.compress_quant_layer(kv_layer, layer_id)

    def finalize_codec(self, q_layers, metas, request_id, original_dtype, original_shape):
        return self._manager.finalize_codec(q_layers, metas, request_id, original_dtype,
                                            original_shape)

    def compress_layer_full(self, kv_layer, layer_id):
        return self._manager.compress_layer_full(kv_layer, layer_id)

    def finalize_layer_group(self, q_perms, cmetas, member_tids, member_blocks, layer_id):
        return self._manager.finalize_layer_group(q_perms, cmetas, member_tids, member_blocks,
                                                  layer_id)

    def decompress_layer_group(self, compressed):
        return self._manager.decompress_layer_group(compressed)

    def finalize_chunked(self, chunks, chunk_metas, request_id, original_dtype, original_shape):
        return self._manager.finalize_chunked(chunks, chunk_metas, request_id, original_dtype,
                                              original_shape)

    def compress_paged_requests(self, kv_layers, layer_ids, requests, member_tids=None,
                                trim: bool = True, deferred: bool = False,
                                request_id: str = "grp"):
        """One message for the requests; None when the controller picks no
        compression."""
        mgr, extra = self._paged_manager(kv_layers, requests, request_id)
        if mgr is None:
            return None
        return mgr.compress_paged_requests(kv_layers, layer_ids, requests, member_tids,
                                           trim=trim, deferred=deferred, extra_meta=extra)

    def send_paged_requests(self, transport, request_id, layer_names, kv_layers, layer_ids,
                            requests, member_tids=None) -> Optional[dict]:
        """Compress and send one message (see
        ``FusedCompressionManager.send_paged_requests``: straight into the
        consumer's ring on the NVLink transport).  None, with nothing sent,
        when the controller picks no compression for it (the caller sends
        the raw KV)."""
        mgr, extra = self._paged_manager(kv_layers, requests, request_id)
        if mgr is None:
            return None
        return mgr.send_paged_requests(transport, request_id, layer_names, kv_layers, layer_ids,
                                       requests, member_tids, extra_meta=extra)

    def decompress_paged_requests(self, compressed, dst_layers, dst_requests):
        return self._decode_manager(compressed).decompress_paged_requests(compressed, dst_layers,
                                                                          dst_requests)

    def decompress_members(self, compressed, dst_layers, selection):
        """Grouped message: decode the members in ``selection`` (member
        index -> destination block ids) in one launch."""
        return self._decode_manager(compressed).decompress_members(compressed, dst_layers,
                                                                   selection)

    def warmup(self, block_size: int = 16) -> None:
        if self._manager is not None and hasattr(self._manager, "warmup"):
            self._manager.warmup(block_size)

    # ------------------------------------------------------- controller
    def current_bandwidth_mbps(self) -> float:
        if self._bandwidth_fn is not None:
            try:
                bw = self._bandwidth_fn()
                if bw and bw > 0:
                    return float(bw)
            except Exception as e:  # noqa: BLE001
                logger.warning("bandwidth probe failed: %s", e)
        return float(self._service_cfg.get("bandwidth_mbps", 10_000.0))

    def select_profile(self, volume_bytes: float, request_id: str):
        """Controller decision for one request: (profile or None, context)."""
        B = self.current_bandwidth_mbps()
        profile, ctx = self._controller.select_profile(
            volume_bytes, B, float(self._service_cfg.get("t_model_ms", 0.0)),
            float(self._service_cfg.get("slo_ms", float("inf"))),
            float(self._service_cfg.get("accuracy_requirement", 0.9)))
        self._last_contexts[request_id] = (time.monotonic(), ctx)
        self._evict_stale_contexts()
        return profile, ctx

    def _compress_controller(self, x: torch.Tensor, request_id: str, meta: dict):
        profile, ctx = self.select_profile(float(x.numel() * x.element_size()), request_id)
        if profile is None:
            logger.debug("controller: no compression for %s (%s)", request_id, ctx.get("reason"))
            return None
        meta["ctrl_profile_cfg"] = profile.compression_config
        meta["ctrl_profile_id"] = profile.profile_id
        mgr, conf = self._get_cached_manager(profile.compression_config)
        return mgr.compress_all_layers(x, request_id, conf, meta)

    def update_controller(self, request_id: str, observed_latency_ms: float) -> None:
        if self._controller is None:
            return
        entry = self._last_contexts.pop(request_id, None)
        if entry is not None:
            self._controller.update(entry[1], observed_latency_ms)

    def get_controller_stats(self) -> Optional[dict]:
        return None if self._controller is None else self._controller.get_statistics()

    def save_controller_state(self) -> None:
        if self._controller is not None and getattr(self, "_bandit_state_path", None):
            self._controller.save_state(self._bandit_state_path)

    def _evict_stale_contexts(self) -> None:
        cutoff = time.monotonic() - self._CONTEXT_TTL_S
        stale = [k for k, (t, _) in self._last_contexts.items() if t < cutoff]
        for k in stale:
            self._last_contexts.pop(k, None)
        if stale:
            logger.warning("evicted %d stale controller contexts", len(stale))
