"""vLLM V1 configuration for the compressed KV connector (two-engine PD).

The prefill engine is the producer, the decode engine the consumer; both must
see the same ``transfer_id`` for a logical request (the router derives it from
its own request id).  ``compression`` is one of ``None`` (raw transfer),
``"default"``, a custom pipeline dict or a controller dict; see
``kvserve_hpdps_b200/compression/config.py`` for the keys.

Homogeneous TP uses one channel per TP rank at ``base_port + tp_rank``.
"""

from __future__ import annotations

from typing import Any, Optional

CONNECTOR_MODULE = "kvserve_hpdps_b200.connector.compressed_kv_connector"
CONNECTOR_NAME = "CompressedKVConnector"
ROLES = {"kv_producer": 0, "kv_consumer": 1}


def make_kv_transfer_config(*, role: str, decode_host: str = "127.0.0.1", base_port: int = 25010,
                            compression: Any = "default", transport: str = "auto",
                            overlap: Optional[str] = None,
                            load_failure_policy: str = "recompute"):
    """KVTransferConfig for one side.  ``transport``: auto (NVLink P2P ring
    when the two GPUs can map each other, else NCCL), p2p or nccl.
    ``load_failure_policy``: what the decode engine does with a request whose
    KV did not arrive intact (the connector reports its blocks): recompute
    them from the prompt, or fail the request."""
    from vllm.config import KVTransferConfig
    if role not in ROLES:
        raise ValueError(f"role must be one of {sorted(ROLES)}, got {role!r}")
    extra: dict = {"compression": compression, "transport": transport}
    if overlap:
        extra["overlap"] = overlap
    return KVTransferConfig(kv_connector=CONNECTOR_NAME, kv_connector_module_path=CONNECTOR_MODULE,
                            kv_role=role, kv_rank=ROLES[role], kv_parallel_size=2,
                            kv_ip=decode_host, kv_port=base_port,
                            kv_connector_extra_config=extra,
                            kv_load_failure_policy=load_failure_policy)


def make_sampling_params(*, transfer_id: str, max_tokens: int = 32, temperature: float = 0.0):
    """SamplingParams carrying the PD transfer id."""
    from vllm import SamplingParams
    return SamplingParams(max_tokens=max_tokens, temperature=temperature,
                          extra_args={"kv_transfer_params": {"transfer_id": transfer_id}})


CUSTOM_PIPELINE = {
    "enabled": True,
    "pipeline": ["transformer", "quantizer", "codec"],
    "transformer_config": {"transform_type": "hadamard", "seed": 0x3333},
    "quantizer_config": {"hybrid_ratio": 0.3, "high_key_max_value": 16,
                         "high_value_max_value": 16, "low_key_max_value": 12,
                         "low_value_max_value": 8, "axis_key": "channel",
                         "axis_value": "token", "split_type": "head"},
    "codec_config": {"codec_type": "rans"},
}

CONTROLLER = {
    "mode": "controller",
    "library_path": "profile_library.json",
    "epsilon": 0.1,
    "alpha": 0.2,
    "service_config": {"bandwidth_mbps": 10000, "slo_ms": 200, "accuracy_requirement": 0.92,
                       "t_model_ms": 0},
}
