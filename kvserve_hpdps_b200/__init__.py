"""kvserve_hpdps_b200: a Blackwell-native (sm_100a) KV-cache transfer and
compression connector for disaggregated prefill/decode serving on vLLM V1.

The public connector class is ``CompressedKVConnector`` (import path
``kvserve_hpdps_b200.connector.compressed_kv_connector``), loaded by vLLM via
``KVTransferConfig(kv_connector_module_path=...)``.  It is imported lazily so
that the compression, controller and transport layers stay usable without
vLLM (reference parity: kvserve_v1/__init__.py:1-6).
"""

__version__ = "0.1.0"

__all__ = ["CompressedKVConnector", "__version__"]


def __getattr__(name):
    if name == "CompressedKVConnector":
        from kvserve_hpdps_b200.connector.compressed_kv_connector import (
            CompressedKVConnector)
        return CompressedKVConnector
    raise AttributeError(name)
