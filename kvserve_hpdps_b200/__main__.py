"""Environment check: ``python -m kvserve_hpdps_b200`` prints one JSON object.

What a deployment needs, checked without launching a kernel:

* the package and torch versions, and whether vLLM's V1 connector base class
  imports (the connector is loaded through ``kv_connector_module_path``);
* the native library: built, loadable, its struct layouts matching the
  Python bindings (checked on load), its CPU rANS coder round-tripping a
  small buffer;
* the GPUs: name, compute capability (the kernels are built for sm_100a
  only, so anything but 10.0 cannot run them), memory;
* NVLink peer access between every pair of visible GPUs (the ring transport
  needs it; without it the connector's ``auto`` transport picks NCCL).

Exit code 0 when the fused path can run on every visible GPU, 1 otherwise
(2 when no GPU is visible).
"""

from __future__ import annotations

import json
import sys


def report() -> dict:
    import torch

    import kvserve_hpdps_b200 as pkg
    out: dict = {"package": pkg.__version__, "torch": torch.__version__,
                 "cuda_build": torch.version.cuda}
    try:
        import vllm
        from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorBase_V1  # noqa
        out["vllm"] = {"version": vllm.__version__, "connector_api": True}
    except Exception as e:  # noqa: BLE001 - vLLM is optional
        out["vllm"] = {"version": None, "connector_api": False, "error": str(e)[:200]}
    from kvserve_hpdps_b200.ops import _lib
    try:
        lb = _lib.lib()
        out["native"] = {"path": _lib.LIB_PATH, "loaded": True,
                         "version": int(lb.kvs_library_version())}
        from kvserve_hpdps_b200.compression.codec import decode_bytes, encode_bytes
        probe = (torch.arange(5000) % 7).to(torch.uint8)  # the CPU coder, no GPU needed
        out["native"]["cpu_codec_ok"] = bool(torch.equal(
            decode_bytes(encode_bytes(probe, "rans")), probe))
    except (RuntimeError, OSError) as e:
        out["native"] = {"path": _lib.LIB_PATH, "loaded": False, "error": str(e)[:300]}
    gpus = []
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    for i in range(n):
        p = torch.cuda.get_device_properties(i)
        gpus.append({"index": i, "name": p.name, "capability": f"{p.major}.{p.minor}",
                     "memory_gb": round(p.total_memory / 2 ** 30, 1), "sms": p.multi_processor_count,
                     "fused_path": (p.major, p.minor) == (10, 0)})
    out["gpus"] = gpus
    if n > 1:
        out["peer_access"] = {f"{a}->{b}": bool(torch.cuda.can_device_access_peer(a, b))
                              for a in range(n) for b in range(n) if a != b}
    return out


def exit_code(rep: dict) -> int:
    if not rep["gpus"]:
        return 2
    ok = rep["native"].get("loaded") and all(g["fused_path"] for g in rep["gpus"])
    return 0 if ok else 1


def main() -> int:
    rep = report()
    print(json.dumps(rep, indent=2))
    return exit_code(rep)


if __name__ == "__main__":
    sys.exit(main())
