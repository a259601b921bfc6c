"""CPU-only compression round trip (no GPU, no transfer).

The quantizer + codec fallback path on a Qwen2.5-7B-shaped layer stack:
synthetic KV [28 layers, 2 (K/V), 2048 tokens, 4 KV heads, 128] in bf16 from a
seeded N(0, 1), with 4 fixed channels per head of K scaled by 12 (outlier
channels); hybrid_ratio 0.3, high key/value levels 16, low key levels 12.
Runs the generic Transform -> Quantizer -> Codec pipeline (PyTorch on the
CPU, the own rANS codec from the native library's CPU path) and prints one
JSON line: compressed bytes, compression ratio, relative MSE and cosine of
the reconstruction, and the CPU wall time of each direction.

Example::

  python examples/cpu_roundtrip.py
  python examples/cpu_roundtrip.py --pipeline quantizer,codec --codec bitpack
  python examples/cpu_roundtrip.py --mode default
  # one TP rank's share of a 32K-token Qwen2.5-32B TP4 request (2 GiB, 8-layer chunks)
  python examples/cpu_roundtrip.py --layers 64 --tokens 32768 --heads 2 \
      --model Qwen2.5-32B-Instruct --tp-size 4 --tp-rank 1
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--tokens", type=int, default=2048)
    ap.add_argument("--heads", type=int, default=4, help="KV heads of this rank")
    ap.add_argument("--model", default="Qwen2.5-7B-Instruct",
                    help="head-score table (Qwen2.5-32B-Instruct: 64 layers x 8 KV heads)")
    ap.add_argument("--tp-size", type=int, default=1)
    ap.add_argument("--tp-rank", type=int, default=0)
    ap.add_argument("--pipeline", default="transformer,quantizer,codec")
    ap.add_argument("--codec", default="rans", help="rans | bitpack | nvcomp | lc")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--mode", default="custom", choices=("custom", "default"),
                    help="default: the 'default' compression spec (on the CPU the adapter runs "
                         "the fused path's generic twin)")
    args = ap.parse_args(argv)
    from kvserve_hpdps_b200.compression.manager import KVCompressionAdapter
    from kvserve_hpdps_b200.compression.oracle import error_metrics
    L, T, H, D = args.layers, args.tokens, args.heads, 128
    g = torch.Generator().manual_seed(args.seed)
    kv = torch.randn((L, 2, T, H, D), generator=g)
    outlier = torch.randperm(D, generator=g)[:4]
    kv[:, 0, :, :, outlier] *= 12.0
    kv = kv.to(torch.bfloat16)
    spec = {"enabled": True, "pipeline": args.pipeline.split(","), "backend": "generic",
            "transformer_config": {"transform_type": "hadamard", "seed": 0x3333},
            "quantizer_config": {"model_name": args.model, "hybrid_ratio": 0.3,
                                 "high_key_max_value": 16, "high_value_max_value": 16,
                                 "low_key_max_value": 12, "low_value_max_value": 16,
                                 "axis_key": "channel", "axis_value": "token",
                                 "split_type": "head"},
            "codec_config": {"codec_type": args.codec}, "min_compress_size": 0}
    if args.mode == "default":
        spec = "default"
    ad = KVCompressionAdapter(spec, H, D, model_name=args.model, num_layers=L,
                              tp_rank=args.tp_rank, tp_size=args.tp_size)
    x = kv.view(L, 2, 1, T, H, D)
    t0 = time.perf_counter()
    cd = ad.compress(x, "cpu-roundtrip")
    t1 = time.perf_counter()
    out = ad.decompress(cd)
    t2 = time.perf_counter()
    from kvserve_hpdps_b200.compression.wire import build_wire
    nbytes = build_wire(cd).nbytes
    err = error_metrics(x.float(), out.float())
    print(json.dumps({
        "config": f"CPU round trip, {args.model} shapes [{L}, 2, {T}, {H}, 128] "
                  f"(TP rank {args.tp_rank}/{args.tp_size}), " + (
            "hybrid 0.3, high 16/16, low key 12" if isinstance(spec, dict) else
            "default spec (hybrid 0.8, levels 12/8 high, 6/4 low, Hadamard, rANS)"),
        "mode": args.mode,
        "pipeline": spec["pipeline"] if isinstance(spec, dict) else
        ad._cpu_fallback()[1].pipeline,
        "codec": args.codec if isinstance(spec, dict) else "default",
        "original_bytes": kv.numel() * 2, "compressed_bytes": int(nbytes),
        "compression_ratio": round(kv.numel() * 2 / nbytes, 3),
        "rel_mse": err["rel_mse"], "cosine": err["cosine"],
        "compress_s": round(t1 - t0, 3), "decompress_s": round(t2 - t1, 3)}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
