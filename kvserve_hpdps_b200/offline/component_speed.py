"""Component speed of the compression kernels (encode / decode GB/s).

The reference measures each stage separately (Hadamard, quantizer, codec)
over 1K-32K tokens and records GB/s of original KV
(kvserve_v1/offline_search/evaluation/component_speed/*.py, results/*.csv).
Here the stages are the fused kernels of this package:

* ``quant``:   paged gather + Hadamard (tcgen05) + stats + quantize
               (one stats launch and one quantize launch per call);
* ``dequant``: dequantize + inverse Hadamard + paged scatter;
* ``rans_enc`` / ``rans_dec``: the interleaved rANS codec over the codes;
* ``lc_enc`` / ``lc_dec``: the LC-style BIT_2 + RZE_1 codec over the codes;
* ``block_copy``: the paged gather of raw KV (the uncompressed path).

``--methods custom,kivi,cachegen,hadamard,minmax`` times the offline methods
instead (the reference's kivi_speed.py, cachegen-*_speed.py,
hadamard_speed.py and quantizer_speed.py), on any device, through the
caches the accuracy harness uses: ``compress`` is a fresh cache's prefill
update over every layer, ``reconstruct`` the first decode step (one token per
layer), which rebuilds the layer's KV from its codes.  ``hadamard`` is the
per-head randomized Hadamard (transform / inverse) and ``minmax`` the
reference quantizer formula per (head, channel) for keys and per token for
values (quantize / dequantize).  CUDA figures are event times; CPU figures
are wall time.

Every fused-stage figure is CUDA-event time on the launching stream after warm-up,
averaged over ``--iters`` launches; the input of a full request (28 layers,
8K tokens, 4 heads: 470 MB) is larger than L2, so no flush is needed at
that size.  Rates are GB/s of ORIGINAL bf16 KV (the reference's unit).

Usage::

  python -m kvserve_hpdps_b200.offline.component_speed --layers 28 --tokens 8192
  python -m kvserve_hpdps_b200.offline.component_speed --only quant --layers 2 --iters 3
  python -m kvserve_hpdps_b200.offline.component_speed --methods kivi,cachegen --tokens 4096
"""

from __future__ import annotations

import argparse
import json
import sys

import torch

STAGES = ("quant", "dequant", "rans_enc", "rans_dec", "lc_enc", "lc_dec", "block_copy")
PEER_STAGES = ("quant_peer", "rans_enc_peer")
METHODS = ("custom", "kivi", "cachegen", "hadamard", "minmax")


def _timeit(fn, iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def _timeit_on(device: torch.device, fn, iters: int, warmup: int = 3) -> float:
    """Mean ms per call: CUDA events on the current stream, else wall time."""
    if device.type == "cuda":
        return _timeit(fn, iters, warmup)
    import time
    for _ in range(warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(iters):
        fn()
    return (time.perf_counter() - t0) * 1e3 / iters


def run_methods(methods: tuple[str, ...] = METHODS, layers: int = 28, tokens: int = 8192,
                heads: int = 4, head_dim: int = 128, iters: int = 5, warmup: int = 2,
                device: str | None = None, dtype: torch.dtype = torch.bfloat16,
                seed: int = 1) -> list[dict]:
    """Compress / reconstruct times of the offline methods on random KV with
    outlier key channels (``[1, heads, tokens, head_dim]`` per layer)."""
    from kvserve_hpdps_b200.compression.head_scores import synthetic_scores
    from kvserve_hpdps_b200.offline.caches import HeadHadamard
    from kvserve_hpdps_b200.offline.caches.common import minmax_codes, minmax_values
    from kvserve_hpdps_b200.offline.lm_harness import make_cache
    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    g = torch.Generator(device="cpu").manual_seed(seed)
    ks, vs = [], []
    for _ in range(layers):
        k = torch.randn(1, heads, tokens, head_dim, generator=g)
        k[..., :4] *= 12.0
        ks.append(k.to(dev, dtype))
        vs.append(torch.randn(1, heads, tokens, head_dim, generator=g).to(dev, dtype))
    nk = torch.randn(1, heads, 1, head_dim, generator=g).to(dev, dtype)
    nbytes = layers * 2 * tokens * heads * head_dim * ks[0].element_size()
    scores = synthetic_scores(layers, heads)
    params = {"custom": dict(transform_type="hadamard", heads_selection=0.5,
                             high_key_max_value=16, high_value_max_value=16,
                             low_key_max_value=8, low_value_max_value=8),
              "kivi": dict(nbits=2, q_group_size=32, residual_length=128),
              "cachegen": dict(quantization_level=1)}
    rows = []

    def row(method, phase, ms, **kw):
        rows.append({"method": method, "phase": phase, "ms": round(ms, 4),
                     "gbps": round(nbytes / ms / 1e6, 3), "layers": layers, "tokens": tokens,
                     "heads": heads, "device": dev.type, **kw})

    for m in methods:
        if m in params:
            def prefill(m=m):
                c = make_cache(m, layers, scores if m == "custom" else None, **params[m])
                for l in range(layers):
                    c.update(ks[l], vs[l], l)
                return c

            def decode(c):
                for l in range(layers):
                    c.update(nk, nk, l)

            row(m, "compress", _timeit_on(dev, prefill, iters, warmup))
            caches = [prefill() for _ in range(iters + warmup)]
            it = iter(caches)
            row(m, "reconstruct", _timeit_on(dev, lambda: decode(next(it)), iters, warmup),
                compression_ratio=round(float(caches[0].compute_compression_ratio()), 3)
                if hasattr(caches[0], "compute_compression_ratio") else None)
        elif m == "hadamard":
            had = HeadHadamard()
            ys = [had.transform(ks[l], l) for l in range(layers)]
            row(m, "compress", _timeit_on(dev, lambda: [had.transform(ks[l], l)
                                                         for l in range(layers)
                                                         for _ in (0, 1)], iters, warmup))
            row(m, "reconstruct", _timeit_on(dev, lambda: [had.inverse(ys[l], l)
                                                            for l in range(layers)
                                                            for _ in (0, 1)], iters, warmup))
        elif m == "minmax":
            def quant():
                return [(minmax_codes(ks[l], 16, [2]), minmax_codes(vs[l], 16, [1, 3]))
                        for l in range(layers)]
            packs = quant()
            row(m, "compress", _timeit_on(dev, quant, iters, warmup))
            row(m, "reconstruct", _timeit_on(dev, lambda: [(minmax_values(*a), minmax_values(*b))
                                                            for a, b in packs],
                                             iters, warmup))
        else:
            raise ValueError(f"unknown method {m!r}; expected one of {METHODS}")
    return rows


def run(layers: int = 28, tokens: int = 8192, heads: int = 4, iters: int = 10,
        only: tuple[str, ...] = STAGES, engine: int = 0, seed: int = 1,
        key_levels=(12, 6, 6, 6), value_levels=(8, 4, 4, 4), warmup: int = 3,
        code_width: int = 8, hybrid_ratio: float | None = None,
        peer: int | None = None) -> list[dict]:
    """Stage timings.  With ``hybrid_ratio`` the per-layer plans are the
    default compression mode's (head-score mask at that ratio, nibble codes)
    instead of the fixed ``key_levels``/``value_levels``.  With ``peer`` (a
    second GPU of this process) the stages ``quant_peer`` and
    ``rans_enc_peer`` time the producer kernels of the direct transfer path:
    the quantize kernel storing its codes into that GPU's memory over NVLink
    (message checksum on), and the rANS encoder whose compaction kernel
    stores the coded stream there."""
    from kvserve_hpdps_b200.models.synthetic import paged_workload
    from kvserve_hpdps_b200.ops import kernels as K
    wl = paged_workload(layers, [tokens], heads, device="cuda", seed=seed, fill=False)
    wl.cache.normal_()
    wl.cache[:, 0, :, :, :, :4].mul_(12.0)  # outlier channels in K
    kl = list(key_levels)[:heads] + [key_levels[-1]] * max(0, heads - len(key_levels))
    vl = list(value_levels)[:heads] + [value_levels[-1]] * max(0, heads - len(value_levels))
    cw = code_width if code_width != 8 else None
    if hybrid_ratio is None:
        plans = [K.make_layer_plan(heads, kl, vl, 0x3333, l, code_width=cw) for l in range(layers)]
    else:
        from kvserve_hpdps_b200.compression.config import get_default_compression_config
        from kvserve_hpdps_b200.compression.fused_manager import FusedCompressionManager
        cfg = get_default_compression_config()
        qc = dict(cfg["quantizer_config"], model_name="Qwen2.5-7B-Instruct",
                  hybrid_ratio=float(hybrid_ratio))
        mgr = FusedCompressionManager(heads, 128, qc, cfg["codec_config"], num_layers=layers)
        plans = [mgr.plan(l) for l in range(layers)]
        code_width = mgr.code_width
    slots = K.LayerSlots([wl.cache[l] for l in range(layers)], plans)
    items = K.WorkItems(slots, [(l, wl.block_ids[0], tokens) for l in range(layers)])
    dst = torch.zeros_like(wl.cache)
    dslots = K.LayerSlots([dst[l] for l in range(layers)], plans)
    nbytes = layers * 2 * tokens * heads * 128 * 2
    codes, meta = K.quantize(slots, items, engine=engine)
    n = codes.numel()
    stream = K.rans_encode(codes)
    rows = []

    def row(stage, ms, **kw):
        rows.append({"stage": stage, "ms": round(ms, 4), "gbps": round(nbytes / ms / 1e6, 1),
                     "layers": layers, "tokens": tokens, "heads": heads, **kw})

    if "quant" in only:
        row("quant", _timeit(lambda: K.quantize(slots, items, codes=codes, meta=meta,
                                                engine=engine), iters, warmup), engine=engine)
    if "dequant" in only:
        row("dequant", _timeit(lambda: K.dequantize(codes, meta, dslots, items, engine=engine),
                               iters, warmup), engine=engine)
    if "rans_enc" in only:
        out = torch.empty(K.rans_max_bytes(n), dtype=torch.uint8, device="cuda")
        row("rans_enc", _timeit(lambda: K.rans_encode(codes, out=out, trim=False), iters, warmup),
            code_bytes=n, stream_bytes=int(stream.numel()),
            bits_per_code=round(8 * stream.numel() / n, 4))
    if "rans_dec" in only:
        dec = torch.empty(n, dtype=torch.uint8, device="cuda")
        row("rans_dec", _timeit(lambda: K.rans_decode(stream, n, out=dec), iters, warmup),
            exact=bool(torch.equal(K.rans_decode(stream, n), codes)))
    if "lc_enc" in only or "lc_dec" in only:
        lc_stream = K.lc_encode(codes)
        if "lc_enc" in only:
            row("lc_enc", _timeit(lambda: K.lc_encode(codes, trim=False), iters, warmup),
                stream_bytes=int(lc_stream.numel()),
                bits_per_code=round(8 * lc_stream.numel() / n, 4))
        if "lc_dec" in only:
            dec_lc = torch.empty(n, dtype=torch.uint8, device="cuda")
            row("lc_dec", _timeit(lambda: K.lc_decode(lc_stream, n, out=dec_lc), iters, warmup),
                exact=bool(torch.equal(K.lc_decode(lc_stream, n), codes)))
    if peer is not None and ("quant_peer" in only or "rans_enc_peer" in only):
        from kvserve_hpdps_b200.parallel.p2p import DeviceRegion, enable_peer_access
        from kvserve_hpdps_b200.parallel.p2p_transport import tensor_view
        here = torch.cuda.current_device()
        enable_peer_access(here, peer)
        torch.cuda.set_device(here)
        region = DeviceRegion(peer, 16 + K.rans_max_bytes(n) + 4096)
        torch.cuda.set_device(here)
        ck = torch.zeros(2, dtype=torch.int64, device="cuda")
        if "quant_peer" in only:
            codes_peer = tensor_view(region.ptr, n, torch.uint8, [n], peer)
            row("quant_peer", _timeit(lambda: K.quantize(slots, items, codes=codes_peer, meta=meta,
                                                         engine=engine, ck=ck), iters, warmup),
                engine=engine, peer=peer, code_bytes_over_link=n)
        if "rans_enc_peer" in only:
            row("rans_enc_peer", _timeit(lambda: K.rans_encode_message(
                codes.data_ptr(), n, region.ptr + 16, torch.device("cuda", here),
                prefix=[0, 1, n & 0xFFFFFFFF, n >> 32], msg_off=16, ck=ck), iters, warmup),
                peer=peer, stream_bytes_over_link=int(stream.numel()))
        torch.cuda.synchronize()
        region.close()
    if "block_copy" in only:
        flat = torch.empty(nbytes // layers, dtype=torch.uint8, device="cuda")
        blocks = torch.tensor(wl.block_ids[0], dtype=torch.int32, device="cuda")

        def copy_all():
            for l in range(layers):
                K.block_copy(wl.cache[l], blocks, flat.data_ptr(), True)
        row("block_copy", _timeit(copy_all, iters, warmup))
    K.dequantize(codes, meta, dslots, items, engine=engine)
    err = K.kv_error(wl.cache[:, :, wl.block_ids[0]], dst[:, :, wl.block_ids[0]])
    # order-0 entropy of the code bytes: the size an ideal per-buffer entropy
    # coder would reach, against which the chunked coder is judged
    hist = torch.bincount(codes, minlength=256).double()
    p = hist[hist > 0] / n
    entropy = float(-(p * torch.log2(p)).sum())
    rows.append({"stage": "summary", "code_width": code_width, "original_bytes": nbytes,
                 "entropy_bits_per_code_byte": round(entropy, 4),
                 "rans_bits_per_code_byte": round(8 * stream.numel() / n, 4),
                 "compressed_bytes": int(stream.numel() + meta.numel()),
                 "compression_ratio": round(nbytes / (stream.numel() + meta.numel()), 3),
                 "rel_mse": err["rel_mse"], "cosine": err["cosine"],
                 "device_error": K.read_device_error(wl.cache.device)})
    return rows


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="component speed of the compression kernels")
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--heads", type=int, default=4)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--engine", type=int, default=0, help="0 = tcgen05, 1 = SIMT")
    ap.add_argument("--only", default=",".join(STAGES))
    ap.add_argument("--code-width", type=int, default=8,
                    help="bits per code in the code buffer (4: two codes per rANS symbol)")
    ap.add_argument("--hybrid-ratio", type=float, default=None,
                    help="use the default mode's per-layer plans at this hybrid_ratio")
    ap.add_argument("--methods", default=None,
                    help=f"time offline methods instead of the fused stages: {','.join(METHODS)}")
    ap.add_argument("--device", default=None, help="--methods device (default: cuda if present)")
    ap.add_argument("--peer", type=int, default=None,
                    help="second GPU for the direct-path stages (--only quant_peer,rans_enc_peer)")
    args = ap.parse_args(argv)
    if args.methods:
        for r in run_methods(tuple(args.methods.split(",")), args.layers, args.tokens, args.heads,
                             iters=args.iters, warmup=args.warmup, device=args.device):
            print(json.dumps(r))
        return 0
    if not torch.cuda.is_available():
        print(json.dumps({"unavailable": "no CUDA device"}))
        return 0
    for r in run(args.layers, args.tokens, args.heads, args.iters,
                 tuple(args.only.split(",")), args.engine, warmup=args.warmup,
                 code_width=args.code_width, hybrid_ratio=args.hybrid_ratio, peer=args.peer):
        print(json.dumps(r))
    return 0


if __name__ == "__main__":
    sys.exit(main())
