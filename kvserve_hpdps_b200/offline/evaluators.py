"""Evaluators of the offline search: compression ratio, reconstruction error,
proxy accuracy and codec speed of a candidate configuration.

The reference evaluates CR with HF-model prefills and its nvCOMP codec and
accuracy with lm-eval (kvserve_v1/offline_search/evaluation/param_search/
cr_evaluator.py, acc_evaluator.py).  Without datasets or checkpoints this
framework evaluates on KV tensors (synthetic, or captured from any model):

* CR: bytes of the fused path's output (codes after the codec + fp16
  metadata) against bf16 input, measured with the real kernels;
* reconstruction error: rel-MSE / cosine / max-abs from the fused metric
  kernel;
* proxy accuracy: fidelity of attention outputs -- for random queries per
  layer and head, the cosine between softmax(QK^T/sqrt(d))V computed with
  the original and with the reconstructed K, V (1.0 = identical);
  ``logit_agreement`` compares next-token logits of a model when one is
  available;
* speed: encode / decode device time -> harmonic speed S in MB/s of
  original KV, as the controller's profiles expect.
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass
from typing import Optional

import torch

from kvserve_hpdps_b200.compression.config import get_default_compression_config
from kvserve_hpdps_b200.offline.search_space import Candidate


@dataclass
class EvalResult:
    candidate: Candidate
    compression_ratio: float
    rel_mse: float
    cosine: float
    accuracy: float
    encode_mbps: Optional[float] = None
    decode_mbps: Optional[float] = None

    @property
    def harmonic_speed_mbps(self) -> Optional[float]:
        if not self.encode_mbps or not self.decode_mbps:
            return None
        return self.encode_mbps * self.decode_mbps / (self.encode_mbps + self.decode_mbps)

    def as_dict(self) -> dict:
        return {"candidate": self.candidate.key(), "config": self.candidate.quantizer_config(),
                "compression_ratio": self.compression_ratio, "rel_mse": self.rel_mse,
                "cosine": self.cosine, "accuracy": self.accuracy,
                "encode_mbps": self.encode_mbps, "decode_mbps": self.decode_mbps,
                "harmonic_speed_mbps": self.harmonic_speed_mbps}


def attention_fidelity(k_ref: torch.Tensor, v_ref: torch.Tensor, k_rec: torch.Tensor,
                       v_rec: torch.Tensor, n_queries: int = 64, seed: int = 0) -> float:
    """Mean cosine of attention outputs with original vs reconstructed KV.

    k/v: [tokens, H, D].  Queries ~ N(0, 1) scaled like keys."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    T, H, D = k_ref.shape
    q = torch.randn((H, n_queries, D), generator=g).to(k_ref.device, torch.float32)
    q = q * k_ref.float().std()
    outs = []
    for kk, vv in ((k_ref, v_ref), (k_rec, v_rec)):
        kf, vf = kk.float().permute(1, 0, 2), vv.float().permute(1, 0, 2)
        w = torch.softmax(q @ kf.transpose(1, 2) / math.sqrt(D), dim=-1)
        outs.append(w @ vf)
    cos = torch.nn.functional.cosine_similarity(outs[0].flatten(1), outs[1].flatten(1), dim=-1)
    return float(cos.mean())


def candidate_spec(c: Candidate, model_name: Optional[str], codec: str = "rans") -> dict:
    spec = get_default_compression_config()
    spec["pipeline"] = ["transformer", "quantizer", "codec"]
    spec["transformer_config"] = {"transform_type": "hadamard", "seed": 0x3333}
    spec["quantizer_config"] = c.quantizer_config(model_name)
    spec["codec_config"] = {"codec_type": codec}
    spec["min_compress_size"] = 0
    return spec


class KVEvaluator:
    """Evaluate candidates on a stack of KV tensors [L, 2, tokens, H, D]."""

    def __init__(self, kv: torch.Tensor, model_name: Optional[str] = None,
                 codec: str = "rans", measure_speed: bool = True, n_queries: int = 64):
        if kv.dim() != 5:
            raise ValueError("kv must be [L, 2, tokens, H, D]")
        self.kv = kv.to(torch.bfloat16)
        self.model_name = model_name
        self.codec = codec
        self.measure_speed = measure_speed and kv.is_cuda
        self.n_queries = n_queries
        L, _, T, H, D = kv.shape
        bs = 16
        nb = (T + bs - 1) // bs
        pad = nb * bs - T
        x = self.kv
        if pad:
            x = torch.cat([x, torch.zeros((L, 2, pad, H, D), dtype=x.dtype, device=x.device)], 2)
        self.stacked = x.view(L, 2, nb, bs, H, D).contiguous()
        self.tokens = T

    def evaluate(self, c: Candidate) -> EvalResult:
        from kvserve_hpdps_b200.compression.manager import KVCompressionAdapter
        L, _, nb, bs, H, D = self.stacked.shape
        spec = candidate_spec(c, self.model_name, self.codec)
        if not self.stacked.is_cuda:
            spec["backend"] = "generic"  # the fused kernels need a GPU
        ad = KVCompressionAdapter(spec, H, D, model_name=self.model_name, num_layers=L)
        cd = ad.compress(self.stacked, "search")
        rec = ad.decompress(cd)
        from kvserve_hpdps_b200.compression.wire import build_wire
        wire_bytes = build_wire(cd).nbytes
        orig = self.stacked.numel() * 2
        ref = self.stacked.view(L, 2, nb * bs, H, D)[:, :, :self.tokens]
        got = rec.view(L, 2, nb * bs, H, D)[:, :, :self.tokens]
        from kvserve_hpdps_b200.ops import kernels as K
        err = K.kv_error(ref.contiguous(), got.contiguous()) if ref.is_cuda else \
            __import__("kvserve_hpdps_b200.compression.oracle", fromlist=["error_metrics"]).error_metrics(ref, got)
        fid = sum(attention_fidelity(ref[l, 0], ref[l, 1], got[l, 0], got[l, 1], self.n_queries, l)
                  for l in range(L)) / L
        enc = dec = None
        if self.measure_speed:
            enc, dec = self._speed(ad)
        return EvalResult(c, orig / wire_bytes, err["rel_mse"], err["cosine"], fid, enc, dec)

    def _speed(self, ad, iters: int = 3) -> tuple[float, float]:
        x = self.stacked
        ad.decompress(ad.compress(x, "w"))
        torch.cuda.synchronize()
        mb = x.numel() * 2 / (1024 * 1024)
        t0 = time.perf_counter()
        for _ in range(iters):
            cd = ad.compress(x, "s")
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        for _ in range(iters):
            ad.decompress(cd)
        torch.cuda.synchronize()
        t2 = time.perf_counter()
        return mb * iters / (t1 - t0), mb * iters / (t2 - t1)


def logit_agreement(model, input_ids: torch.Tensor, kv_transform) -> dict:
    """Top-1 agreement / KL of next-token logits between a model's prefill
    with its own KV and with ``kv_transform(k, v, layer) -> (k', v')``
    applied to the cached KV (HF ``DynamicCache`` models).  Uses the fused
    logit-agreement kernel on CUDA."""
    from kvserve_hpdps_b200.ops import kernels as K
    with torch.no_grad():
        out = model(input_ids[:, :-1], use_cache=True)
        cache = out.past_key_values
        ref = model(input_ids[:, -1:], past_key_values=cache, use_cache=True).logits[:, -1]
        out2 = model(input_ids[:, :-1], use_cache=True)
        c2 = out2.past_key_values
        for l in range(len(c2.layers) if hasattr(c2, "layers") else len(c2)):
            layer = c2.layers[l] if hasattr(c2, "layers") else None
            if layer is not None:
                layer.keys, layer.values = kv_transform(layer.keys, layer.values, l)
        approx = model(input_ids[:, -1:], past_key_values=c2, use_cache=True).logits[:, -1]
    if ref.is_cuda:
        return K.logit_agreement(ref.float(), approx.float())
    lr, la = torch.log_softmax(ref.double(), -1), torch.log_softmax(approx.double(), -1)
    return {"top1_agreement": float((ref.argmax(-1) == approx.argmax(-1)).float().mean()),
            "kl_mean": float((lr.exp() * (lr - la)).sum(-1).mean()), "rows": ref.shape[0]}
