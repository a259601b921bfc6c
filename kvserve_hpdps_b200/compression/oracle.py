"""CPU oracle of the fused producer/consumer math (plain PyTorch, float32).

Every device kernel of the fused path is tested against these functions.  The
math is the reference's ``compress_v3`` / ``decompress_v3``
(kvserve_v1/tilelang_ops/kv_hadamard_quant.py:1307-1486) with two documented
choices of this framework:

* quantization multiplies by the correctly rounded reciprocal of the scale
  instead of dividing by it (the two differ only when the quotient lies
  within one ulp of a rounding boundary);
* codes are clamped to ``levels-1`` instead of ``levels`` (``levels`` is the
  reference's ``max_value``).  The top code ``levels`` can only be produced by
  bf16 rounding pushing a value past the maximum, and ``levels-1`` is then the
  nearer reconstruction; the cap keeps every code inside ceil(log2(levels))
  bits.  Pass ``clamp_top=False`` for the reference's cap.

Key codes: per (head, channel) min/max over the valid tokens of the request
layer.  Value codes: per token, min/max over all channels of the heads that
share a level count (one group per distinct level count).  The transformed
value is rounded to bf16 before quantization, as the reference stores its
intermediate in bf16.
"""

from __future__ import annotations

from typing import Optional

import torch

from kvserve_hpdps_b200.compression.signs import fwht_fp32

EPS_RANGE = 1e-5


def _bf16_round(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32)


def _quant(val: torch.Tensor, mn: torch.Tensor, scale: torch.Tensor,
           top: torch.Tensor) -> torch.Tensor:
    rcp = 1.0 / scale
    q = torch.floor((val - mn) * rcp + 0.5)
    q = torch.minimum(torch.clamp(q, min=0.0), top)
    return q.to(torch.uint8)


def forward_transform(x: torch.Tensor, signs: Optional[torch.Tensor]) -> torch.Tensor:
    """[..., H, D] -> float32 transformed (signs [H, D] or None = identity)."""
    xf = x.to(torch.float32)
    if signs is None:
        return xf
    return fwht_fp32(xf * signs.to(torch.float32))


def compress_layer(kv_layer: torch.Tensor, key_levels: torch.Tensor,
                   value_levels: torch.Tensor, signs: Optional[torch.Tensor],
                   n_valid: Optional[int] = None, clamp_top: bool = True) -> dict:
    """Quantize one request layer ``[2, B, bs, H, D]``.

    Returns ``codes`` uint8 ``[2, H, B, bs, D]`` (heads-outer, the wire order)
    and the float32 metadata: ``key_min``/``key_scale`` ``[H, D]``,
    ``value_min``/``value_scale`` ``[G, rows]`` with ``groups`` (head lists).
    """
    _, B, bs, H, D = kv_layer.shape
    rows = B * bs
    nv = rows if n_valid is None else int(n_valid)
    kl = key_levels.to(torch.float32).reshape(H)
    vl = value_levels.to(torch.float32).reshape(H)

    kt = forward_transform(kv_layer[0].reshape(rows, H, D), signs)
    kmin = kt[:nv].amin(dim=0)
    kmax = kt[:nv].amax(dim=0)
    kscale = torch.clamp(kmax - kmin, min=EPS_RANGE) / (kl[:, None] - 1.0)
    ktop = (kl - 1.0 if clamp_top else kl)[None, :, None].expand(1, H, D)
    qk = _quant(_bf16_round(kt), kmin[None], kscale[None], ktop)

    vt = forward_transform(kv_layer[1].reshape(rows, H, D), signs)
    rmin = vt.amin(dim=2)
    rmax = vt.amax(dim=2)
    groups: list[list[int]] = []
    gid: dict[float, int] = {}
    for h, v in enumerate(vl.tolist()):
        if v not in gid:
            gid[v] = len(gid)
            groups.append([])
        groups[gid[v]].append(h)
    G = len(groups)
    vmin = torch.empty((G, rows), dtype=torch.float32)
    vscale = torch.empty((G, rows), dtype=torch.float32)
    qv = torch.empty((rows, H, D), dtype=torch.uint8)
    vtb = _bf16_round(vt)
    for g, hs in enumerate(groups):
        lev = float(vl[hs[0]])
        gmin = rmin[:, hs].amin(dim=1)
        gmax = rmax[:, hs].amax(dim=1)
        sc = torch.clamp(gmax - gmin, min=EPS_RANGE) / (lev - 1.0)
        vmin[g], vscale[g] = gmin, sc
        top = torch.tensor(lev - 1.0 if clamp_top else lev)
        qv[:, hs, :] = _quant(vtb[:, hs, :], gmin[:, None, None], sc[:, None, None], top)

    codes = torch.stack([qk.reshape(B, bs, H, D), qv.reshape(B, bs, H, D)], 0)
    return {
        "codes": codes.permute(0, 3, 1, 2, 4).contiguous(),
        "key_min": kmin, "key_scale": kscale,
        "value_min": vmin, "value_scale": vscale, "groups": groups,
    }


def dequant_bf16(q: torch.Tensor, scale: torch.Tensor, mn: torch.Tensor) -> torch.Tensor:
    """bf16 dequantization exactly as the reference computes it: the codes,
    scale and min are bf16 and each of ``q*scale`` and ``+min`` rounds to
    bf16 (kv_hadamard_quant.py:1431-1472)."""
    return q.to(torch.bfloat16) * scale.to(torch.bfloat16) + mn.to(torch.bfloat16)


def decompress_layer(codes: torch.Tensor, key_min: torch.Tensor, key_scale: torch.Tensor,
                     value_min: torch.Tensor, value_scale: torch.Tensor,
                     groups: list[list[int]], signs: Optional[torch.Tensor]) -> torch.Tensor:
    """Inverse of :func:`compress_layer` from heads-outer codes ``[2, H, B, bs, D]``.

    ``key_*`` are [H, D]; ``value_*`` are [G, rows].  Metadata is first
    rounded to fp16 (the wire precision) and then to bf16.  Returns bf16
    ``[2, B, bs, H, D]``.
    """
    _, H, B, bs, D = codes.shape
    rows = B * bs
    c = codes.permute(0, 2, 3, 1, 4).reshape(2, rows, H, D)
    kmin = key_min.to(torch.float16)
    ksc = key_scale.to(torch.float16)
    dk = dequant_bf16(c[0], ksc[None], kmin[None])
    dv = torch.empty((rows, H, D), dtype=torch.bfloat16)
    vmin = value_min.to(torch.float16)
    vsc = value_scale.to(torch.float16)
    for g, hs in enumerate(groups):
        dv[:, hs, :] = dequant_bf16(c[1][:, hs, :], vsc[g][:, None, None], vmin[g][:, None, None])
    out = []
    for d in (dk, dv):
        if signs is None:
            out.append(d)
        else:
            y = fwht_fp32(d.to(torch.float32)).to(torch.bfloat16)
            out.append(y * signs.to(torch.bfloat16))
    return torch.stack(out, 0).reshape(2, B, bs, H, D)


def error_metrics(ref: torch.Tensor, approx: torch.Tensor) -> dict:
    """rel-MSE (||a-r||^2/||r||^2), cosine similarity, max |a-r| in float64."""
    r = ref.to(torch.float64).flatten()
    a = approx.to(torch.float64).flatten()
    d = a - r
    rn = float((r * r).sum())
    an = float((a * a).sum())
    return {
        "rel_mse": float((d * d).sum()) / max(rn, 1e-300),
        "mse": float((d * d).mean()),
        "cosine": float((r * a).sum()) / max((rn * an) ** 0.5, 1e-300),
        "max_abs": float(d.abs().max()) if d.numel() else 0.0,
    }
