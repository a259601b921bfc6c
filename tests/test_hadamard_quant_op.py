"""Reference-compatible op API (KVHadamardQuantOp): the per-row legacy form
on CPU, compress_v3 / decompress_v3 on the GPU against the fused manager."""

import pytest
import torch

from kvserve_hpdps_b200.compression.signs import rademacher_signs
from kvserve_hpdps_b200.ops.hadamard_quant_op import KVHadamardQuantOp, make_rademacher_signs


def _kv(shape, seed=0, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g).to(torch.bfloat16).to(device)


def test_signs_match_reference_seeding():
    s = make_rademacher_signs(3, 4, 128, device="cpu", dtype=torch.float32)
    assert torch.equal(s, rademacher_signs(3, 4, 128, 0xC0FEBABE))


@pytest.mark.parametrize("quant_type", ["absmax", "minmax"])
def test_legacy_per_row_round_trip(quant_type):
    op = KVHadamardQuantOp(num_heads=4, head_dim=128, quant_type=quant_type,
                           model_name="Qwen2.5-7B-Instruct", hybrid_ratio=0.5)
    kv = _kv((3, 16, 4, 128))
    q, meta = op.compress(kv, layer_id=2, is_key=True)
    assert q.shape == kv.shape and q.dtype == torch.uint8
    m = meta["max_vals"]
    assert int(q.max()) <= int(2 * m.max() if quant_type == "absmax" else m.max())
    out = op.decompress(q, meta, layer_id=2)
    cos = torch.nn.functional.cosine_similarity(out.float().flatten(), kv.float().flatten(), dim=0)
    assert float(cos) > 0.98
    with pytest.raises(ValueError):
        KVHadamardQuantOp(quant_type="zip")


@pytest.mark.gpu
def test_compress_v3_matches_fused_round_trip():
    op = KVHadamardQuantOp(num_heads=4, head_dim=128, model_name="Qwen2.5-7B-Instruct",
                           hybrid_ratio=0.5, high_key_max_value=16, high_value_max_value=16,
                           low_key_max_value=8, low_value_max_value=8, num_layers=28)
    x = _kv((2, 5, 16, 4, 128), seed=3, device="cuda")
    q, meta = op.compress_v3(x, 7)
    assert q.shape == x.shape and q.dtype == torch.uint8
    assert meta["key_meta"]["min_val"].shape == (4, 128)
    heads = sorted(int(h) for g in meta["value_meta"]["per_group_meta"].values()
                   for h in g["head_idx"])
    assert heads == [0, 1, 2, 3]
    for lev, g in meta["value_meta"]["per_group_meta"].items():
        for h in g["head_idx"].tolist():
            assert float(meta["value_max_vals"][h]) == lev
    out = op.decompress_v3(q, meta, 7)
    ref = torch.empty_like(x)
    batch = op._mgr.quantize_paged([x], [7], [(list(range(5)), 80)])
    op._mgr.dequantize_paged(batch, [ref])
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    cos = torch.nn.functional.cosine_similarity(out.float().flatten(), x.float().flatten(), dim=0)
    assert float(cos) > 0.95
