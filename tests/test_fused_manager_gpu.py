"""Grouped multi-request messages of the fused manager on the GPU: packed
metadata layout, wire round trip, whole-message and member-subset decode,
and decode of the per-item metadata layout."""

import pytest
import torch

from kvserve_hpdps_b200.compression.fused_manager import FusedCompressionManager
from kvserve_hpdps_b200.compression.wire import build_wire, restore_from_wire
from kvserve_hpdps_b200.models.synthetic import gather_request, paged_workload

pytestmark = pytest.mark.gpu

QC = {"model_name": "Qwen2.5-7B-Instruct", "hybrid_ratio": 0.8, "high_key_max_value": 12,
      "high_value_max_value": 8, "low_key_max_value": 6, "low_value_max_value": 4}


def _setup(L=4, tokens=(300, 1024, 17)):
    H = 4
    src = paged_workload(L, list(tokens), H, device="cuda", seed=5)
    dst = paged_workload(L, list(tokens), H, device="cuda", seed=9, fill=False)
    mgr = FusedCompressionManager(H, 128, QC, {"codec_type": "rans"}, num_layers=28)
    reqs = [(b, t) for b, t in zip(src.block_ids, tokens)]
    dreqs = [(b, t) for b, t in zip(dst.block_ids, tokens)]
    return src, dst, mgr, reqs, dreqs


def _expected(mgr, src, reqs, L):
    """Reconstruction through the plain paged round trip (no message)."""
    batch = mgr.quantize_paged([src.cache[l] for l in range(L)], list(range(L)), reqs)
    ref = torch.zeros_like(src.cache)
    mgr.dequantize_paged(batch, [ref[l] for l in range(L)])
    return ref


def _to_items_layout(mgr, cd):
    """Rewrite a packed message into the per-item metadata layout."""
    md = dict(cd.metadata)
    plans = mgr._message_plans(md)
    _, moffs = mgr._message_offsets(md, plans)
    R = len(md["member_tids"])
    bs = md["block_size"]
    meta = md["quantization_params"][0]
    qp = []
    for i, off in enumerate(moffs):
        plan = plans[i // R]
        qp.append(mgr.canon_meta(meta, off, plan, md["member_blocks"][i % R] * bs))
    md["layout"] = "items"
    md["quantization_params"] = qp
    md.pop("layer_plans")
    return type(cd)(request_id=cd.request_id, layer_id=cd.layer_id,
                    compressed_tensor=cd.compressed_tensor, metadata=md,
                    original_size=cd.original_size, compressed_size=cd.compressed_size)


def test_grouped_message_round_trip_and_members():
    L = 4
    src, dst, mgr, reqs, dreqs = _setup(L)
    ref = _expected(mgr, src, reqs, L)
    cd = mgr.compress_paged_requests([src.cache[l] for l in range(L)], list(range(L)), reqs,
                                     member_tids=["a", "b", "c"])
    assert cd.metadata["layout"] == "items_packed"
    assert len(cd.metadata["quantization_params"]) == 1
    wire = build_wire(cd)
    assert len(wire.aux_tensors) == 1  # all items' metadata in one tensor
    back = restore_from_wire(wire)
    for variant in (back, _to_items_layout(mgr, back)):
        dst.cache.zero_()
        mgr.decompress_paged_requests(variant, [dst.cache[l] for l in range(L)], dreqs)
        torch.cuda.synchronize()
        for (sb, t), (db, _) in zip(reqs, dreqs):
            for l in range(L):
                a = gather_request(ref[l], sb).view(2, -1, 4, 128)[:, :t]
                b = gather_request(dst.cache[l], db).view(2, -1, 4, 128)[:, :t]
                assert torch.equal(a, b)
        # members 0 and 2 only
        dst.cache.zero_()
        mgr.decompress_members(variant, [dst.cache[l] for l in range(L)],
                               {0: dreqs[0][0], 2: dreqs[2][0]})
        torch.cuda.synchronize()
        for m in (0, 2):
            (sb, t), (db, _) = reqs[m], dreqs[m]
            for l in range(L):
                a = gather_request(ref[l], sb).view(2, -1, 4, 128)[:, :t]
                b = gather_request(dst.cache[l], db).view(2, -1, 4, 128)[:, :t]
                assert torch.equal(a, b)
        untouched = gather_request(dst.cache[0], dreqs[1][0])
        assert int(untouched.abs().sum()) == 0


@pytest.mark.parametrize("codec", ["lc", "bitpack", "none"])
def test_paged_message_round_trip_other_codecs(codec):
    """The grouped paged message with the LC, bitpack and raw stream codecs
    reconstructs what the plain paged round trip reconstructs."""
    L = 2
    src, dst, _, reqs, dreqs = _setup(L)
    mgr = FusedCompressionManager(4, 128, QC, {"codec_type": codec}, num_layers=28)
    ref = _expected(mgr, src, reqs, L)
    cd = mgr.compress_paged_requests([src.cache[l] for l in range(L)], list(range(L)), reqs,
                                     member_tids=["a", "b", "c"])
    back = restore_from_wire(build_wire(cd))
    mgr.decompress_paged_requests(back, [dst.cache[l] for l in range(L)], dreqs)
    torch.cuda.synchronize()
    for (sb, t), (db, _) in zip(reqs, dreqs):
        for l in range(L):
            a = gather_request(ref[l], sb).view(2, -1, 4, 128)[:, :t]
            b = gather_request(dst.cache[l], db).view(2, -1, 4, 128)[:, :t]
            assert torch.equal(a, b)


@pytest.mark.parametrize("symbol_bits", [4, 8])
def test_dense_and_layer_group_apis_match_paged_round_trip(symbol_bits):
    """The reference-compatible dense APIs (whole request, per-layer groups of
    several requests, chunked layers) reconstruct exactly what the paged
    round trip reconstructs, with nibble or byte codes under the codec."""
    L, H, B, bs = 3, 4, 6, 16
    mgr = FusedCompressionManager(H, 128, QC, {"codec_type": "rans", "symbol_bits": symbol_bits},
                                  num_layers=28)
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn((L, 2, B, bs, H, 128), generator=g, device="cuda").to(torch.bfloat16)
    x[:, 0, :, :, :, :3] *= 12
    # reference: paged round trip of the same data
    ref = torch.empty_like(x)
    batch = mgr.quantize_paged([x[l] for l in range(L)], list(range(L)), [(list(range(B)), B * bs)])
    mgr.dequantize_paged(batch, [ref[l] for l in range(L)])
    # whole request
    cd = mgr.compress_all_layers(x, "r")
    out = mgr.decompress_all_layers(cd)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    # one layer, two members in one codec call
    q0, m0 = mgr.compress_quant_layer(x[1], 1)
    q1, m1 = mgr.compress_quant_layer(x[1, :, :2].contiguous(), 1)
    grp = mgr.finalize_layer_group([q0, q1], [m0, m1], ["a", "b"], [B, 2], 1)
    outs = dict(mgr.decompress_layer_group(grp))
    torch.cuda.synchronize()
    assert torch.equal(outs["a"], ref[1])
    # chunked per-layer bodies
    chunks, metas = zip(*[mgr.compress_layer_full(x[l], l) for l in range(L)])
    cdc = mgr.finalize_chunked(list(chunks), list(metas), "r", "bfloat16", list(x.shape))
    outc = mgr.decompress_all_layers(cdc)
    torch.cuda.synchronize()
    assert torch.equal(outc, ref)
