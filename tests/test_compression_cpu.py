"""CPU tests of the compression layer: signs, head masks, oracle math, the
lossless codecs (CPU implementation of the device stream format), the wire
envelope, the generic pipeline and the adapter's mode dispatch."""

import math

import pytest
import torch

from kvserve_hpdps_b200.compression import codec as C
from kvserve_hpdps_b200.compression import head_scores as HS
from kvserve_hpdps_b200.compression import oracle, signs
from kvserve_hpdps_b200.compression.config import CompressedKVData, validate_spec
from kvserve_hpdps_b200.compression.wire import build_wire, restore_from_wire
from kvserve_hpdps_b200.ops import kernels as K


def test_rademacher_signs_follow_the_seeding_rule():
    s = signs.rademacher_signs(layer_id=3, num_heads=4, head_dim=128, base_seed=0x3333)
    g = torch.Generator().manual_seed(0x3333 ^ (3 << 16) ^ 2)
    b = torch.randint(0, 2, (128,), generator=g, dtype=torch.int8).float() * 2 - 1
    assert torch.equal(s[2], b)
    assert set(s.unique().tolist()) == {-1.0, 1.0}
    from kvserve_hpdps_b200.compression.transformer import HadamardTransform
    ref_api = HadamardTransform(0x3333).get_rademacher_signs(3, 4, 128, torch.device("cpu"),
                                                              torch.float32)
    assert ref_api.shape == (1, 1, 4, 128) and torch.equal(ref_api[0, 0], s)


def test_fwht_is_orthonormal_and_self_inverse():
    x = torch.randn(5, 3, 128)
    y = signs.fwht_fp32(x)
    assert torch.allclose(signs.fwht_fp32(y), x, atol=1e-5)
    assert torch.allclose(y.norm(dim=-1), x.norm(dim=-1), rtol=1e-5)
    # non power-of-two head dims are transformed per power-of-two chunk
    z = torch.randn(2, 96)
    assert torch.allclose(signs.fwht_fp32(signs.fwht_fp32(z)), z, atol=1e-5)
    assert signs.pow2_chunks(100) == [64, 32, 4]


def test_head_masks_and_tp_slicing():
    scores = HS.get_scores_from_csv("Qwen2.5-7B-Instruct")
    assert scores.shape == (28, 4)
    m = HS.head_low_mask(scores, 0.3)
    assert int(m.sum()) == round(112 * 0.3)
    low_scores = scores[m]
    assert float(low_scores.max()) <= float(scores[~m].min())
    assert HS.slice_for_tp(m, 2, tp_rank=1, tp_size=2).shape == (28, 2)
    assert torch.equal(HS.slice_for_tp(m, 2, 1, 2), m[:, 2:4])
    with pytest.raises(ValueError):
        HS.slice_for_tp(m, 3)
    lm = HS.layer_low_mask(28)
    assert int(lm.sum()) == round(28 * 0.33) and bool(lm[-1]) and not bool(lm[0])
    assert bool(HS.layer_low_mask(1).all())  # round(0.33) == 0 marks every layer low
    assert HS.get_scores_from_csv("Meta-Llama-3-8B").shape == (32, 8)


def test_hybrid_plan_levels():
    p = HS.HybridPrecisionPlan(None, 4, "Qwen2.5-7B-Instruct", 0.8, 12, 8, 6, 4)
    kl, vl = p.key_levels, p.value_levels
    assert set(kl.unique().tolist()) <= {12.0, 6.0} and set(vl.unique().tolist()) <= {8.0, 4.0}
    assert int((kl == 6).sum()) == round(112 * 0.8)
    goh, heads = p.value_groups_for(0)
    assert sorted(h for g in heads for h in g) == [0, 1, 2, 3]
    q = HS.HybridPrecisionPlan(28, 4, "no-such-model", 0.8, 12, 8, 6, 4)
    assert bool((q.key_levels == 12).all())


def test_oracle_quantization_semantics():
    torch.manual_seed(0)
    kv = (torch.randn(2, 3, 16, 2, 128) * 2).to(torch.bfloat16)
    s = signs.rademacher_signs(1, 2, 128, 0x3333)
    r = oracle.compress_layer(kv, torch.tensor([12.0, 6.0]), torch.tensor([8.0, 4.0]), s)
    c = r["codes"]
    assert int(c[0, 0].max()) <= 11 and int(c[0, 1].max()) <= 5
    assert int(c[1, 0].max()) <= 7 and int(c[1, 1].max()) <= 3
    # key scale = range / (levels - 1) per (head, channel)
    kt = oracle.forward_transform(kv[0].reshape(-1, 2, 128), s)
    exp = torch.clamp(kt.amax(0) - kt.amin(0), min=1e-5) / torch.tensor([11.0, 5.0])[:, None]
    assert torch.allclose(r["key_scale"], exp)
    rec = oracle.decompress_layer(c, r["key_min"], r["key_scale"], r["value_min"],
                                  r["value_scale"], r["groups"], s)
    err = oracle.error_metrics(kv, rec)
    assert err["cosine"] > 0.85
    r2 = oracle.compress_layer(kv, torch.tensor([12.0, 6.0]), torch.tensor([8.0, 4.0]), s,
                               clamp_top=False)
    assert int(r2["codes"][0, 0].max()) <= 12


@pytest.mark.parametrize("n", [1, 513, 32768, 70001])
def test_cpu_rans_roundtrip(n):
    g = torch.Generator().manual_seed(n)
    p = torch.tensor([0.05, 0.45, 0.45, 0.05])
    x = torch.multinomial(p, n, replacement=True, generator=g).to(torch.uint8)
    s = K.rans_encode(x)
    assert torch.equal(K.rans_decode(s, n), x)
    if n > 10000:
        ent = -(p * p.log2()).sum().item()
        assert s.numel() * 8 / n < ent * 1.1 + 0.05


def test_cpu_rans_detects_corruption():
    x = torch.randint(0, 4, (40000,), dtype=torch.uint8)
    s = K.rans_encode(x).clone()
    bad = s.clone()
    bad[0] ^= 0xFF
    with pytest.raises(RuntimeError):
        K.rans_decode(bad, x.numel())
    with pytest.raises(RuntimeError):
        K.rans_decode(s, x.numel() + 1)


@pytest.mark.parametrize("codec", ["none", "rans", "bitpack"])
def test_codec_stage_roundtrip_cpu(codec):
    x = torch.randint(0, 11, (2, 4, 3, 16, 128), dtype=torch.uint8)
    enc = C.encode_bytes(x, codec)
    assert C.parse_header(enc) == (codec, x.numel())
    out = C.decode_bytes(enc).view(x.shape)
    assert torch.equal(out, x)
    if codec == "bitpack":
        assert enc.numel() < x.numel() * 0.6


def test_codec_name_mapping():
    assert C.resolve_codec("nvcomp", "ANS") == "rans"
    assert C.resolve_codec("nvcomp", "Bitcomp") == "bitpack"
    assert C.resolve_codec("lc") == "lc"
    with pytest.raises(ValueError):
        C.resolve_codec("nvcomp", "Brotli")
    codec = C.KVServeCodec(codec_type="nvcomp", nvcomp_algorithm="ANS", data_type="|u1")
    x = torch.randint(0, 5, (1000,), dtype=torch.uint8)
    assert torch.equal(codec.decode(0, codec.encode(0, x), "uint8", [1000], "cpu"), x)


@pytest.mark.parametrize("n", [1, 63, 16384, 16385, 70000])
def test_lc_codec_round_trip_and_format(n):
    """BIT_2 + RZE_1: lossless at any size; small codes compress, random
    bytes fall back to raw chunks; the stream names its codec."""
    from kvserve_hpdps_b200.compression import lc
    g = torch.Generator().manual_seed(n)
    x = torch.randint(0, 16, (n,), generator=g, dtype=torch.uint8)
    codec = C.LCCodec()
    enc = codec.encode(0, x)
    assert C.parse_header(enc) == ("lc", n)
    assert torch.equal(codec.decode(0, enc, "uint8", [n], "cpu"), x)
    if n >= 16384:
        assert enc.numel() < 0.7 * n
    r = torch.randint(0, 256, (n,), generator=g, dtype=torch.uint8)
    s = lc.encode(r.numpy())
    assert s.size <= lc.max_bytes(n)
    assert torch.equal(torch.from_numpy(lc.decode(s, n)), r)
    with pytest.raises(ValueError):
        lc.decode(s[:16], n)


def test_bitpack_matches_native_layout():
    codes = torch.randint(0, 8, (9, 128), dtype=torch.uint8)
    assert torch.equal(C._bitpack_rows(codes, 3), K.bitpack(codes, 3))
    assert torch.equal(C._bitunpack_rows(K.bitpack(codes, 3), 3), codes)


def test_wire_roundtrip_single_and_byte_chunks():
    body = torch.arange(1000, dtype=torch.int32)
    meta = {"request_id": "r1", "quantization_params": [
        {"key_meta": {"min_val": torch.randn(2, 3), "axis": "channel"},
         "value_meta": {"per_group_list": [{"head_idx": torch.tensor([0, 1])}]}}]}
    cd = CompressedKVData("r1", 3, body, meta, 4000, 4000)
    for max_chunk in (1 << 20, 1000):
        w = build_wire(cd, max_chunk)
        assert w.meta["body_mode"] == ("single" if max_chunk > 4000 else "byte_chunks")
        assert len(w.aux_tensors) == 2
        back = restore_from_wire(w)
        assert torch.equal(back.compressed_tensor, body)
        qp = back.metadata["quantization_params"][0]
        assert torch.equal(qp["key_meta"]["min_val"], meta["quantization_params"][0]["key_meta"]["min_val"])
        assert back.request_id == "r1"


def test_wire_chunked_and_rejects_tensor_outside_qparams():
    cd = CompressedKVData("r", 1, None, {"request_id": "r"}, 10, 4, is_chunked=True,
                          chunks=[torch.zeros(2, dtype=torch.uint8), torch.ones(2, dtype=torch.uint8)],
                          chunk_metadata=[{"quantization_params": [torch.zeros(1)]}, {}])
    w = build_wire(cd)
    back = restore_from_wire(w)
    assert back.is_chunked and len(back.chunks) == 2
    assert torch.equal(back.chunk_metadata[0]["quantization_params"][0], torch.zeros(1))
    bad = CompressedKVData("r", 1, torch.zeros(1), {"stray": torch.zeros(1)}, 1, 1)
    with pytest.raises(TypeError):
        build_wire(bad)


def test_validate_spec():
    validate_spec(None)
    validate_spec("default")
    validate_spec({"pipeline": ["quantizer", "codec"], "quantizer_config": {"hybrid_ratio": 0.5}})
    with pytest.raises(ValueError):
        validate_spec({"pipeline": ["compressor"]})
    with pytest.raises(ValueError):
        validate_spec({"quantizer_config": {"hybrid_ratio": 1.5}})
    with pytest.raises(ValueError):
        validate_spec({"mode": "controller"})


GENERIC = {"enabled": True, "pipeline": ["transformer", "quantizer", "codec"],
           "transformer_config": {"transform_type": "hadamard", "seed": 0x3333},
           "quantizer_config": {"model_name": "Qwen2.5-7B-Instruct", "hybrid_ratio": 0.3,
                                "high_key_max_value": 16, "high_value_max_value": 16,
                                "low_key_max_value": 12, "low_value_max_value": 12,
                                "axis_key": "token", "axis_value": "token", "split_type": "head"},
           "codec_config": {"codec_type": "nvcomp", "nvcomp_algorithm": "ANS"},
           "min_compress_size": 0}


def test_generic_pipeline_roundtrip_cpu():
    from kvserve_hpdps_b200.compression.manager import KVCompressionAdapter
    from kvserve_hpdps_b200.compression.pipeline_manager import CompressionManager
    ad = KVCompressionAdapter(GENERIC, num_kv_heads=4, head_size=128)
    assert isinstance(ad.manager, CompressionManager)
    x = torch.randn(3, 2, 2, 16, 4, 128).to(torch.bfloat16)
    c = ad.compress(x, "req")
    assert c is not None and c.compressed_size < x.numel() * 2 / 3
    y = ad.decompress(c)
    assert y.shape == x.shape
    cos = torch.nn.functional.cosine_similarity(x.float().flatten(), y.float().flatten(), dim=0)
    assert float(cos) > 0.97


def test_generic_quantizer_matches_reference_formula():
    from kvserve_hpdps_b200.compression.quantizer import dequantize, quantize
    x = torch.randn(4, 16, 2, 128).to(torch.bfloat16)
    q, m = quantize(12, x, "channel")
    mx = x.amax(dim=(0, 1), keepdim=True)
    mn = x.amin(dim=(0, 1), keepdim=True)
    sc = (mx - mn).clamp(min=1e-5) / 11
    exp = ((x - mn) / sc).round().clamp(0, 12).to(torch.uint8)
    assert torch.equal(q, exp)
    assert torch.equal(dequantize(q, m), q.to(torch.bfloat16) * sc + mn)


def test_adapter_routes_compatible_custom_pipelines_to_fused():
    from kvserve_hpdps_b200.compression.fused_manager import FusedCompressionManager
    from kvserve_hpdps_b200.compression.manager import (KVCompressionAdapter, add_sentinel,
                                                        is_compressed_layer_names, strip_sentinel)
    spec = dict(GENERIC)
    spec["quantizer_config"] = dict(GENERIC["quantizer_config"], axis_key="channel")
    ad = KVCompressionAdapter(spec, num_kv_heads=4, head_size=128)
    assert isinstance(ad.manager, FusedCompressionManager)
    assert ad.supports_overlap() and ad.supports_paged()
    ad2 = KVCompressionAdapter("default", num_kv_heads=4, head_size=128,
                               model_name="Qwen2.5-7B-Instruct")
    assert ad2.manager.base_seed == 0x3333 and ad2.manager.codec == "rans"
    names = add_sentinel(["a", "b"])
    assert is_compressed_layer_names(names) and strip_sentinel(names) == ["a", "b"]


def test_cpu_roundtrip_example_runs(capsys):
    """The CPU-only round trip example (quantizer + codec fallback path) at a
    reduced size: prints a compression ratio above 2 and a close
    reconstruction."""
    import importlib.util
    import json
    import os
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                        "examples", "cpu_roundtrip.py")
    spec = importlib.util.spec_from_file_location("cpu_roundtrip", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.main(["--layers", "2", "--tokens", "256"]) == 0
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["compression_ratio"] > 2.0 and line["cosine"] > 0.98
    assert mod.main(["--layers", "2", "--tokens", "256", "--mode", "default"]) == 0
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["mode"] == "default" and line["compression_ratio"] > 3.0 and line["cosine"] > 0.9


def test_split_helpers_match_the_quantizer_layout():
    """head_split / head_restore / head_reconstruct and the layer forms
    invert each other, and the generic quantizer packs LOW heads first in
    exactly the order head_split gives."""
    from kvserve_hpdps_b200.compression import split as S
    from kvserve_hpdps_b200.compression.quantizer import KVServeQuantizer
    x = torch.randn(3, 16, 4, 128).to(torch.bfloat16)
    mask = torch.tensor([[True, False, True, False], [False, False, False, False]])
    low, high = S.head_split(0, x, mask)
    assert torch.equal(low, x[:, :, [0, 2]]) and torch.equal(high, x[:, :, [1, 3]])
    packed = torch.cat([low, high], dim=2)
    lo2, hi2 = S.head_restore(0, packed, mask)
    assert torch.equal(lo2, low) and torch.equal(hi2, high)
    assert torch.equal(S.head_reconstruct(0, lo2, hi2, mask), x)
    lo3, hi3 = S.head_split(1, x, mask)  # no LOW head in layer 1
    assert lo3.shape[2] == 0 and torch.equal(S.head_reconstruct(1, lo3, hi3, mask), x)
    lm = torch.tensor([False, True])
    a, b = S.layer_split(1, x, lm)
    assert a is x and b.numel() == 0 and S.layer_reconstruct(1, a, b, lm) is x
    a, b = S.layer_restore(0, x, lm)
    assert a.numel() == 0 and b is x and S.layer_reconstruct(0, a, b, lm) is x
    for bad in (None, mask.float()):
        with pytest.raises(ValueError):
            S.head_split(0, x, bad)
        with pytest.raises(ValueError):
            S.layer_split(0, x, None if bad is None else lm.float())
    qz = KVServeQuantizer(model_name="Qwen2.5-7B-Instruct", hybrid_ratio=0.5,
                          axis_key="token", axis_value="token")
    m = qz.head_scores_mask
    layer = next(i for i in range(m.shape[0]) if 0 < int(m[i].sum()) < m.shape[1])
    kv = torch.randn(2, 3, 16, m.shape[1], 128).to(torch.bfloat16)
    q, meta = qz.quantize(layer, kv)
    lo_k, hi_k = S.head_restore(layer, q[0], m)
    from kvserve_hpdps_b200.compression.quantizer import quantize
    want_lo, _ = quantize(qz.low_key_max_value, S.head_split(layer, kv[0], m)[0], "token")
    want_hi, _ = quantize(qz.high_key_max_value, S.head_split(layer, kv[0], m)[1], "token")
    assert torch.equal(lo_k, want_lo) and torch.equal(hi_k, want_hi)


def test_reference_module_paths_alias_this_package():
    """With the compat directory on PYTHONPATH every reference module path
    imports (in a child process, so the alias never meets a real
    ``kvserve_v1`` here) and exposes the same objects as this package."""
    import os
    import subprocess
    import sys

    import kvserve_hpdps_b200.compat as compat
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = "\n".join([
        "import importlib, kvserve_v1",
        "from kvserve_v1 import _ALIASES",
        "for a in _ALIASES: importlib.import_module('kvserve_v1.' + a)",
        "from kvserve_v1.connector.compressed_kv_connector import CompressedKVConnector as A",
        "from kvserve_hpdps_b200.connector.compressed_kv_connector import "
        "CompressedKVConnector as B",
        "assert A is B and kvserve_v1.CompressedKVConnector is B",
        "from kvserve_v1.compression.tilelang_manager import TileLangCompressionManager as T",
        "from kvserve_hpdps_b200.compression.fused_manager import FusedCompressionManager as F",
        "assert T is F",
        "from kvserve_v1.compression.quantizer.split_func import head_restore",
        "from kvserve_v1.compression.codec.nvcomp_func import nvCOMPCodec",
        "from kvserve_v1.compression.controller.analytical_model import AnalyticalModel",
        "from kvserve_v1.compression.compression_manager import DEFAULT_COMPRESSION_CONFIG",
        "import kvserve_v1.compression.wire as w, kvserve_hpdps_b200.compression.wire as w2",
        "assert w.build_wire is w2.build_wire and w._unpack is w2._unpack",
        "from kvserve_v1.offline_search.src.cache.cache_utils import CustomCache, HadamardTransform",
        "from kvserve_hpdps_b200.offline import caches as OC",
        "assert CustomCache is OC.CustomCache and HadamardTransform is OC.HeadHadamard",
        "from kvserve_v1.compression.transformer import HadamardTransform as RT",
        "from kvserve_hpdps_b200.compression.transformer import HadamardTransform as CT",
        "assert RT is CT",
        "from kvserve_v1.offline_search.duo_config.duo_config import duo_attention_on_the_fly as D",
        "from kvserve_hpdps_b200.offline.duo_scores import duo_scores_on_the_fly",
        "assert D is duo_scores_on_the_fly",
        "from kvserve_v1.offline_search.evaluation.param_search.acc_evaluator import "
        "AccuracyEvaluator as AE",
        "from kvserve_v1.offline_search.evaluation.param_search.cr_evaluator import "
        "CompressionEvaluator as CE",
        "from kvserve_hpdps_b200.offline import param_search as PS",
        "assert AE is PS.AccuracyEvaluator and CE is PS.CompressionEvaluator",
        "print('ALIASES', len(_ALIASES))",
    ])
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([compat.path(), root]))
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=300, cwd=str(root))
    assert out.returncode == 0, out.stderr[-2000:]
    assert "ALIASES" in out.stdout


def test_codec_ops_are_registered_torch_operators():
    """torch.ops.kvserve codecs: round trip on CPU, fake (meta) shapes with a
    data-dependent stream length, and torch.library.opcheck."""
    from torch._subclasses.fake_tensor import FakeTensorMode
    from torch.fx.experimental.symbolic_shapes import ShapeEnv

    import kvserve_hpdps_b200.ops.library  # noqa: F401 - registers the ops
    x = torch.randint(0, 12, (70000,), dtype=torch.uint8)
    ops = torch.ops.kvserve
    for enc, dec in ((ops.rans_encode, ops.rans_decode), (ops.lc_encode, ops.lc_decode)):
        s = enc(x)
        assert s.dtype == torch.uint8 and s.numel() < x.numel()
        assert torch.equal(dec(s, x.numel()), x)
        torch.library.opcheck(enc.default, (x,))
        torch.library.opcheck(dec.default, (s, x.numel()))
    with FakeTensorMode(shape_env=ShapeEnv()):
        fs = ops.rans_encode(torch.empty(1000, dtype=torch.uint8))
        assert fs.dtype == torch.uint8 and not isinstance(fs.shape[0], int)
        assert ops.lc_decode(fs, 1000).shape == (1000,)


@pytest.mark.parametrize("split_type", ["head", "layer"])
@pytest.mark.parametrize("axes", [("channel", "token"), ("token", "token"), ("tensor", "channel")])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_quantize_into_matches_quantize(split_type, axes, dtype):
    """The generic pipeline's direct-write quantizer gives the same codes (in
    the heads-outer layout) and metadata as quantize + permute."""
    from kvserve_hpdps_b200.compression.quantizer import KVServeQuantizer
    qz = KVServeQuantizer(model_name="Qwen2.5-7B-Instruct", hybrid_ratio=0.5,
                          high_key_max_value=16, high_value_max_value=12,
                          low_key_max_value=8, low_value_max_value=6,
                          axis_key=axes[0], axis_value=axes[1], split_type=split_type)
    g = torch.Generator().manual_seed(3)
    for layer in (0, 3, 27):  # layer split: 27 is LOW, 0 and 3 HIGH
        x = (torch.randn(2, 5, 16, 4, 128, generator=g) * 3).to(dtype)
        q, m = qz.quantize(layer, x)
        out = torch.full((2, 4, 5, 16, 128), 255, dtype=torch.uint8)
        m2 = qz.quantize_into(layer, x, out)
        assert torch.equal(out, q.permute(0, 3, 1, 2, 4))
        assert list(m2) == list(m)
        for k in m:
            if isinstance(m[k], dict):
                for f in m[k]:
                    a, b = m[k][f], m2[k][f]
                    assert (a is None and b is None) or (torch.is_tensor(a) and torch.equal(a, b)) \
                        or a == b, (k, f)
            else:
                assert m[k] == m2[k]
        # and back: the direct-write dequantizer equals dequantize
        codes = q  # [2, blocks, block_size, heads, dim], LOW heads first
        back = torch.full((2, 5, 16, 4, 128), float("nan"), dtype=dtype)
        qz.dequantize_into(layer, codes, m, back)
        assert torch.equal(back, qz.dequantize(layer, codes, m))


def test_cpu_rans_threads_and_corrupt_streams(monkeypatch):
    """The CPU coder runs chunks on host threads: the stream is the same
    bytes for one thread and for many, and corrupt or truncated streams are
    rejected with an error (every read and write is bounds-checked)."""
    g = torch.Generator().manual_seed(5)
    x = torch.randint(0, 6, (300000,), dtype=torch.uint8, generator=g)
    x[40000:72768] = torch.randint(0, 256, (32768,), dtype=torch.uint8, generator=g)  # raw chunk
    many = K.rans_encode(x)
    monkeypatch.setenv("KVS_CPU_THREADS", "1")
    one = K.rans_encode(x)
    assert torch.equal(one, many)
    assert torch.equal(K.rans_decode(one, x.numel()), x)
    monkeypatch.delenv("KVS_CPU_THREADS")
    rejected = 0
    for i in range(300):
        bad = many.clone()
        if i % 3 == 0:
            bad = bad[:int(torch.randint(0, bad.numel(), (1,), generator=g))].clone()
        else:
            pos = torch.randint(0, 96 if i % 3 == 1 else bad.numel(), (4,), generator=g)
            bad[pos] ^= torch.randint(1, 256, (4,), dtype=torch.uint8, generator=g)
        try:
            out = K.rans_decode(bad, x.numel())
            assert out.numel() == x.numel()
        except RuntimeError:
            rejected += 1
    assert rejected > 100


def test_native_cpu_lc_matches_reference_and_rejects_corruption():
    """The native CPU LC coder writes the numpy reference's stream byte for
    byte (codes, raw chunks, tails) and rejects corrupt streams."""
    from kvserve_hpdps_b200.compression import lc
    g = torch.Generator().manual_seed(9)
    x = torch.randint(0, 6, (90001,), dtype=torch.uint8, generator=g)
    x[20000:40000] = torch.randint(0, 256, (20000,), dtype=torch.uint8, generator=g)
    s = K.lc_encode(x)
    assert torch.equal(s, torch.from_numpy(lc.encode(x.numpy())))
    assert torch.equal(K.lc_decode(s, x.numel()), x)
    assert torch.equal(torch.from_numpy(lc.decode(s.numpy(), x.numel())), x)
    rejected = 0
    for i in range(200):
        bad = s[:int(torch.randint(0, s.numel(), (1,), generator=g))].clone() if i % 2 else s.clone()
        if i % 2 == 0:
            pos = torch.randint(0, bad.numel(), (3,), generator=g)
            bad[pos] ^= torch.randint(1, 256, (3,), dtype=torch.uint8, generator=g)
        try:
            assert K.lc_decode(bad, x.numel()).numel() == x.numel()
        except ValueError:
            rejected += 1
    assert rejected >= 100


def test_default_mode_falls_back_to_the_generic_pipeline_on_cpu():
    """Default mode builds the fused manager; a CPU tensor goes through its
    generic twin (same quantizer settings, Hadamard seed and codec) instead
    of failing on CUDA initialisation, and the message decodes back."""
    from kvserve_hpdps_b200.compression.manager import KVCompressionAdapter
    ad = KVCompressionAdapter("default", 4, 128, model_name="Qwen2.5-7B-Instruct", num_layers=28)
    assert ad.manager.backend == "kvs_fused"
    g = torch.Generator().manual_seed(2)
    x = torch.randn(28, 2, 3, 16, 4, 128, generator=g)
    x[:, 0, ..., :4] *= 12
    x = x.to(torch.bfloat16)
    cd = ad.compress(x, "r1")
    assert cd.metadata["backend"] == "generic" and cd.metadata.get("transformer_applied")
    assert cd.original_size / cd.compressed_size > 3
    mgr, conf = ad._cpu_fallback()
    assert conf.quantizer_config["hybrid_ratio"] == ad.manager.quantizer_config["hybrid_ratio"]
    assert mgr.transformer.seed == 0x3333
    out = ad.decompress(cd)
    assert out.shape == x.shape
    cos = torch.nn.functional.cosine_similarity(out.float().flatten(), x.float().flatten(), dim=0)
    assert float(cos) > 0.95


def test_nvcomp_names_map_to_own_coders_and_say_so():
    """The reference's nvCOMP algorithm names resolve to this framework's own
    coders; an unknown name is rejected by the spec validator with the
    mapping in the error text."""
    from kvserve_hpdps_b200.compression.codec import resolve_codec
    from kvserve_hpdps_b200.compression.config import validate_spec
    assert resolve_codec("nvcomp", "Bitcomp") == "bitpack"
    assert {resolve_codec("nvcomp", a) for a in
            ("ANS", "Cascaded", "Deflate", "GDeflate", "LZ4", "Zstd")} == {"rans"}
    spec = {"enabled": True, "pipeline": ["quantizer", "codec"],
            "codec_config": {"codec_type": "nvcomp", "nvcomp_algorithm": "Snappy"}}
    with pytest.raises(ValueError, match="LZ4, Zstd -> rans"):
        validate_spec(spec)
    spec["codec_config"]["nvcomp_algorithm"] = "LZ4"
    validate_spec(spec)
