"""User pipeline components selected by name (``*_impl``) on the CPU."""

import pytest
import torch

from kvserve_hpdps_b200.compression.components import (Quantizer, register_component,
                                                       resolve_component)
from kvserve_hpdps_b200.compression.config import validate_spec
from kvserve_hpdps_b200.compression.manager import KVCompressionAdapter, use_fused
from kvserve_hpdps_b200.compression.wire import build_wire, restore_from_wire


class PassThrough:
    """The custom quantizer of the reference's connector README: codes are
    the input itself, the metadata names its dtype."""

    def __init__(self, **kwargs):
        self.scale = kwargs.get("scale", 1.0)

    def update_params(self, **kwargs):
        self.scale = kwargs.get("scale", self.scale)

    def quantize(self, layer_id, tensor, **kwargs):
        return tensor, {"original_dtype": str(tensor.dtype).replace("torch.", "")}

    def dequantize(self, layer_id, tensor, meta, **kwargs):
        return tensor


class Int8Quantizer(Quantizer):
    """Symmetric per-layer int8 codes with an fp32 scale in the metadata."""

    def quantize(self, layer_id, tensor, **kwargs):
        s = tensor.float().abs().amax().clamp(min=1e-8) / 127
        return (tensor.float() / s).round().to(torch.int8), {"scale": s.reshape(1)}

    def dequantize(self, layer_id, tensor, meta, **kwargs):
        return tensor.float() * meta["scale"]


class Negate:
    def transform(self, layer_id, tensor, **kwargs):
        return -tensor

    def inverse(self, layer_id, tensor, **kwargs):
        return -tensor

    def update_params(self, **kwargs):
        pass


def _kv(seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(2, 2, 3, 16, 4, 128, generator=g).to(torch.bfloat16)


def _round_trip(spec, kv):
    ad = KVCompressionAdapter(spec, 4, 128)
    cd = ad.compress(kv, "r")
    w = build_wire(cd)
    return ad.decompress(restore_from_wire(w)), w.nbytes


def test_registered_quantizer_round_trips_exactly():
    register_component("quantizer", "my_quantizer", PassThrough)
    spec = {"enabled": True, "pipeline": ["quantizer", "codec"], "quantizer_impl": "my_quantizer",
            "quantizer_config": {"scale": 1.0}, "codec_config": {"codec_type": "rans"}}
    validate_spec(spec)
    assert not use_fused(spec)
    kv = _kv()
    out, nbytes = _round_trip(spec, kv)
    assert torch.equal(out, kv) and nbytes > 0


def test_import_path_components_with_metadata_tensors():
    register_component("transformer", "negate", Negate)
    spec = {"enabled": True, "pipeline": ["transformer", "quantizer", "codec"],
            "transformer_impl": "negate",
            "quantizer_impl": f"{__name__}:Int8Quantizer",
            "quantizer_config": {}, "codec_config": {"codec_type": "rans"}}
    kv = _kv(1)
    out, nbytes = _round_trip(spec, kv)
    cos = torch.nn.functional.cosine_similarity(out.float().flatten(), kv.float().flatten(), 0)
    assert float(cos) > 0.99 and nbytes < kv.numel() * 2 * 0.6  # int8 codes + rANS
    assert resolve_component("quantizer", "kvserve_hpdps_b200.compression.quantizer."
                                          "KVServeQuantizer").__name__ == "KVServeQuantizer"


def test_bad_component_names_are_rejected():
    with pytest.raises(ValueError, match="unknown quantizer_impl"):
        resolve_component("quantizer", "nope")
    with pytest.raises(ValueError, match="cannot be imported"):
        resolve_component("codec", "no_such_module:Codec")
    with pytest.raises(TypeError, match="lacks"):
        register_component("codec", "bad", PassThrough)
    with pytest.raises(ValueError, match="kind"):
        register_component("scheduler", "x", PassThrough)
    with pytest.raises(ValueError, match="unknown quantizer_impl"):
        validate_spec({"pipeline": ["quantizer"], "quantizer_impl": "nope"})
    assert resolve_component("quantizer", None) is None
