"""Wire-level interoperability with the reference implementation (installed
in ``baseline/_ref``; skipped without it): a message compressed by either
framework's quantizer pipeline and carried in its wire envelope is restored
and decompressed by the other into the same KV.  Runs in a child process so
that the reference package never enters this test session."""

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")

CODE = r"""
import sys
sys.path.insert(0, ROOT)
sys.path.insert(0, REF)
import torch
from kvserve_hpdps_b200.compression import wire as OW
from kvserve_hpdps_b200.compression.manager import KVCompressionAdapter as Ours
from kvserve_v1.compression import wire as RW
from kvserve_v1.compression.manager import KVCompressionAdapter as Ref
L, T, H, D = 4, 256, 4, 128
g = torch.Generator().manual_seed(0)
x = torch.randn((L, 2, 1, T, H, D), generator=g)
x[:, 0, ..., :4] *= 12
x = x.to(torch.bfloat16)
qc = {"model_name": "Qwen2.5-7B-Instruct", "hybrid_ratio": 0.3, "high_key_max_value": 16,
      "high_value_max_value": 16, "low_key_max_value": 12, "low_value_max_value": 16,
      "axis_key": "channel", "axis_value": "token", "split_type": "head"}
ours = Ours({"enabled": True, "pipeline": ["quantizer"], "backend": "generic",
             "quantizer_config": qc, "min_compress_size": 0}, H, D,
            model_name="Qwen2.5-7B-Instruct", num_layers=28)
ref = Ref({"enabled": True, "pipeline": ["quantizer"], "quantizer_config": qc}, H, D,
          model_name="Qwen2.5-7B-Instruct")
cd = ours.compress(x, "a")
w = OW.build_wire(cd, 512 << 20)
by_ref = ref.decompress(RW.restore_from_wire(RW.CompressedWire(w.meta, w.body_chunks,
                                                               w.aux_tensors)))
assert torch.equal(by_ref.reshape(-1), ours.decompress(cd).reshape(-1)), "ours -> reference"
rc = ref.compress(x, "b")
rw = RW.build_wire(rc, 512 << 20)
by_ours = ours.decompress(OW.restore_from_wire(OW.CompressedWire(rw.meta, rw.body_chunks,
                                                                 rw.aux_tensors)))
assert torch.equal(by_ours.reshape(-1), ref.decompress(rc).reshape(-1)), "reference -> ours"
assert torch.equal(cd.compressed_tensor.view(torch.uint8).reshape(-1),
                   rc.compressed_tensor.view(torch.uint8).reshape(-1)), "bodies"
print("INTEROP OK")
"""


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "kvserve_v1")),
                    reason="reference not installed in baseline/_ref")
def test_wire_messages_cross_between_the_frameworks():
    code = CODE.replace("ROOT", repr(ROOT)).replace("REF", repr(REF))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=600, cwd="/tmp" if os.path.isdir("/tmp") else ROOT)
    assert out.returncode == 0 and "INTEROP OK" in out.stdout, out.stderr[-3000:]
