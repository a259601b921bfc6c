"""Property-based checks of the CPU codecs (rANS, LC, bit-pack) through the
public container API: every byte string round-trips, for any size and
symbol distribution; a corrupted stream is rejected or decodes to some
bytes, never crashes the process."""

import pytest
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from kvserve_hpdps_b200.compression.codec import decode_bytes, encode_bytes

CODECS = ["rans", "lc", "none"]


@st.composite
def byte_strings(draw):
    n = draw(st.integers(min_value=1, max_value=70000))
    kind = draw(st.sampled_from(["uniform", "skewed", "constant", "sparse", "nibbles"]))
    g = torch.Generator().manual_seed(draw(st.integers(0, 2 ** 31 - 1)))
    if kind == "uniform":
        x = torch.randint(0, 256, (n,), generator=g)
    elif kind == "skewed":
        x = torch.clamp(torch.randn(n, generator=g).abs() * draw(st.floats(0.1, 40.0)), 0, 255)
    elif kind == "constant":
        x = torch.full((n,), draw(st.integers(0, 255)))
    elif kind == "sparse":
        x = torch.randint(0, 256, (n,), generator=g) * (torch.rand(n, generator=g) < 0.03)
    else:
        x = torch.randint(0, 16, (n,), generator=g)
    return x.to(torch.uint8)


@pytest.mark.parametrize("codec", CODECS)
@settings(max_examples=40, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(data=byte_strings())
def test_round_trip(codec, data):
    stream = encode_bytes(data, codec)
    assert torch.equal(decode_bytes(stream), data)


@pytest.mark.parametrize("codec", ["rans", "lc"])
@settings(max_examples=40, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(data=byte_strings(), where=st.floats(0.0, 1.0), flip=st.integers(1, 255))
def test_corrupted_stream_never_crashes(codec, data, where, flip):
    stream = encode_bytes(data, codec).clone()
    i = 16 + int(where * (stream.numel() - 17))  # inside the coded body
    stream[i] ^= flip
    try:
        out = decode_bytes(stream)
    except (RuntimeError, ValueError):
        return  # rejected
    assert out.dtype == torch.uint8 and out.numel() == data.numel()
