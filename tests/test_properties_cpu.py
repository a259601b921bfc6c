"""Property-based checks on the CPU: the codecs (rANS, LC) through the
public container API (every byte string round-trips, for any size and
symbol distribution; a corrupted stream is rejected or decodes to some
bytes, never crashes the process), the wire envelope over arbitrary
metadata, the ring allocator's no-overlap invariant and the search
driver's invariants."""

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
@settings(max_examples=40, deadline=None, derandomize=True, suppress_health_check=[HealthCheck.too_slow])
@given(data=byte_strings())
def test_round_trip(codec, data):
    stream = encode_bytes(data, codec)
    assert torch.equal(decode_bytes(stream), data)


@pytest.mark.parametrize("codec", ["rans", "lc"])
@settings(max_examples=40, deadline=None, derandomize=True, suppress_health_check=[HealthCheck.too_slow])
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


def _same(a, b):
    if torch.is_tensor(a):
        return torch.is_tensor(b) and a.dtype == b.dtype and a.shape == b.shape and \
            torch.equal(a, b)
    if isinstance(a, dict):
        return isinstance(b, dict) and a.keys() == b.keys() and all(_same(a[k], b[k]) for k in a)
    if isinstance(a, (list, tuple)):
        return isinstance(b, (list, tuple)) and len(a) == len(b) and all(map(_same, a, b))
    return a == b


@st.composite
def metadata(draw, depth=0):
    leaf = st.one_of(st.integers(-2 ** 40, 2 ** 40), st.booleans(), st.text(max_size=8),
                     st.floats(allow_nan=False, allow_infinity=False), st.none(),
                     st.builds(lambda n, d: torch.arange(n).to(d), st.integers(0, 12),
                               st.sampled_from([torch.float16, torch.int64, torch.uint8,
                                                torch.float32])))
    if depth >= 2:
        return draw(leaf)
    return draw(st.one_of(
        leaf, st.lists(st.deferred(lambda: metadata(depth=depth + 1)), max_size=3),
        st.dictionaries(st.text("abcdefgh_", min_size=1, max_size=6),
                        st.deferred(lambda: metadata(depth=depth + 1)), max_size=3)))


PLAIN = st.dictionaries(st.text("abcdefgh_", min_size=1, max_size=6),
                        st.one_of(st.integers(-2 ** 40, 2 ** 40), st.text(max_size=8),
                                  st.lists(st.integers(0, 9), max_size=4)), max_size=3)


@settings(max_examples=60, deadline=None, derandomize=True, suppress_health_check=[HealthCheck.too_slow])
@given(qp=st.lists(metadata(), max_size=4), plain=PLAIN,
       n=st.integers(0, 5000), chunk=st.sampled_from([16, 1000, 4096, 1 << 20]))
def test_wire_envelope_round_trips_any_metadata(qp, plain, n, chunk):
    """Tensors anywhere under ``quantization_params`` travel as aux tensors
    behind placeholders (the wire contract allows them nowhere else); bodies
    above the chunk bound are split into byte chunks."""
    meta = dict(plain, quantization_params=qp)
    from kvserve_hpdps_b200.compression.config import CompressedKVData
    from kvserve_hpdps_b200.compression.wire import build_wire, restore_from_wire
    body = (torch.arange(n) % 251).to(torch.uint8)
    cd = CompressedKVData(request_id="r", layer_id=3, compressed_tensor=body,
                          metadata=dict(meta, request_id="r"), original_size=2 * n,
                          compressed_size=n)
    w = build_wire(cd, chunk)
    if n > chunk:
        assert w.meta["body_mode"] == "byte_chunks" and len(w.body_chunks) > 1
    back = restore_from_wire(w)
    assert torch.equal(back.compressed_tensor.reshape(-1), body)
    assert _same(back.metadata, cd.metadata), (back.metadata, cd.metadata)


@settings(max_examples=60, deadline=None, derandomize=True)
@given(ops=st.lists(st.tuples(st.booleans(), st.integers(1, 3000), st.integers(0, 10 ** 6)),
                    max_size=60))
def test_ring_allocator_never_overlaps(ops):
    """Random reservations and returns (including repeated returns): live
    regions never overlap, stay inside the ring, and free + live bytes always
    equal the capacity."""
    from kvserve_hpdps_b200.parallel.p2p_transport import RingAllocator, _align
    cap = 16384
    al = RingAllocator(cap)
    live: list[tuple[int, int]] = []
    for alloc, size, pick in ops:
        if alloc or not live:
            off = al.try_alloc(size)
            if off is not None:
                n = _align(size)
                assert 0 <= off and off + n <= cap
                assert all(off + n <= o or o + s <= off for o, s in live)
                live.append((off, n))
        else:
            o, s = live.pop(pick % len(live))
            assert al.release(o, s)
            assert not al.release(o, s)  # a second return is refused
        assert al.free_bytes() + sum(s for _, s in live) == cap


@settings(max_examples=25, deadline=None, derandomize=True, suppress_health_check=[HealthCheck.too_slow])
@given(budget=st.integers(1, 12), thr=st.floats(0.5, 1.0), noise=st.integers(0, 2 ** 31 - 1))
def test_search_invariants(budget, thr, noise):
    """The constraint-aware search never exceeds its budget, never evaluates
    a candidate twice, and its best is the highest-CR feasible evaluation."""
    import random as _r

    from kvserve_hpdps_b200.offline.bo import ConstraintAwareBO, predicted_cr
    from kvserve_hpdps_b200.offline.search_space import enumerate_space
    rng = _r.Random(noise)
    pool = enumerate_space({"hybrid_ratio": [0.0, 0.5, 1.0], "high_key_max_value": [16, 8],
                            "high_value_max_value": [16, 8], "low_key_max_value": [8, 4],
                            "low_value_max_value": [8, 4]})

    def evaluate(c):  # accuracy falls with compression, plus noise
        cr = predicted_cr(c)
        return {"accuracy": max(0.0, 1.0 - 0.02 * cr + rng.uniform(-0.02, 0.02)),
                "compression_ratio": cr}
    res = ConstraintAwareBO(pool, evaluate, thr, budget=budget).run()
    keys = [h["candidate"] for h in res["history"]]
    assert len(keys) == res["evaluations"] <= budget and len(set(keys)) == len(keys)
    feas = [h for h in res["history"] if h["accuracy"] >= thr]
    if feas:
        assert res["best"] is not None and res["best"]["compression_ratio"] == max(
            h["compression_ratio"] for h in feas)
    else:
        assert res["best"] is None
