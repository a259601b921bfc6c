"""The no-allocation rANS encoder, called through its exported C symbol.

Callers that cannot allocate device memory when they encode (a serving
engine that reserved most of the GPU for its KV cache at start-up, or an
embedder with a fixed memory budget) use ``kvs_rans_encode_noalloc``: its
scratch is a fixed file-scope device array of the library, so the caller
provides only the input and the output.  This file is named to be collected
last so that a run stopping at the first failure has already run every
other test.
"""

import ctypes

import pytest
import torch

from kvserve_hpdps_b200.ops import _lib
from kvserve_hpdps_b200.ops import kernels as K

pytestmark = pytest.mark.gpu


def _symbols():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    enc = lib.kvs_rans_encode_noalloc
    enc.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_uint64,
                    ctypes.c_void_p]
    enc.restype = ctypes.c_int
    mx = lib.kvs_rans_encode_noalloc_max_symbols
    mx.argtypes = []
    mx.restype = ctypes.c_uint64
    cap = lib.kvs_rans_max_bytes
    cap.argtypes = [ctypes.c_uint64, ctypes.c_uint32]
    cap.restype = ctypes.c_uint64
    return enc, mx, cap


def _symbols_input(n, seed):
    g = torch.Generator().manual_seed(seed)
    p = torch.tensor([0.01, 0.09, 0.4, 0.4, 0.09, 0.01])
    x = torch.multinomial(p, n, replacement=True, generator=g).to(torch.uint8)
    x[: n // 7] = torch.randint(0, 256, (n // 7,), generator=g, dtype=torch.uint8)
    return x.cuda()


def test_noalloc_encoder_matches_allocating_encoder_twice():
    enc, _, cap = _symbols()
    stream = torch.cuda.current_stream().cuda_stream
    # two calls in a row: the shared scratch keeps the first call's contents
    for n, seed in ((3_000_017, 1), (1_000_000, 2)):
        x = _symbols_input(n, seed)
        expected = K.rans_encode(x)  # the existing (caller-provided scratch) entry point
        c = int(cap(n, 32768))
        out = torch.empty(c, dtype=torch.uint8, device="cuda")
        rc = enc(x.data_ptr(), n, out.data_ptr(), c, stream)
        assert rc == 0, rc
        torch.cuda.synchronize()
        size = int(out[24:32].cpu().view(torch.int64).item())
        # a lossless coder: the tolerance is exact equality
        assert size == expected.numel()
        assert torch.equal(out[:size], expected)
        assert torch.equal(K.rans_decode(out[:size], n), x)


def test_noalloc_encoder_at_its_limit():
    """An input of exactly the maximum size fills the scratch to its last
    staging slot and uses every record-size entry; part of it is random
    bytes, so some chunks take the raw fallback."""
    enc, mx, cap = _symbols()
    n = int(mx())
    x = _symbols_input(n, 3)
    expected = K.rans_encode(x)
    c = int(cap(n, 32768))
    out = torch.empty(c, dtype=torch.uint8, device="cuda")
    rc = enc(x.data_ptr(), n, out.data_ptr(), c, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, rc
    torch.cuda.synchronize()
    size = int(out[24:32].cpu().view(torch.int64).item())
    assert size == expected.numel()
    assert torch.equal(out[:size], expected)
    assert torch.equal(K.rans_decode(out[:size], n), x)


def test_noalloc_encoder_rejects_inputs_beyond_its_scratch():
    enc, mx, cap = _symbols()
    limit = int(mx())
    x = torch.zeros(16, dtype=torch.uint8, device="cuda")
    out = torch.zeros(16, dtype=torch.uint8, device="cuda")
    rc = enc(x.data_ptr(), limit + 1, out.data_ptr(), int(cap(limit + 1, 32768)),
             torch.cuda.current_stream().cuda_stream)
    assert rc == -3
    assert int(out.sum()) == 0  # nothing was launched
