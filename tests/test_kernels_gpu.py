"""Numerics of the sm_100a kernels against the float32 CPU oracle.

Every test here needs a CUDA device.  All transform engines are checked:
engine 0 (persistent TMA + tcgen05.mma), engine 2 (tcgen05, one CTA per
tile) and engine 1 (SIMT butterfly).  Codes may
differ from the oracle by one step where the transform's summation order
moves a value across a rounding boundary; the tests bound how often.
"""

import pytest
import torch

from kvserve_hpdps_b200.compression import oracle
from kvserve_hpdps_b200.models.synthetic import gather_request, paged_workload
from kvserve_hpdps_b200.ops import kernels as K

pytestmark = pytest.mark.gpu

ENGINES = [K.ENGINE_TCGEN05, K.ENGINE_SIMT, K.ENGINE_TCGEN05_TILE, K.ENGINE_TCGEN05_PERSISTENT]


def _plan(H, layer_id=5, packed=False, seed=0x3333):
    kl = [12.0 if h % 2 == 0 else 6.0 for h in range(H)]
    vl = [8.0 if h % 3 == 0 else 4.0 for h in range(H)]
    return K.make_layer_plan(H, kl, vl, seed, layer_id, packed=packed)


def _segments(codes, batch, plan, r):
    """[2, H, rows, 128] uint8 codes of request r (unpacked, CPU)."""
    c = codes.cpu()
    code_off = batch.layout(plan)[0][r]
    rows = batch.n_rows[r]
    H = plan.num_heads
    out = torch.empty((2, H, rows, 128), dtype=torch.uint8)
    for kv in range(2):
        for h in range(H):
            s = kv * H + h
            bits = (plan.key_bits if kv == 0 else plan.value_bits)[h]
            start = code_off + rows * plan.seg_prefix[s]
            seg = c[start:start + rows * 16 * bits]
            out[kv, h] = seg.view(rows, 128) if bits == 8 else K.bitunpack(seg, bits)
    return out


def _meta(meta, batch, plan, r):
    m = meta.cpu()
    off = batch.layout(plan)[1][r]
    rows, H, G = batch.n_rows[r], plan.num_heads, plan.n_groups
    f = m[off:off + plan.meta_bytes(rows)].view(torch.float16)
    kmin = f[:H * 128].view(H, 128)
    ksc = f[H * 128:2 * H * 128].view(H, 128)
    vmin = f[2 * H * 128:2 * H * 128 + G * rows].view(G, rows)
    vsc = f[2 * H * 128 + G * rows:].view(G, rows)
    return kmin, ksc, vmin, vsc


def _check_codes(got, exp, max_frac=2e-3):
    d = (got.to(torch.int16) - exp.to(torch.int16)).abs()
    assert int(d.max()) <= 1, f"code mismatch larger than one step: {int(d.max())}"
    frac = float((d != 0).float().mean())
    assert frac <= max_frac, f"too many code mismatches: {frac:.2e}"


@pytest.mark.parametrize("engine", ENGINES)
@pytest.mark.parametrize("H", [1, 2, 4, 8])
@pytest.mark.parametrize("packed", [False, True])
def test_quantize_matches_oracle(engine, H, packed):
    tokens = [300, 128, 37]
    wl = paged_workload(1, tokens, H, block_size=16, device="cuda", seed=H + 10 * packed)
    layer = wl.cache[0]
    plan = _plan(H, packed=packed)
    batch = K.RequestBatch(wl.block_ids, wl.n_tokens, 16, layer.device)
    codes, meta = K.quantize_layer(layer, batch, plan, engine=engine)
    torch.cuda.synchronize()
    K.check_device_error(layer.device)
    for r, t in enumerate(tokens):
        dense = gather_request(layer, wl.block_ids[r]).cpu()
        ref = oracle.compress_layer(dense, torch.tensor(plan.key_levels),
                                    torch.tensor(plan.value_levels), plan.signs, n_valid=t)
        rows = batch.n_rows[r]
        got = _segments(codes, batch, plan, r)
        exp = ref["codes"].reshape(2, H, rows, 128)
        _check_codes(got, exp)
        kmin, ksc, vmin, vsc = _meta(meta, batch, plan, r)
        torch.testing.assert_close(kmin.float(), ref["key_min"].half().float(), rtol=2e-3, atol=2e-3)
        torch.testing.assert_close(ksc.float(), ref["key_scale"].half().float(), rtol=2e-3, atol=1e-5)
        torch.testing.assert_close(vmin.float()[:, :t], ref["value_min"].half().float()[:, :t],
                                   rtol=2e-3, atol=2e-3)
        torch.testing.assert_close(vsc.float()[:, :t], ref["value_scale"].half().float()[:, :t],
                                   rtol=2e-3, atol=1e-5)


def _oracle_buffers(dense_list, plan, batch, tokens):
    """Codes/meta buffers in the device layout built from the oracle."""
    _, _, cbytes, mbytes = batch.layout(plan)
    codes = torch.zeros(cbytes, dtype=torch.uint8)
    meta = torch.zeros(mbytes, dtype=torch.uint8)
    refs = []
    H = plan.num_heads
    for r, dense in enumerate(dense_list):
        ref = oracle.compress_layer(dense, torch.tensor(plan.key_levels),
                                    torch.tensor(plan.value_levels), plan.signs, n_valid=tokens[r])
        refs.append(ref)
        rows = batch.n_rows[r]
        off = batch.layout(plan)[0][r]
        cr = ref["codes"].reshape(2, H, rows, 128)
        for kv in range(2):
            for h in range(H):
                bits = (plan.key_bits if kv == 0 else plan.value_bits)[h]
                start = off + rows * plan.seg_prefix[kv * H + h]
                seg = cr[kv, h].contiguous().view(-1) if bits == 8 else K.bitpack(cr[kv, h], bits).view(-1)
                codes[start:start + seg.numel()] = seg
        moff = batch.layout(plan)[1][r]
        f = torch.cat([ref["key_min"].half().flatten(), ref["key_scale"].half().flatten(),
                       ref["value_min"].half().flatten(), ref["value_scale"].half().flatten()])
        meta[moff:moff + f.numel() * 2] = f.view(torch.uint8)
    return codes, meta, refs


@pytest.mark.parametrize("engine", ENGINES)
@pytest.mark.parametrize("H", [2, 4, 8])
@pytest.mark.parametrize("packed", [False, True])
def test_dequantize_matches_oracle(engine, H, packed):
    tokens = [260, 64]
    wl = paged_workload(1, tokens, H, block_size=16, device="cuda", seed=3 * H)
    layer = wl.cache[0]
    plan = _plan(H, layer_id=2, packed=packed)
    dense = [gather_request(layer, b).cpu() for b in wl.block_ids]
    dst = paged_workload(1, tokens, H, block_size=16, device="cuda", seed=99, fill=False,
                         extra_blocks=5)
    batch = K.RequestBatch(dst.block_ids, tokens, 16, layer.device)
    codes, meta, refs = _oracle_buffers(dense, plan, batch, tokens)
    K.dequantize_layer(codes.cuda(), meta.cuda(), dst.cache[0], batch, plan, engine=engine)
    torch.cuda.synchronize()
    K.check_device_error(layer.device)
    for r, t in enumerate(tokens):
        ref = refs[r]
        exp = oracle.decompress_layer(ref["codes"], ref["key_min"], ref["key_scale"],
                                      ref["value_min"], ref["value_scale"], ref["groups"],
                                      plan.signs)
        got = gather_request(dst.cache[0], dst.block_ids[r]).cpu()
        nb = len(dst.block_ids[r])
        g = got.view(2, nb * 16, H, 128)[:, :t].float()
        e = exp.view(2, nb * 16, H, 128)[:, :t].float()
        torch.testing.assert_close(g, e, rtol=1.6e-2, atol=2e-3)


@pytest.mark.parametrize("engine", ENGINES)
def test_round_trip_error_close_to_oracle(engine):
    H, tokens = 4, [1024, 333]
    wl = paged_workload(1, tokens, H, block_size=16, device="cuda", seed=5)
    layer = wl.cache[0]
    plan = _plan(H, layer_id=7)
    batch = K.RequestBatch(wl.block_ids, tokens, 16, layer.device)
    codes, meta = K.quantize_layer(layer, batch, plan, engine=engine)
    dst = torch.zeros_like(layer)
    K.dequantize_layer(codes, meta, dst, batch, plan, engine=engine)
    torch.cuda.synchronize()
    K.check_device_error(layer.device)
    for r, t in enumerate(tokens):
        src = gather_request(layer, wl.block_ids[r])
        rec = gather_request(dst, wl.block_ids[r])
        nb = len(wl.block_ids[r])
        s = src.view(2, nb * 16, H, 128)[:, :t]
        g = rec.view(2, nb * 16, H, 128)[:, :t]
        got = K.kv_error(s, g)
        ref = oracle.compress_layer(src.cpu(), torch.tensor(plan.key_levels),
                                    torch.tensor(plan.value_levels), plan.signs, n_valid=t)
        exp_rec = oracle.decompress_layer(ref["codes"], ref["key_min"], ref["key_scale"],
                                          ref["value_min"], ref["value_scale"], ref["groups"],
                                          plan.signs)
        exp = oracle.error_metrics(s.cpu(), exp_rec.view(2, nb * 16, H, 128)[:, :t])
        assert abs(got["cosine"] - exp["cosine"]) < 2e-3
        assert abs(got["rel_mse"] - exp["rel_mse"]) < 2e-2 * max(exp["rel_mse"], 1e-6) + 1e-4


@pytest.mark.parametrize("engine", ENGINES)
def test_multi_layer_launch_matches_oracle(engine):
    """One launch over several layers with different plans (levels, signs,
    packing) and several requests per layer."""
    H, tokens, L = 4, [200, 96], 3
    wl = paged_workload(L, tokens, H, device="cuda", seed=77)
    plans = [
        K.make_layer_plan(H, [12, 6, 12, 6], [8, 4, 4, 8], 0x3333, 0),
        K.make_layer_plan(H, [16, 16, 16, 16], [16, 16, 16, 16], 0x3333, 1, packed=True),
        K.make_layer_plan(H, [6, 6, 12, 12], [4, 4, 8, 8], None, 2),
    ]
    slots = K.LayerSlots([wl.cache[l] for l in range(L)], plans)
    items = K.WorkItems(slots, [(l, b, t) for l in range(L) for b, t in zip(wl.block_ids, tokens)])
    codes, meta = K.quantize(slots, items, engine=engine)
    dst = torch.zeros_like(wl.cache)
    dslots = K.LayerSlots([dst[l] for l in range(L)], plans)
    K.dequantize(codes, meta, dslots, items, engine=engine)
    torch.cuda.synchronize()
    K.check_device_error(wl.cache.device)
    for r, (l, blocks, t) in enumerate(items.items):
        plan = plans[l]
        dense = gather_request(wl.cache[l], blocks).cpu()
        ref = oracle.compress_layer(dense, torch.tensor(plan.key_levels),
                                    torch.tensor(plan.value_levels), plan.signs, n_valid=t)
        rows = items.n_rows[r]
        cr = items.item_codes(codes, r).cpu()
        got = torch.empty((2, H, rows, 128), dtype=torch.uint8)
        for kv in range(2):
            for h in range(H):
                bits = (plan.key_bits if kv == 0 else plan.value_bits)[h]
                st = rows * plan.seg_prefix[kv * H + h]
                seg = cr[st:st + rows * 16 * bits]
                got[kv, h] = seg.view(rows, 128) if bits == 8 else K.bitunpack(seg, bits)
        _check_codes(got, ref["codes"].reshape(2, H, rows, 128))
        exp = oracle.decompress_layer(ref["codes"], ref["key_min"], ref["key_scale"],
                                      ref["value_min"], ref["value_scale"], ref["groups"],
                                      plan.signs)
        rec = gather_request(dst[l], blocks).cpu()
        nb = len(blocks)
        torch.testing.assert_close(rec.view(2, nb * 16, H, 128)[:, :t].float(),
                                   exp.view(2, nb * 16, H, 128)[:, :t].float(),
                                   rtol=1.6e-2, atol=4e-3)


def test_engines_agree():
    H, tokens = 4, [512]
    wl = paged_workload(1, tokens, H, device="cuda", seed=11)
    plan = _plan(H)
    batch = K.RequestBatch(wl.block_ids, tokens, 16, wl.cache.device)
    c0, m0 = K.quantize_layer(wl.cache[0], batch, plan, engine=K.ENGINE_TCGEN05)
    c1, m1 = K.quantize_layer(wl.cache[0], batch, plan, engine=K.ENGINE_SIMT)
    torch.cuda.synchronize()
    _check_codes(c0.cpu(), c1.cpu())


@pytest.mark.parametrize("packed", [False, True])
def test_persistent_engines_bit_exact_vs_tile_engine(packed):
    """The persistent kernels (warp-specialized and not) walk many jobs per CTA (image reloads at
    layer/head changes, key statistics carried across tiles, odd token
    counts, partial tiles): codes, metadata and reconstruction must equal
    the one-CTA-per-tile engine bit for bit."""
    H, L = 4, 6
    tokens = [1, 130, 2047, 4096, 777]
    wl = paged_workload(L, tokens, H, device="cuda", seed=123)
    plans = [K.make_layer_plan(H, [12, 6, 16, 6][:H], [8, 4, 4, 16][:H], 0x3333, l,
                               packed=packed) for l in range(L)]
    slots = K.LayerSlots([wl.cache[l] for l in range(L)], plans)
    items = K.WorkItems(slots, [(l, b, t) for l in range(L) for b, t in zip(wl.block_ids, tokens)])
    outs = []
    for engine in (K.ENGINE_TCGEN05_TILE, K.ENGINE_TCGEN05, K.ENGINE_TCGEN05_PERSISTENT):
        codes, meta = K.quantize(slots, items, engine=engine)
        dst = torch.zeros_like(wl.cache)
        dslots = K.LayerSlots([dst[l] for l in range(L)], plans)
        K.dequantize(codes, meta, dslots, items, engine=engine)
        torch.cuda.synchronize()
        K.check_device_error(wl.cache.device)
        outs.append((codes.clone(), meta.clone(), dst))
    for o in outs[1:]:
        assert torch.equal(outs[0][0], o[0]), "codes differ"
        assert torch.equal(outs[0][1], o[1]), "metadata differ"
        for l in range(L):
            for b, t in zip(wl.block_ids, tokens):
                a = gather_request(outs[0][2][l], b).view(2, -1, H, 128)[:, :t]
                c = gather_request(o[2][l], b).view(2, -1, H, 128)[:, :t]
                assert torch.equal(a, c), f"reconstruction differs (layer {l}, {t} tokens)"


@pytest.mark.parametrize("n", [1, 511, 4096, 32768, 100000, 300001])
@pytest.mark.parametrize("dist", ["skewed", "uniform256", "constant"])
def test_rans_gpu_matches_cpu(n, dist):
    g = torch.Generator().manual_seed(n)
    if dist == "skewed":
        p = torch.tensor([0.02, 0.18, 0.3, 0.3, 0.18, 0.02])
        x = torch.multinomial(p, n, replacement=True, generator=g).to(torch.uint8)
    elif dist == "uniform256":
        x = torch.randint(0, 256, (n,), generator=g, dtype=torch.uint8)
    else:
        x = torch.full((n,), 3, dtype=torch.uint8)
    cpu_stream = K.rans_encode(x)
    gpu_stream = K.rans_encode(x.cuda())
    torch.cuda.synchronize()
    assert torch.equal(gpu_stream.cpu(), cpu_stream), "device and host streams differ"
    y = K.rans_decode(gpu_stream, n)
    torch.cuda.synchronize()
    K.check_device_error(y.device)
    assert torch.equal(y.cpu(), x)
    assert torch.equal(K.rans_decode(cpu_stream, n), x)


def test_block_copy_gather_scatter():
    H, tokens = 4, [80, 33]
    wl = paged_workload(1, tokens, H, device="cuda", seed=21)
    layer = wl.cache[0]
    blocks = torch.tensor(wl.block_ids[0], dtype=torch.int32, device="cuda")
    flat = torch.empty((2, blocks.numel(), 16, H, 128), dtype=torch.bfloat16, device="cuda")
    K.block_copy(layer, blocks, flat.data_ptr(), gather=True)
    torch.cuda.synchronize()
    assert torch.equal(flat, gather_request(layer, wl.block_ids[0]))
    dst = torch.zeros_like(layer)
    K.block_copy(dst, blocks, flat.data_ptr(), gather=False)
    torch.cuda.synchronize()
    assert torch.equal(gather_request(dst, wl.block_ids[0]), flat)


@pytest.mark.parametrize("layout", ["flash_attn", "flashinfer", "hnd"])
def test_raw_paged_transfer_round_trip(layout):
    """One-launch raw gather of several (layer, blocks) items into the
    stacked flat layout, its fused message checksum, and the scatter back."""
    L, H, nb = 3, 4, 12
    g = torch.Generator(device="cuda").manual_seed(4)
    if layout == "flash_attn":
        layers = [torch.randn((2, nb, 16, H, 128), generator=g, device="cuda").to(torch.bfloat16)
                  for _ in range(L)]
    elif layout == "flashinfer":
        layers = [torch.randn((nb, 2, 16, H, 128), generator=g, device="cuda").to(torch.bfloat16)
                  for _ in range(L)]
    else:  # head-major blocks: [nb, 2, H, bs, D] storage seen as [nb, 2, bs, H, D]
        layers = [torch.randn((nb, 2, H, 16, 128), generator=g, device="cuda")
                  .to(torch.bfloat16).transpose(2, 3) for _ in range(L)]
    blocks = [7, 2, 11, 0, 5]
    raw = K.RawItems(layers, [(l, blocks) for l in range(L)])
    assert raw.block_order == ("hnd" if layout == "hnd" else "nhd")
    flat = torch.empty(raw.flat_bytes, dtype=torch.uint8, device="cuda")
    ck = torch.empty(2, dtype=torch.int64, device="cuda")
    trailer = torch.zeros(2, dtype=torch.int64, device="cuda")
    flag = torch.zeros(4, dtype=torch.int32, device="cuda")
    K.paged_raw(raw, flat.data_ptr(), True, flag_ptr=flag.data_ptr(), flag_value=9,
                trailer_ptr=trailer.data_ptr(), checksum=ck)
    torch.cuda.synchronize()
    assert K.read_device_error(flat.device) == 0
    assert int(flag[0]) == 9
    idx = torch.tensor(blocks, device="cuda")
    for l in range(L):
        t = layers[l]
        part = flat[raw.item_offsets[l]:raw.item_offsets[l] + 2 * len(blocks) * raw.block_bytes]
        if layout == "flash_attn":
            exp = t[:, idx]
        else:
            exp = t[idx].transpose(0, 1)
        if layout == "hnd":
            exp = exp.transpose(2, 3)  # bytes of a block are in [H, bs, D] order
        assert torch.equal(part.view(torch.bfloat16).view(exp.shape), exp.contiguous())
    ref = torch.empty(2, dtype=torch.int64, device="cuda")
    K.checksum([(flat.data_ptr(), 0, raw.flat_bytes)], ref)
    torch.cuda.synchronize()
    assert torch.equal(ck, ref) and torch.equal(trailer, ref)
    dst = [torch.zeros_like(t) for t in layers]
    draw = K.RawItems(dst, [(l, [1, 3, 4, 8, 10]) for l in range(L)])
    K.paged_raw(draw, flat.data_ptr(), False)
    torch.cuda.synchronize()
    for l in range(L):
        for a, b in zip(blocks, [1, 3, 4, 8, 10]):
            if layout == "flash_attn":
                assert torch.equal(dst[l][:, b], layers[l][:, a])
            else:
                assert torch.equal(dst[l][b], layers[l][a])
    # a block id that turns bad after the host check is recorded and skipped
    off = draw._ptrs[3] - draw._desc.data_ptr()  # first block-table entry
    draw._desc[off:off + 4] = torch.tensor([100], dtype=torch.int32).view(torch.uint8).cuda()
    K.paged_raw(draw, flat.data_ptr(), False)
    torch.cuda.synchronize()
    assert K.read_device_error(flat.device) == 3


def test_kv_error_matches_cpu():
    g = torch.Generator().manual_seed(3)
    a = torch.randn(10007, generator=g).to(torch.bfloat16)
    b = (a.float() + 0.01 * torch.randn(10007, generator=g)).to(torch.bfloat16)
    got = K.kv_error(a.cuda(), b.cuda())
    exp = oracle.error_metrics(a, b)
    for k in ("rel_mse", "cosine", "max_abs"):
        assert abs(got[k] - exp[k]) <= 1e-6 + 1e-5 * abs(exp[k])


def test_logit_agreement():
    g = torch.Generator().manual_seed(4)
    r = torch.randn(8, 1000, generator=g)
    a = r.clone()
    a[3] += 5 * torch.randn(1000, generator=g)
    out = K.logit_agreement(r.cuda(), a.cuda())
    lp_r, lp_a = torch.log_softmax(r.double(), -1), torch.log_softmax(a.double(), -1)
    kl = (lp_r.exp() * (lp_r - lp_a)).sum(-1).mean()
    agree = (r.argmax(-1) == a.argmax(-1)).float().mean()
    assert abs(out["kl_mean"] - float(kl)) < 1e-4
    assert abs(out["top1_agreement"] - float(agree)) < 1e-6


def test_wait_flag_times_out_with_error_status():
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    K.read_device_error(flag.device)  # clear
    K.wait_flag(flag.data_ptr(), 1, flag.device, timeout_s=0.05)
    torch.cuda.synchronize()
    assert K.read_device_error(flag.device) == 2
    K.set_flag(flag.data_ptr(), 1, flag.device)
    K.wait_flag(flag.data_ptr(), 1, flag.device, timeout_s=0.05)
    torch.cuda.synchronize()
    assert K.read_device_error(flag.device) == 0


@pytest.mark.parametrize("engine", ENGINES)
def test_head_major_block_layout_matches_token_major(engine):
    """vLLM's FlashInfer cache on B200 is [nb, 2, bs, H, D] with a head-major
    (HND) block: the kernels must read and write it exactly like the
    token-major (NHD) form of the same logical values."""
    H, L = 4, 2
    tokens = [200, 33]
    wl = paged_workload(L, tokens, H, device="cuda", seed=21)
    nb, bs = wl.cache.shape[2], wl.cache.shape[3]
    # same logical values in a FlashInfer-ordered, head-major cache
    hnd = []
    for l in range(L):
        storage = torch.empty((nb, 2, H, bs, 128), dtype=torch.bfloat16, device="cuda")
        view = storage.permute(0, 1, 3, 2, 4)  # logical [nb, 2, bs, H, D], HND strides
        view.copy_(wl.cache[l].permute(1, 0, 2, 3, 4))
        hnd.append(view)
    plans = [K.make_layer_plan(H, [12, 6, 16, 6], [8, 4, 4, 16], 0x3333, l) for l in range(L)]
    items_spec = [(l, b, t) for l in range(L) for b, t in zip(wl.block_ids, tokens)]
    s_nhd = K.LayerSlots([wl.cache[l] for l in range(L)], plans)
    s_hnd = K.LayerSlots(hnd, plans)
    c0, m0 = K.quantize(s_nhd, K.WorkItems(s_nhd, items_spec), engine=engine)
    c1, m1 = K.quantize(s_hnd, K.WorkItems(s_hnd, items_spec), engine=engine)
    torch.cuda.synchronize()
    K.check_device_error(wl.cache.device)
    assert torch.equal(c0, c1) and torch.equal(m0, m1)
    dst_nhd = torch.zeros_like(wl.cache)
    dst_hnd = [torch.zeros((nb, 2, H, bs, 128), dtype=torch.bfloat16,
                           device="cuda").permute(0, 1, 3, 2, 4) for _ in range(L)]
    d0 = K.LayerSlots([dst_nhd[l] for l in range(L)], plans)
    d1 = K.LayerSlots(dst_hnd, plans)
    K.dequantize(c0, m0, d0, K.WorkItems(d0, items_spec), engine=engine)
    K.dequantize(c1, m1, d1, K.WorkItems(d1, items_spec), engine=engine)
    torch.cuda.synchronize()
    K.check_device_error(wl.cache.device)
    for l in range(L):
        for b, t in zip(wl.block_ids, tokens):
            idx = torch.tensor(b, device="cuda")
            a = dst_nhd[l][:, idx].reshape(2, -1, H, 128)[:, :t]
            c = dst_hnd[l][idx].permute(1, 0, 2, 3, 4).reshape(2, -1, H, 128)[:, :t]
            assert torch.equal(a, c)


def test_message_checksum_detects_corruption():
    """Producer checksum of a message's segments vs the consumer's
    recomputation over its landed copy: equal copies pass, one flipped byte
    records ERR_CORRUPT (host-injected corruption; nothing faults)."""
    dev = torch.device("cuda")
    g = torch.Generator(device="cuda").manual_seed(5)
    parts = [torch.randint(0, 256, (n,), generator=g, device=dev, dtype=torch.uint8)
             for n in (1000, 4096, 37)]
    offs, o = [], 0
    for p in parts:
        offs.append(o)
        o += (p.numel() + 255) // 256 * 256
    ring = torch.zeros(o + 256, dtype=torch.uint8, device=dev)
    ck = torch.empty(2, dtype=torch.int64, device=dev)
    K.checksum([(p.data_ptr(), off, p.numel()) for p, off in zip(parts, offs)], ck)
    for p, off in zip(parts, offs):
        ring[off:off + p.numel()] = p
    ring[o:o + 16] = ck.view(torch.uint8)
    segs = [(ring.data_ptr() + off, off, p.numel()) for p, off in zip(parts, offs)]
    K.read_device_error(dev)
    K.verify_checksum(segs, ring.data_ptr() + o, dev)
    assert K.read_device_error(dev) == 0
    ring[offs[1] + 777] ^= 0x10
    K.verify_checksum(segs, ring.data_ptr() + o, dev)
    assert K.read_device_error(dev) == 4  # ERR_CORRUPT
    # a misaligned source checksums like the aligned one
    buf = torch.zeros(4096 + 3, dtype=torch.uint8, device=dev)
    buf[3:] = parts[1]
    ck2 = torch.empty(2, dtype=torch.int64, device=dev)
    K.checksum([(buf.data_ptr() + 3, 0, 4096)], ck2)
    ck3 = torch.empty(2, dtype=torch.int64, device=dev)
    K.checksum([(parts[1].data_ptr(), 0, 4096)], ck3)
    assert torch.equal(ck2, ck3)


def test_error_monitor_reports_without_waiting():
    """A bounded flag wait that runs out (nothing sets the flag) records a
    timeout; the non-blocking monitor reports it at a later poll."""
    dev = torch.device("cuda")
    K.read_device_error(dev)
    mon = K.ErrorMonitor(dev)
    assert mon.poll() == 0
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    K.wait_flag(flag.data_ptr(), 7, dev, timeout_s=0.05)
    torch.cuda.synchronize()
    code = 0
    for _ in range(3):
        code = code or mon.poll()
        torch.cuda.synchronize()
    assert code == 2  # ready-flag timeout
    assert K.read_device_error(dev) == 0  # the monitor cleared the word


@pytest.mark.parametrize("engine", ENGINES)
def test_bad_block_id_is_recorded_not_followed(engine):
    """A device block-table entry outside the cache (set after the host
    check passed) records a bounds error: dequantize skips that block's rows
    and writes the others, quantize reads block 0 in its place."""
    H, tokens = 2, [64, 48]
    wl = paged_workload(1, tokens, H, block_size=16, device="cuda", seed=3)
    layer = wl.cache[0]
    plan = _plan(H)
    slots = K.LayerSlots.single(layer, plan)
    items = K.WorkItems(slots, [(0, b, n) for b, n in zip(wl.block_ids, tokens)])
    codes, meta = K.quantize(slots, items, engine=engine)
    torch.cuda.synchronize()
    assert K.read_device_error(layer.device) == 0
    dst = torch.zeros_like(layer)
    dslots = K.LayerSlots.single(dst, plan)
    ditems = K.WorkItems(dslots, [(0, b, n) for b, n in zip(wl.block_ids, tokens)])
    ditems._ints[1] = dst.shape[1] + 3  # entry 1 = second block of request 0
    K.dequantize(codes, meta, dslots, ditems, engine=engine)
    torch.cuda.synchronize()
    assert K.read_device_error(dst.device) == 3
    assert int(dst[:, wl.block_ids[0][1]].abs().sum()) == 0
    for b in (wl.block_ids[0][0], wl.block_ids[1][0]):
        assert float(dst[:, b].float().abs().sum()) > 0
    items._ints[0] = -5
    K.quantize(slots, items, engine=engine)
    torch.cuda.synchronize()
    assert K.read_device_error(layer.device) == 3


@pytest.mark.parametrize("n", [1, 1000, 16384, 16385, 300000])
def test_lc_gpu_matches_cpu_reference(n):
    """Device BIT_2 + RZE_1 writes the numpy reference's stream byte for byte
    and decodes it; a corrupt stream records ERR_CORRUPT instead of reading
    outside it."""
    from kvserve_hpdps_b200.compression import lc
    g = torch.Generator().manual_seed(n)
    x = torch.randint(0, 16, (n,), generator=g, dtype=torch.uint8)
    x[: n // 3] = torch.randint(0, 256, (n // 3,), generator=g, dtype=torch.uint8)  # raw chunks too
    ref = torch.from_numpy(lc.encode(x.numpy()))
    s = K.lc_encode(x.cuda())
    torch.cuda.synchronize()
    assert torch.equal(s.cpu(), ref)
    out = K.lc_decode(s, n)
    torch.cuda.synchronize()
    assert K.read_device_error(out.device) == 0
    assert torch.equal(out.cpu(), x)
    bad = s.clone()
    bad[0] ^= 0xFF
    K.lc_decode(bad, n)
    torch.cuda.synchronize()
    assert K.read_device_error(out.device) == 4
    K.lc_decode(s[:32], n)
    torch.cuda.synchronize()
    assert K.read_device_error(out.device) == 4


def test_rans_decode_rejects_corrupt_streams():
    """A corrupt header, directory or length records ERR_CORRUPT; the decoder
    never reads or writes outside the buffers it was given."""
    g = torch.Generator().manual_seed(7)
    x = torch.randint(0, 6, (200000,), generator=g, dtype=torch.uint8).cuda()
    s = K.rans_encode(x)
    out = K.rans_decode(s, x.numel())
    torch.cuda.synchronize()
    assert K.read_device_error(out.device) == 0 and torch.equal(out, x)
    for field, value in ((0, 0x12345678), (4, 1 << 20), (16, 1 << 30), (24, 1 << 40)):
        bad = s.clone()
        bad[field:field + 4] = torch.tensor([value & 0xFFFFFFFF], dtype=torch.int64) \
            .to(torch.int32).view(torch.uint8).cuda()
        K.rans_decode(bad, x.numel())
        torch.cuda.synchronize()
        assert K.read_device_error(out.device) == 4, field
    dir0 = s.clone()  # first record offset far past the stream
    dir0[32:40] = torch.tensor([1 << 40], dtype=torch.int64).view(torch.uint8).cuda()
    K.rans_decode(dir0, x.numel())
    torch.cuda.synchronize()
    assert K.read_device_error(out.device) == 4
    K.rans_decode(s[:1000], x.numel())  # truncated: the header's total exceeds the buffer
    torch.cuda.synchronize()
    assert K.read_device_error(out.device) == 4


def test_step_errors_read_every_step_one_step_late():
    """StepErrors: each push copies and clears the error word; check(keep=1)
    reports a step's error once the next step has been pushed, check(0) the
    last one."""
    dev = torch.device("cuda", 0)
    K.read_device_error(dev)  # clear
    errs = K.StepErrors(dev)
    errs.push()
    errs.check(keep=1)  # nothing older than the newest
    K.workspace(dev).err[0] = 7  # step 2 fails
    errs.push()
    errs.check(keep=1)  # step 1 was clean
    errs.push()  # step 3: the word was cleared by step 2's push
    with pytest.raises(RuntimeError, match="device error 7"):
        errs.check(keep=1)
    errs.check(0)
    assert K.read_device_error(dev) == 0
