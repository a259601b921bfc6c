"""Host-side validation of work-item block ids against the paged cache."""

import pytest
import torch

from kvserve_hpdps_b200.ops import kernels as K


def _slots(layout):
    H, nb = 2, 6
    shape = (2, nb, 16, H, 128) if layout == "flash_attn" else (nb, 2, 16, H, 128)
    plan = K.make_layer_plan(H, [12.0, 6.0], [8.0, 4.0], 0x3333, 0)
    return K.LayerSlots.single(torch.zeros(shape, dtype=torch.bfloat16), plan)


@pytest.mark.parametrize("layout", ["flash_attn", "flashinfer"])
def test_block_ids_inside_cache_accepted(layout):
    items = K.WorkItems(_slots(layout), [(0, [5, 0, 3], 40), (0, [1], 16)])
    assert items.n_rows == [48, 16]


@pytest.mark.parametrize("layout", ["flash_attn", "flashinfer"])
@pytest.mark.parametrize("bad", [6, 100, -1])
def test_block_ids_outside_cache_rejected(layout, bad):
    with pytest.raises(ValueError, match="outside the 6 blocks"):
        K.WorkItems(_slots(layout), [(0, [0, 1], 32), (0, [2, bad], 20)])


def test_raw_items_layout_and_checks():
    layers = [torch.zeros((2, 6, 16, 2, 64), dtype=torch.bfloat16) for _ in range(3)]
    raw = K.RawItems(layers, [(l, [4, 0]) for l in range(3)])
    assert raw.block_bytes == 16 * 2 * 64 * 2
    assert raw.item_offsets == [0, 4 * raw.block_bytes, 8 * raw.block_bytes]
    assert raw.flat_bytes == 12 * raw.block_bytes and raw.n_units == 12
    assert raw.block_order == "nhd" and raw.flat_shape(1) == (2, 2, 16, 2, 64)
    with pytest.raises(ValueError, match="outside the 6 blocks"):
        K.RawItems(layers, [(0, [6])])
    with pytest.raises(ValueError, match="outside the 3 layers"):
        K.RawItems(layers, [(3, [1])])
    with pytest.raises(ValueError, match="not dense"):
        K.RawItems([torch.zeros((2, 6, 16, 2, 128), dtype=torch.bfloat16)[..., :64]], [(0, [1])])


def test_work_item_tables_match_per_item_layout():
    """The vectorised table build against a per-item loop over the plans:
    block table (one copy per shared block list), list offsets, tokens,
    rows, tile prefix, slot, and 16-byte aligned code/metadata offsets."""
    H = 2
    plans = [K.make_layer_plan(H, [12.0, 6.0], [8.0, 4.0], 0x3333, 0),
             K.make_layer_plan(H, [12.0, 12.0], [8.0, 8.0], 0x3333, 1, code_width=4),
             K.make_layer_plan(H, [16.0, 6.0], [6.0, 4.0], 0x3333, 2)]
    layers = [torch.zeros((2, 9, 16, H, 128), dtype=torch.bfloat16),
              torch.zeros((7, 2, 16, H, 128), dtype=torch.bfloat16),
              torch.zeros((2, 5, 32, H, 128), dtype=torch.bfloat16)]
    slots = K.LayerSlots(layers, plans)
    shared = [8, 0, 3, 5, 1, 2, 4, 6, 7]  # 144 tokens at block size 16: two tiles
    items = [(0, shared, 140), (1, [6, 2], 20), (0, shared, 144),
             (2, torch.tensor([4, 0, 1]), 70), (1, [0], 1), (2, [], 0)]
    w = K.WorkItems(slots, items)
    bt, off, code_off, meta_off, row_off = [], [], [], [], []
    seen: dict[int, int] = {}
    c = m = r = 0
    prefix = [0]
    for s, b, n in items:
        ids = [int(x) for x in b]
        if id(b) not in seen:
            seen[id(b)] = len(bt)
            bt += ids
        off.append(seen[id(b)])
        rows = len(ids) * layers[s].shape[2]
        code_off.append(c)
        meta_off.append(m)
        row_off.append(r)
        c += (rows * plans[s].row_bytes() + 15) // 16 * 16
        m += (plans[s].meta_bytes(rows) + 15) // 16 * 16
        r += rows
        prefix.append(prefix[-1] + (rows + K.TILE_ROWS - 1) // K.TILE_ROWS)
    R = len(items)
    ints = w._ints.tolist()
    o = w._o
    assert ints[o["bt"]:o["bt"] + len(bt)] == bt and o["off"] == len(bt)
    assert ints[o["off"]:o["off"] + R] == off
    assert ints[o["ntok"]:o["ntok"] + R] == [n for _, _, n in items]
    assert ints[o["rows"]:o["rows"] + R] == [row_off[i + 1] - row_off[i] for i in range(R - 1)] \
        + [r - row_off[-1]]
    assert ints[o["prefix"]:o["prefix"] + R + 1] == prefix
    assert ints[o["slot"]:o["slot"] + R] == [s for s, _, _ in items]
    assert w._longs.tolist() == code_off + meta_off + row_off
    assert (w.code_bytes, w.meta_bytes, w.total_rows, w.total_tiles) == (c, m, r, prefix[-1])
    assert all(x % 16 == 0 for x in code_off + meta_off)
    # explicit offsets: the end of the furthest item bounds the buffers
    w2 = K.WorkItems(slots, items[:2], code_offsets=[4096, 0], meta_offsets=[0, 1024])
    assert w2.code_bytes == 4096 + 144 * plans[0].row_bytes()
    assert w2.meta_bytes == 1024 + plans[1].meta_bytes(32)
    with pytest.raises(ValueError):
        K.WorkItems(slots, items[:2], code_offsets=[8, 0])
    with pytest.raises(ValueError):
        K.WorkItems(slots, items[:2], meta_offsets=[0])


def test_code_and_metadata_buffers_cover_the_items():
    """Buffers shorter than the extents the work items address are refused
    before any launch (a message whose layout does not match the requests)."""
    from types import SimpleNamespace

    import pytest
    import torch

    from kvserve_hpdps_b200.ops import kernels as K
    items = SimpleNamespace(code_bytes=4096, meta_bytes=1056)
    K._check_extents(torch.empty(4096, dtype=torch.uint8), torch.empty(528, dtype=torch.float16),
                     items)
    with pytest.raises(ValueError, match="shorter"):
        K._check_extents(torch.empty(4080, dtype=torch.uint8),
                         torch.empty(1056, dtype=torch.uint8), items)
    with pytest.raises(ValueError, match="shorter"):
        K._check_extents(torch.empty(8192, dtype=torch.uint8),
                         torch.empty(1040, dtype=torch.uint8), items)
