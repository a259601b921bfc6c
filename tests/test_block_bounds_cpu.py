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
