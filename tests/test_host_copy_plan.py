"""CPU checks of run_from_host's copy plan: the layer groups cover every layer once, in order, single
layers first; the pitched copies of a row range move exactly those rows of every layer (one copy
for a run of layers that continue each other in memory on both sides, one per layer otherwise) and
leave the other rows alone. The copies are applied here with memmove on host tensors."""
import ctypes

import torch

from reki_megakernel_b200.mk_expert import _copy_groups, _rows2d


def apply(entries):
    for dst, dp, src, sp, w, h in entries:
        assert w <= dp and w <= sp and h >= 1
        for i in range(h):
            ctypes.memmove(dst + i * dp, src + i * sp, w)


def test_groups_cover_every_layer_once_in_order():
    for L in range(1, 16):
        g = _copy_groups(L)
        assert g[0] == (0, 1)
        flat = [l for l0, l1 in g for l in range(l0, l1)]
        assert flat == list(range(L)), (L, g)
        assert all(l1 > l0 for l0, l1 in g)
    assert _copy_groups(10) == [(0, 1), (1, 2), (2, 4), (4, 6), (6, 10)]


def test_row_range_of_contiguous_layers_is_one_copy():
    dev = torch.zeros(4, 6, 3, 5)   # stands for the device block of one kind: 4 layers of 6 rows
    host = torch.arange(4 * 6 * 15, dtype=torch.float32).reshape(4, 6, 3, 5)
    e = _rows2d([dev[l] for l in range(1, 4)], [host[l] for l in range(1, 4)], 2, 5)
    assert len(e) == 1 and e[0][5] == 3 and e[0][4] == 3 * 15 * 4
    apply(e)
    assert torch.equal(dev[1:, 2:5], host[1:, 2:5])
    assert (dev[0] == 0).all() and (dev[1:, :2] == 0).all() and (dev[1:, 5:] == 0).all()


def test_range_clipped_to_the_rows_and_empty_ranges_skipped():
    dev = torch.zeros(2, 4, 8)
    host = torch.ones(2, 4, 8)
    e = _rows2d([dev[0], dev[1]], [host[0], host[1]], 1, 1 << 30)  # memory rows from kv_start to the end
    apply(e)
    assert (dev[:, 1:] == 1).all() and (dev[:, :1] == 0).all()
    assert _rows2d([dev[0]], [host[0]], 4, 1 << 30) == [] and _rows2d([dev[0]], [host[0]], 0, 0) == []


def test_separate_host_allocations_stay_separate():
    dev = torch.zeros(3, 4, 2)
    hosts = [torch.full((4, 2), float(l + 1)) for l in range(3)]  # separate allocations
    e = _rows2d([dev[l] for l in range(3)], hosts, 0, 3)
    assert len(e) == 3 and all(x[5] == 1 for x in e)
    apply(e)
    for l in range(3):
        assert (dev[l, :3] == l + 1).all() and (dev[l, 3] == 0).all()
