"""CPU checks of run_from_host's copy plan: the layer groups cover every layer once, in order, single
layers first; consecutive per-layer copies merge exactly when both sides continue each other in
memory, and the merged copy spans the same bytes."""
import torch

from reki_megakernel_b200.mk_expert import _copy_groups, _merged


def test_groups_cover_every_layer_once_in_order():
    for L in range(1, 16):
        g = _copy_groups(L)
        assert g[0] == (0, 1)
        flat = [l for l0, l1 in g for l in range(l0, l1)]
        assert flat == list(range(L)), (L, g)
        assert all(l1 > l0 for l0, l1 in g)
    assert _copy_groups(10) == [(0, 1), (1, 2), (2, 4), (4, 6), (6, 10)]


def test_contiguous_layers_merge_into_one_copy():
    dev = torch.zeros(4, 3, 5)   # stands for the device block of one kind
    host = torch.arange(60, dtype=torch.float32).reshape(4, 3, 5)
    m = _merged([(dev[l], host[l]) for l in range(1, 4)])
    assert len(m) == 1
    d, h = m[0]
    assert d.data_ptr() == dev[1].data_ptr() and h.data_ptr() == host[1].data_ptr()
    assert d.numel() == h.numel() == 45
    d.copy_(h)
    assert torch.equal(dev[1:], host[1:]) and torch.equal(dev[0], torch.zeros(3, 5))


def test_non_contiguous_sources_stay_separate():
    dev = torch.zeros(3, 4)
    hosts = [torch.full((4,), float(l)) for l in range(3)]  # separate allocations
    m = _merged([(dev[l], hosts[l]) for l in range(3)])
    assert len(m) == 3
    gapped = torch.zeros(6, 4)
    m = _merged([(gapped[2 * l], hosts[l]) for l in range(3)])  # destinations not adjacent
    assert len(m) == 3
