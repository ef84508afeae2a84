"""CPU check of the host-side weight packing (``reki_megakernel_b200.packing``) that callers of
``mkx_run_static`` use to lay out the weights themselves.

The expected position of every source element is restated here from the documented layout rule
(column pairs split over the CTAs, ``[K/16][R][16]`` per CTA with the mma.sync A-fragment order of
the 16 k of a block; the down projection split in NGRP K-slice groups first) and compared with
what ``pack_weights`` produced: each packed buffer must be exactly that permutation of its source.
"""
import numpy as np
import pytest
import torch

from reki_megakernel_b200.packing import NGRP, pack_weights
from reki_megakernel_b200.synthetic import ExpertDims, make_weights


def _perm16(kk: np.ndarray) -> np.ndarray:
    """Position of k within a 16-element block: k 0,1,8,9, 2,3,10,11, ... are stored in order."""
    return ((kk & 7) >> 1) * 4 + (kk >> 3) * 2 + (kk & 1)


def _split(N: int, G: int):
    """First row and row count of every CTA when N rows are split in column pairs over G CTAs."""
    P = N // 2
    lo = (np.arange(G + 1) * P) // G
    return 2 * lo[:-1], 2 * (lo[1:] - lo[:-1])


def _positions(L: int, N: int, K: int, G: int, nm: int = 1, m: int = 0) -> np.ndarray:
    """Packed element offset of W[l, n, k] for matrix m of an nm-matrix stage, shape [L, N, K]."""
    r0, R = _split(N, G)
    owner = np.searchsorted(r0 + R, np.arange(N), side="right")  # CTA whose rows hold n
    assert np.all((r0[owner] <= np.arange(N)) & (np.arange(N) < r0[owner] + R[owner]))
    n = np.arange(N)[:, None]
    k = np.arange(K)[None, :]
    o = owner[:, None]
    within = (k // 16) * R[o] * 16 + (n - r0[o]) * 16 + _perm16(k % 16)
    per_layer = nm * r0[o] * K + m * R[o] * K + within
    return np.arange(L)[:, None, None] * (nm * N * K) + per_layer[None]


def _down_positions(L: int, N: int, I: int, G: int) -> np.ndarray:
    KS = I // NGRP
    out = np.empty((L, N, I), dtype=np.int64)
    for j in range(NGRP):
        gn = ((j + 1) * G) // NGRP - (j * G) // NGRP
        pos = _positions(L, N, KS, gn)                       # layer stride N * KS inside the group
        l = np.arange(L)[:, None, None]
        out[:, :, j * KS:(j + 1) * KS] = (pos - l * N * KS) + l * N * I + j * N * KS
    return out


def _check(buf: torch.Tensor, src: torch.Tensor, pos: np.ndarray):
    flat = buf.view(torch.int16).numpy()
    assert flat.size == pos.size
    assert np.array_equal(np.sort(pos.reshape(-1)), np.arange(pos.size)), "positions are not a permutation"
    np.testing.assert_array_equal(flat[pos.reshape(-1)], src.contiguous().view(torch.int16).numpy().reshape(-1))


@pytest.mark.parametrize("G", [148, 37, 7])
def test_packed_buffers_are_the_documented_permutation(G):
    d = ExpertDims(L=2, H=128, NH=2, HD=64, I=512, A=32)
    w = make_weights(d, seed=3)
    pk = pack_weights(w, G)
    L, H, I = d.L, d.H, d.I
    _check(pk["w"][0], w.wqkv, _positions(L, 3 * H, H, G))
    _check(pk["w"][1], w.wo, _positions(L, H, H, G))
    _check(pk["w"][2], w.wqca, _positions(L, H, H, G))
    _check(pk["w"][3], w.woca, _positions(L, H, H, G))
    # gate and up rows of a CTA back to back: one buffer holding both matrices
    gu = pk["w"][4].view(torch.int16).numpy()
    pg, pu = _positions(L, I, H, G, nm=2, m=0), _positions(L, I, H, G, nm=2, m=1)
    both = np.concatenate([pg.reshape(-1), pu.reshape(-1)])
    assert np.array_equal(np.sort(both), np.arange(gu.size))
    np.testing.assert_array_equal(gu[pg.reshape(-1)], w.wg.view(torch.int16).numpy().reshape(-1))
    np.testing.assert_array_equal(gu[pu.reshape(-1)], w.wu.view(torch.int16).numpy().reshape(-1))
    _check(pk["w"][5], w.wd, _down_positions(L, H, I, G))


def test_fp32_tail_and_norm_buffers():
    d = ExpertDims(L=2, H=128, NH=2, HD=64, I=512, A=32)
    w = make_weights(d, seed=4)
    pk = pack_weights(w, 148)
    H = d.H
    torch.testing.assert_close(pk["nrm"], torch.stack([1.0 + w.qn.float(), 1.0 + w.kn.float(), 1.0 + w.qcan.float()]),
                               rtol=0, atol=0)
    tail = pk["tailw"]
    torch.testing.assert_close(tail[:8 * H].view(8, H), w.win.float()[:8], rtol=0, atol=0)
    torch.testing.assert_close(tail[8 * H:9 * H], w.bin.float(), rtol=0, atol=0)
    torch.testing.assert_close(tail[9 * H:9 * H + w.bout.numel()], w.bout.float(), rtol=0, atol=0)
    torch.testing.assert_close(pk["wout"], w.wout.float(), rtol=0, atol=0)
