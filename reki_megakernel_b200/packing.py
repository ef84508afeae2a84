"""Host-side packing of the expert weights into the kernel's layout (for ``mkx_run_static``).

``mkx_create`` packs on the device into memory it allocates. A caller that cannot allocate device
memory runs ``mkx_run_static`` instead and must hand it the packed weights in memory it already owns;
``pack_weights`` produces them on the CPU (once, e.g. at build time), to be copied into that memory.

Layout, per weight stage ([L, N, K] row-major bf16; gate/up interleaved per CTA): the N output rows are
split in column pairs over the G CTAs (CTA i owns pairs [i P / G, (i+1) P / G), P = N / 2); each CTA's
R rows are stored at element offset r0 * K of the layer (gate/up: 2 r0 K, gate rows then up rows) as
[K / 16][R][16], the 16 k of a block in the order the mma.sync A fragment reads them
(k 0,1,8,9, 2,3,10,11, 4,5,12,13, 6,7,14,15).

The down projection (Wd [L, H, I]) is split in two levels: the G CTAs form NGRP = 4 contiguous
groups (group j = CTAs [j G / 4, (j+1) G / 4)), group j owns the K-slice [j I / 4, (j+1) I / 4) for
all H rows, and inside a layer group j's block (H x I / 4 elements, at offset j H I / 4) holds the
slice split over the group's CTAs in the layout above.
"""
from __future__ import annotations

import torch

from .synthetic import ExpertWeights

AO = 8
TAIL_FLOATS_EXTRA = 32
NGRP = 4


def _perm16() -> torch.Tensor:
    """inv[pos] = k: the source k stored at position pos of a 16-element block."""
    pos = [((kk & 7) >> 1) * 4 + (kk >> 3) * 2 + (kk & 1) for kk in range(16)]
    inv = [0] * 16
    for kk, p in enumerate(pos):
        inv[p] = kk
    return torch.tensor(inv)


def _pack(mats: list[torch.Tensor], G: int) -> torch.Tensor:
    L, N, K = mats[0].shape
    P = N // 2
    nm = len(mats)
    inv = _perm16()
    out = torch.empty(L, nm * N * K, dtype=torch.bfloat16)
    for i in range(G):
        lo, hi = (i * P) // G, ((i + 1) * P) // G
        r0, R = 2 * lo, 2 * (hi - lo)
        for m, w in enumerate(mats):
            c = w[:, r0:r0 + R, :].reshape(L, R, K // 16, 16).permute(0, 2, 1, 3)[..., inv]
            base = nm * r0 * K + m * R * K
            out[:, base:base + R * K] = c.reshape(L, R * K)
    return out.reshape(-1)


def _pack_down(wd: torch.Tensor, G: int) -> torch.Tensor:
    L, N, I = wd.shape
    KS = I // NGRP
    out = torch.empty(L, N * I, dtype=torch.bfloat16)
    for j in range(NGRP):
        gn = ((j + 1) * G) // NGRP - (j * G) // NGRP
        out[:, j * N * KS:(j + 1) * N * KS] = _pack([wd[:, :, j * KS:(j + 1) * KS]], gn).reshape(L, N * KS)
    return out.reshape(-1)


def pack_weights(w: ExpertWeights, grid: int) -> dict:
    """CPU tensors in the kernel's layout for ``grid`` CTAs: ``w`` (6 bf16 buffers: QKV, O, CA-Q,
    CA-O, gate+up, down), ``nrm`` fp32 [3, L, HD] = 1 + norm weights, ``tailw`` fp32 (action_in_proj
    rows 0..7 transposed, its bias, the output bias padded to 32), ``wout`` fp32 [A, H]."""
    c = {k: v.detach().cpu() for k, v in w.tensors().items()}
    H = w.dims.H
    packed = [_pack([c["wqkv"]], grid), _pack([c["wo"]], grid), _pack([c["wqca"]], grid), _pack([c["woca"]], grid),
              _pack([c["wg"], c["wu"]], grid), _pack_down(c["wd"], grid)]
    nrm = torch.stack([1.0 + c[k].float() for k in ("qn", "kn", "qcan")]).contiguous()
    tail = torch.zeros(AO * H + H + TAIL_FLOATS_EXTRA, dtype=torch.float32)
    tail[:AO * H] = c["win"].float()[:AO].reshape(-1)
    tail[AO * H:AO * H + H] = c["bin"].float()
    tail[AO * H + H:AO * H + H + c["bout"].numel()] = c["bout"].float()
    return {"w": packed, "nrm": nrm, "tailw": tail, "wout": c["wout"].float().contiguous()}
