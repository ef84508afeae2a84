"""CPU restatement of the cross-attention K/V preparation ("register_prepare") — test
infrastructure only: imported by tests/, __graft_entry__.smoke() and bench.py's CPU legs, never by
the product path.

Parity unpinned: the producer of the reference's cross-attention K/V (Kyutai's
``register_prepare``, described in README.md:279-281 as the 31 M-weight projection of the 2048-wide
VLM source) is not part of the reference checkout. The reference megakernel only consumes its
output (``past.cross_attn_kv``, src/mk_expert.py:486-495): per layer K [SP, NH, HD] and V, K already
head-normed and rotated, which is what the cross-attention stage expects
(src/mk_expert.py:225-251, "K arrives already normed/rotated"). This restatement fixes the math the
library implements:

    k = src . Wk^T ; K = bf16( RoPE( RMSNorm_HD(k) * (1 + kn) ) ) ; V = bf16( src . Wv^T )

on bf16 src and weights with float64 accumulation here (the GPU accumulates in fp32), fp32-level
norm and rotate-half RoPE with the expert's cos/sin tables, one bf16 rounding at the end.
"""
from __future__ import annotations

import torch


def prepare_oracle(wkv: torch.Tensor, kn: torch.Tensor, src: torch.Tensor, cos: torch.Tensor,
                   sin: torch.Tensor, eps: float = 1e-6):
    """wkv [L, 2, H, src_dim] bf16, kn [L, HD], src [S, src_dim] bf16, cos/sin [S, HD] fp32 ->
    (K, V) bf16 [L, S, NH, HD] with NH = H / HD."""
    L, _, H, D = wkv.shape
    HD = kn.shape[1]
    NH = H // HD
    S = src.shape[0]
    x = src.double()
    ks, vs = [], []
    c = cos.double()[:, None, :]
    s_ = sin.double()[:, None, :]
    for l in range(L):
        k = (x @ wkv[l, 0].double().T).reshape(S, NH, HD)
        v = (x @ wkv[l, 1].double().T).reshape(S, NH, HD)
        k = k * torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + eps) * (1.0 + kn[l].double())
        rot = torch.cat([-k[..., HD // 2:], k[..., :HD // 2]], dim=-1)
        k = k * c + rot * s_
        ks.append(k.float().to(torch.bfloat16))
        vs.append(v.float().to(torch.bfloat16))
    return torch.stack(ks), torch.stack(vs)
