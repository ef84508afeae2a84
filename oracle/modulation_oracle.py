"""CPU restatement of the per-step modulation network ("_step_modulations") — test infrastructure
only: imported by tests/, __graft_entry__.smoke() and bench.py's CPU legs, never by the product path.

Parity unpinned: the reference's expert takes its per-step AdaRMS modulation rows from Kyutai's
``RekiFlowModel._step_modulations(num_steps, state_cond) -> (mods, dt)`` (called by ``install``,
src/mk_expert.py:527-535), which is not part of the reference checkout. The reference fixes only
the output: ``mods [N, MODW]`` with MODW = 3L*3H + 2H, per layer [scale, shift, gate] of the SA, CA
and MLP blocks, then [scale, shift] of the final norm (the offsets the megakernel reads,
src/mk_expert.py:336-340,423), and dt. This restatement fixes the math the library implements:

    t_s = 1 - s/N ; temb_s = [cos(1000 t_s f_i), sin(1000 t_s f_i)], f_i = 10000^(-i/(tdim/2))
    e_s = 8 (W_t temb_s + W_s state) ; a_s = bf16(silu(e_s)) ; mods_s = bf16(W_m a_s + b_m) ; dt = 1/N

in float64 here (the GPU: fp32 conditioning, fp32 accumulation of the bf16 projection), with the
two bf16 roundings at the same points.
"""
from __future__ import annotations

import math

import torch


def conditioning_oracle(w_t: torch.Tensor, w_s: torch.Tensor, state: torch.Tensor, N: int) -> torch.Tensor:
    """Projection input a [N, H] (bf16 values, returned as float64)."""
    tdim = w_t.shape[1]
    half = tdim // 2
    t = 1.0 - torch.arange(N, dtype=torch.float64) / N
    f = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float64) / half)
    ang = 1000.0 * t[:, None] * f[None, :]
    temb = torch.cat([ang.cos(), ang.sin()], dim=1)
    e = 8.0 * (temb @ w_t.double().T + state.double().reshape(1, -1) @ w_s.double().T)
    a = e / (1.0 + torch.exp(-e))
    return a.to(torch.bfloat16).double()


def modulation_oracle(w_t: torch.Tensor, w_s: torch.Tensor, w_m: torch.Tensor, b_m: torch.Tensor,
                      state: torch.Tensor, N: int):
    """(mods [N, MODW] bf16, dt float) of an N-step predict."""
    a = conditioning_oracle(w_t, w_s, state, N)
    mods = a @ w_m.double().T + b_m.double()[None, :]
    return mods.to(torch.bfloat16), 1.0 / N
