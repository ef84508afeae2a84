"""CPU oracle of the register pass, the register-memory carry and the whole 10-step predict.
TEST INFRASTRUCTURE ONLY: imported by tests/, never by the product path.

Parity unpinned. The reference megakernel runs Euler steps 2..N; step 1 -- the action rows together
with the current frame's register rows, which yields that frame's register K/V -- and the register
cache that carries frames from predict to predict are Kyutai's (``_expert_first_step`` and
``_register_cache``, bound and read at ``src/mk_expert.py:527-533`` and
``src/profile_breakdown.py:97-100``; described in the reference README as "register rows with plain
norms, segmented varlen attention over the register buffer, the register K/V output"), and are not
in the reference checkout. This file fixes the restatement the library implements:

* register pass (``register_pass``): R register rows through every layer with the action rows' math
  but plain norms and residuals (AdaRMS scale = shift = 0, gates 1: ``plain_row``); in each layer
  the rows' own K (per-head RMSNorm with 1 + k_norm, RoPE, bf16) and V are written into the memory
  rows [PM - R, PM) first, then the rows attend over the memory rows [kv_start, PM) -- older frames
  and the current frame -- and over the cross-attention source; no output besides the memory;
* carry (``roll_frames``): before each predict the memory moves up by one frame (R rows), the oldest
  frame drops out; after predict p (0-based) ``min(p + 1, PM / R)`` frames are valid, so
  kv_start = PM - R * min(p + 1, PM / R) (``frames_valid``);
* step 1 of the action rows is the same computation as steps 2..N (memory of the current and older
  frames, own rows), so the whole predict is N Euler steps from the noise with the modulation rows
  of all N steps (``predict``).

Rounding points are the action rows' (``OracleExpert``): bf16 at every Linear output, gated residual
and norm, fp32 softmax statistics, P rounded before P V.
"""
from __future__ import annotations

import torch

from oracle.expert_oracle import OracleExpert
from oracle.modulation_oracle import modulation_oracle
from oracle.prepare_oracle import prepare_oracle
from reki_megakernel_b200.synthetic import rope_cos_sin


def plain_row(d) -> torch.Tensor:
    """The modulation row of the register rows [MODW] fp32: scale and shift 0, every gate 1."""
    m = torch.zeros(d.MODW)
    H = d.H
    for l in range(d.L):
        for blk in range(3):
            o = 9 * H * l + 3 * H * blk + 2 * H
            m[o:o + H] = 1.0
    return m


def frames_valid(p: int, PM: int, R: int) -> int:
    """Frames in the memory during predict p (0-based), the current one included."""
    return min(p + 1, PM // R)


def kv_start_of(p: int, PM: int, R: int) -> int:
    return PM - R * frames_valid(p, PM, R)


def roll_frames(memk: torch.Tensor, memv: torch.Tensor, R: int) -> None:
    """Moves every layer's memory rows [R, PM) to [0, PM - R) in place (the oldest frame drops)."""
    for m in (memk, memv):
        m[:, :-R] = m[:, R:].clone()


def register_pass(orc: OracleExpert, reg_in: torch.Tensor, memk: torch.Tensor, memv: torch.Tensor, kv_start: int,
                  kca: torch.Tensor, vca: torch.Tensor, S: int, sa_pe, ca_pe) -> torch.Tensor:
    """Writes the register K/V of every layer into memk / memv [L, PM, NH, HD] rows [PM - R, PM)
    (in place) and returns the register rows after the last layer [R, H]."""
    R = reg_in.shape[0]
    PM = memk.shape[1]
    ep = dict(memk=memk, memv=memv, kv_start=kv_start, kca=kca, vca=vca, S=S, sa_cos=sa_pe[0].float(),
              sa_sin=sa_pe[1].float(), ca_cos=ca_pe[0].float(), ca_sin=ca_pe[1].float())
    h = reg_in.float()
    mrow = plain_row(orc.d).to(h.device)
    for l in range(orc.d.L):
        h, _ = orc.layer(l, h, mrow, ep, frame_row0=PM - R)
    return h


class PredictOracle:
    """A sequence of whole predicts carrying the register memory: for predict p, given the VLM
    source rows, the proprio state and the flow noise -- roll the memory, prepare the
    cross-attention K/V, the modulation rows, the register pass, then N Euler steps of the action
    rows from the noise. Producers: ``prepare_oracle`` and ``modulation_oracle``."""

    def __init__(self, orc: OracleExpert, prep_w, mod_w, reg_in: torch.Tensor, *, N: int = 10, PM: int = 96,
                 R: int = 32, T: int = 10, action_dim: int = 7):
        d = orc.d
        self.orc, self.prep_w, self.mod_w, self.reg_in = orc, prep_w, mod_w, reg_in
        self.N, self.PM, self.R, self.T, self.action_dim = N, PM, R, T, action_dim
        self.memk = torch.zeros((d.L, PM, d.NH, d.HD), dtype=torch.bfloat16)
        self.memv = torch.zeros_like(self.memk)
        self.p = 0
        self.reg_sa = rope_cos_sin(torch.arange(R) + (PM - R), d.HD)
        self.reg_ca = rope_cos_sin(torch.arange(R), d.HD)
        self.act_sa = rope_cos_sin(torch.arange(T) + PM, d.HD)
        self.act_ca = rope_cos_sin(torch.arange(T), d.HD)

    def predict(self, src: torch.Tensor, state: torch.Tensor, noise: torch.Tensor, kv=None, mods_dt=None) -> torch.Tensor:
        """src [S, src_dim] bf16, state [sdim], noise [T, A] fp32 -> actions [T, A] fp32. ``kv`` = (K, V)
        [L, >= S, NH, HD] and ``mods_dt`` = (mods [N, MODW], dt) replace the two producers' outputs
        (to check the rest against a device run's own producer outputs)."""
        d = self.orc.d
        S = src.shape[0]
        roll_frames(self.memk, self.memv, self.R)
        ks = kv_start_of(self.p, self.PM, self.R)
        if kv is None:
            cos, sin = rope_cos_sin(torch.arange(S), d.HD)
            kca, vca = prepare_oracle(self.prep_w.wkv, self.prep_w.kn, src, cos, sin, self.prep_w.eps)
        else:
            kca, vca = (t.cpu() for t in kv)
        if mods_dt is None:
            mw = self.mod_w
            mods, dt = modulation_oracle(mw.w_t, mw.w_s, mw.w_m, mw.b_m, state, self.N)
        else:
            mods, dt = mods_dt[0].cpu(), float(mods_dt[1])
        register_pass(self.orc, self.reg_in, self.memk, self.memv, ks, kca, vca, S, self.reg_sa, self.reg_ca)
        ep = dict(x=noise.float(), mods=torch.cat([mods[:1], mods]).float(), dt=dt, memk=self.memk,
                  memv=self.memv, kv_start=ks, kca=kca, vca=vca, S=S, sa_cos=self.act_sa[0], sa_sin=self.act_sa[1],
                  ca_cos=self.act_ca[0], ca_sin=self.act_ca[1], action_dim=self.action_dim)
        self.p += 1
        return self.orc.run_episode(ep)
