"""CPU oracle for the REKI action-expert Euler loop, steps 2..N.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import this module, and only as the checker or the timed CPU baseline. The product path
(``reki_megakernel_b200``) never calls it and fails loudly when its CUDA library is missing.

What it restates (file:line in the reference project ``muninn-huginn/reki-megakernel``):

* mode ``"bf16"`` follows the reference megakernel's rounding points exactly
  (``src/mk_expert.py:26-29``): bf16 GEMM inputs with fp32 accumulation and one bf16 rounding per
  Linear output (``:106-159``, ``:348``, ``:378``); AdaRMS input rounded to bf16 (``:119``); gated
  residuals ``bf16(res + bf16(acc) * gate)`` (``:162-172``); per-head RMSNorm with weight ``1 + w``
  then rotate-half RoPE, rounded after the norm and after the rotation (``:175-193``);
  self-attention over memory rows ``[cu_kv[0], PM)`` concatenated with the action rows, single
  softmax, ``P`` rounded to bf16 before ``P V`` (``:196-222``); cross-attention with an online
  softmax over 64-row blocks (``:225-251``); ``g = bf16(silu(bf16(gate)) * bf16(up))`` (``:403-413``);
  fp32 step tail: final AdaRMS rounded to bf16, fp32 out-projection, Euler update of the padded
  action state, fp32 in-projection rounded to bf16 (``:254-299``; ``archive/mk_expert_v1.py:196-228``);
  per-step modulation rows laid out ``[sa(scale,shift,gate), ca(...), mlp(...)] x L, final(scale,
  shift)`` (``:336-340``, ``:423``); loop order ``FIRST tail, for s: for l: 8 stages; tail``
  (``:326-426``).
* mode ``"fp32"`` is the same expert in plain fp32 (weights upcast once, no intermediate rounding):
  the eager CPU expert used as the timed CPU baseline.

Parity status: pinned against the reference's own Triton kernel run on identical seeded inputs
(``tests/golden/make_golden.py`` runs ``src/mk_expert.py`` through Triton's CPU interpreter; the
fixtures it wrote live in ``tests/golden/``). Kyutai's original expert is not available, so parity
against it is unpinned.
"""
from __future__ import annotations

import torch

from reki_megakernel_b200.synthetic import ExpertWeights, StepInputs

AO = 8          # real action dims carried through the loop (``src/mk_expert.py:478``)
CA_BLOCK = 64   # cross-attention block of the reference's online softmax (``src/mk_expert.py:478`` BS)


def _bf(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).float()


class OracleExpert:
    """fp32 copies of the weights plus the per-step math; ``run`` integrates steps 2..N."""

    def __init__(self, w: ExpertWeights, mode: str = "bf16", device="cpu"):
        if mode not in ("bf16", "fp32"):
            raise ValueError(mode)
        self.mode = mode
        self.d = w.dims
        self.dev = torch.device(device)
        f = lambda t: t.detach().to(self.dev, torch.float32).contiguous()  # noqa: E731
        self.wqkv, self.wo, self.wqca, self.woca = f(w.wqkv), f(w.wo), f(w.wqca), f(w.woca)
        self.wg, self.wu, self.wd = f(w.wg), f(w.wu), f(w.wd)
        self.qn, self.kn, self.qcan = f(w.qn), f(w.kn), f(w.qcan)
        self.win, self.bin, self.wout, self.bout = f(w.win), f(w.bin), f(w.wout), f(w.bout)
        self.eps, self.qk_eps = float(w.eps), float(w.qk_eps)

    # ---- helpers -----------------------------------------------------------------------------
    def _r(self, t):
        return _bf(t) if self.mode == "bf16" else t

    def _adarms(self, h, scale, shift):
        """AdaRMS: rsqrt(mean(h^2) + eps) * h * (1 + scale) + shift (``src/mk_expert.py:93-122``)."""
        rstd = torch.rsqrt(h.pow(2).sum(-1, keepdim=True) / h.shape[-1] + self.eps)
        return self._r(h * rstd * (1.0 + scale) + shift)

    def _linear(self, a, w):
        return self._r(a @ w.T)

    def _gated(self, res, acc, gate):
        return self._r(res + self._r(acc) * gate)

    def _norm_rope(self, x, w, cos, sin):
        """Per-head RMSNorm (weight 1 + w) then rotate-half RoPE (``src/mk_expert.py:175-193``)."""
        HD = x.shape[-1]
        r = torch.rsqrt(x.pow(2).sum(-1, keepdim=True) / HD + self.qk_eps)
        xn = self._r(x * r * (1.0 + w))
        perm = (torch.arange(HD, device=x.device) + HD // 2) % HD
        xpn = self._r(x[..., perm] * r * (1.0 + w[perm]))
        sign = torch.where(torch.arange(HD, device=x.device) < HD // 2, -1.0, 1.0)
        return self._r(xn * cos + sign * xpn * sin)

    # ---- attention ---------------------------------------------------------------------------
    def _sa(self, l, qkv, memk, memv, kv_start, cos, sin, own: bool = True):
        """Self-attention of the action rows over [memory rows kv_start..PM || own rows]
        (``src/mk_expert.py:196-222``); ``own=False``: the memory rows only (the register pass, whose
        rows are already in the memory)."""
        d = self.d
        H, NH, HD = d.H, d.NH, d.HD
        scale = HD ** -0.5
        T = qkv.shape[0]
        y = torch.empty(T, H, device=qkv.device)
        for h in range(NH):
            sl = slice(h * HD, (h + 1) * HD)
            q = self._norm_rope(qkv[:, sl], self.qn[l], cos, sin)
            k = self._norm_rope(qkv[:, H + h * HD: H + (h + 1) * HD], self.kn[l], cos, sin)
            v = qkv[:, 2 * H + h * HD: 2 * H + (h + 1) * HD]
            mk = memk[l, kv_start:, h].float()
            mv = memv[l, kv_start:, h].float()
            if not own:
                k, v = k[:0], v[:0]
            s1 = (q @ mk.T) * scale
            s2 = (q @ k.T) * scale
            ninf = torch.full((T, 1), -float("inf"), device=q.device)
            mx = torch.maximum(s1.amax(1, keepdim=True) if s1.shape[1] else ninf,
                               s2.amax(1, keepdim=True) if s2.shape[1] else ninf)
            p1 = torch.exp(s1 - mx)
            p2 = torch.exp(s2 - mx)
            den = p1.sum(1, keepdim=True) + p2.sum(1, keepdim=True)
            o = (self._r(p1) @ mv + self._r(p2) @ v) / den
            y[:, sl] = self._r(o)
        return y

    def _ca(self, l, qca, kca, vca, S, cos, sin):
        """Cross-attention over the S valid rows of the cached source K/V, online softmax in
        64-row blocks (``src/mk_expert.py:225-251``)."""
        d = self.d
        H, NH, HD = d.H, d.NH, d.HD
        scale = HD ** -0.5
        T = qca.shape[0]
        y = torch.empty(T, H, device=qca.device)
        for h in range(NH):
            sl = slice(h * HD, (h + 1) * HD)
            q = self._norm_rope(qca[:, sl], self.qcan[l], cos, sin)
            k_all = kca[l, :S, h].float()
            v_all = vca[l, :S, h].float()
            if self.mode == "fp32":
                s = (q @ k_all.T) * scale
                p = torch.softmax(s, dim=1)
                y[:, sl] = p @ v_all
                continue
            mx = torch.full((T, 1), -float("inf"), device=q.device)
            den = torch.zeros(T, 1, device=q.device)
            acc = torch.zeros(T, HD, device=q.device)
            for s0 in range(0, S, CA_BLOCK):
                k = k_all[s0:s0 + CA_BLOCK]
                v = v_all[s0:s0 + CA_BLOCK]
                s = (q @ k.T) * scale
                mn = torch.maximum(mx, s.amax(1, keepdim=True))
                alpha = torch.exp(mx - mn)
                p = torch.exp(s - mn)
                den = den * alpha + p.sum(1, keepdim=True)
                acc = acc * alpha + self._r(p) @ v
                mx = mn
            y[:, sl] = self._r(acc / den)
        return y

    # ---- one episode ---------------------------------------------------------------------------
    def layer(self, l, h, mrow, ep, frame_row0: int | None = None):
        """One expert layer (8 stages of ``src/mk_expert.py:342-421``). Returns (h_out, parts).

        ``frame_row0`` set: the register pass -- the rows' own K (norm + RoPE, rounded) and V are first
        written into ``ep["memk"]`` / ``ep["memv"]`` rows [frame_row0, frame_row0 + rows) of layer l,
        then the self-attention reads the memory rows only."""
        d = self.d
        H, NH, HD = d.H, d.NH, d.HD
        m_sa = mrow[(3 * l) * 3 * H:]
        m_ca = m_sa[3 * H:]
        m_mlp = m_ca[3 * H:]
        a = self._adarms(h, m_sa[:H], m_sa[H:2 * H])
        qkv = self._linear(a, self.wqkv[l])
        if frame_row0 is not None:
            R = qkv.shape[0]
            for hh in range(NH):
                k = self._norm_rope(qkv[:, H + hh * HD: H + (hh + 1) * HD], self.kn[l], ep["sa_cos"], ep["sa_sin"])
                ep["memk"][l, frame_row0:frame_row0 + R, hh] = k.to(ep["memk"].dtype)
                ep["memv"][l, frame_row0:frame_row0 + R, hh] = qkv[:, 2 * H + hh * HD: 2 * H + (hh + 1) * HD].to(
                    ep["memv"].dtype)
        y = self._sa(l, qkv, ep["memk"], ep["memv"], ep["kv_start"], ep["sa_cos"], ep["sa_sin"],
                     own=frame_row0 is None)
        h2 = self._gated(h, y @ self.wo[l].T, m_sa[2 * H:3 * H])
        a = self._adarms(h2, m_ca[:H], m_ca[H:2 * H])
        qca = self._linear(a, self.wqca[l])
        y = self._ca(l, qca, ep["kca"], ep["vca"], ep["S"], ep["ca_cos"], ep["ca_sin"])
        h3 = self._gated(h2, y @ self.woca[l].T, m_ca[2 * H:3 * H])
        a = self._adarms(h3, m_mlp[:H], m_mlp[H:2 * H])
        gf = self._r(a @ self.wg[l].T)
        uf = self._r(a @ self.wu[l].T)
        g = self._r(gf / (1.0 + torch.exp(-gf)) * uf)
        hout = self._gated(h3, g @ self.wd[l].T, m_mlp[2 * H:3 * H])
        return hout, dict(qkv=qkv, h2=h2, qca=qca, h3=h3, g=g)

    def in_proj(self, xpad):
        """h0 = bf16(xpad[:, :AO] @ Win[:AO] + bin), fp32 products (``src/mk_expert.py:280-293``)."""
        hacc = self.bin[None, :].expand(xpad.shape[0], -1).clone()
        for a in range(AO):
            hacc = hacc + xpad[:, a:a + 1] * self.win[a][None, :]
        return self._r(hacc)

    def velocity(self, h, modf):
        """v = AdaRMS_final(h) (rounded) @ Wout^T + bout in fp32 (``src/mk_expert.py:271-299``)."""
        H = self.d.H
        o = self._adarms(h, modf[:H], modf[H:2 * H])
        return o @ self.wout.T + self.bout[None, :]

    def run_episode(self, ep: dict, trace: list | None = None) -> torch.Tensor:
        """Steps 2..N of one episode. ``ep``: x [T, A], mods [N, MODW], dt, memk/memv
        [L, PM, NH, HD], kv_start, kca/vca [L, SP, NH, HD], S, cos/sin [T, HD], action_dim."""
        d = self.d
        L, H = d.L, d.H
        adim = ep["action_dim"]
        x = ep["x"].float().clone()
        T, A = x.shape
        mods = ep["mods"].float()
        dt = float(ep["dt"])
        keep = (torch.arange(A, device=x.device) < adim)[None, :]
        h = self.in_proj(torch.where(keep, x, 0.0))
        n_steps = mods.shape[0] - 1
        for s in range(n_steps):
            mrow = mods[1 + s]
            for l in range(L):
                h, parts = self.layer(l, h, mrow, ep)
                if trace is not None:
                    trace.append(dict(step=s, layer=l, h=h.clone(), **parts))
            v = self.velocity(h, mrow[3 * L * 3 * H:])
            x = torch.where(keep, x, 0.0) + dt * v
            h = self.in_proj(torch.where(keep, x, 0.0))
        return x

    def run(self, inp: StepInputs, trace: list | None = None) -> torch.Tensor:
        """All episodes of ``inp``; returns [B, T, A] fp32 (the state after step N)."""
        outs = []
        for b in range(inp.x.shape[0]):
            e = inp.episode(b).to(self.dev)
            ep = dict(x=e.x[0], mods=e.mods[0], dt=e.dt[0], memk=e.memk[0], memv=e.memv[0],
                      kv_start=int(e.kv_start[0]), kca=e.kca[0], vca=e.vca[0], S=int(e.S[0]),
                      sa_cos=e.sa_cos[0].float(), sa_sin=e.sa_sin[0].float(),
                      ca_cos=e.ca_cos[0].float(), ca_sin=e.ca_sin[0].float(), action_dim=inp.action_dim)
            outs.append(self.run_episode(ep, trace if b == 0 else None))
        return torch.stack(outs)


def _native_layer(h, m_sa, m_ca, m_mlp, wqkv, wo, wqca, woca, wg, wu, wd, qn, kn, qcan, memk, memv, kca, vca,
                  sa_cos, sa_sin, ca_cos, ca_sin, eps: float, qk_eps: float):
    """One expert layer on native bf16 tensors (see ``NativeBf16Expert``). h [T, H] bf16; m_* [3H]
    fp32 (scale, shift, gate); weights bf16 [N, K]; qn / kn / qcan fp32 [HD] (offsets, scale 1 + w);
    memk / memv [M, NH, HD] bf16 (valid rows only); kca / vca [S, NH, HD] bf16 (valid rows only);
    cos / sin fp32 [T, HD]. Returns h after the layer, bf16."""
    T, H = h.shape
    NH, HD = memk.shape[1], memk.shape[2]
    bf = torch.bfloat16

    def adarms(x, sc, sh):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * (1.0 + sc) + sh).to(bf)

    def norm_rope(x, w, cos, sin):
        xf = x.float()
        xn = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + qk_eps) * (1.0 + w)).to(bf).float()
        rot = torch.cat([-xn[..., HD // 2:], xn[..., :HD // 2]], -1)
        return (xn * cos[:, None] + rot * sin[:, None]).to(bf)

    def attend(q, k, v):  # q [T, NH, HD], k / v [N, NH, HD] -> [T, H]
        o = torch.nn.functional.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None],
                                                             v.transpose(0, 1)[None])
        return o[0].transpose(0, 1).reshape(T, H)

    def gated(res, o, gate):
        return (res.float() + o.float() * gate).to(bf)

    qkv = adarms(h, m_sa[:H], m_sa[H:2 * H]) @ wqkv.T
    q = norm_rope(qkv[:, :H].reshape(T, NH, HD), qn, sa_cos, sa_sin)
    k = norm_rope(qkv[:, H:2 * H].reshape(T, NH, HD), kn, sa_cos, sa_sin)
    v = qkv[:, 2 * H:].reshape(T, NH, HD)
    y = attend(q, torch.cat([memk, k], 0), torch.cat([memv, v], 0))
    h2 = gated(h, y @ wo.T, m_sa[2 * H:3 * H])
    qc = norm_rope((adarms(h2, m_ca[:H], m_ca[H:2 * H]) @ wqca.T).reshape(T, NH, HD), qcan, ca_cos, ca_sin)
    h3 = gated(h2, attend(qc, kca, vca) @ woca.T, m_ca[2 * H:3 * H])
    a = adarms(h3, m_mlp[:H], m_mlp[H:2 * H])
    g = (torch.nn.functional.silu((a @ wg.T).float()) * (a @ wu.T).float()).to(bf)
    return gated(h3, g @ wd.T, m_mlp[2 * H:3 * H])


class NativeBf16Expert:
    """The expert written the way a PyTorch model runs it in bf16, an implementation independent of
    the oracle's rounding model: bf16 Linear layers (library GEMMs with fp32 accumulation and bf16
    output), AdaRMS and gated residuals in fp32 rounded to bf16, per-head RMSNorm + rotate-half RoPE,
    attention through ``scaled_dot_product_attention`` on bf16 q / k / v, SiLU-gated MLP, and the
    oracle's fp32 step tail (``src/mk_expert.py:254-299``). ``compile=True`` runs every layer through
    ``torch.compile`` (Inductor): the stand-in for the reference's compiled expert, which
    ``src/test_mk.py:36-40`` compares with its eager expert and the megakernel (Kyutai's model is not
    available here). Test infrastructure; meant for a CUDA device."""

    def __init__(self, w: ExpertWeights, device="cuda", compile: bool = False):
        self.tail = OracleExpert(w, "bf16", device)
        self.dev = torch.device(device)
        bf = torch.bfloat16
        g = lambda t: t.detach().to(self.dev, bf).contiguous()  # noqa: E731
        self.w = dict(wqkv=g(w.wqkv), wo=g(w.wo), wqca=g(w.wqca), woca=g(w.woca), wg=g(w.wg), wu=g(w.wu), wd=g(w.wd))
        f = lambda t: t.detach().to(self.dev, torch.float32).contiguous()  # noqa: E731
        self.qn, self.kn, self.qcan = f(w.qn), f(w.kn), f(w.qcan)
        self.d = w.dims
        self.eps, self.qk_eps = float(w.eps), float(w.qk_eps)
        self.fn = torch.compile(_native_layer, dynamic=False) if compile else _native_layer

    def run(self, inp: StepInputs) -> torch.Tensor:
        d = self.d
        L, H = d.L, d.H
        outs = []
        for b in range(inp.x.shape[0]):
            e = inp.episode(b).to(self.dev)
            adim = inp.action_dim
            x = e.x[0].float().clone()
            mods = e.mods[0].float()
            dt = float(e.dt[0])
            ks, S = int(e.kv_start[0]), int(e.S[0])
            keep = (torch.arange(x.shape[1], device=self.dev) < adim)[None, :]
            h = self.tail.in_proj(torch.where(keep, x, 0.0)).to(torch.bfloat16)
            for s in range(mods.shape[0] - 1):
                mrow = mods[1 + s]
                for l in range(L):
                    m = mrow[9 * H * l:]
                    h = self.fn(h, m[:3 * H], m[3 * H:6 * H], m[6 * H:9 * H],
                                *(self.w[k][l] for k in ("wqkv", "wo", "wqca", "woca", "wg", "wu", "wd")),
                                self.qn[l], self.kn[l], self.qcan[l], e.memk[0, l, ks:], e.memv[0, l, ks:],
                                e.kca[0, l, :S], e.vca[0, l, :S], e.sa_cos[0].float(), e.sa_sin[0].float(),
                                e.ca_cos[0].float(), e.ca_sin[0].float(), self.eps, self.qk_eps)
                v = self.tail.velocity(h.float(), mrow[9 * H * L:])
                x = torch.where(keep, x, 0.0) + dt * v
                h = self.tail.in_proj(torch.where(keep, x, 0.0)).to(torch.bfloat16)
            outs.append(x)
        return torch.stack(outs)


def chunk_diff(a: torch.Tensor, b: torch.Tensor, action_dim: int = 7) -> dict:
    """max / mean |a - b| over the real action dims (``src/compare.py:16-25``)."""
    d = (a[..., :action_dim].float() - b[..., :action_dim].float()).abs()
    return {"max_abs": float(d.max()), "mean_abs": float(d.mean())}
