"""Episode-batch path: Euler steps 2..N of B independent episodes with one weight stream
(``include/mkx_batch.h``).

The reference megakernel serves one episode per launch (``ExpertMegakernel.run`` asserts
``x_t.shape[0] == 1``, src/mk_expert.py:488); its benchmark configuration also asks for 1, 8, 32 and
128 episodes per GPU. ``BatchedExpert`` stacks the episodes' action rows into M = B * T token rows and
runs every dense stage as one tcgen05 GEMM over all of them, so the 212 MB of weights cross HBM once
per Euler step for the whole batch instead of once per episode. Per episode the math is the
reference's (same stages and rounding points); inputs are the reference's ``run`` inputs stacked
over episodes, with each episode's own register memory, cross-attention K/V, modulation rows, noise,
dt, first valid memory row and source length.

There is no CPU fallback: the CUDA library must load.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .synthetic import ExpertWeights, StepInputs

AO = 8
TP = 16


class BatchedExpert:
    """``BatchedExpert(weights, max_episodes).run(inputs) -> x_out [B, T, A]``."""

    def __init__(self, weights: ExpertWeights, max_episodes: int, device=None):
        w = weights
        d = w.dims
        self.dims = d
        dev = torch.device(device) if device is not None else w.wqkv.device
        if dev.type != "cuda":
            raise ValueError("BatchedExpert needs the expert weights on a CUDA device")
        self.device = dev
        self.max_episodes = int(max_episodes)
        self._lib = _lib.load()
        t = {k: v.to(dev).contiguous() for k, v in w.tensors().items()}
        for k in ("wqkv", "wo", "wqca", "woca", "wg", "wu", "wd", "qn", "kn", "qcan"):
            if t[k].dtype != torch.bfloat16:
                raise ValueError(f"{k} must be bf16")
        for k in ("win", "bin", "wout", "bout"):
            t[k] = t[k].float().contiguous()
        dims = _lib.Dims(L=d.L, H=d.H, NH=d.NH, HD=d.HD, I=d.I, A=d.A, eps=float(w.eps), qk_eps=float(w.qk_eps),
                         max_rows=TP, grid=0)
        wts = _lib.Weights(**{f[0]: t[f[0]].data_ptr() for f in _lib.Weights._fields_})
        h = C.c_void_p()
        with torch.cuda.device(dev):
            torch.cuda.synchronize(dev)
            _lib.check(self._lib.mkx_batch_create(C.byref(dims), C.byref(wts), self.max_episodes, dev.index or 0,
                                                  C.byref(h)), "mkx_batch_create")
        self._h = h
        del t

    def launches(self, B: int, T: int, n_steps: int) -> int:
        """Kernel launches one ``run`` enqueues."""
        return int(self._lib.mkx_batch_launches(self._h, int(B), int(T), int(n_steps)))

    def run(self, inp: StepInputs, out: torch.Tensor | None = None) -> torch.Tensor:
        """Steps 2..N of every episode of ``inp`` (all tensors on the expert's device). ``inp.mods``
        [B, N, MODW] bf16; memory K/V [B, L, PM, NH, HD] valid from ``inp.kv_start[b]``;
        cross-attention K/V [B, L, SP, NH, HD] valid below ``inp.S[b]``. Returns x_out [B, T, A] fp32
        (``out`` when given); asynchronous on the current stream, graph-capturable."""
        d = self.dims
        x = inp.x
        if x.dim() != 3 or x.shape[2] != d.A or x.dtype != torch.float32:
            raise ValueError(f"x must be fp32 [B, T, {d.A}]")
        B, T = x.shape[0], x.shape[1]
        if not (1 <= B <= self.max_episodes) or not (1 <= T <= TP) or not (1 <= inp.action_dim <= AO):
            raise ValueError(f"B={B} (<= {self.max_episodes}), T={T} (<= {TP}), action_dim={inp.action_dim} (<= {AO})")
        MODW = 9 * d.L * d.H + 2 * d.H
        if inp.mods.dim() != 3 or inp.mods.shape[0] != B or inp.mods.shape[2] != MODW or inp.mods.shape[1] < 2:
            raise ValueError(f"mods must be [B, N >= 2, {MODW}]")
        if inp.mods.dtype != torch.bfloat16:
            raise ValueError("mods must be bf16")
        n_steps = inp.mods.shape[1] - 1
        PM, SP = inp.memk.shape[2], inp.kca.shape[2]
        shapes = {"memk": (B, d.L, PM, d.NH, d.HD), "memv": (B, d.L, PM, d.NH, d.HD),
                  "kca": (B, d.L, SP, d.NH, d.HD), "vca": (B, d.L, SP, d.NH, d.HD)}
        for k, shp in shapes.items():
            v = getattr(inp, k)
            if tuple(v.shape) != shp or v.dtype != torch.bfloat16:
                raise ValueError(f"{k} must be bf16 {list(shp)}")
        for k in ("sa_cos", "sa_sin", "ca_cos", "ca_sin"):
            v = getattr(inp, k)
            if tuple(v.shape) != (B, T, d.HD) or v.dtype != torch.float32:
                raise ValueError(f"{k} must be fp32 [B, T, {d.HD}]")
        ts = {k: getattr(inp, k) for k in ("x", "mods", "dt", "memk", "memv", "kca", "vca", "sa_cos", "sa_sin",
                                            "ca_cos", "ca_sin")}
        ts["kv_start"] = inp.kv_start.to(torch.int32)
        ts["S"] = inp.S.to(torch.int32)
        for k, v in ts.items():
            if v.device != self.device:
                raise ValueError(f"{k} must be on the expert's device {self.device}")
            if not v.is_contiguous():
                raise ValueError(f"{k} must be contiguous")
        if ts["dt"].dtype != torch.float32 or ts["dt"].numel() != B:
            raise ValueError("dt must be fp32 [B]")
        if ts["kv_start"].numel() != B or ts["S"].numel() != B:
            raise ValueError("kv_start and S need one value per episode")
        if out is None:
            out = torch.empty((B, T, d.A), dtype=torch.float32, device=self.device)
        elif tuple(out.shape) != (B, T, d.A) or out.dtype != torch.float32 or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous fp32 [B, T, {d.A}] tensor")
        bi = _lib.BatchInputs(
            x_in=ts["x"].data_ptr(), x_out=out.data_ptr(), mods=ts["mods"].data_ptr(), dt=ts["dt"].data_ptr(),
            memk=ts["memk"].data_ptr(), memv=ts["memv"].data_ptr(), kv_start=ts["kv_start"].data_ptr(), mem_rows=PM,
            kca=ts["kca"].data_ptr(), vca=ts["vca"].data_ptr(), src_rows=ts["S"].data_ptr(), ca_rows=SP,
            sa_cos=ts["sa_cos"].data_ptr(), sa_sin=ts["sa_sin"].data_ptr(), ca_cos=ts["ca_cos"].data_ptr(),
            ca_sin=ts["ca_sin"].data_ptr(), B=B, T=T, n_steps=n_steps, action_dim=int(inp.action_dim))
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(self._lib.mkx_batch_run(self._h, C.byref(bi), C.c_void_p(stream)), "mkx_batch_run")
        self._keep = ts  # converted tensors stay alive until the next call
        return out

    def register_pass(self, reg_in: torch.Tensor, memk: torch.Tensor, memv: torch.Tensor, kv_start: torch.Tensor,
                      kca: torch.Tensor, vca: torch.Tensor, src_rows: torch.Tensor, sa_pe, ca_pe) -> None:
        """The current frame's R register rows through every layer with plain norms
        (``include/mkx_batch.h``, ``mkx_batch_register_pass``): writes each layer's register K / V
        into memory rows [PM - R, PM) of ``memk`` / ``memv`` [L, PM, NH, HD] bf16 (in place), the
        self-attention reading rows [kv_start, PM). ``reg_in`` [R, H] bf16 (R a multiple of 16);
        ``kca`` / ``vca`` [L, SP, NH, HD] bf16 valid below ``src_rows``; ``kv_start`` and ``src_rows``
        one-element int32 device tensors; ``sa_pe`` / ``ca_pe`` (cos, sin) fp32 [R, HD]. Asynchronous
        on the current stream, graph-capturable; shares the handle's buffers with ``run``."""
        d = self.dims
        if reg_in.dim() != 2 or reg_in.shape[1] != d.H or reg_in.dtype != torch.bfloat16:
            raise ValueError(f"reg_in must be bf16 [R, {d.H}]")
        R = reg_in.shape[0]
        if R < 16 or R % 16 or R > 16 * self.max_episodes:
            raise ValueError(f"R={R} must be a multiple of 16 in 16..{16 * self.max_episodes}")
        PM, SP = memk.shape[1], kca.shape[1]
        for k, v, shp in (("memk", memk, (d.L, PM, d.NH, d.HD)), ("memv", memv, (d.L, PM, d.NH, d.HD)),
                          ("kca", kca, (d.L, SP, d.NH, d.HD)), ("vca", vca, (d.L, SP, d.NH, d.HD))):
            if tuple(v.shape) != shp or v.dtype != torch.bfloat16:
                raise ValueError(f"{k} must be bf16 {list(shp)}")
        if PM < R:
            raise ValueError(f"the memory ({PM} rows) must hold the frame's {R} rows")
        tabs = [*sa_pe, *ca_pe]
        for t in tabs:
            if tuple(t.shape) != (R, d.HD) or t.dtype != torch.float32:
                raise ValueError(f"RoPE tables must be fp32 [{R}, {d.HD}]")
        ints = (kv_start, src_rows)
        for t in ints:
            if t.dtype != torch.int32 or t.numel() < 1:
                raise ValueError("kv_start and src_rows must be int32 device tensors")
        for t in (reg_in, memk, memv, kca, vca, *tabs, *ints):
            if t.device != self.device:
                raise ValueError(f"every tensor must be on the expert's device {self.device}")
            if not t.is_contiguous():
                raise ValueError("every tensor must be contiguous")
        ri = _lib.RegisterInputs(
            reg_in=reg_in.data_ptr(), memk=memk.data_ptr(), memv=memv.data_ptr(), kv_start=kv_start.data_ptr(),
            mem_rows=PM, kca=kca.data_ptr(), vca=vca.data_ptr(), src_rows=src_rows.data_ptr(), ca_rows=SP,
            sa_cos=tabs[0].data_ptr(), sa_sin=tabs[1].data_ptr(), ca_cos=tabs[2].data_ptr(), ca_sin=tabs[3].data_ptr(),
            R=R)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(self._lib.mkx_batch_register_pass(self._h, C.byref(ri), C.c_void_p(stream)),
                   "mkx_batch_register_pass")

    STATE = {"h": 0, "a": 1, "qkv": 2, "y": 3, "g": 4, "x": 5}

    def state(self, name: str, rows: int, cols: int) -> torch.Tensor:
        """A copy of the first ``rows`` x ``cols`` of an activation buffer (``STATE`` names; bf16,
        the action state fp32): inspection for tests, synchronous."""
        dt = torch.float32 if name == "x" else torch.bfloat16
        t = torch.empty((rows, cols), dtype=dt, device=self.device)
        _lib.check(self._lib.mkx_batch_copy_state(self._h, self.STATE[name], C.c_void_p(t.data_ptr()),
                                                  t.numel() * t.element_size()), "mkx_batch_copy_state")
        return t

    def check_device_error(self) -> None:
        code = C.c_int(0)
        st = self._lib.mkx_batch_last_error(self._h, C.byref(code))
        if st == _lib.MKX_ERR_DEVICE:
            raise _lib.MkxError("batched expert", st, f"device code 0x{code.value:x}")
        _lib.check(st, "mkx_batch_last_error")

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.mkx_batch_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass
