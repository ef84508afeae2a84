"""Per-step modulation rows on the GPU (``_step_modulations``): the AdaRMS [scale, shift, gate]
vectors of every layer and step that ``ExpertMegakernel.run`` reads as ``mods [N, MODW]``
(src/mk_expert.py:336-340,423), computed by two kernels of ``include/mkx_mods.h`` (conditioning,
then an HBM-bound projection streaming the 108.5 MB modulation weight once for all N steps).

``StepModulations(weights)(num_steps, state_cond) -> (mods, dt)`` mirrors the model callable that
``install`` binds (``model._step_modulations``, src/mk_expert.py:527-535); the network itself is a
restatement (Kyutai's is not in the reference). There is no CPU fallback: the CUDA library must load.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .synthetic import ModulationWeights

NMAX = 16


def check_out(MODW: int, device, num_steps: int, out) -> None:
    """What ``StepModulations.run`` checks of caller-owned outputs before it hands their pointers to
    the library, which cannot see sizes or devices: mods a contiguous [N, MODW] bf16 tensor and dt a
    float32 tensor of at least one value, both on ``device``. Raises ValueError."""
    if out is None:
        return
    if len(out) != 2:
        raise ValueError("out must be a (mods, dt) pair")
    mods, dt = out
    if (mods.device != device or mods.dtype != torch.bfloat16 or tuple(mods.shape) != (num_steps, MODW)
            or not mods.is_contiguous()):
        raise ValueError(f"out mods must be a contiguous [{num_steps}, {MODW}] bf16 tensor on {device}")
    if dt.device != device or dt.dtype != torch.float32 or dt.numel() < 1:
        raise ValueError(f"out dt must be a float32 tensor of at least one value on {device}")


class StepModulations:
    """``StepModulations(weights)(num_steps, state) -> (mods [N, MODW] bf16, dt [1] fp32)`` on the
    weights' device."""

    def __init__(self, weights: ModulationWeights, device=None):
        self.lib = _lib.load()
        dev = torch.device(device) if device is not None else weights.w_m.device
        if dev.type != "cuda":
            raise ValueError("StepModulations needs CUDA tensors")
        d = weights.dims
        self.dims = d
        self.device = dev
        w_t = weights.w_t.to(dev, torch.float32).contiguous()
        w_s = weights.w_s.to(dev, torch.float32).contiguous()
        w_m = weights.w_m.to(dev, torch.bfloat16).contiguous()
        b_m = weights.b_m.to(dev, torch.float32).contiguous()
        if w_m.shape != (d.MODW, d.H) or b_m.shape != (d.MODW,):
            raise ValueError(f"w_m must be [{d.MODW}, {d.H}] and b_m [{d.MODW}]")
        self.sdim = weights.sdim
        md = _lib.ModsDims(H=d.H, L=d.L, tdim=weights.tdim, sdim=weights.sdim)
        h = C.c_void_p()
        _lib.check(self.lib.mkx_mods_create(C.byref(md), w_t.data_ptr(), w_s.data_ptr(), w_m.data_ptr(),
                                            b_m.data_ptr(), dev.index or 0, C.byref(h)), "mkx_mods_create")
        self.h = h
        self.MODW = self.lib.mkx_mods_width(h)

    def run(self, num_steps: int, state: torch.Tensor, out=None):
        if not 1 <= num_steps <= NMAX:
            raise ValueError(f"num_steps must be in 1..{NMAX}")
        state = state.reshape(-1)
        if state.numel() != self.sdim:
            raise ValueError(f"state must have {self.sdim} values")
        state = state.to(self.device, torch.float32).contiguous()
        if out is None:
            mods = torch.empty((num_steps, self.MODW), dtype=torch.bfloat16, device=self.device)
            dt = torch.empty((1,), dtype=torch.float32, device=self.device)
        else:
            check_out(self.MODW, self.device, num_steps, out)
            mods, dt = out
        st = self.lib.mkx_mods_run(self.h, num_steps, state.data_ptr(), mods.data_ptr(), dt.data_ptr(),
                                   torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(st, "mkx_mods_run")
        self._keep = state  # alive until the stream reaches the launch
        return mods, dt

    __call__ = run

    def projection_input(self) -> torch.Tensor:
        """The last run's projection input a [16, H] bf16 (rows >= N zero), on the current stream."""
        a = torch.empty((NMAX, self.dims.H), dtype=torch.bfloat16, device=self.device)
        _lib.check(self.lib.mkx_mods_input(self.h, a.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream),
                   "mkx_mods_input")
        return a

    def check_device_error(self):
        code = C.c_int(0)
        _lib.check(self.lib.mkx_mods_last_error(self.h, C.byref(code)), "mkx_mods_last_error")
        if code.value != 0:
            raise _lib.MkxError("modulation kernels", _lib.MKX_ERR_DEVICE, f"error word {code.value:#x}")

    def close(self):
        if getattr(self, "h", None):
            self.lib.mkx_mods_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass
