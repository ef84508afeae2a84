"""Cross-attention K/V preparation on the GPU (``register_prepare``): every layer's K and V of the
cross-attention stage, projected once per predict from the VLM source rows by one tcgen05 GEMM
(``include/mkx_prepare.h``), in the layout ``ExpertMegakernel.run`` reads from
``past.cross_attn_kv`` (src/mk_expert.py:486-495). The reference megakernel has no counterpart: it
consumes K/V that Kyutai's model prepared (README.md:279-281).

There is no CPU fallback: the CUDA library must load.
"""
from __future__ import annotations

import ctypes as C
from types import SimpleNamespace

import torch

from . import _lib
from .synthetic import PrepareWeights, rope_cos_sin


def check_run_args(dims, device, S: int, SP: int, cos: torch.Tensor, sin: torch.Tensor, out) -> None:
    """What ``RegisterPrepare.run`` checks before it hands raw pointers to the library, which cannot
    see sizes or devices: SP >= S, RoPE tables [>= S, HD] fp32 and, when given, the outputs
    [L, SP, NH, HD] bf16, all contiguous on ``device``. Raises ValueError."""
    if SP < S:
        raise ValueError(f"SP={SP} must be >= S={S}")
    for name, t in (("cos", cos), ("sin", sin)):
        if t.device != device or t.dtype != torch.float32 or t.dim() != 2 or t.shape[0] < S or t.shape[1] != dims.HD:
            raise ValueError(f"{name} must be [>= {S}, {dims.HD}] fp32 on {device}")
    if out is not None:
        shape = (dims.L, SP, dims.NH, dims.HD)
        if len(out) != 2:
            raise ValueError("out must be a (k, v) pair")
        for name, t in zip(("k", "v"), out):
            if t.device != device or t.dtype != torch.bfloat16 or tuple(t.shape) != shape or not t.is_contiguous():
                raise ValueError(f"out {name} must be a contiguous {list(shape)} bf16 tensor on {device}")


class RegisterPrepare:
    """``RegisterPrepare(weights).run(src) -> (k, v)``, both [L, SP, NH, HD] bf16 on src's device."""

    def __init__(self, weights: PrepareWeights, device=None):
        self.lib = _lib.load()
        dev = torch.device(device) if device is not None else weights.wkv.device
        if dev.type != "cuda":
            raise ValueError("RegisterPrepare needs CUDA tensors")
        d = weights.dims
        self.dims = d
        self.device = dev
        self.wkv = weights.wkv.to(dev, torch.bfloat16).contiguous()
        self.kn = weights.kn.to(dev, torch.float32).contiguous()
        pd = _lib.PrepDims(L=d.L, H=d.H, NH=d.NH, HD=d.HD, src_dim=d.src_dim, eps=float(weights.eps))
        h = C.c_void_p()
        _lib.check(self.lib.mkx_prep_create(C.byref(pd), self.wkv.data_ptr(), self.kn.data_ptr(),
                                            dev.index or 0, C.byref(h)), "mkx_prep_create")
        self.h = h
        self._tables = {}

    def tables(self, S: int):
        """RoPE tables of source positions 0..S-1 (fp32 [S, HD])."""
        t = self._tables.get(S)
        if t is None:
            c, s = rope_cos_sin(torch.arange(S), self.dims.HD)
            t = (c.to(self.device).contiguous(), s.to(self.device).contiguous())
            self._tables[S] = t
        return t

    def run(self, src: torch.Tensor, cos: torch.Tensor | None = None, sin: torch.Tensor | None = None,
            SP: int | None = None, out=None):
        d = self.dims
        if src.dim() != 2 or src.shape[1] != d.src_dim or src.dtype != torch.bfloat16 or src.device != self.device:
            raise ValueError(f"src must be [S, {d.src_dim}] bf16 on {self.device}")
        src = src.contiguous()
        S = src.shape[0]
        SP = SP or S
        if cos is None or sin is None:
            cos, sin = self.tables(S)
        check_run_args(d, self.device, S, SP, cos, sin, out)
        if out is None:
            k = torch.empty((d.L, SP, d.NH, d.HD), dtype=torch.bfloat16, device=self.device)
            v = torch.empty_like(k)
        else:
            k, v = out
        st = self.lib.mkx_prep_run(self.h, src.data_ptr(), S, cos.contiguous().data_ptr(), sin.contiguous().data_ptr(),
                                   k.data_ptr(), v.data_ptr(), SP, torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(st, "mkx_prep_run")
        return k, v

    def check_device_error(self):
        code = C.c_int(0)
        _lib.check(self.lib.mkx_prep_last_error(self.h, C.byref(code)), "mkx_prep_last_error")
        if code.value != 0:
            raise _lib.MkxError("register_prepare kernel", _lib.MKX_ERR_DEVICE, f"error word {code.value:#x}")

    def close(self):
        if getattr(self, "h", None):
            self.lib.mkx_prep_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def register_prepare(prepare: RegisterPrepare, ca_src: torch.Tensor, mem_kv, *, T: int, kv_start: int = 0,
                     SP: int | None = None, out=None):
    """``register_prepare`` under the reference's name: what the reference megakernel says it reads
    from Kyutai's step-1 side (``src/mk_expert.py:22-24``: "register_prepare (CA source K/V, cos/sin,
    cu_seqlens)"), built on the GPU, returned as the ``past`` object ``ExpertMegakernel.run`` takes
    (``src/mk_expert.py:486-495``).

    ca_src: [S, src_dim] bf16 VLM source rows; mem_kv: per layer (K, V) [PM, NH, HD] bf16 register
    memory (rows >= kv_start valid, already normed and rotated); T: action rows. Returns
    ``past.cross_attn_kv`` (per layer K, V [SP, NH, HD], from one tcgen05 launch), and
    ``past.register_step`` with ``mem_kv``, ``sa_pe`` (RoPE of the action rows at positions
    PM .. PM + T - 1, after the memory), ``ca_pe`` (positions 0 .. T - 1), ``cu_kv`` = [kv_start, PM]
    and ``cu_src`` = [0, S] (int32, device). Asynchronous on the current stream; ``out`` = (k, v)
    reuses K/V buffers (graph capture)."""
    d, dev = prepare.dims, prepare.device
    S = ca_src.shape[0]
    if len(mem_kv) != d.L:
        raise ValueError(f"mem_kv needs {d.L} (K, V) pairs")
    PM = mem_kv[0][0].shape[0]
    if not 0 <= kv_start <= PM:
        raise ValueError(f"kv_start={kv_start} must be in 0..{PM}")
    k, v = prepare.run(ca_src, SP=SP, out=out)
    sa = tuple(t.to(dev) for t in rope_cos_sin(torch.arange(T) + PM, d.HD))
    ca = tuple(t.to(dev) for t in rope_cos_sin(torch.arange(T), d.HD))
    step = {"mem_kv": list(mem_kv), "sa_pe": sa, "ca_pe": ca,
            "cu_kv": torch.tensor([kv_start, PM], dtype=torch.int32, device=dev),
            "cu_src": torch.tensor([0, S], dtype=torch.int32, device=dev)}
    return SimpleNamespace(register_step=step, cross_attn_kv=[(k[l], v[l]) for l in range(d.L)])
