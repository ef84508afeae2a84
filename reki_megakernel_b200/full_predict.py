"""A whole predict of the action expert -- all N Euler steps and the register-memory carry -- as one
CUDA graph replay.

The reference megakernel serves Euler steps 2..N (``ExpertMegakernel.run``, src/mk_expert.py:483-515);
``install`` leaves step 1, the modulation rows and ``register_prepare`` to Kyutai's compiled
callables (src/mk_expert.py:521-536), and the register cache carries 3 frames of 32 register rows
from predict to predict (``_register_cache.append_frame``, src/profile_breakdown.py:97-100). Kyutai's
code is absent from the reference checkout; the parts here restate it (parity unpinned; the CPU
restatement is ``oracle/register_oracle.py``):

1. carry: the memory moves up by one frame (two device copies per K / V), the oldest frame drops
   (a side branch of the graph beside ``RegisterPrepare``, joined before the register pass);
2. ``RegisterPrepare``: every layer's cross-attention K/V from the VLM source rows (one tcgen05 launch);
3. ``StepModulations``: the AdaRMS rows of all N steps (two launches, on a side branch of the graph
   that overlaps steps 1, 2 and 4);
4. register pass (``BatchedExpert.register_pass``): the frame's R register rows through every layer
   with plain norms, writing their K/V into the newest frame's memory rows (tcgen05 GEMMs, 11
   launches per layer);
5. the action rows: all N Euler steps in ONE persistent ``expert_kernel`` launch from the flow noise
   (the modulation rows behind a placeholder row 0, so the launch's steps 1..N read rows 1..N); step
   1 is the same computation as steps 2..N over the memory that now holds the current frame.

Inputs sit in static device buffers that ``__call__`` refills before each replay; the predict count
(how many frames are valid) is a device word set before the replay.
"""
from __future__ import annotations

from types import SimpleNamespace

import torch

from .batch import BatchedExpert
from .mk_expert import ExpertMegakernel
from .modulations import StepModulations
from .prepare import RegisterPrepare
from .synthetic import register_rope, rope_cos_sin


class FullPredict:
    """``FullPredict(mk, batched, prepare, modulations, reg_in, S=...)(src, state, noise) -> [1, T, A]``.

    mk: the persistent expert; batched: a ``BatchedExpert`` of >= R / 16 episodes (its handle runs the
    register pass); reg_in: [R, H] bf16 register rows; PM = frames x R memory rows; S source rows;
    N Euler steps; T action rows. ``reset()`` starts a new episode (empty memory)."""

    def __init__(self, mk: ExpertMegakernel, batched: BatchedExpert, prepare: RegisterPrepare,
                 modulations: StepModulations, reg_in: torch.Tensor, *, S: int, num_steps: int = 10, T: int = 10,
                 frames: int = 3, action_dim: int = 7, SP: int | None = None, graph: bool = True):
        dev = mk.device
        if any(x.device != dev for x in (batched, prepare, modulations)):
            raise ValueError("every part must live on one device")
        d = prepare.dims
        R = reg_in.shape[0]
        PM = frames * R
        if not 1 <= num_steps <= 15:
            raise ValueError("num_steps must be in 1..15")
        self.mk, self.batched, self.prepare, self.modulations = mk, batched, prepare, modulations
        self.N, self.S, self.T, self.R, self.PM, self.action_dim = num_steps, S, T, R, PM, action_dim
        SP = SP or S
        L, NH, HD = d.L, d.NH, d.HD
        z = lambda *shape, dt=torch.bfloat16: torch.zeros(shape, dtype=dt, device=dev)  # noqa: E731
        self.reg_in = reg_in.to(dev, torch.bfloat16).contiguous()
        self.memk, self.memv = z(L, PM, NH, HD), z(L, PM, NH, HD)
        self.tmp = z(L, PM - R, NH, HD)
        self.src = z(S, d.src_dim)
        self.state = z(modulations.sdim, dt=torch.float32)
        self.noise = z(1, T, mk.A, dt=torch.float32)
        self.k, self.v = z(L, SP, NH, HD), z(L, SP, NH, HD)
        self.mods = z(num_steps + 1, modulations.MODW)  # row 0: placeholder, never read
        self.dt = z(1, dt=torch.float32)
        self.cu_kv = torch.tensor([PM - R, PM], dtype=torch.int32, device=dev)
        self.cu_src = torch.tensor([0, S], dtype=torch.int32, device=dev)
        self.cos, self.sin = (t.to(dev) for t in rope_cos_sin(torch.arange(S), HD))
        rs = [t.to(dev).contiguous() for t in register_rope(d, PM, R)]
        self.reg_sa, self.reg_ca = (rs[0], rs[1]), (rs[2], rs[3])
        sa = tuple(t.to(dev) for t in rope_cos_sin(torch.arange(T) + PM, HD))
        ca = tuple(t.to(dev) for t in rope_cos_sin(torch.arange(T), HD))
        self.past = SimpleNamespace(
            register_step={"mem_kv": [(self.memk[l], self.memv[l]) for l in range(L)], "sa_pe": sa, "ca_pe": ca,
                           "cu_kv": self.cu_kv, "cu_src": self.cu_src},
            cross_attn_kv=[(self.k[l], self.v[l]) for l in range(L)])
        self.p = 0
        self.side = torch.cuda.Stream(dev)
        self.carry = torch.cuda.Stream(dev)
        self.graph = None
        if graph:
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                for _ in range(2):
                    self._body()
            torch.cuda.current_stream(dev).wait_stream(side)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.out = self._body()
            self.reset()

    def _body(self) -> torch.Tensor:
        R = self.R
        main = torch.cuda.current_stream(self.mk.device)
        # the modulation rows need nothing from the other parts: a side branch that runs on the SMs
        # the register pass's small launches leave idle, joined before the Euler steps
        self.side.wait_stream(main)
        with torch.cuda.stream(self.side):
            self.modulations.run(self.N, self.state, out=(self.mods[1:], self.dt))
        # the carry (frames move up by one, the oldest drops) on a second branch: register_prepare
        # does not touch the memory, and its 120 CTAs leave SMs for the copies; joined before the
        # register pass, which writes the newest frame
        self.carry.wait_stream(main)
        with torch.cuda.stream(self.carry):
            for m in (self.memk, self.memv):
                self.tmp.copy_(m[:, R:])
                m[:, :-R].copy_(self.tmp)
        self.prepare.run(self.src, self.cos, self.sin, SP=self.k.shape[1], out=(self.k, self.v))
        main.wait_stream(self.carry)
        self.batched.register_pass(self.reg_in, self.memk, self.memv, self.cu_kv[:1], self.k, self.v,
                                   self.cu_src[1:], self.reg_sa, self.reg_ca)
        main.wait_stream(self.side)
        return self.mk.run(self.noise, self.mods, self.dt, self.past, self.action_dim)

    def reset(self) -> None:
        """A new episode: empty register memory, predict count 0."""
        self.memk.zero_()
        self.memv.zero_()
        self.p = 0

    def frames_valid(self) -> int:
        """Frames the next predict attends to (the current one included)."""
        return min(self.p + 1, self.PM // self.R)

    def __call__(self, src: torch.Tensor, state: torch.Tensor, noise: torch.Tensor) -> torch.Tensor:
        """One predict: src [S, src_dim] bf16, state [sdim], noise [1, T, A] fp32 (any device). Returns
        the graph's output tensor [1, T, A] (overwritten by the next call); asynchronous."""
        self.src.copy_(src, non_blocking=True)
        self.state.copy_(state.reshape(-1), non_blocking=True)
        self.noise.copy_(noise.reshape(self.noise.shape), non_blocking=True)
        self.cu_kv[:1].fill_(self.PM - self.R * self.frames_valid())
        self.p += 1
        if self.graph is not None:
            self.graph.replay()
            return self.out
        return self._body()

    def check_device_errors(self) -> None:
        self.mk.check_device_error()
        self.batched.check_device_error()
        self.prepare.check_device_error()
        self.modulations.check_device_error()
