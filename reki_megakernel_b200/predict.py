"""The GPU half of a predict after Euler step 1, captured as one CUDA graph.

The reference captures the expert in CUDA graphs around Kyutai's step functions (``ExpertGraphs``,
README.md:127-128; ``install`` rebinds ``_expert_actions`` inside it, src/mk_expert.py:521-536) and
lists the host glue around it as remaining work (README.md:284-286). Here the three GPU parts of a
predict that follow the VLM prefill and Euler step 1 run as one graph replay:

1. ``StepModulations(N, state)``: the AdaRMS rows of every layer and step (``mods [N, MODW]``, dt);
2. ``RegisterPrepare(src)``: every layer's cross-attention K/V from the VLM source rows;
3. ``ExpertMegakernel.run(x_t, mods, dt, past, action_dim)``: Euler steps 2..N.

Step 1 (Kyutai's ``_expert_first_step``: the action rows plus the register rows, which also yields the
current frame's register K/V) is not in the reference checkout; its output ``x_t`` and the register
memory K/V are inputs here. All inputs live in static device buffers that ``__call__`` refills
(device-to-device copies, captured nowhere) before each replay.
"""
from __future__ import annotations

from types import SimpleNamespace

import torch

from .mk_expert import ExpertMegakernel
from .modulations import StepModulations
from .prepare import RegisterPrepare
from .synthetic import rope_cos_sin


class PredictGraph:
    """``PredictGraph(mk, prepare, modulations, ...)(src, state, x_t) -> x_out [1, T, A]``.

    memk / memv: the register memory K/V [L, PM, NH, HD] bf16 (device, read in place, valid rows from
    ``kv_start``); S source rows, N Euler steps (N - 1 run in the expert), T action rows."""

    def __init__(self, mk: ExpertMegakernel, prepare: RegisterPrepare, modulations: StepModulations, *,
                 num_steps: int, S: int, T: int, memk: torch.Tensor, memv: torch.Tensor, kv_start: int,
                 action_dim: int, SP: int | None = None):
        dev = mk.device
        if prepare.device != dev or modulations.device != dev:
            raise ValueError("the three parts must live on one device")
        if num_steps < 2:
            raise ValueError("num_steps must be >= 2 (step 1 is not part of the graph)")
        d = prepare.dims
        L, NH, HD, PM = d.L, d.NH, d.HD, memk.shape[1]
        if memk.shape != (L, PM, NH, HD) or memv.shape != memk.shape:
            raise ValueError(f"memory K/V must be [{L}, PM, {NH}, {HD}]")
        self.mk, self.prepare, self.modulations = mk, prepare, modulations
        self.N, self.S, self.T, self.action_dim = num_steps, S, T, action_dim
        SP = SP or S
        self.src = torch.zeros((S, d.src_dim), dtype=torch.bfloat16, device=dev)
        self.state = torch.zeros((modulations.sdim,), dtype=torch.float32, device=dev)
        self.x_t = torch.zeros((1, T, mk.A), dtype=torch.float32, device=dev)
        self.k = torch.zeros((L, SP, NH, HD), dtype=torch.bfloat16, device=dev)
        self.v = torch.zeros_like(self.k)
        self.mods = torch.zeros((num_steps, modulations.MODW), dtype=torch.bfloat16, device=dev)
        self.dt = torch.zeros((1,), dtype=torch.float32, device=dev)
        self.cos, self.sin = (t.to(dev) for t in rope_cos_sin(torch.arange(S), HD))
        sa = tuple(t.to(dev) for t in rope_cos_sin(torch.arange(T) + PM, HD))
        ca = tuple(t.to(dev) for t in rope_cos_sin(torch.arange(T), HD))
        self.past = SimpleNamespace(
            register_step={"mem_kv": [(memk[l], memv[l]) for l in range(L)], "sa_pe": sa, "ca_pe": ca,
                           "cu_kv": torch.tensor([kv_start, PM], dtype=torch.int32, device=dev),
                           "cu_src": torch.tensor([0, S], dtype=torch.int32, device=dev)},
            cross_attn_kv=[(self.k[l], self.v[l]) for l in range(L)])
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                self._body()
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self._body()

    def _body(self) -> torch.Tensor:
        self.prepare.run(self.src, self.cos, self.sin, SP=self.k.shape[1], out=(self.k, self.v))
        self.modulations.run(self.N, self.state, out=(self.mods, self.dt))
        return self.mk.run(self.x_t, self.mods, self.dt, self.past, self.action_dim)

    def __call__(self, src: torch.Tensor, state: torch.Tensor, x_t: torch.Tensor) -> torch.Tensor:
        """Copies the inputs into the graph's buffers, replays, returns the graph's output tensor
        (overwritten by the next call)."""
        self.src.copy_(src)
        self.state.copy_(state.reshape(-1))
        self.x_t.copy_(x_t)
        self.graph.replay()
        return self.out

    def check_device_errors(self) -> None:
        self.mk.check_device_error()
        self.prepare.check_device_error()
        self.modulations.check_device_error()
