"""Drop-in replacement for the reference's ``src/mk_expert.py`` (``ExpertMegakernel``, ``install``).

Same names, arguments and behaviour as the reference launcher:

* ``ExpertMegakernel(model)`` reads the expert from a REKI-shaped model object
  (``src/mk_expert.py:436-481``), packs it once into the CUDA library's own device memory
  (``mkx_create``) and keeps the reference's attributes (``L, NH, HD, H, I, A, TP, nprog, cfg``).
* ``.run(x_t, mods, dt, past, action_dim)`` integrates Euler steps 2..N in one persistent launch on
  the current stream and returns a fresh ``[1, T, A]`` fp32 tensor (``src/mk_expert.py:483-515``).
  It reads ``past.register_step`` (``mem_kv``, ``sa_pe``, ``ca_pe``, ``cu_kv``, ``cu_src``) and
  ``past.cross_attn_kv`` in place: the per-layer K/V tensors are passed by pointer, no stacking copy.
  No host synchronisation happens, so the call can be captured in a CUDA graph (the reference's
  launch sits inside Kyutai's expert graph).
* ``.run_from_host(x_t, mods, dt, past, action_dim)``: the same launch for callers whose inputs sit
  in pinned host memory (no counterpart in the reference). The small inputs are copied ahead of the
  launch; each layer's memory and cross-attention K/V are copied on a side stream while the launch
  already runs, and the kernel waits (bounded) for a per-layer readiness word before its first read
  of them, so the copies overlap the first Euler step instead of preceding the launch.
* ``.barriers(n_steps)`` keeps the reference's count ``1 + n_steps (8 L + 1)``
  (``src/mk_expert.py:517-518``): the number of dependent exchange points of one launch.
* ``install(model)`` rebinds ``model._expert_actions`` exactly like ``src/mk_expert.py:521-536``.

Preconditions the reference asserts (``src/mk_expert.py:444,462,464,480,488,496``) raise
``ValueError`` here; a failed CUDA call or a device-side wait that ran out raises ``MkxError``.
There is no CPU path: without ``libmkx.so`` the import fails.
"""
from __future__ import annotations

import ctypes as C
from types import SimpleNamespace

import torch

from . import _lib
from .synthetic import ExpertWeights, weights_from_model

AO = 8     # real action dims the loop carries (src/mk_expert.py:478)
TP = 16    # action rows per launch


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


READY_PERIOD = 0x3FFFFFFF


def ready_value(seq: int) -> int:
    """The readiness-word value of ``run_from_host`` call ``seq`` (1, 2, ...): cycles through
    1..READY_PERIOD, so it is never the buffer's initial 0 and never the previous call's value (the
    launch would otherwise take the previous call's words for this call's K/V)."""
    return (seq - 1) % READY_PERIOD + 1


def _copy_groups(L: int):
    """Layer groups of run_from_host's K/V copies, each group followed by its layers' readiness
    words: single layers first (the launch needs them soonest), larger runs later (fewer copies: each
    costs the host ~2.5 us to enqueue and the copy engine a fixed overhead; the 10 x 0.79 MB of a
    predict's K/V then cross at the engine's full rate well inside the first Euler step)."""
    sizes, out, l = [1, 1, 2, 2], [], 0
    for n in sizes:
        if l >= L:
            break
        out.append((l, min(L, l + n)))
        l = min(L, l + n)
    if l < L:
        out.append((l, L))
    return out


def _rows2d(dev_layers, host_layers, r0: int, r1: int):
    """Pitched copies (dst, dpitch, src, spitch, width, height) of rows [r0, r1) of consecutive layers
    (each a contiguous [rows, ...] tensor, the range clipped to its rows): one copy for each run of
    layers whose device and host tensors both follow each other at one pitch."""
    out = []
    for d, h in zip(dev_layers, host_layers):
        rows = d.shape[0]
        a, z = min(max(r0, 0), rows), min(max(r1, 0), rows)
        if z <= a:
            continue
        rb = (d.numel() // rows) * d.element_size()  # bytes per row
        dp, hp, w = d.data_ptr() + a * rb, h.data_ptr() + a * rb, (z - a) * rb
        pitch = rows * rb
        if out:
            pd, pdp, ph, php, pw, n = out[-1]
            if pw == w and pdp == pitch and php == pitch and pd + n * pitch == dp and ph + n * pitch == hp:
                out[-1] = (pd, pdp, ph, php, pw, n + 1)
                continue
        out.append((dp, pitch, hp, pitch, w, 1))
    return out


class ExpertMegakernel:
    """Packs the expert weights once; ``run`` integrates Euler steps 2..N in one launch."""

    def __init__(self, model=None, *, weights: ExpertWeights | None = None, max_rows: int = TP, grid: int = 0,
                 device=None):
        w = weights if weights is not None else weights_from_model(model)
        d = w.dims
        self.L, self.NH, self.HD, self.H, self.I, self.A = d.L, d.NH, d.HD, d.H, d.I, d.A
        self.TP = TP
        self.eps, self.qk_eps = float(w.eps), float(w.qk_eps)
        dev = torch.device(device) if device is not None else w.wqkv.device
        if dev.type != "cuda":
            raise ValueError("ExpertMegakernel needs the expert weights on a CUDA device")
        self.device = dev
        lib = _lib.load()
        self._lib = lib
        t = {k: v.to(dev).contiguous() for k, v in w.tensors().items()}
        for k in ("wqkv", "wo", "wqca", "woca", "wg", "wu", "wd", "qn", "kn", "qcan"):
            if t[k].dtype != torch.bfloat16:
                raise ValueError(f"{k} must be bf16")
        for k in ("win", "bin", "wout", "bout"):
            t[k] = t[k].float().contiguous()
        dims = _lib.Dims(L=d.L, H=d.H, NH=d.NH, HD=d.HD, I=d.I, A=d.A, eps=self.eps, qk_eps=self.qk_eps,
                         max_rows=max_rows, grid=grid)
        wts = _lib.Weights(**{f[0]: t[f[0]].data_ptr() for f in _lib.Weights._fields_})
        handle = C.c_void_p()
        with torch.cuda.device(dev):
            torch.cuda.synchronize(dev)  # the packing kernels read the weights on another stream
            _lib.check(lib.mkx_create(C.byref(dims), C.byref(wts), dev.index or 0, C.byref(handle)), "mkx_create")
        self._h = handle
        del t
        g, smem = C.c_int(), C.c_int()
        _lib.check(lib.mkx_launch_shape(self._h, C.byref(g), C.byref(smem)), "mkx_launch_shape")
        self.nprog = g.value
        self.cfg = dict(grid=g.value, threads=256, smem_bytes=smem.value, max_rows=max_rows, AO=AO)
        self._dt_cache: dict = {}

    # ------------------------------------------------------------------------------------------
    def _dt_tensor(self, dt) -> torch.Tensor:
        if isinstance(dt, torch.Tensor):
            if dt.device != self.device:
                raise ValueError("dt must be on the expert's device")
            return dt.reshape(-1)[:1].float() if dt.dtype != torch.float32 else dt.reshape(-1)
        key = float(dt)
        if key not in self._dt_cache:
            self._dt_cache[key] = torch.tensor([key], dtype=torch.float32, device=self.device)
        return self._dt_cache[key]

    def run(self, x_t: torch.Tensor, mods: torch.Tensor, dt, past, action_dim: int,
            trace: torch.Tensor | None = None, prof: torch.Tensor | None = None,
            kv_ready: torch.Tensor | None = None, kv_ready_value: int = 0) -> torch.Tensor:
        """x_t: [1, T, A] fp32 after Euler step 1; mods: [N, MODW] (row 0 = step 1, used already);
        returns x_t after step N (padded dims as the reference: 0 + dt * v). kv_ready (optional,
        int32 [L] on the device): the launch reads layer l's K/V only once kv_ready[l] equals
        kv_ready_value (see ``run_from_host``)."""
        si, out, keep = self._step_inputs(x_t, mods, dt, past, action_dim, trace, prof, kv_ready, kv_ready_value)
        self._launch(si)
        return out

    def _launch(self, si) -> None:
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(self._lib.mkx_run(self._h, C.byref(si), C.c_void_p(stream)), "mkx_run")

    def _step_inputs(self, x_t, mods, dt, past, action_dim, trace, prof, kv_ready, kv_ready_value):
        """Validated launch descriptor, the fresh output tensor, and the tensors the descriptor points
        to that were made here (kept alive by the caller until the launch is enqueued)."""
        step = past.register_step
        if x_t.dim() != 3 or x_t.shape[0] != 1 or x_t.shape[2] != self.A:
            raise ValueError(f"x_t must be [1, T, {self.A}], got {tuple(x_t.shape)}")
        T = x_t.shape[1]
        if not (1 <= T <= self.cfg["max_rows"]) or not (1 <= action_dim <= AO):
            raise ValueError(f"T={T} must be in 1..{self.cfg['max_rows']} and action_dim={action_dim} in 1..{AO}")
        if mods.dim() != 2 or mods.shape[1] != 9 * self.L * self.H + 2 * self.H or mods.shape[0] < 2:
            raise ValueError(f"mods must be [N >= 2, {9 * self.L * self.H + 2 * self.H}], got {tuple(mods.shape)}")
        n_steps = mods.shape[0] - 1
        mem = step["mem_kv"]
        ca = past.cross_attn_kv
        if len(mem) != self.L or len(ca) != self.L:
            raise ValueError("need one memory and one cross-attention K/V pair per layer")

        def kv_rows(t: torch.Tensor):
            if t.dim() == 4 and t.shape[0] == 1:
                t = t[0]
            if t.dim() != 3 or t.shape[1] != self.NH or t.shape[2] != self.HD or t.dtype != torch.bfloat16:
                raise ValueError(f"K/V must be bf16 [rows, {self.NH}, {self.HD}], got {t.dtype} {tuple(t.shape)}")
            if t.stride(2) != 1 or t.stride(1) != self.HD:
                raise ValueError("K/V heads must be contiguous")
            if t.device != self.device:
                raise ValueError("K/V must be on the expert's device")
            return t
        memk = [kv_rows(m[0]) for m in mem]
        memv = [kv_rows(m[1]) for m in mem]
        kca = [kv_rows(k[0]) for k in ca]
        vca = [kv_rows(k[1]) for k in ca]
        PM = memk[0].shape[0]
        mstride = memk[0].stride(0)
        cstride = kca[0].stride(0)
        if any(m.shape[0] != PM or m.stride(0) != mstride for m in memk + memv):
            raise ValueError("memory K/V of all layers must share rows and row stride")
        if any(k.stride(0) != cstride for k in kca + vca):
            raise ValueError("cross-attention K/V of all layers must share the row stride")

        def pe(t: torch.Tensor):
            t = t.reshape(-1, self.HD)
            if t.shape[0] != T:
                raise ValueError(f"RoPE tables must be [T={T}, {self.HD}], got {tuple(t.shape)}")
            return t.float().contiguous() if t.dtype != torch.float32 else t.contiguous()
        sa_cos, sa_sin = (pe(t) for t in step["sa_pe"])
        ca_cos, ca_sin = (pe(t) for t in step["ca_pe"])
        cu_kv = step["cu_kv"].to(torch.int32).contiguous()
        cu_src = step["cu_src"].to(torch.int32).contiguous()
        if cu_kv.numel() < 2 or cu_src.numel() < 2:
            raise ValueError("cu_kv and cu_src need two values each")
        # the library sees only pointers: a tensor on another device would be read through a bad address
        placed = (("x_t", x_t), ("mods", mods), ("sa_pe", sa_cos), ("sa_pe", sa_sin), ("ca_pe", ca_cos),
                  ("ca_pe", ca_sin), ("cu_kv", cu_kv), ("cu_src", cu_src))
        for name, t in placed:
            if t.device != self.device:
                raise ValueError(f"{name} must be on the expert's device {self.device}, got {t.device}")
        x_in = x_t.reshape(T, self.A)
        x_in = x_in.float().contiguous() if x_in.dtype != torch.float32 else x_in.contiguous()
        if mods.dtype not in (torch.bfloat16, torch.float32):
            mods = mods.float()
        mods = mods.contiguous()
        if mods.data_ptr() % 16:  # the modulation rows are bulk-copied (TMA): 16-byte aligned source
            mods = mods.clone()
        dt_t = self._dt_tensor(dt)
        out = torch.empty(T, self.A, dtype=torch.float32, device=self.device)
        if trace is not None:
            if trace.dtype != torch.bfloat16 or trace.numel() != n_steps * self.L * T * self.H or not trace.is_contiguous():
                raise ValueError("trace must be a contiguous bf16 tensor of n_steps * L * T * H elements")
        si = _lib.StepInputs()
        si.x_in, si.x_out, si.mods = x_in.data_ptr(), out.data_ptr(), mods.data_ptr()
        si.mods_fp32 = 1 if mods.dtype == torch.float32 else 0
        si.dt = dt_t.data_ptr()
        for l in range(self.L):
            si.memk[l], si.memv[l] = memk[l].data_ptr(), memv[l].data_ptr()
            si.kca[l], si.vca[l] = kca[l].data_ptr(), vca[l].data_ptr()
        si.mem_rows, si.mem_row_stride, si.ca_row_stride = PM, mstride, cstride
        si.ca_rows = min(k.shape[0] for k in kca + vca)
        si.cu_kv, si.cu_src = cu_kv.data_ptr(), cu_src.data_ptr()
        si.sa_cos, si.sa_sin, si.ca_cos, si.ca_sin = (t.data_ptr() for t in (sa_cos, sa_sin, ca_cos, ca_sin))
        si.T, si.n_steps, si.action_dim = T, n_steps, int(action_dim)
        if kv_ready is not None:
            if kv_ready.dtype != torch.int32 or kv_ready.numel() < self.L or kv_ready.device != self.device:
                raise ValueError(f"kv_ready must be an int32 tensor of >= {self.L} values on the expert's device")
            si.kv_ready, si.kv_ready_value = kv_ready.data_ptr(), int(kv_ready_value)
        si.trace_h = trace.data_ptr() if trace is not None else None
        if prof is not None:
            need = self.nprog * (1 + self.barriers(n_steps))
            if prof.dtype != torch.int64 or prof.numel() < need or not prof.is_contiguous():
                raise ValueError(f"prof must be a contiguous int64 tensor of >= {need} elements")
            si.prof = prof.data_ptr()
        keep = (x_in, mods, dt_t, sa_cos, sa_sin, ca_cos, ca_sin, cu_kv, cu_src)
        return si, out.reshape(1, T, self.A), keep

    def run_from_host(self, x_t: torch.Tensor, mods: torch.Tensor, dt, past, action_dim: int) -> torch.Tensor:
        """``run`` with every input in pinned host memory (``past`` as for ``run``, its tensors on the
        host; dt a float or a one-element tensor). Returns the device result like ``run``.

        On the current stream the small inputs (x_t, mods, dt, RoPE tables, cu_kv, cu_src) are copied
        in; on a side stream that first waits for this handle's previous launch (it read the same
        buffers), per group of layers the memory and cross-attention K/V rows the launch reads
        (memory rows from cu_kv[0], source rows below cu_src[1]: one pitched copy per kind and group)
        and a 4-byte readiness word, all plain host-to-device copies issued by the library (a kernel
        on that stream would wait for the SMs the launch holds); then the launch is enqueued on the
        current stream. ``last_h2d_bytes`` is the number of bytes the call copied in. The launch waits for
        layer l's word before reading its K/V, so the K/V copies run under the first Euler step
        instead of ahead of the launch. Successive calls may come from different current streams:
        each call's copies wait for the previous call's launch. The host tensors must stay alive
        until the streams have used them."""
        dev = self.device
        st = past.register_step
        host = {"x": x_t, "mods": mods, "sa_cos": st["sa_pe"][0], "sa_sin": st["sa_pe"][1],
                "ca_cos": st["ca_pe"][0], "ca_sin": st["ca_pe"][1], "cu_kv": st["cu_kv"], "cu_src": st["cu_src"]}
        if len(st["mem_kv"]) != self.L or len(past.cross_attn_kv) != self.L:
            raise ValueError("need one memory and one cross-attention K/V pair per layer")
        kv = [(m[0], m[1], c[0], c[1]) for m, c in zip(st["mem_kv"], past.cross_attn_kv)]
        objs = tuple(host.values()) + tuple(x for layer in kv for x in layer) + (dt,)
        last = getattr(self, "_host_last", None)
        if last is not None and len(last[0]) == len(objs) and all(a is b for a, b in zip(last[0], objs)):
            # the very tensor objects of the last call (a control loop refilling its pinned buffers):
            # their shapes, strides and addresses were checked then; only the contents are new
            host, seen = last[1], last[2]
        else:
            if isinstance(dt, torch.Tensor):
                host["dt"] = dt.reshape(-1)[:1]
            tensors = list(host.values()) + [x for layer in kv for x in layer]
            key = tuple((k, tuple(v.shape), v.dtype) for k, v in host.items()) + tuple(
                (tuple(t.shape), t.dtype) for layer in kv for t in layer)
            seen = (key, tuple(t.data_ptr() for t in tensors), tuple(t.stride() for t in tensors))
        self._host_last = None  # set again once this call's checks have passed
        if seen != getattr(self, "_host_seen", None):  # the same host tensors as last call: checked then
            tensors = list(host.values()) + [x for layer in kv for x in layer]
            storages = {}
            for t in tensors:
                if t.device.type != "cpu" or not t.is_contiguous():
                    raise ValueError("run_from_host takes contiguous host tensors")
                storages[t.untyped_storage().data_ptr()] = t
            if not all(t.is_pinned() for t in storages.values()):
                raise ValueError("run_from_host takes tensors in pinned host memory")
            self._host_seen = seen
        key = seen[0]
        b = getattr(self, "_host_bufs", None)
        if b is None or b["key"] != key:
            b = {"key": key,
                 "in": {k: torch.empty(v.shape, dtype=v.dtype, device=dev) for k, v in host.items()},
                 "kv": self._device_kv(kv, dev),
                 "ready": torch.zeros(self.L, dtype=torch.int32, device=dev),
                 "ring": torch.zeros((64, self.L), dtype=torch.int32).pin_memory(),
                 "ring_done": [None] * 64, "seq": 0,
                 "copy": torch.cuda.Stream(dev), "prev": None, "prev_stream": None}
            self._host_bufs = b
            # the buffers were created (zeroed) on the current stream: the side stream's first
            # copies must not overtake that
            b["copy"].wait_stream(torch.cuda.current_stream(dev))
        main = torch.cuda.current_stream(dev)
        if b["prev"] is not None and b["prev_stream"] != main:
            main.wait_event(b["prev"])  # the previous launch, on another stream, still reads b["in"]
        # the kernel reads memory rows [kv_start, PM) and source rows [0, S) only: the others stay
        # on the host (their device rows keep whatever they held, which no launch reads). Here the
        # two values are on the host, so a kv_start the kernel would read out of bounds with is refused.
        if host["cu_kv"].numel() < 2 or host["cu_src"].numel() < 2:
            raise ValueError("cu_kv and cu_src need two values each")
        rows = (int(host["cu_kv"][0]), int(host["cu_src"][1]))
        pm = min(layer[0].shape[0] for layer in kv)
        if not 0 <= rows[0] <= pm or rows[1] < 1:
            raise ValueError(f"kv_start={rows[0]} must be in 0..{pm} and S={rows[1]} at least 1")
        plan = b.get("plan")
        if plan is None or plan["seen"] != seen or plan["rows"] != rows:
            # the copy lists for these host tensors and row ranges, as library-call arguments built
            # once; the readiness words' sources (the ring row of the call) are patched in per call
            side, ready_at = [], []
            for l0, l1 in _copy_groups(self.L):
                for j in range(4):  # memory K, V, cross-attention K, V of layers l0..l1-1
                    r0, r1 = (rows[0], 1 << 30) if j < 2 else (0, rows[1])
                    side += _rows2d([b["kv"][l][j] for l in range(l0, l1)], [kv[l][j] for l in range(l0, l1)], r0, r1)
                ready_at.append((len(side), l0, l1))
                w = 4 * (l1 - l0)
                side.append((b["ready"][l0:l1].data_ptr(), w, b["ring"][0][l0:l1].data_ptr(), w, w, 1))
            small = [(b["in"][k], v) for k, v in host.items()]
            plan = {"seen": seen, "rows": rows, "small": self._h2d_args(small), "side": self._h2d2_args(side),
                    "ready_at": ready_at,
                    "bytes": sum(v.numel() * v.element_size() for _, v in small) + sum(e[4] * e[5] for e in side)}
            b["plan"] = plan
        self._h2d_run(plan["small"], main)
        b["seq"] += 1
        value = ready_value(b["seq"])
        slot = b["seq"] % 64
        if b["ring_done"][slot] is not None:
            b["ring_done"][slot].synchronize()  # that slot's words were copied out 64 calls ago
        row = b["ring"][slot]
        row.fill_(value)
        cs = b["copy"]
        if b["prev"] is not None:
            cs.wait_event(b["prev"])  # the previous launch has finished with the buffers
        side = plan["side"]
        for idx, l0, l1 in plan["ready_at"]:  # this call's ring row
            side[3][idx] = row[l0:l1].data_ptr()
        self._h2d2_run(side, cs)  # enqueued before the launch: the copies start while it is prepared
        self.last_h2d_bytes = plan["bytes"]
        ev = torch.cuda.Event()
        ev.record(cs)
        if b.get("si") is None or b["dt_key"] != (None if "dt" in host else float(dt)):
            # the device buffers never change for this buffer set: validate and describe them once
            d = b["in"]
            dpast = SimpleNamespace(
                register_step={"mem_kv": [(b["kv"][l][0], b["kv"][l][1]) for l in range(self.L)],
                               "sa_pe": (d["sa_cos"], d["sa_sin"]), "ca_pe": (d["ca_cos"], d["ca_sin"]),
                               "cu_kv": d["cu_kv"], "cu_src": d["cu_src"]},
                cross_attn_kv=[(b["kv"][l][2], b["kv"][l][3]) for l in range(self.L)])
            b["si"], _, b["si_keep"] = self._step_inputs(d["x"], d["mods"], d["dt"] if "dt" in d else dt, dpast,
                                                         action_dim, None, None, b["ready"], value)
            b["dt_key"] = None if "dt" in host else float(dt)
            si = b["si"]
            direct = {"x": si.x_in, "mods": si.mods, "sa_cos": si.sa_cos, "sa_sin": si.sa_sin, "ca_cos": si.ca_cos,
                      "ca_sin": si.ca_sin, "cu_kv": si.cu_kv, "cu_src": si.cu_src}
            if any(d[k].data_ptr() != v for k, v in direct.items()) or ("dt" in d and d["dt"].data_ptr() != si.dt):
                b["si"] = None
                raise ValueError("run_from_host needs inputs that need no conversion: x_t and tables fp32, "
                                 "mods bf16 or fp32, cu_kv / cu_src int32, dt fp32")
        si = b["si"]
        if not 1 <= int(action_dim) <= AO:
            raise ValueError(f"action_dim={action_dim} must be in 1..{AO}")
        out = torch.empty((1, int(si.T), self.A), dtype=torch.float32, device=dev)
        si.x_out, si.action_dim, si.kv_ready_value = out.data_ptr(), int(action_dim), int(value)
        self._launch(si)
        done = torch.cuda.Event()
        done.record(main)
        b["ring_done"][slot] = ev
        b["prev"], b["prev_stream"] = done, main
        self._host_last = (objs, host, seen)
        return out

    @staticmethod
    def _device_kv(kv, dev):
        """Device K/V buffers for run_from_host: per kind (memory K, V, cross-attention K, V) one
        allocation holding every layer back to back, so a run of layers can be one copy."""
        out = [[None] * 4 for _ in kv]
        for j in range(4):
            shapes = [tuple(layer[j].shape) for layer in kv]
            dt = kv[0][j].dtype
            if all(sh == shapes[0] for sh in shapes) and all(layer[j].dtype == dt for layer in kv):
                whole = torch.empty((len(kv),) + shapes[0], dtype=dt, device=dev)
                for l in range(len(kv)):
                    out[l][j] = whole[l]
            else:
                for l, layer in enumerate(kv):
                    out[l][j] = torch.empty(layer[j].shape, dtype=layer[j].dtype, device=dev)
        return [tuple(o) for o in out]

    @staticmethod
    def _h2d_args(pairs):
        """(n, dst, src, bytes) library-call arguments of host-to-device copies (dst, src)."""
        n = len(pairs)
        dst = (C.c_void_p * n)(*[dd.data_ptr() for dd, _ in pairs])
        src = (C.c_void_p * n)(*[ss.data_ptr() for _, ss in pairs])
        nb = (C.c_size_t * n)(*[ss.numel() * ss.element_size() for _, ss in pairs])
        return [n, dst, src, nb]

    @staticmethod
    def _h2d2_args(entries):
        """[n, dst, dpitch, src, spitch, width, height] library-call arguments of pitched copies."""
        n = len(entries)
        cols = list(zip(*entries)) if entries else [()] * 6
        kinds = (C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t)
        return [n] + [(k * n)(*c) for k, c in zip(kinds, cols)]

    def _h2d2_run(self, args, stream) -> None:
        """The pitched copies of `args` (from _h2d2_args) in order on `stream`, one library call."""
        n, dst, dp, src, sp, w, h = args
        _lib.check(self._lib.mkx_h2d_copies_2d(n, dst, dp, src, sp, w, h, C.c_void_p(stream.cuda_stream)),
                   "mkx_h2d_copies_2d")

    def _h2d_run(self, args, stream) -> None:
        """The copies of `args` (from _h2d_args) in order on `stream`, one library call for all."""
        n, dst, src, nb = args
        _lib.check(self._lib.mkx_h2d_copies(n, dst, src, nb, C.c_void_p(stream.cuda_stream)), "mkx_h2d_copies")

    def _h2d(self, pairs, stream) -> None:
        """Host-to-device copies (dst, src) in order on `stream`, one library call for all."""
        self._h2d_run(self._h2d_args(pairs), stream)

    def barriers(self, n_steps: int) -> int:
        return int(self._lib.mkx_sync_points(self._h, int(n_steps)))

    # ---- status / test hooks ------------------------------------------------------------------
    def status(self) -> tuple[int, int]:
        """(error code, stage counter) from the device; synchronous."""
        code, stages = C.c_int(), C.c_longlong()
        self._lib.mkx_last_error(self._h, C.byref(code), C.byref(stages))
        return code.value, stages.value

    def check_device_error(self) -> None:
        code, stages = C.c_int(), C.c_longlong()
        st = self._lib.mkx_last_error(self._h, C.byref(code), C.byref(stages))
        if st == _lib.MKX_ERR_DEVICE:
            raise _lib.MkxError("expert_kernel", st, f"device code 0x{code.value:x} (cta << 16 | kind << 8 | stage)")
        _lib.check(st, "mkx_last_error")

    def clear_error(self) -> None:
        _lib.check(self._lib.mkx_clear_error(self._h), "mkx_clear_error")

    def set_timeout(self, seconds: float) -> None:
        _lib.check(self._lib.mkx_set_timeout_ns(self._h, int(seconds * 1e9)), "mkx_set_timeout_ns")

    def set_fault_injection(self, stage: int) -> None:
        _lib.check(self._lib.mkx_set_fault_injection(self._h, int(stage)), "mkx_set_fault_injection")

    def set_launch_sequence(self, seq: int) -> None:
        """Test hook: the handle's launch sequence number (exchange tags are seq * 4096 + instance + 1
        in 32 bits, so seq and seq + 2**20 give the same tags)."""
        _lib.check(self._lib.mkx_set_launch_sequence(self._h, int(seq) & 0xFFFFFFFF), "mkx_set_launch_sequence")

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.mkx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def install(model) -> ExpertMegakernel:
    """Route ``RekiFlowModel._expert_actions`` (what ``ExpertGraphs`` captures) through the megakernel
    for steps 2..N; modulations, register_prepare and step 1 stay the model's own callables
    (``src/mk_expert.py:521-536``)."""
    mk = ExpertMegakernel(model)
    model._mk = mk

    def _expert_actions(noise, cross_attn_cache, register_cache, state_cond, action_dim, num_steps):
        if noise.shape[0] != 1:
            raise ValueError("the megakernel path runs batch 1")
        mods, dt = model._step_modulations(num_steps, state_cond)
        x_t, cur_k, cur_v = model._expert_first_step(noise, cross_attn_cache, register_cache, mods[:1], dt, action_dim)
        if num_steps > 1:
            x_t = mk.run(x_t, mods, dt, cross_attn_cache, action_dim)
        return x_t, cur_k, cur_v

    model._expert_actions = _expert_actions
    return mk
