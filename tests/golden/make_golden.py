"""Generate golden fixtures by running the REFERENCE megakernel on identical seeded inputs.

    python tests/golden/make_golden.py --ref <reference checkout> [--configs small full]

(``--ref`` defaults to the ``REKI_REFERENCE`` environment variable.)

The reference's Triton kernel (``src/mk_expert.py``, class ``ExpertMegakernel`` and kernel
``expert_megakernel``) is imported unmodified from the reference checkout and executed on the CPU
through Triton's interpreter (``TRITON_INTERPRET=1``). Three interpreter behaviours are adjusted so
the run computes what the GPU computes, and nothing in the reference's code is changed:

* bf16 ``tl.dot`` operands are stored as raw uint16 bit patterns by the interpreter, which then
  multiplies the integers; here they are widened to fp32 first (fp32 accumulation, as on the GPU).
* fp32 -> bf16 casts truncate in the interpreter; here they round to nearest even, as the GPU's
  ``cvt.rn.bf16.f32`` does.
* The interpreter runs programs one after another, so the kernel's software grid barrier
  (``_arrive`` / ``_wait``, ``src/mk_expert.py:43-76``) would spin forever. Each program runs in its
  own thread and the two barrier helpers are replaced by a ``threading.Barrier`` over all programs
  (same ordering guarantee: no program starts stage k + 1 before all finished stage k). The L2
  prefetch (``PF``, inline PTX) is switched off with the reference's own config flag; it never
  changes results (``results/gpus/b200/tune_v5.json``: identical max |d| with PF on and off).

The reference needs ``torch.cuda.get_device_properties(..).multi_processor_count``; the script
reports ``NPROG`` programs (the result does not depend on it: every tile is computed the same way
by whichever program owns it).

Outputs ``tests/golden/ref_<config>.npz``: the reference's final action state, the scratch buffers
it leaves behind (last layer of the last step), and the configuration; the inputs themselves are
regenerated from the stored seeds by ``reki_megakernel_b200.synthetic``.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time
from pathlib import Path
from types import SimpleNamespace

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from reki_megakernel_b200.synthetic import ExpertDims, make_inputs, make_model, make_weights  # noqa: E402

NPROG = 72  # the reference's minimum: H / BT + A - AO programs (src/mk_expert.py:480)

CONFIGS = {
    # One layer, one Euler step: isolates every stage's rounding points (near bit-exact check).
    "layer": dict(dims=dict(L=1, I=1024), inputs=dict(T=5, n_steps=1, frame_slots=2, frames_valid=1,
                                                     S=100, action_dim=6, seed=3, noise_seed=77)),
    # L=2 layers, MLP 1024, 5 action rows, odd source length, shorter memory, 3 Euler steps.
    "small": dict(dims=dict(L=2, I=1024), inputs=dict(T=5, n_steps=3, frame_slots=2, frames_valid=1,
                                                     S=100, action_dim=6, seed=3, noise_seed=77)),
    # REKI's expert at BASELINE configs[1]: 10 layers, 10 action rows, 2 of 3 register frames valid,
    # 160 source rows, 9 Euler steps.
    "full": dict(dims=dict(), inputs=dict(T=10, n_steps=9, S=160, action_dim=7, seed=0, noise_seed=1234)),
}


def _patch_interpreter():
    import triton.language as tl
    from triton.runtime import interpreter as it

    def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
        t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)
        return t.view(torch.int16).numpy().view(np.uint16)

    def bf16_bits_to_f32(a: np.ndarray) -> np.ndarray:
        return (a.astype(np.uint32) << 16).view(np.float32)

    orig_cast = it.InterpreterBuilder.cast_impl
    orig_fp = it.InterpreterBuilder.create_fp_to_fp

    def cast_impl(self, src, dst_type):
        s, d = src.dtype.scalar, dst_type.scalar
        if s == tl.float32 and d == tl.bfloat16:
            return it.TensorHandle(f32_to_bf16_bits(src.data), d)
        if s == tl.bfloat16 and d == tl.float32:
            return it.TensorHandle(bf16_bits_to_f32(src.data), d)
        return orig_cast(self, src, dst_type)

    def create_fp_to_fp(self, src, dst_type, rounding_mode):
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
            return it.TensorHandle(f32_to_bf16_bits(src.data), dst_type.scalar)
        return orig_fp(self, src, dst_type, rounding_mode)

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        ad = bf16_bits_to_f32(a.data) if a.dtype.scalar == tl.bfloat16 else a.data.astype(np.float32)
        bd = bf16_bits_to_f32(b.data) if b.dtype.scalar == tl.bfloat16 else b.data.astype(np.float32)
        return it.TensorHandle(np.matmul(ad, bd, dtype=np.float32) + d.data, d.dtype.scalar)

    it.InterpreterBuilder.cast_impl = cast_impl
    it.InterpreterBuilder.create_si_to_fp = lambda self, s, t: cast_impl(self, s, t)
    it.InterpreterBuilder.create_fp_ext = lambda self, s, t: cast_impl(self, s, t)
    it.InterpreterBuilder.create_fp_trunc = lambda self, s, t: cast_impl(self, s, t)
    it.InterpreterBuilder.create_fp_to_fp = create_fp_to_fp
    it.InterpreterBuilder.create_dot = create_dot

    # Thread-local program ids: each program of the grid runs in its own thread.
    tls = threading.local()
    it.InterpreterBuilder.grid_idx = property(lambda self: getattr(tls, "idx", None),
                                              lambda self, v: setattr(tls, "idx", v))

    def threaded_call(self, *args_dev, **kwargs):
        import inspect
        argspec = inspect.getfullargspec(self.fn)
        kwargs = {k: v for k, v in kwargs.items() if k in argspec.args}
        args_hst, kwargs_hst = self._init_args_hst(args_dev, kwargs)
        scope = it._patch_lang(self.fn)
        errors = []
        try:
            args = inspect.getcallargs(self.fn, *args_hst, **kwargs_hst)
            args = {n: a if n in self.constexprs else it._implicit_cvt(a) for n, a in args.items()}
            grid = self.grid(args) if callable(self.grid) else self.grid
            grid = tuple(grid) + (1,) * (3 - len(grid))
            assert grid[1] == grid[2] == 1
            it.interpreter_builder.set_grid_dim(*grid)

            def body(pid):
                try:
                    it.interpreter_builder.set_grid_idx(pid, 0, 0)
                    self.fn(**args)
                except BaseException as e:  # noqa: BLE001
                    errors.append(e)
                    _BARRIER.abort()
            ths = [threading.Thread(target=body, args=(p,)) for p in range(grid[0])]
            for t in ths:
                t.start()
            for t in ths:
                t.join()
        finally:
            scope.restore()
        if errors:
            raise errors[0]
        self._restore_args_dev(args_dev, args_hst, kwargs, kwargs_hst)

    it.GridExecutor.__call__ = threaded_call


_BARRIER = threading.Barrier(NPROG)
_BARRIER_COUNT = [0]
_COUNT_LOCK = threading.Lock()


def _arrive(bar_ptr):
    return None


def _wait(bar_ptr, nb, nprog, prof_ptr, pid, POLL, PROFILE):
    with _COUNT_LOCK:
        _BARRIER_COUNT[0] += 1
    _BARRIER.wait()


def run_reference(ref_src: Path, cfg: dict):
    _patch_interpreter()
    sys.path.insert(0, str(ref_src))
    import mk_expert as ref  # the reference module, unmodified
    ref._arrive = _arrive
    ref._wait = _wait

    dims = ExpertDims(**cfg["dims"])
    w = make_weights(dims, seed=0)
    inp = make_inputs(dims, poison=True, **cfg["inputs"])
    model = make_model(w)
    orig_props = torch.cuda.get_device_properties
    torch.cuda.get_device_properties = lambda dev=None: SimpleNamespace(multi_processor_count=NPROG)
    try:
        mk = ref.ExpertMegakernel(model)
    finally:
        torch.cuda.get_device_properties = orig_props
    mk.cfg["PF"] = False
    T = inp.x.shape[1]
    past = SimpleNamespace(
        register_step={"mem_kv": [(inp.memk[0, l], inp.memv[0, l]) for l in range(dims.L)],
                       "sa_pe": (inp.sa_cos[0], inp.sa_sin[0]), "ca_pe": (inp.ca_cos[0], inp.ca_sin[0]),
                       "cu_kv": torch.tensor([int(inp.kv_start[0]), 0], dtype=torch.int32),
                       "cu_src": torch.tensor([0, int(inp.S[0])], dtype=torch.int32)},
        cross_attn_kv=[(inp.kca[0, l], inp.vca[0, l]) for l in range(dims.L)])
    _BARRIER_COUNT[0] = 0
    t0 = time.time()
    with torch.no_grad():
        x = mk.run(inp.x[0:1].reshape(1, T, dims.A), inp.mods[0], inp.dt[0:1], past, inp.action_dim)
    el = time.time() - t0
    n_steps = inp.mods.shape[1] - 1
    res = dict(
        x_out=x[0].numpy().astype(np.float32),
        h_last=mk.hh[1, :T].view(torch.int16).numpy().view(np.uint16),
        h2_last=mk.h2[:T].view(torch.int16).numpy().view(np.uint16),
        h3_last=mk.h3[:T].view(torch.int16).numpy().view(np.uint16),
        qkv_last=mk.qkv[:T].view(torch.int16).numpy().view(np.uint16),
        qca_last=mk.qca[:T].view(torch.int16).numpy().view(np.uint16),
        g_last=mk.g[:T].view(torch.int16).numpy().view(np.uint16),
        barriers=np.int64(_BARRIER_COUNT[0] // NPROG), expected_barriers=np.int64(mk.barriers(n_steps)),
    )
    return res, el


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("REKI_REFERENCE"),
                    help="root of the reference checkout (the directory holding src/mk_expert.py)")
    ap.add_argument("--configs", nargs="*", default=list(CONFIGS))
    a = ap.parse_args()
    if not a.ref:
        ap.error("--ref (or REKI_REFERENCE) must name the reference checkout")
    out_dir = Path(__file__).resolve().parent
    for name in a.configs:
        cfg = CONFIGS[name]
        res, el = run_reference(Path(a.ref) / "src", cfg)
        np.savez_compressed(out_dir / f"ref_{name}.npz", config=json.dumps(cfg), **res)
        print(f"{name}: {el:.1f} s, barriers {int(res['barriers'])} (expected {int(res['expected_barriers'])}), "
              f"max|x| {np.abs(res['x_out']).max():.4f}", flush=True)


if __name__ == "__main__":
    main()
