"""Parity of the CUDA megakernel (through the C ABI via ``ExpertMegakernel``) with the CPU oracle and
with the reference kernel's golden outputs, plus the launch invariants the reference checks
(``src/test_mk.py:41-51``: max |d| against the other implementations, barrier-count invariant).

Tolerance: max |d| <= 1e-2 and mean |d| <= 1.5e-3 on the real action dims of
the chunk, as is, for every loop length (the synthetic action_out_proj is drawn at std 0.005, see
``synthetic.make_weights``). The rounding-level check is per layer: every traced layer output is
compared with the oracle's layer applied to the kernel's own traced input (teacher forcing).
"""
import pytest
import torch

from oracle.expert_oracle import OracleExpert
from reki_megakernel_b200.synthetic import ExpertDims, make_inputs, make_past, make_weights

from _cases import GOLDEN_FILES, TOL_MAX, TOL_MEAN, chunk_err, golden_case

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module")
def full():
    from reki_megakernel_b200.mk_expert import ExpertMegakernel
    dims = ExpertDims()
    w = make_weights(dims, seed=0)
    mk = ExpertMegakernel(weights=w.to(DEV))
    return dims, w, mk, OracleExpert(w, "bf16")


@pytest.fixture(scope="module")
def small():
    from reki_megakernel_b200.mk_expert import ExpertMegakernel
    dims = ExpertDims(L=2, I=1024)
    w = make_weights(dims, seed=0)
    mk = ExpertMegakernel(weights=w.to(DEV))
    return dims, w, mk, OracleExpert(w, "bf16")


def run_mk(mk, inp, b=0, **kw):
    d = inp.to(DEV)
    past = make_past(d, b)
    out = mk.run(d.x[b:b + 1], d.mods[b], d.dt[b:b + 1], past, d.action_dim, **kw)
    torch.cuda.synchronize()
    mk.check_device_error()
    return out[0].cpu()


def test_full_config_vs_oracle(full):
    dims, w, mk, orc = full
    inp = make_inputs(dims, poison=True)   # T=10, 9 steps, S=160, 2 of 3 frames
    out = run_mk(mk, inp)
    ref = orc.run(inp)[0]
    mx, mean = chunk_err(out, ref, inp.action_dim)
    print(f"kernel vs bf16 oracle, BASELINE configs[1]: max {mx:.3e}, mean {mean:.3e}")
    assert mx <= TOL_MAX and mean <= TOL_MEAN, (mx, mean)
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("name", ["layer", "small", "full"])
def test_vs_reference_golden(name, full, small):
    path = GOLDEN_FILES[name]
    if not path.exists():
        pytest.skip(f"{path.name} not generated")
    dims, w, inp, z = golden_case(path)
    if name == "full":
        mk = full[2]
    elif name == "small":
        mk = small[2]
    else:
        from reki_megakernel_b200.mk_expert import ExpertMegakernel
        mk = ExpertMegakernel(weights=w.to(DEV))
    out = run_mk(mk, inp)
    ref = torch.from_numpy(z["x_out"])
    mx, mean = chunk_err(out, ref, inp.action_dim)
    print(f"kernel vs reference kernel ({name}): max {mx:.3e}, mean {mean:.3e}")
    assert mx <= TOL_MAX and mean <= TOL_MEAN, (mx, mean)
    if name == "layer":  # one layer, one step: every stage's rounding points line up
        assert mx <= 1e-3, mx


def test_per_layer_teacher_forced(full):
    """Per-layer bf16 error without accumulation: the oracle's layer l applied to the kernel's own
    traced output of layer l - 1 must reproduce the kernel's traced output of layer l."""
    dims, w, mk, orc = full
    inp = make_inputs(dims, n_steps=2, poison=True)
    T = inp.x.shape[1]
    trace = torch.zeros(2 * dims.L * T * dims.H, dtype=torch.bfloat16, device=DEV)
    run_mk(mk, inp, trace=trace)
    got = trace.view(2, dims.L, T, dims.H).float().cpu()
    e = inp.episode(0)
    ep = dict(memk=e.memk[0], memv=e.memv[0], kv_start=int(e.kv_start[0]), kca=e.kca[0], vca=e.vca[0],
              S=int(e.S[0]), sa_cos=e.sa_cos[0], sa_sin=e.sa_sin[0], ca_cos=e.ca_cos[0], ca_sin=e.ca_sin[0])
    worst_rel, worst_mean, worst_frac = 0.0, 0.0, 1.0
    for s_ in range(2):
        mrow = inp.mods[0, 1 + s_].float()
        for l in range(1, dims.L):
            ref, _ = orc.layer(l, got[s_, l - 1], mrow, ep)
            g = got[s_, l]
            d = (g - ref).abs()
            worst_rel = max(worst_rel, float(d.max() / ref.abs().max()))      # vs the layer's scale
            worst_mean = max(worst_mean, float(d.mean() / ref.abs().mean()))
            worst_frac = min(worst_frac, float((g == ref).float().mean()))
    print(f"teacher-forced layers: worst max rel {worst_rel:.3e}, worst mean rel {worst_mean:.3e}, "
          f"worst bit-identical fraction {worst_frac:.4f}")
    # 8 dense stages per layer: an early 1-ulp flip perturbs every later accumulation, so some
    # outputs differ by an ulp; the errors must stay at that level (bf16 ulp = 2^-8 relative).
    assert worst_rel <= 1.6e-2 and worst_mean <= 3e-3 and worst_frac >= 0.5, (worst_rel, worst_mean, worst_frac)


@pytest.mark.parametrize("T,adim,n_steps,S,frames", [
    (1, 7, 2, 160, 2), (8, 7, 2, 160, 2), (9, 3, 2, 64, 3), (16, 8, 2, 65, 1), (10, 1, 1, 1, 2),
    (10, 7, 2, 300, 2), (10, 7, 1, 1024, 2)])
def test_edge_shapes(small, T, adim, n_steps, S, frames):
    dims, w, mk, orc = small
    inp = make_inputs(dims, T=T, action_dim=adim, n_steps=n_steps, S=S, frames_valid=frames, poison=True, seed=5)
    out = run_mk(mk, inp)
    ref = orc.run(inp)[0]
    mx, mean = chunk_err(out, ref, adim)
    assert torch.isfinite(out).all()
    assert mx <= TOL_MAX and mean <= TOL_MEAN, (T, adim, S, mx, mean)
    # padded dims (>= action_dim) are 0 + dt * v at the last step, as in the reference
    mxp, _ = chunk_err(out[:, adim:], ref[:, adim:], out.shape[1] - adim)
    assert mxp <= TOL_MAX


@pytest.mark.parametrize("frame_slots,frames_valid", [(8, 6), (8, 8)])
def test_long_memory_several_chunks(small, frame_slots, frames_valid):
    """256 memory rows (192 or 256 valid keys): self-attention runs over more than one key chunk."""
    dims, w, mk, orc = small
    inp = make_inputs(dims, T=10, n_steps=2, frame_slots=frame_slots, frames_valid=frames_valid, S=200,
                      poison=True, seed=7)
    out = run_mk(mk, inp)
    ref = orc.run(inp)[0]
    mx, mean = chunk_err(out, ref, inp.action_dim)
    assert torch.isfinite(out).all()
    assert mx <= TOL_MAX and mean <= TOL_MEAN, (frame_slots, frames_valid, mx, mean)


def test_fp32_mods_bitwise_equal(small):
    """fp32 modulations holding exactly the bf16 values give bit-identical outputs."""
    dims, w, mk, _ = small
    inp = make_inputs(dims, seed=9)
    a = run_mk(mk, inp)
    inp.mods = inp.mods.float()
    b = run_mk(mk, inp)
    assert torch.equal(a, b)


@pytest.mark.parametrize("where", ["x_t", "mods", "dt", "sa_pe", "ca_pe", "cu_kv", "cu_src", "mem_kv", "cross_kv"])
def test_host_tensors_are_rejected_before_launch(small, where):
    """Every tensor ``run`` hands to the library by pointer must be on the expert's device: one left
    in host memory raises ValueError and nothing is launched; the next correct call still matches."""
    dims, w, mk, _ = small
    inp = make_inputs(dims, seed=13)
    good = run_mk(mk, inp)
    d = inp.to(DEV)
    past = make_past(d)
    x, mods, dt = d.x[:1], d.mods[0], d.dt[:1]
    st = past.register_step
    if where == "x_t":
        x = x.cpu()
    elif where == "mods":
        mods = mods.cpu()
    elif where == "dt":
        dt = dt.cpu()
    elif where in ("sa_pe", "ca_pe"):
        st[where] = tuple(t.cpu() for t in st[where])
    elif where in ("cu_kv", "cu_src"):
        st[where] = st[where].cpu()
    elif where == "mem_kv":
        st["mem_kv"] = [(k.cpu(), v) for k, v in st["mem_kv"]]
    else:
        past.cross_attn_kv = [(k, v.cpu()) for k, v in past.cross_attn_kv]
    with pytest.raises(ValueError):
        mk.run(x, mods, dt, past, d.action_dim)
    assert torch.equal(run_mk(mk, inp), good)


def test_deterministic_and_repeatable(small):
    dims, w, mk, _ = small
    inp = make_inputs(dims, seed=11)
    a = run_mk(mk, inp)
    b = run_mk(mk, inp)
    c = run_mk(mk, make_inputs(dims, seed=12))
    d = run_mk(mk, inp)
    assert torch.equal(a, b) and torch.equal(a, d) and not torch.equal(a, c)


def test_stage_count_invariant(full):
    """Every CTA walks every stage: sum of per-CTA stage counts == grid * barriers(n_steps)
    (``src/test_mk.py:44-45``: 108,040 = 148 * 730 on B200)."""
    dims, w, mk, _ = full
    inp = make_inputs(dims)
    mk.clear_error()
    run_mk(mk, inp)
    code, stages = mk.status()
    assert code == 0
    assert mk.barriers(9) == 730
    assert stages == mk.nprog * mk.barriers(9), (stages, mk.nprog)


def test_cuda_graph_capture(small):
    dims, w, mk, _ = small
    inp = make_inputs(dims, seed=21).to(DEV)
    past = make_past(inp)
    eager = mk.run(inp.x[:1], inp.mods[0], inp.dt[:1], past, inp.action_dim).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        mk.run(inp.x[:1], inp.mods[0], inp.dt[:1], past, inp.action_dim)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = mk.run(inp.x[:1], inp.mods[0], inp.dt[:1], past, inp.action_dim)
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    mk.check_device_error()


def test_exchange_tags_after_the_sequence_wraps(small):
    """Exchange tags repeat every 2^20 launches. A launch with 16 action rows, then one with 10 (it
    clears rows 10-15 of every exchange buffer, which it does not use), then, 2^20 sequence numbers
    after the first (set through the test hook instead of a million launches), one with 16 rows
    again: its tags equal the first launch's, and its output must still equal a fresh handle's,
    bit for bit -- no word of the first launch is taken for one of the third's."""
    from reki_megakernel_b200.mk_expert import ExpertMegakernel
    dims, w, mk, _ = small
    third = make_inputs(dims, T=16, n_steps=1, poison=True, seed=53)
    fresh = ExpertMegakernel(weights=w.to(DEV))
    want = run_mk(fresh, third)
    fresh.close()
    seq = 5000
    mk.set_launch_sequence(seq)
    run_mk(mk, make_inputs(dims, T=16, n_steps=1, poison=True, seed=51))
    run_mk(mk, make_inputs(dims, T=10, n_steps=1, poison=True, seed=52))
    mk.set_launch_sequence(seq + (1 << 20))
    assert torch.equal(run_mk(mk, third), want)


def test_timeout_reports_error_and_recovers(small):
    """A withheld exchange word (test hook, nothing faults) makes the bounded waits run out: the
    launch returns, the error word is set, and the next launch after clear_error is correct."""
    from reki_megakernel_b200._lib import MkxError
    dims, w, mk, _ = small
    inp = make_inputs(dims, seed=31)
    good = run_mk(mk, inp)
    mk.set_timeout(0.05)
    mk.set_fault_injection(1)
    d = inp.to(DEV)
    mk.run(d.x[:1], d.mods[0], d.dt[:1], make_past(d), d.action_dim)
    torch.cuda.synchronize()
    code, _ = mk.status()
    assert code != 0 and ((code >> 8) & 0xff) == 1, hex(code)   # kind 1: a wait timed out
    with pytest.raises(MkxError):
        mk.check_device_error()
    mk.set_fault_injection(0)
    mk.set_timeout(2.0)
    mk.clear_error()
    again = run_mk(mk, inp)
    assert torch.equal(again, good)


def test_install_routes_expert_actions(small):
    """``install(model)`` replaces ``_expert_actions`` and keeps step 1 / modulations the model's."""
    from reki_megakernel_b200.mk_expert import install
    from reki_megakernel_b200.synthetic import make_model
    dims, w, _, orc = small
    inp = make_inputs(dims, seed=41, n_steps=2).to(DEV)
    model = make_model(w.to(DEV))
    calls = {}

    def step_modulations(num_steps, state_cond):
        calls["mods"] = num_steps
        return inp.mods[0], inp.dt[:1]

    def first_step(noise, cache, reg, mods1, dt, adim):
        calls["first"] = True
        return inp.x[:1], "k", "v"
    model._step_modulations = step_modulations
    model._expert_first_step = first_step
    mk = install(model)
    x, k, v = model._expert_actions(inp.x[:1], make_past(inp), None, None, inp.action_dim, inp.n_steps + 1)
    torch.cuda.synchronize()
    assert calls == {"mods": inp.n_steps + 1, "first": True} and (k, v) == ("k", "v")
    ref = orc.run(inp.to("cpu"))[0]
    mx, mean = chunk_err(x[0], ref, inp.action_dim)
    assert mx <= TOL_MAX and mean <= TOL_MEAN
    mk.close()
