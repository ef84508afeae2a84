"""Per-step modulation rows on the GPU (conditioning + HBM-bound projection) against their CPU
restatement (parity unpinned: Kyutai's ``_step_modulations`` is not in the reference).

Checked stage by stage, each against the oracle on the same input:
* conditioning a = bf16(silu(8 e)): the GPU computes the timestep embedding in double and e in fp32
  (256-long dot products), the oracle all in float64. Bar: >= 99 % of a bit-identical, every element
  within one bf16 ulp (2^-7 of its magnitude) plus 2^-14 of its row's RMS.
* projection mods = bf16(W_m a + b_m), given the GPU's own bf16 a: fp32 accumulation (GPU) against
  float64 (oracle) of the same bf16 products. Bar: >= 99 % bit-identical, every output within one
  bf16 ulp plus 2^-14 of its row's RMS.
* end to end against the oracle's own a: a conditioning element whose rounding flipped moves an
  output by about 2^-13 of its row's RMS. Bar: every output within one bf16 ulp plus 2^-11 of its
  row's RMS.
dt = 1/N exactly."""
import pytest
import torch

from oracle.modulation_oracle import conditioning_oracle, modulation_oracle
from reki_megakernel_b200.synthetic import ExpertDims, make_modulation_weights, make_state

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _check(got, ref, min_exact, rms_frac):
    g, r = got.float().cpu(), ref.float()
    exact = (g == r).float().mean().item()
    rms = r.pow(2).mean(-1, keepdim=True).sqrt()
    tol = r.abs() * 2.0 ** -7 + rms * rms_frac + 1e-30
    worst = ((g - r).abs() / tol).max().item()
    assert exact >= min_exact and worst <= 1.0, (exact, worst)
    return exact


def _check_stages(sm, w, st, N, mods):
    """Conditioning vs its oracle; projection vs the oracle on the GPU's own input; end to end."""
    a_gpu = sm.projection_input().cpu()
    a_ref = conditioning_oracle(w.w_t, w.w_s, st, N)
    assert (a_gpu[N:] == 0).all()
    _check(a_gpu[:N], a_ref, 0.99, 2.0 ** -14)
    proj = (a_gpu[:N].double() @ w.w_m.double().T + w.b_m.double()[None, :]).to(torch.bfloat16)
    _check(mods, proj, 0.99, 2.0 ** -14)
    ref, _ = modulation_oracle(w.w_t, w.w_s, w.w_m, w.b_m, st, N)
    _check(mods, ref, 0.0, 2.0 ** -11)


@pytest.fixture(scope="module")
def full():
    from reki_megakernel_b200.modulations import StepModulations
    d = ExpertDims()
    w = make_modulation_weights(d, seed=0)
    sm = StepModulations(w.to(DEV))
    yield d, w, sm
    sm.close()


@pytest.mark.parametrize("N", [1, 2, 8, 9, 10, 16])
def test_modulations_match_oracle(full, N):
    d, w, sm = full
    st = make_state(w.sdim, seed=N)
    mods, dt = sm(N, st.to(DEV))
    torch.cuda.synchronize()
    assert mods.shape == (N, d.MODW) and mods.dtype == torch.bfloat16
    _check_stages(sm, w, st, N, mods)
    rdt = 1.0 / N
    assert dt.item() == torch.tensor(rdt, dtype=torch.float32).item()


def test_small_model_and_out_buffers():
    from reki_megakernel_b200.modulations import StepModulations
    d = ExpertDims(L=2)
    w = make_modulation_weights(d, seed=5, tdim=128, sdim=33)
    sm = StepModulations(w.to(DEV))
    st = make_state(33, seed=5)
    mods = torch.full((10, d.MODW), 7.0, dtype=torch.bfloat16, device=DEV)
    dt = torch.zeros(1, device=DEV)
    sm(10, st.to(DEV), out=(mods, dt))
    torch.cuda.synchronize()
    _check_stages(sm, w, st, 10, mods)
    assert dt.item() == pytest.approx(0.1)
    sm.close()


def test_graph_capture_and_feeds_the_expert(full):
    """Captured in a CUDA graph; its rows drive ExpertMegakernel.run like the oracle's rows do. The two
    row sets differ by one bf16 ulp in ~1 % of their entries, which the 9 integrated Euler steps of the
    synthetic expert carry to a few 1e-3 of the action chunk; rows read at a wrong step or offset give
    differences of order 1. Bar: max |d| <= 5e-2, mean <= 1e-2, and the run is bitwise repeatable."""
    from oracle.expert_oracle import chunk_diff
    from reki_megakernel_b200.mk_expert import ExpertMegakernel
    from reki_megakernel_b200.synthetic import make_inputs, make_past, make_weights
    d, w, sm = full
    st = make_state(w.sdim, seed=11).to(DEV)
    eager, _ = sm(10, st)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        sm(10, st)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        mods, dt = sm(10, st)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(mods, eager)

    ref, _ = modulation_oracle(w.w_t, w.w_s, w.w_m, w.b_m, st.cpu(), 10)
    mk = ExpertMegakernel(weights=make_weights(d, seed=0).to(DEV))
    inp = make_inputs(d).to(DEV)
    past = make_past(inp)
    out_gpu = mk.run(inp.x[:1], mods, dt, past, inp.action_dim)
    again = mk.run(inp.x[:1], mods.clone(), dt, past, inp.action_dim)
    out_ref = mk.run(inp.x[:1], ref.to(DEV), torch.tensor([0.1], device=DEV), past, inp.action_dim)
    torch.cuda.synchronize()
    mk.check_device_error()
    assert torch.equal(out_gpu, again)
    err = chunk_diff(out_gpu[0].cpu(), out_ref[0].cpu(), inp.action_dim)
    assert err["max_abs"] <= 5e-2 and err["mean_abs"] <= 1e-2, err
    mk.close()
