"""The restated modulation network's CPU oracle (parity unpinned: Kyutai's ``_step_modulations`` is
not in the reference): its output contract and its rounding points, on small shapes."""
import torch

from oracle.modulation_oracle import conditioning_oracle, modulation_oracle
from reki_megakernel_b200.synthetic import ExpertDims, make_modulation_weights, make_state


def test_output_contract():
    d = ExpertDims(L=2)
    w = make_modulation_weights(d, seed=1)
    st = make_state(w.sdim, seed=1)
    mods, dt = modulation_oracle(w.w_t, w.w_s, w.w_m, w.b_m, st, 10)
    assert mods.shape == (10, 9 * d.L * d.H + 2 * d.H) == (10, d.MODW) and mods.dtype == torch.bfloat16
    assert dt == 0.1
    assert torch.isfinite(mods.float()).all()


def test_projection_input_is_bf16_silu_of_the_conditioning():
    d = ExpertDims(L=1)
    w = make_modulation_weights(d, seed=2)
    st = make_state(w.sdim, seed=2)
    a = conditioning_oracle(w.w_t, w.w_s, st, 4)
    assert torch.equal(a, a.to(torch.bfloat16).double())          # rounded once to bf16
    # step 0 has t = 1: the embedding is cos / sin of 1000 f_i
    half = w.tdim // 2
    f = torch.tensor([10000.0 ** (-i / half) for i in range(half)], dtype=torch.float64)
    temb = torch.cat([(1000.0 * f).cos(), (1000.0 * f).sin()])
    e = 8.0 * (w.w_t.double() @ temb + w.w_s.double() @ st.double())
    ref = (e * torch.sigmoid(e)).to(torch.bfloat16).double()
    assert torch.equal(a[0], ref)


def test_steps_differ_and_state_matters():
    d = ExpertDims(L=1)
    w = make_modulation_weights(d, seed=3)
    m1, _ = modulation_oracle(w.w_t, w.w_s, w.w_m, w.b_m, make_state(w.sdim, seed=3), 5)
    m2, _ = modulation_oracle(w.w_t, w.w_s, w.w_m, w.b_m, make_state(w.sdim, seed=4), 5)
    assert not torch.equal(m1[0], m1[1]) and not torch.equal(m1, m2)
