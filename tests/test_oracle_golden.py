"""The CPU oracle pinned against the reference's own kernel (CPU only).

``tests/golden/ref_*.npz`` were written by ``tests/golden/make_golden.py``, which runs the reference's
Triton kernel (``src/mk_expert.py``) unmodified on identical seeded inputs; each file holds the final
action state and the kernel's last-layer scratch buffers (qkv, h2, qca, h3, g, h of the last layer of
the last Euler step, bf16 bit patterns). The inputs are regenerated here from the stored seeds and the
oracle (``oracle/expert_oracle.py``, mode "bf16") runs on the CPU.

* one layer, one step: every stage's rounding points line up, so the action state agrees to fp32
  rounding (<= 1e-6) and >= 99.9 % of every scratch buffer is bit-identical (the rest one-ulp flips
  from a different fp32 summation order: within 2^-8 of the buffer's largest magnitude);
* 2 layers x 3 steps and the full configuration (10 layers x 9 steps): the one-ulp flips compound
  through the Euler loop, so the chunk is checked with the north-star tolerance (max 1e-2, mean
  1.5e-3 on the real action dims, as is).
"""
import pytest
import torch

from _cases import GOLDEN_FILES, TOL_MAX, TOL_MEAN, bf16_from_u16, chunk_err, golden_case
from oracle.expert_oracle import OracleExpert

BUFFERS = (("h", "h_last"), ("h2", "h2_last"), ("h3", "h3_last"), ("qkv", "qkv_last"), ("qca", "qca_last"),
           ("g", "g_last"))


def _run(name):
    path = GOLDEN_FILES[name]
    if not path.exists():
        pytest.skip(f"{path.name} not generated")
    dims, w, inp, z = golden_case(path)
    trace = []
    x = OracleExpert(w, "bf16").run(inp, trace=trace)[0]
    return inp, z, x, trace[-1]


def test_one_layer_matches_the_reference_kernel_stage_by_stage():
    inp, z, x, last = _run("layer")
    mx, _ = chunk_err(x, torch.from_numpy(z["x_out"]), inp.x.shape[2])
    assert mx <= 1e-6, mx
    for key, buf in BUFFERS:
        got = last[key].float()
        ref = bf16_from_u16(z[buf]).reshape(got.shape)
        same = (got == ref).float().mean().item()
        worst = ((got - ref).abs().max() / ref.abs().max()).item()
        assert same >= 0.999 and worst <= 2.0 ** -8, (key, same, worst)


def test_two_layers_three_steps_within_tolerance():
    inp, z, x, _ = _run("small")
    mx, mean = chunk_err(x, torch.from_numpy(z["x_out"]), inp.action_dim)
    assert mx <= TOL_MAX and mean <= TOL_MEAN, (mx, mean)


def test_full_configuration_within_tolerance():
    inp, z, x, _ = _run("full")
    mx, mean = chunk_err(x, torch.from_numpy(z["x_out"]), inp.action_dim)
    assert mx <= TOL_MAX and mean <= TOL_MEAN, (mx, mean)
    assert int(z["barriers"]) == int(z["expected_barriers"])  # the reference run walked every barrier
