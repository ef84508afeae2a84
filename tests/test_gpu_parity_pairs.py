"""Pairwise parity at BASELINE configs[1] (10 layers, 10 action rows, 9 Euler steps, S = 160) between
the megakernel and four independent implementations of steps 2..10, the way the reference's own
check compares its megakernel with Kyutai's eager and compiled expert (``src/test_mk.py:34-51``,
``results/gpus/b200/test_mk.json:8-13``):

* ``mk``        -- this library's kernel (``ExpertMegakernel.run`` through the C ABI);
* ``reference`` -- the reference's Triton kernel, run on the same seeded inputs by
                   ``tests/golden/make_golden.py`` (fixture ``ref_full.npz``);
* ``oracle``    -- the bf16 CPU oracle (the reference kernel's rounding points);
* ``eager``     -- the oracle in plain fp32, on the GPU;
* ``compiled``  -- the expert on native bf16 tensors (library GEMMs, SDPA attention) through
                   ``torch.compile``, on the GPU (the stand-in for the compiled expert).

Every pair must meet the north-star bar on the real action dims, unscaled: max |d| <= 1e-2 and
mean |d| <= 1.5e-3. The errors are printed; with MKX_PARITY_JSON set they are also written there as
JSON, in the reference's key style (``max|a-b| action dims``).
"""
import itertools
import json
import os

import pytest
import torch

from _cases import GOLDEN_FILES, TOL_MAX, TOL_MEAN, chunk_err, golden_case

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_pairwise_parity_baseline_config():
    from oracle.expert_oracle import NativeBf16Expert, OracleExpert
    from reki_megakernel_b200.mk_expert import ExpertMegakernel
    from reki_megakernel_b200.synthetic import make_past

    path = GOLDEN_FILES["full"]
    dims, w, inp, z = golden_case(path)          # configs[1] inputs regenerated from the fixture's seeds
    d = inp.to(DEV)
    mk = ExpertMegakernel(weights=w.to(DEV))
    out = {"mk": mk.run(d.x[:1], d.mods[0], d.dt[:1], make_past(d), d.action_dim)[0]}
    torch.cuda.synchronize()
    mk.check_device_error()
    out["reference"] = torch.from_numpy(z["x_out"])
    out["oracle"] = OracleExpert(w, "bf16").run(inp)[0]
    with torch.no_grad():
        out["eager"] = OracleExpert(w, "fp32", DEV).run(inp)[0]
        out["compiled"] = NativeBf16Expert(w, DEV, compile=True).run(inp)[0]
    torch.cuda.synchronize()
    adim = inp.action_dim
    res = {"config": "BASELINE configs[1]: L=10, T=10, 9 Euler steps, S=160, 2 of 3 register frames, batch 1",
           "tolerance": {"max": TOL_MAX, "mean": TOL_MEAN}}
    bad = []
    for a, b in itertools.combinations(out, 2):
        mx, mean = chunk_err(out[a], out[b], adim)
        res[f"max|{a}-{b}| action dims"] = mx
        res[f"mean|{a}-{b}| action dims"] = mean
        if not (mx <= TOL_MAX and mean <= TOL_MEAN):
            bad.append((a, b, mx, mean))
    res["max_abs_x action dims"] = float(out["mk"][:, :adim].abs().max())
    print(json.dumps(res, indent=1))
    if os.environ.get("MKX_PARITY_JSON"):
        with open(os.environ["MKX_PARITY_JSON"], "w") as f:
            json.dump(res, f, indent=1)
    assert not bad, bad
