"""The register pass and the whole carried predict (all 10 Euler steps, 3 register
frames x 32 rows carried over 20 consecutive seeded predicts) against the CPU restatement in
``oracle/register_oracle.py`` (parity unpinned: Kyutai's step 1 and register cache are absent from
the reference).

Tolerances. Action chunks: the north-star bar, max |d| <= 1e-2 and mean |d| <= 1.5e-3 on the real
action dims. Register K / V written by the pass: the register rows run with unit gates, so every
layer adds O(1) updates to the residual and the bf16 rounding noise grows layer by layer (the bf16
and fp32 restatements end about 1e-2 apart in mean on these O(1) values). The device result is held
to that noise: per layer, mean |device - bf16 oracle| <= 1.3 x mean |bf16 oracle - fp32 oracle| +
1e-4 and max <= 1.5 x that max + 1.6e-2; the first layer's K / V (identical inputs, fp32
accumulation in another order) at least 99 % bit-identical. Rows outside the frame and rows below
kv_start (NaN) must stay untouched and unread."""
import pytest
import torch

from reki_megakernel_b200.synthetic import (ExpertDims, make_modulation_weights, make_prepare_weights, make_register_rows,
                                            make_source, make_state, make_weights, register_rope)

from _cases import TOL_MAX, TOL_MEAN, chunk_err

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def assert_within_noise(got, ref, ref32, what):
    """got vs the bf16 oracle, bounded by the bf16 oracle's own distance from the fp32 oracle."""
    e = (got.float() - ref.float()).abs()
    n = (ref.float() - ref32.float()).abs()
    assert float(e.mean()) <= 1.3 * float(n.mean()) + 1e-4, (what, float(e.mean()), float(n.mean()))
    assert float(e.max()) <= 1.5 * float(n.max()) + 1.6e-2, (what, float(e.max()), float(n.max()))
    return float(e.max()), float(e.mean()), float(n.mean())


def _u16(t):
    return t.contiguous().view(torch.int16)


@pytest.fixture(scope="module", params=["small", "full"])
def parts(request):
    from oracle.expert_oracle import OracleExpert
    from reki_megakernel_b200.batch import BatchedExpert
    d = ExpertDims(L=2, I=1024) if request.param == "small" else ExpertDims()
    w = make_weights(d, seed=0)
    bx = BatchedExpert(w.to(DEV), max_episodes=2)
    yield request.param, d, w, bx, OracleExpert(w, "bf16"), OracleExpert(w, "fp32")
    bx.close()


def _pass_inputs(d, PM=96, R=32, frames=2, S=100, SP=128, seed=0):
    g = torch.Generator().manual_seed(seed + 5)
    memk = torch.randn((d.L, PM, d.NH, d.HD), generator=g).to(torch.bfloat16)
    memv = torch.randn((d.L, PM, d.NH, d.HD), generator=g).to(torch.bfloat16)
    ks = PM - R * frames
    memk[:, :ks] = float("nan")
    memv[:, :ks] = float("nan")
    memk[:, PM - R:] = float("nan")  # overwritten before the self-attention reads it
    memv[:, PM - R:] = float("nan")
    kca = torch.randn((d.L, SP, d.NH, d.HD), generator=g).to(torch.bfloat16)
    vca = torch.randn((d.L, SP, d.NH, d.HD), generator=g).to(torch.bfloat16)
    kca[:, S:] = float("nan")
    vca[:, S:] = float("nan")
    return memk, memv, ks, kca, vca, S


@pytest.mark.parametrize("frames,S", [(1, 100), (2, 160), (3, 1)])
def test_register_pass_writes_the_frame(parts, frames, S):
    from oracle.register_oracle import register_pass
    name, d, w, bx, orc, orc32 = parts
    PM, R = 96, 32
    memk, memv, ks, kca, vca, S = _pass_inputs(d, PM, R, frames, S, SP=max(64, -(-S // 64) * 64), seed=frames)
    reg = make_register_rows(d, R, seed=frames)
    rope = register_rope(d, PM, R)
    gk, gv = memk.clone().to(DEV), memv.clone().to(DEV)
    bx.register_pass(reg.to(DEV), gk, gv, torch.tensor([ks], dtype=torch.int32, device=DEV), kca.to(DEV), vca.to(DEV),
                     torch.tensor([S], dtype=torch.int32, device=DEV), tuple(t.to(DEV) for t in rope[:2]),
                     tuple(t.to(DEV) for t in rope[2:]))
    torch.cuda.synchronize()
    bx.check_device_error()
    gk, gv = gk.cpu(), gv.cpu()
    rk, rv = memk.clone(), memv.clone()
    register_pass(orc, reg, rk, rv, ks, kca, vca, S, rope[:2], rope[2:])
    fk32, fv32 = memk.clone(), memv.clone()
    register_pass(orc32, reg, fk32, fv32, ks, kca, vca, S, rope[:2], rope[2:])
    # rows outside the frame untouched, bit for bit (NaN patterns included)
    assert torch.equal(_u16(gk[:, :PM - R]), _u16(memk[:, :PM - R]))
    assert torch.equal(_u16(gv[:, :PM - R]), _u16(memv[:, :PM - R]))
    fk, fv = gk[:, PM - R:], gv[:, PM - R:]
    assert torch.isfinite(fk.float()).all() and torch.isfinite(fv.float()).all()
    worst = (0.0, 0.0, 0.0)
    for l in range(d.L):
        for got, ref, r32, what in ((fk[l], rk[l, PM - R:], fk32[l, PM - R:], f"K{l}"),
                                    (fv[l], rv[l, PM - R:], fv32[l, PM - R:], f"V{l}")):
            mx, mean, noise = assert_within_noise(got, ref, r32, (name, what))
            worst = (max(worst[0], mx), max(worst[1], mean), max(worst[2], noise))
    for got, ref in ((fk[0], rk[0, PM - R:]), (fv[0], rv[0, PM - R:])):
        same0 = float((_u16(got) == _u16(ref)).float().mean())
        assert same0 >= 0.99, same0
    print(f"{name} frames={frames} S={S}: K/V worst max {worst[0]:.3e} mean {worst[1]:.3e} "
          f"(bf16-fp32 oracle mean up to {worst[2]:.3e})")


def test_register_pass_rejects_bad_arguments(parts):
    name, d, w, bx, orc, orc32 = parts
    memk, memv, ks, kca, vca, S = _pass_inputs(d)
    z = lambda *s: torch.zeros(s, dtype=torch.float32, device=DEV)  # noqa: E731
    one = torch.tensor([0], dtype=torch.int32, device=DEV)
    args = lambda reg, R=32: (reg, memk.to(DEV), memv.to(DEV), one, kca.to(DEV), vca.to(DEV), one,  # noqa: E731
                              (z(R, d.HD), z(R, d.HD)), (z(R, d.HD), z(R, d.HD)))
    with pytest.raises(ValueError):
        bx.register_pass(*args(torch.zeros((24, d.H), dtype=torch.bfloat16, device=DEV), 24))  # not a multiple of 16
    with pytest.raises(ValueError):
        bx.register_pass(*args(torch.zeros((48, d.H), dtype=torch.bfloat16, device=DEV), 48))  # > 16 * max_episodes
    with pytest.raises(ValueError):
        bx.register_pass(*args(torch.zeros((32, d.H), dtype=torch.bfloat16)))                  # host tensor


def _predictors(d, w, bx, S, graph=True, T=10, frames=3):
    from reki_megakernel_b200.full_predict import FullPredict
    from reki_megakernel_b200.mk_expert import ExpertMegakernel
    from reki_megakernel_b200.modulations import StepModulations
    from reki_megakernel_b200.prepare import RegisterPrepare
    mk = ExpertMegakernel(weights=w.to(DEV))
    rp = RegisterPrepare(make_prepare_weights(d, seed=0).to(DEV))
    sm = StepModulations(make_modulation_weights(d, seed=0).to(DEV))
    fp = FullPredict(mk, bx, rp, sm, make_register_rows(d, 32).to(DEV), S=S, num_steps=10, T=T, frames=frames,
                     graph=graph)
    return fp, (mk, rp, sm)


def _predict_inputs(d, p, S, sdim=7, T=10):
    src = make_source(S, d.src_dim, seed=100 + p)
    state = make_state(sdim, seed=100 + p)
    noise = torch.randn((1, T, d.A), generator=torch.Generator().manual_seed(1234 + p))
    return src, state, noise


def test_carried_predicts_match_the_oracle(parts):
    """20 consecutive predicts (small expert) / 4 (full expert) carrying the memory: each action
    chunk against the restated predict fed with the device's own cross-attention K/V and modulation
    rows (those kernels have their own parity tests); the memory after the last predict too."""
    from oracle.register_oracle import PredictOracle
    name, d, w, bx, orc, orc32 = parts
    S = 160
    n = 20 if name == "small" else 4
    fp, keep = _predictors(d, w, bx, S)
    mk_po = lambda o: PredictOracle(o, make_prepare_weights(d, seed=0), make_modulation_weights(d, seed=0),  # noqa: E731
                                    make_register_rows(d, 32), N=10, PM=96, R=32, T=10, action_dim=7)
    po, po32 = mk_po(orc), mk_po(orc32)
    worst = (0.0, 0.0)
    for p in range(n):
        src, state, noise = _predict_inputs(d, p, S)
        got = fp(src.to(DEV), state.to(DEV), noise.to(DEV)).clone()
        torch.cuda.synchronize()
        fp.check_device_errors()
        kv, md = (fp.k, fp.v), (fp.mods[1:], fp.dt.item())
        ref = po.predict(src, state, noise[0], kv=kv, mods_dt=md)
        po32.predict(src, state, noise[0], kv=kv, mods_dt=md)
        mx, mean = chunk_err(got[0], ref, 7)
        worst = (max(worst[0], mx), max(worst[1], mean))
        assert torch.isfinite(got).all()
        assert mx <= TOL_MAX and mean <= TOL_MEAN, (name, p, mx, mean)
    for got, ref, r32, what in ((fp.memk.cpu(), po.memk, po32.memk, "K"), (fp.memv.cpu(), po.memv, po32.memv, "V")):
        mx, mean, noise = assert_within_noise(got, ref, r32, (name, what))
    print(f"{name}: {n} predicts, worst chunk max {worst[0]:.3e} mean {worst[1]:.3e}; memory V max {mx:.3e} "
          f"mean {mean:.3e} (bf16-fp32 oracle mean {noise:.3e})")


def test_full_predict_with_the_oracle_producers(parts):
    """Predicts 0-2 against the restatement with its own producers (prepare and modulation oracles),
    nothing taken from the device."""
    from oracle.register_oracle import PredictOracle
    name, d, w, bx, orc, orc32 = parts
    if name != "full":
        pytest.skip("full expert only")
    S = 160
    fp, keep = _predictors(d, w, bx, S)
    po = PredictOracle(orc, make_prepare_weights(d, seed=0), make_modulation_weights(d, seed=0),
                       make_register_rows(d, 32), N=10, PM=96, R=32, T=10, action_dim=7)
    for p in range(3):
        src, state, noise = _predict_inputs(d, p, S)
        got = fp(src.to(DEV), state.to(DEV), noise.to(DEV)).clone()
        torch.cuda.synchronize()
        ref = po.predict(src, state, noise[0])
        mx, mean = chunk_err(got[0], ref, 7)
        print(f"predict {p}: max {mx:.3e} mean {mean:.3e}")
        assert mx <= TOL_MAX and mean <= TOL_MEAN, (p, mx, mean)


def test_graph_replays_equal_eager_predicts(parts):
    """The captured predict and the same parts called eagerly give bit-identical chunks and memory
    over successive predicts (every kernel is deterministic); reset() starts the memory over."""
    name, d, w, bx, orc, orc32 = parts
    if name != "small":
        pytest.skip("small expert only")
    S = 64
    fg, keep1 = _predictors(d, w, bx, S, graph=True)
    fe, keep2 = _predictors(d, w, bx, S, graph=False)
    for p in range(4):
        src, state, noise = (t.to(DEV) for t in _predict_inputs(d, p, S))
        a = fg(src, state, noise).clone()
        b = fe(src, state, noise).clone()
        torch.cuda.synchronize()
        assert torch.equal(a, b), p
        assert torch.equal(fg.memk, fe.memk) and torch.equal(fg.memv, fe.memv), p
    first = fg(*(t.to(DEV) for t in _predict_inputs(d, 0, S))).clone()
    fg.reset()
    again = fg(*(t.to(DEV) for t in _predict_inputs(d, 0, S))).clone()
    fe.reset()
    ref0 = fe(*(t.to(DEV) for t in _predict_inputs(d, 0, S))).clone()
    torch.cuda.synchronize()
    assert torch.equal(again, ref0)
    assert not torch.equal(first, again)  # the 5th predict saw three frames of memory


@pytest.mark.parametrize("S,T,frames", [(1, 10, 3), (300, 16, 2), (64, 1, 1)])
def test_carried_predict_shapes(parts, S, T, frames):
    """Source lengths 1 and 300, 16 and 1 action rows, 2 frames and a single frame (kv_start 0 from
    the first predict, nothing carried): 5 predicts each against the restatement."""
    from oracle.register_oracle import PredictOracle
    name, d, w, bx, orc, orc32 = parts
    if name != "small":
        pytest.skip("small expert only")
    fp, keep = _predictors(d, w, bx, S, T=T, frames=frames)
    po = PredictOracle(orc, make_prepare_weights(d, seed=0), make_modulation_weights(d, seed=0),
                       make_register_rows(d, 32), N=10, PM=32 * frames, R=32, T=T, action_dim=7)
    for p in range(5):
        src, state, noise = _predict_inputs(d, p, S, T=T)
        got = fp(src.to(DEV), state.to(DEV), noise.to(DEV)).clone()
        torch.cuda.synchronize()
        fp.check_device_errors()
        ref = po.predict(src, state, noise[0], kv=(fp.k, fp.v), mods_dt=(fp.mods[1:], fp.dt.item()))
        mx, mean = chunk_err(got[0], ref, 7)
        assert torch.isfinite(got).all()
        assert mx <= TOL_MAX and mean <= TOL_MEAN, (S, T, frames, p, mx, mean)

