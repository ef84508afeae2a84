"""CPU checks of the register-pass / carry restatement (``oracle/register_oracle.py``) on a tiny expert:
the plain modulation row, the frame schedule, the roll, and that the pass writes exactly the
current frame's rows, reads nothing below kv_start and carries frames up one slot per predict."""
import torch

from oracle.expert_oracle import OracleExpert
from oracle.register_oracle import PredictOracle, kv_start_of, plain_row, register_pass, roll_frames
from reki_megakernel_b200.synthetic import (ExpertDims, make_modulation_weights, make_prepare_weights, make_register_rows,
                                            make_source, make_state, make_weights, register_rope)

D = ExpertDims(L=2, H=128, NH=2, HD=64, I=256, src_dim=128)


def test_plain_row_has_unit_gates_and_no_scale_or_shift():
    m = plain_row(D).reshape(-1)
    H = D.H
    assert m.numel() == D.MODW
    for l in range(D.L):
        for blk in range(3):
            o = 9 * H * l + 3 * H * blk
            assert (m[o:o + 2 * H] == 0).all() and (m[o + 2 * H:o + 3 * H] == 1).all()
    assert (m[9 * H * D.L:] == 0).all()


def test_frame_schedule():
    assert [kv_start_of(p, 96, 32) for p in range(5)] == [64, 32, 0, 0, 0]
    assert [kv_start_of(p, 64, 16) for p in range(6)] == [48, 32, 16, 0, 0, 0]


def test_roll_moves_every_frame_up_one_slot():
    k = torch.arange(2 * 6 * 2 * 3, dtype=torch.float32).reshape(2, 6, 2, 3)
    v = -k.clone()
    k0, v0 = k.clone(), v.clone()
    roll_frames(k, v, 2)
    assert torch.equal(k[:, :4], k0[:, 2:]) and torch.equal(v[:, :4], v0[:, 2:])
    assert torch.equal(k[:, 4:], k0[:, 4:])  # the newest slot is rewritten by the pass


def test_register_pass_writes_the_frame_and_reads_no_row_below_kv_start():
    w = make_weights(D, seed=0)
    orc = OracleExpert(w, "bf16")
    PM, R = 96, 32
    g = torch.Generator().manual_seed(3)
    memk = torch.randn((D.L, PM, D.NH, D.HD), generator=g).to(torch.bfloat16)
    memv = torch.randn((D.L, PM, D.NH, D.HD), generator=g).to(torch.bfloat16)
    memk[:, :32] = float("nan")
    memv[:, :32] = float("nan")
    memk[:, 64:] = float("nan")
    memv[:, 64:] = float("nan")
    k0, v0 = memk.clone(), memv.clone()
    kca = torch.randn((D.L, 40, D.NH, D.HD), generator=g).to(torch.bfloat16)
    vca = torch.randn((D.L, 40, D.NH, D.HD), generator=g).to(torch.bfloat16)
    kca[:, 33:] = float("nan")
    vca[:, 33:] = float("nan")
    reg = make_register_rows(D, R)
    rope = register_rope(D, PM, R)
    h = register_pass(orc, reg, memk, memv, 32, kca, vca, 33, rope[:2], rope[2:])
    assert torch.isfinite(h).all()
    assert torch.isfinite(memk[:, 64:].float()).all() and torch.isfinite(memv[:, 64:].float()).all()
    u = lambda t: t.view(torch.int16)  # noqa: E731
    assert torch.equal(u(memk[:, :64]), u(k0[:, :64])) and torch.equal(u(memv[:, :64]), u(v0[:, :64]))
    # layer 0's V is the V third of QKV of the plain-normed register rows
    a = orc._adarms(reg.float(), torch.zeros(D.H), torch.zeros(D.H))
    v_ref = orc._linear(a, orc.wqkv[0])[:, 2 * D.H:].reshape(R, D.NH, D.HD)
    assert torch.equal(memv[0, 64:].float(), v_ref)


def test_predicts_carry_frames_up():
    w = make_weights(D, seed=0)
    po = PredictOracle(OracleExpert(w, "bf16"), make_prepare_weights(D), make_modulation_weights(D),
                       make_register_rows(D, 32), N=3, PM=96, R=32, T=4, action_dim=7)
    frames = []
    for p in range(3):
        src = make_source(20, D.src_dim, seed=p)
        x = po.predict(src, make_state(7, seed=p), torch.randn((4, D.A), generator=torch.Generator().manual_seed(p)))
        assert torch.isfinite(x).all()
        frames.append(po.memk[:, 64:].clone())
    assert torch.equal(po.memk[:, 32:64], frames[1]) and torch.equal(po.memk[:, :32], frames[0])
    assert not torch.equal(frames[1], frames[2])
