"""Cross-attention K/V preparation (tcgen05 GEMM + fused head norm / RoPE) against its CPU
restatement (parity unpinned: the reference checkout has no producer of these K/V).

The GPU accumulates the 2048-long dot products on the tensor cores (fp32 accumulator, whose
additions truncate: ~1e-5 relative after 128 K-steps), the oracle in float64; both round once to
bf16. Bar: at least 97 % of the outputs bit-identical, and every output within one bf16 ulp of the
oracle (2^-7 of its magnitude) plus 2^-14 of its head row's RMS (the accumulation error carried
through the head norm and the RoPE cancellation)."""
import pytest
import torch

from oracle.prepare_oracle import prepare_oracle
from reki_megakernel_b200.synthetic import ExpertDims, make_prepare_weights, make_source, rope_cos_sin

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _check(got, ref):
    g, r = got.float().cpu(), ref.float()
    exact = (g == r).float().mean().item()
    rms = r.pow(2).mean(-1, keepdim=True).sqrt()
    tol = r.abs() * 2.0 ** -7 + rms * 2.0 ** -14 + 1e-30
    worst = ((g - r).abs() / tol).max().item()
    assert exact >= 0.97 and worst <= 1.0, (exact, worst)
    return exact


def _run(L, S, SP=None, seed=0):
    from reki_megakernel_b200.prepare import RegisterPrepare
    d = ExpertDims(L=L)
    pw = make_prepare_weights(d, seed=seed)
    src = make_source(S, d.src_dim, seed=seed)
    rp = RegisterPrepare(pw.to(DEV))
    k, v = rp.run(src.to(DEV), SP=SP)
    torch.cuda.synchronize()
    rp.check_device_error()
    c, s = rope_cos_sin(torch.arange(S), d.HD)
    rk, rv = prepare_oracle(pw.wkv, pw.kn, src, c, s, pw.eps)
    return rp, k, v, rk, rv


@pytest.mark.parametrize("L,S", [(1, 1), (2, 7), (2, 16), (2, 100), (10, 160), (2, 256), (2, 300), (2, 1024)])
def test_prepare_matches_oracle(L, S):
    rp, k, v, rk, rv = _run(L, S)
    _check(k[:, :S], rk)
    _check(v[:, :S], rv)
    assert torch.isfinite(k.float()).all() and torch.isfinite(v.float()).all()
    rp.close()


def test_padding_rows_untouched():
    from reki_megakernel_b200.prepare import RegisterPrepare
    d = ExpertDims(L=2)
    pw = make_prepare_weights(d, seed=3)
    src = make_source(50, d.src_dim, seed=3).to(DEV)
    rp = RegisterPrepare(pw.to(DEV))
    k = torch.full((d.L, 64, d.NH, d.HD), 7.0, dtype=torch.bfloat16, device=DEV)
    v = torch.full_like(k, -3.0)
    rp.run(src, SP=64, out=(k, v))
    torch.cuda.synchronize()
    rp.check_device_error()
    assert (k[:, 50:] == 7.0).all() and (v[:, 50:] == -3.0).all()
    assert not (k[:, :50] == 7.0).all()
    rp.close()


def test_unaligned_rope_tables_rejected():
    """The epilogue reads the RoPE tables as 16-byte vectors: a table that does not start on a 16-byte
    boundary is refused before the launch."""
    from reki_megakernel_b200 import _lib
    from reki_megakernel_b200.prepare import RegisterPrepare
    d = ExpertDims(L=1)
    rp = RegisterPrepare(make_prepare_weights(d, seed=0).to(DEV))
    src = make_source(8, d.src_dim, seed=0).to(DEV)
    c, s = (t.to(DEV) for t in rope_cos_sin(torch.arange(9), d.HD))
    cu = c.reshape(-1)[1:1 + 8 * d.HD].view(8, d.HD)  # 4 bytes past a 16-byte boundary
    su = s.reshape(-1)[1:1 + 8 * d.HD].view(8, d.HD)
    with pytest.raises(_lib.MkxError):
        rp.run(src, cu, su)
    with pytest.raises(_lib.MkxError):
        rp.run(src, c[:8], su)
    rp.run(src, c[:8], s[:8])  # aligned: accepted
    torch.cuda.synchronize()
    rp.check_device_error()
    rp.close()


def test_prepare_graph_capture_and_feeds_the_expert():
    """Captured in a CUDA graph; its K/V are the layout ExpertMegakernel reads."""
    from reki_megakernel_b200.prepare import RegisterPrepare
    d = ExpertDims(L=2)
    pw = make_prepare_weights(d, seed=5)
    src = make_source(160, d.src_dim, seed=5).to(DEV)
    rp = RegisterPrepare(pw.to(DEV))
    eager = rp.run(src)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        rp.run(src)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        k, v = rp.run(src)
    g.replay()
    torch.cuda.synchronize()
    rp.check_device_error()
    assert torch.equal(k, eager[0]) and torch.equal(v, eager[1])
    assert k.shape == (d.L, 160, d.NH, d.HD) and k.stride(1) == d.NH * d.HD   # one K row per source row
    rp.close()


def test_register_prepare_callable_builds_the_expert_past():
    """``register_prepare(prepare, src, mem_kv, T=..., kv_start=...)`` returns the ``past`` the expert
    reads: its K/V equal ``RegisterPrepare.run``'s, its tables and cu_seqlens are the ones the
    synthetic inputs use, and the expert run on it equals the run on an equivalent hand-built past."""
    from reki_megakernel_b200.mk_expert import ExpertMegakernel
    from reki_megakernel_b200.prepare import RegisterPrepare, register_prepare
    from reki_megakernel_b200.synthetic import make_inputs, make_past, make_weights
    d = ExpertDims(L=2, I=1024)
    S = 96
    rp = RegisterPrepare(make_prepare_weights(d, seed=0).to(DEV))
    src = make_source(S, d.src_dim, seed=4).to(DEV)
    inp = make_inputs(d, T=10, n_steps=2, S=S, SP=S, seed=4).to(DEV)
    mem = [(inp.memk[0, l], inp.memv[0, l]) for l in range(d.L)]
    past = register_prepare(rp, src, mem, T=10, kv_start=int(inp.kv_start[0]))
    k, v = rp.run(src)
    for l in range(d.L):
        assert torch.equal(past.cross_attn_kv[l][0], k[l]) and torch.equal(past.cross_attn_kv[l][1], v[l])
    inp.kca, inp.vca = k[None], v[None]
    ref_past = make_past(inp)
    for key in ("sa_pe", "ca_pe"):
        for a, b in zip(past.register_step[key], ref_past.register_step[key]):
            assert torch.equal(a, b)
    for key in ("cu_kv", "cu_src"):
        assert torch.equal(past.register_step[key], ref_past.register_step[key])
    mk = ExpertMegakernel(weights=make_weights(d, seed=0).to(DEV))
    a = mk.run(inp.x[:1], inp.mods[0], inp.dt[:1], past, inp.action_dim)
    b = mk.run(inp.x[:1], inp.mods[0], inp.dt[:1], ref_past, inp.action_dim)
    torch.cuda.synchronize()
    mk.check_device_error()
    assert torch.equal(a, b)
    mk.close()
    rp.close()
