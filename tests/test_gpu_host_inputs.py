"""Inputs streamed from pinned host memory (``ExpertMegakernel.run_from_host``): the per-layer K/V
copies overlap the launch, which waits (bounded) for a per-layer readiness word before reading
them. The result must equal ``run`` on the same inputs already on the device, bit for bit (the same
kernel on the same data), for successive calls; and a readiness word that never arrives must end the
launch with a reported timeout (nothing faults), after which the handle works again."""
import pytest
import torch

from reki_megakernel_b200.synthetic import ExpertDims, make_inputs, make_past, make_weights

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def full():
    from reki_megakernel_b200.mk_expert import ExpertMegakernel
    dims = ExpertDims()
    mk = ExpertMegakernel(weights=make_weights(dims, seed=0).to(DEV))
    yield dims, mk
    mk.close()


def _pinned_past(inp):
    """The ``past`` of episode 0 with every tensor in pinned host memory."""
    past = make_past(inp)
    pin = lambda t: t.contiguous().pin_memory()  # noqa: E731
    st = past.register_step
    st["mem_kv"] = [(pin(k), pin(v)) for k, v in st["mem_kv"]]
    st["sa_pe"] = tuple(pin(t) for t in st["sa_pe"])
    st["ca_pe"] = tuple(pin(t) for t in st["ca_pe"])
    st["cu_kv"], st["cu_src"] = pin(st["cu_kv"]), pin(st["cu_src"])
    past.cross_attn_kv = [(pin(k), pin(v)) for k, v in past.cross_attn_kv]
    return past


@pytest.mark.parametrize("S", [160, 64])
def test_run_from_host_equals_run(full, S):
    dims, mk = full
    outs = []
    for seed in (1, 2):
        inp = make_inputs(dims, S=S, seed=seed, noise_seed=100 + seed)
        d = inp.to(DEV)
        want = mk.run(d.x[:1], d.mods[0], d.dt[:1], make_past(d), d.action_dim).clone()
        hp = _pinned_past(inp)
        got = mk.run_from_host(inp.x[:1].contiguous().pin_memory(), inp.mods[0].contiguous().pin_memory(),
                               inp.dt[:1].contiguous().pin_memory(), hp, inp.action_dim)
        torch.cuda.synchronize()
        mk.check_device_error()
        assert torch.equal(got, want)
        outs.append(got.clone())
    assert not torch.equal(outs[0], outs[1])


def test_missing_readiness_word_times_out_and_recovers(full):
    from reki_megakernel_b200._lib import MkxError
    dims, mk = full
    inp = make_inputs(dims, n_steps=2, seed=7)
    d = inp.to(DEV)
    good = mk.run(d.x[:1], d.mods[0], d.dt[:1], make_past(d), d.action_dim).clone()
    never = torch.zeros(dims.L, dtype=torch.int32, device=DEV)   # nothing ever writes the value 5
    mk.set_timeout(0.05)
    mk.run(d.x[:1], d.mods[0], d.dt[:1], make_past(d), d.action_dim, kv_ready=never, kv_ready_value=5)
    torch.cuda.synchronize()
    code, _ = mk.status()
    assert code != 0 and ((code >> 8) & 0xff) == 1, hex(code)   # kind 1: a wait timed out
    with pytest.raises(MkxError):
        mk.check_device_error()
    mk.set_timeout(2.0)
    mk.clear_error()
    ready = torch.full((dims.L,), 5, dtype=torch.int32, device=DEV)
    again = mk.run(d.x[:1], d.mods[0], d.dt[:1], make_past(d), d.action_dim, kv_ready=ready, kv_ready_value=5)
    torch.cuda.synchronize()
    mk.check_device_error()
    assert torch.equal(again, good)


def test_run_from_host_on_alternating_streams(full):
    """Successive calls from two different current streams: each call's input copies must wait for
    the previous launch, which ran on the other stream and reads the same device buffers."""
    dims, mk = full
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    cases = [make_inputs(dims, S=160, seed=20 + i, noise_seed=200 + i) for i in range(4)]
    wants = []
    for inp in cases:
        d = inp.to(DEV)
        wants.append(mk.run(d.x[:1], d.mods[0], d.dt[:1], make_past(d), d.action_dim).clone())
    torch.cuda.synchronize()
    hosts = [(inp.x[:1].contiguous().pin_memory(), inp.mods[0].contiguous().pin_memory(),
              inp.dt[:1].contiguous().pin_memory(), _pinned_past(inp), inp.action_dim) for inp in cases]
    gots = []
    for i, h in enumerate(hosts):
        with torch.cuda.stream(streams[i % 2]):
            gots.append(mk.run_from_host(*h))
    torch.cuda.synchronize()
    mk.check_device_error()
    for got, want in zip(gots, wants):
        assert torch.equal(got, want)
