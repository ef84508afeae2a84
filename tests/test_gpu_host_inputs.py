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


def test_run_from_host_copies_only_the_rows_read(full):
    """One set of pinned host buffers refilled in place between calls (a control loop), with
    kv_start and S changing from call to call and NaN in every row the kernel must not read: each
    result equals ``run`` on the same inputs on the device, and the call copies exactly the memory
    rows [kv_start, PM) and the source rows [0, S) of every layer besides the small inputs."""
    dims, mk = full
    cases = [make_inputs(dims, S=S, SP=192, frames_valid=fv, seed=30 + i, noise_seed=300 + i, poison=True)
             for i, (S, fv) in enumerate([(160, 1), (64, 3), (100, 2), (160, 3)])]
    wants = []
    for inp in cases:
        d = inp.to(DEV)
        wants.append(mk.run(d.x[:1], d.mods[0], d.dt[:1], make_past(d), d.action_dim).clone())
    torch.cuda.synchronize()
    pin = lambda t: t.contiguous().pin_memory()  # noqa: E731
    x, mods, dt = pin(cases[0].x[:1]), pin(cases[0].mods[0]), pin(cases[0].dt[:1])
    hp = _pinned_past(cases[0])
    row_bytes = dims.NH * dims.HD * 2
    for inp, want in zip(cases, wants):
        src = make_past(inp)
        x.copy_(inp.x[:1])
        mods.copy_(inp.mods[0])
        dt.copy_(inp.dt[:1])
        for (hk, hv), (k, v) in zip(hp.register_step["mem_kv"], src.register_step["mem_kv"]):
            hk.copy_(k)
            hv.copy_(v)
        for (hk, hv), (k, v) in zip(hp.cross_attn_kv, src.cross_attn_kv):
            hk.copy_(k)
            hv.copy_(v)
        for key in ("cu_kv", "cu_src"):
            hp.register_step[key].copy_(src.register_step[key])
        for key in ("sa_pe", "ca_pe"):
            for t, s in zip(hp.register_step[key], src.register_step[key]):
                t.copy_(s)
        got = mk.run_from_host(x, mods, dt, hp, inp.action_dim)
        torch.cuda.synchronize()
        mk.check_device_error()
        assert torch.equal(got, want)
        st = hp.register_step
        small = sum(t.numel() * t.element_size() for t in (x, mods, dt, st["cu_kv"], st["cu_src"], *st["sa_pe"], *st["ca_pe"]))
        PM, kv0, S = st["mem_kv"][0][0].shape[0], int(st["cu_kv"][0]), int(st["cu_src"][1])
        assert mk.last_h2d_bytes == small + dims.L * 2 * row_bytes * ((PM - kv0) + S) + 4 * dims.L


def test_run_from_host_refuses_out_of_range_row_limits(full):
    """kv_start and S are on the host here: a kv_start outside [0, PM] (the kernel would read outside
    the memory) or S < 1 is refused before anything is copied or launched."""
    dims, mk = full
    inp = make_inputs(dims, seed=40)
    args = (inp.x[:1].contiguous().pin_memory(), inp.mods[0].contiguous().pin_memory(),
            inp.dt[:1].contiguous().pin_memory())
    for kv0, S in ((-1, 160), (97, 160), (32, 0)):
        hp = _pinned_past(inp)
        hp.register_step["cu_kv"][0] = kv0
        hp.register_step["cu_src"][1] = S
        with pytest.raises(ValueError):
            mk.run_from_host(*args, hp, inp.action_dim)
    hp = _pinned_past(inp)
    hp.register_step["cu_src"] = hp.register_step["cu_src"][:1].clone().pin_memory()
    with pytest.raises(ValueError):
        mk.run_from_host(*args, hp, inp.action_dim)
    good = mk.run_from_host(*args, _pinned_past(inp), inp.action_dim)  # the handle still works
    torch.cuda.synchronize()
    mk.check_device_error()
    d = inp.to(DEV)
    assert torch.equal(good, mk.run(d.x[:1], d.mods[0], d.dt[:1], make_past(d), d.action_dim))
