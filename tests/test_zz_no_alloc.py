"""The allocation-free entry point ``mkx_run_static`` against the regular one (``mkx_run``).

``mkx_run_static`` serves callers that cannot allocate device memory themselves (a runtime that hands
out every buffer from an arena reserved at start-up, or a control loop that must not call cudaMalloc
once it runs). It launches the same kernel with its scratch in a static device array, on weights the
caller packed (here with ``reki_megakernel_b200.packing``) and buffers the caller owns.

The test makes two calls in a row through the C ABI, on two different sets of inputs, before any
``ExpertMegakernel`` handle exists in the process (so the first call does the per-device set-up
itself when this file runs alone), then checks each output against ``mkx_run`` on the same inputs.
Same kernel, same packing (the grid is the device's SM count for both), same inputs: the outputs
must be bit-identical. The second call's different inputs make a word left behind by the first
call show up as a mismatch. Collected last on purpose (file name).
"""
import ctypes as C

import pytest
import torch

from reki_megakernel_b200 import _lib
from reki_megakernel_b200.packing import pack_weights
from reki_megakernel_b200.synthetic import ExpertDims, make_inputs, make_past, make_weights

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _step_inputs(inp, past, out):
    """The mkx_step_inputs struct for episode 0 of ``inp`` (all tensors on the device)."""
    st = past.register_step
    si = _lib.StepInputs()
    si.x_in, si.x_out = inp.x[0].data_ptr(), out.data_ptr()
    si.mods, si.mods_fp32, si.dt = inp.mods[0].data_ptr(), 0, inp.dt[:1].data_ptr()
    L = inp.memk.shape[1]
    for l in range(L):
        si.memk[l], si.memv[l] = st["mem_kv"][l][0].data_ptr(), st["mem_kv"][l][1].data_ptr()
        si.kca[l], si.vca[l] = past.cross_attn_kv[l][0].data_ptr(), past.cross_attn_kv[l][1].data_ptr()
    si.mem_rows, si.mem_row_stride = inp.memk.shape[2], st["mem_kv"][0][0].stride(0)
    si.ca_rows, si.ca_row_stride = inp.kca.shape[2], past.cross_attn_kv[0][0].stride(0)
    si.cu_kv, si.cu_src = st["cu_kv"].data_ptr(), st["cu_src"].data_ptr()
    si.sa_cos, si.sa_sin = st["sa_pe"][0].data_ptr(), st["sa_pe"][1].data_ptr()
    si.ca_cos, si.ca_sin = st["ca_pe"][0].data_ptr(), st["ca_pe"][1].data_ptr()
    si.T, si.n_steps, si.action_dim = inp.x.shape[1], inp.n_steps, inp.action_dim
    return si


def test_static_scratch_entry_matches_mkx_run_twice():
    dims = ExpertDims()
    w = make_weights(dims, seed=0)
    grid = torch.cuda.get_device_properties(0).multi_processor_count
    packed = pack_weights(w, grid)                      # the caller's own, already packed weights
    bufs = [t.to(DEV) for t in packed["w"]]
    nrm, tailw, wout = packed["nrm"].to(DEV), packed["tailw"].to(DEV), packed["wout"].to(DEV)
    pw = _lib.PackedWeights()
    for i, t in enumerate(bufs):
        pw.w[i] = t.data_ptr()
    pw.nrm, pw.tailw, pw.wout = nrm.data_ptr(), tailw.data_ptr(), wout.data_ptr()
    d = _lib.Dims(L=dims.L, H=dims.H, NH=dims.NH, HD=dims.HD, I=dims.I, A=dims.A, eps=w.eps, qk_eps=w.qk_eps,
                  max_rows=16, grid=grid)
    lib = _lib.load()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    err = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    calls = [make_inputs(dims, poison=True, seed=2, noise_seed=1234).to(DEV),
             make_inputs(dims, poison=True, seed=3, noise_seed=1300, T=9, action_dim=6).to(DEV)]
    outs = []
    for inp in calls:                                   # two static calls first: no handle exists yet
        past = make_past(inp)
        out = torch.full((inp.x.shape[1], dims.A), float("nan"), device=DEV)
        si = _step_inputs(inp, past, out)
        _lib.check(lib.mkx_run_static(C.byref(d), C.byref(pw), C.byref(si), C.c_void_p(err.data_ptr()), stream),
                   "mkx_run_static")
        torch.cuda.synchronize()
        assert int(err.item()) == 0, hex(int(err.item()))
        outs.append(out)

    from reki_megakernel_b200.mk_expert import ExpertMegakernel
    mk = ExpertMegakernel(weights=w.to(DEV), grid=grid)  # the regular entry point, handle scratch
    for call, (inp, out) in enumerate(zip(calls, outs)):
        ref = mk.run(inp.x[:1], inp.mods[0], inp.dt[:1], make_past(inp), inp.action_dim)[0]
        torch.cuda.synchronize()
        mk.check_device_error()
        assert torch.equal(out, ref), (call, float((out - ref).abs().max()))
    assert not torch.equal(outs[0][:9], outs[1])
    mk.close()


def test_static_scratch_entry_rejects_oversized_mlp():
    d = _lib.Dims(L=2, H=768, NH=12, HD=64, I=4096, A=32, eps=1e-6, qk_eps=1e-6, max_rows=16, grid=0)
    pw, si = _lib.PackedWeights(), _lib.StepInputs()
    si.T = 10
    st = _lib.load().mkx_run_static(C.byref(d), C.byref(pw), C.byref(si), None, None)
    assert st == _lib.MKX_ERR_UNSUPPORTED
    assert b"3072" in _lib.load().mkx_last_cuda_error()
