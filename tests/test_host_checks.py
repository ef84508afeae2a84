"""Argument checks the Python wrappers make before handing raw device pointers to the C library,
which sees no sizes or devices (CPU only: ``meta`` tensors stand for the device's tensors)."""
import pytest
import torch

from reki_megakernel_b200.modulations import check_out
from reki_megakernel_b200.prepare import check_run_args
from reki_megakernel_b200.synthetic import ExpertDims

META = torch.device("meta")
D = ExpertDims(L=2)


def _t(shape, dtype, device=META):
    return torch.empty(shape, dtype=dtype, device=device)


def test_prepare_accepts_matching_buffers():
    cos, sin = _t((50, D.HD), torch.float32), _t((64, D.HD), torch.float32)
    k, v = _t((D.L, 64, D.NH, D.HD), torch.bfloat16), _t((D.L, 64, D.NH, D.HD), torch.bfloat16)
    check_run_args(D, META, 50, 64, cos, sin, (k, v))
    check_run_args(D, META, 50, 50, cos, sin, None)


@pytest.mark.parametrize("bad", ["sp", "cos_rows", "cos_dtype", "cos_device", "k_shape", "v_dtype", "k_device",
                                 "k_strided", "pair"])
def test_prepare_rejects(bad):
    cos, sin = _t((50, D.HD), torch.float32), _t((50, D.HD), torch.float32)
    k, v = _t((D.L, 64, D.NH, D.HD), torch.bfloat16), _t((D.L, 64, D.NH, D.HD), torch.bfloat16)
    S, SP, out = 50, 64, (k, v)
    if bad == "sp":
        SP = 49
    elif bad == "cos_rows":
        cos = _t((49, D.HD), torch.float32)
    elif bad == "cos_dtype":
        cos = _t((50, D.HD), torch.bfloat16)
    elif bad == "cos_device":
        cos = _t((50, D.HD), torch.float32, "cpu")
    elif bad == "k_shape":
        out = (_t((D.L, 63, D.NH, D.HD), torch.bfloat16), v)
    elif bad == "v_dtype":
        out = (k, _t((D.L, 64, D.NH, D.HD), torch.float32))
    elif bad == "k_device":
        out = (_t((D.L, 64, D.NH, D.HD), torch.bfloat16, "cpu"), v)
    elif bad == "k_strided":
        out = (_t((D.L, D.NH, 64, D.HD), torch.bfloat16).transpose(1, 2), v)
    elif bad == "pair":
        out = (k,)
    with pytest.raises(ValueError):
        check_run_args(D, META, S, SP, cos, sin, out)


def test_modulation_outputs():
    W = D.MODW
    check_out(W, META, 9, None)
    check_out(W, META, 9, (_t((9, W), torch.bfloat16), _t((1,), torch.float32)))
    bad = [(_t((8, W), torch.bfloat16), _t((1,), torch.float32)),
           (_t((9, W), torch.float32), _t((1,), torch.float32)),
           (_t((9, W), torch.bfloat16, "cpu"), _t((1,), torch.float32)),
           (_t((W, 9), torch.bfloat16).t(), _t((1,), torch.float32)),
           (_t((9, W), torch.bfloat16), _t((1,), torch.float64)),
           (_t((9, W), torch.bfloat16), _t((0,), torch.float32)),
           (_t((9, W), torch.bfloat16), _t((1,), torch.float32, "cpu")),
           (_t((9, W), torch.bfloat16),)]
    for out in bad:
        with pytest.raises(ValueError):
            check_out(W, META, 9, out)
