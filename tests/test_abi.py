"""The C ABI without a GPU: the library loads, exports every entry point ``include/mkx.h``
declares, its structs have the same layout in C and in the ctypes binding, and argument checks
that need no device reject bad calls."""
import ctypes as C
import re
import shutil
import subprocess
import sys

import pytest

from conftest import ROOT

HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_symbols():
    syms = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        syms |= set(re.findall(r"\b(mkx_[a-z0-9_]+)\s*\(", text))
    return sorted(syms)


def test_library_exports_every_declared_symbol():
    from reki_megakernel_b200 import _lib
    lib = _lib.load()
    syms = declared_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib.SIGNATURES), set(syms) ^ set(_lib.SIGNATURES)
    nm = shutil.which("nm")
    if nm:
        out = subprocess.run([nm, "-D", "--defined-only", str(_lib.lib_path())], capture_output=True, text=True).stdout
        exported = set(re.findall(r"\b(mkx_[a-z0-9_]+)\b", out))
        assert set(syms) <= exported


def _c_layout(struct: str, fields):
    gcc = shutil.which("gcc")
    if not gcc:
        pytest.skip("gcc missing")
    body = "".join(f'printf("{f} %zu\\n", offsetof({struct}, {f}));' for f in fields)
    src = f'#include <stdio.h>\n#include <stddef.h>\n#include "mkx.h"\n#include "mkx_prepare.h"\n#include "mkx_batch.h"\nint main(void){{{body} printf("sizeof %zu\\n", sizeof({struct})); return 0;}}\n'
    import tempfile
    from pathlib import Path
    with tempfile.TemporaryDirectory() as d:
        c = Path(d) / "l.c"
        c.write_text(src)
        exe = Path(d) / "l"
        r = subprocess.run([gcc, "-I", str(ROOT / "include"), "-I", "/usr/local/cuda/include", str(c), "-o", str(exe)],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        out = subprocess.run([str(exe)], capture_output=True, text=True).stdout
    return {k: int(v) for k, v in (line.split() for line in out.splitlines())}


@pytest.mark.parametrize("struct,cls", [("mkx_dims", "Dims"), ("mkx_weights", "Weights"), ("mkx_step_inputs", "StepInputs"),
                                        ("mkx_packed_weights", "PackedWeights"), ("mkx_prep_dims", "PrepDims"),
                                        ("mkx_batch_inputs", "BatchInputs"),
                                        ("mkx_register_inputs", "RegisterInputs")])
def test_struct_layout_matches_c(struct, cls):
    from reki_megakernel_b200 import _lib
    ct = getattr(_lib, cls)
    fields = [f[0] for f in ct._fields_]
    c = _c_layout(struct, fields)
    for f in fields:
        assert getattr(ct, f).offset == c[f], (struct, f, getattr(ct, f).offset, c[f])
    assert C.sizeof(ct) == c["sizeof"]


def test_null_arguments_are_rejected_without_a_device():
    from reki_megakernel_b200 import _lib
    lib = _lib.load()
    h = C.c_void_p()
    assert lib.mkx_create(None, None, 0, C.byref(h)) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_run(None, None, None) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_sync_points(None, 9) == -1
    assert lib.mkx_set_timeout_ns(None, 1) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_set_fault_injection(None, 1) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_set_launch_sequence(None, 1) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_clear_error(None) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_last_error(None, None, None) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_launch_shape(None, None, None) == _lib.MKX_ERR_INVALID_ARG
    d = _lib.Dims(L=10, H=1024, NH=16, HD=64, I=3072, A=32, eps=1e-6, qk_eps=1e-6, max_rows=16, grid=0)
    w = _lib.Weights(*([1] * 14))
    assert lib.mkx_create(C.byref(d), C.byref(w), 0, C.byref(h)) == _lib.MKX_ERR_UNSUPPORTED
    lib.mkx_destroy(None)


def test_static_entry_rejects_a_misaligned_error_word_without_a_device():
    """mkx_run_static copies the launch's 4-byte error word to err_out on the stream; a misaligned
    err_out would only fail later, asynchronously, so the call rejects it up front."""
    from reki_megakernel_b200 import _lib
    lib = _lib.load()
    d = _lib.Dims(L=10, H=768, NH=12, HD=64, I=3072, A=32, eps=1e-6, qk_eps=1e-6, max_rows=16, grid=0)
    pw, si = _lib.PackedWeights(), _lib.StepInputs()
    si.T = 10
    assert lib.mkx_run_static(C.byref(d), C.byref(pw), C.byref(si), C.c_void_p(0x1002), None) == _lib.MKX_ERR_INVALID_ARG
    assert b"aligned" in lib.mkx_last_cuda_error()


def test_batch_arguments_are_rejected_without_a_device():
    from reki_megakernel_b200 import _lib
    lib = _lib.load()
    h = C.c_void_p()
    assert lib.mkx_batch_create(None, None, 8, 0, C.byref(h)) == _lib.MKX_ERR_INVALID_ARG
    d = _lib.Dims(L=10, H=768, NH=12, HD=64, I=3072, A=32, eps=1e-6, qk_eps=1e-6, max_rows=16, grid=0)
    w = _lib.Weights(*([1] * 14))
    assert lib.mkx_batch_create(C.byref(d), C.byref(w), 0, 0, C.byref(h)) == _lib.MKX_ERR_INVALID_ARG  # no episodes
    d.I = 1000                                                                     # not a multiple of 128
    assert lib.mkx_batch_create(C.byref(d), C.byref(w), 8, 0, C.byref(h)) == _lib.MKX_ERR_UNSUPPORTED
    assert lib.mkx_batch_run(None, None, None) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_batch_launches(None, 8, 10, 9) == -1
    assert lib.mkx_batch_last_error(None, None) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_batch_copy_state(None, 0, None, 0) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_batch_register_pass(None, None, None) == _lib.MKX_ERR_INVALID_ARG
    lib.mkx_batch_destroy(None)


def test_prepare_arguments_are_rejected_without_a_device():
    from reki_megakernel_b200 import _lib
    lib = _lib.load()
    h = C.c_void_p()
    assert lib.mkx_prep_create(None, None, None, 0, C.byref(h)) == _lib.MKX_ERR_INVALID_ARG
    d = _lib.PrepDims(L=10, H=1024, NH=16, HD=64, src_dim=2048, eps=1e-6)
    assert lib.mkx_prep_create(C.byref(d), 16, 16, 0, C.byref(h)) == _lib.MKX_ERR_UNSUPPORTED
    d = _lib.PrepDims(L=10, H=768, NH=12, HD=64, src_dim=2000, eps=1e-6)   # not a multiple of 64
    assert lib.mkx_prep_create(C.byref(d), 16, 16, 0, C.byref(h)) == _lib.MKX_ERR_UNSUPPORTED
    assert lib.mkx_prep_run(None, None, 0, None, None, None, None, 0, None) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_prep_last_error(None, None) == _lib.MKX_ERR_INVALID_ARG
    lib.mkx_prep_destroy(None)


def test_modulation_arguments_are_rejected_without_a_device():
    from reki_megakernel_b200 import _lib
    lib = _lib.load()
    h = C.c_void_p()
    assert lib.mkx_mods_create(None, None, None, None, None, 0, C.byref(h)) == _lib.MKX_ERR_INVALID_ARG
    for d in (_lib.ModsDims(H=1024, L=10, tdim=256, sdim=7),    # width the kernels are not built for
              _lib.ModsDims(H=768, L=10, tdim=100, sdim=7),     # embedding width not a multiple of 64
              _lib.ModsDims(H=768, L=10, tdim=256, sdim=65),    # state wider than 64
              _lib.ModsDims(H=768, L=0, tdim=256, sdim=7)):
        assert lib.mkx_mods_create(C.byref(d), 16, 16, 16, 16, 0, C.byref(h)) == _lib.MKX_ERR_UNSUPPORTED
    assert lib.mkx_mods_run(None, 10, None, None, None, None) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_mods_width(None) == 0
    assert lib.mkx_mods_input(None, None, None) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_mods_last_error(None, None) == _lib.MKX_ERR_INVALID_ARG
    lib.mkx_mods_destroy(None)


def test_host_copy_arguments_are_checked_without_a_device():
    from reki_megakernel_b200 import _lib
    lib = _lib.load()
    assert lib.mkx_h2d_copies(-1, None, None, None, None) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_h2d_copies(2, None, None, None, None) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_h2d_copies(0, None, None, None, None) == _lib.MKX_OK   # nothing to copy
    assert lib.mkx_h2d_copies_2d(-1, None, None, None, None, None, None, None) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_h2d_copies_2d(1, None, None, None, None, None, None, None) == _lib.MKX_ERR_INVALID_ARG
    assert lib.mkx_h2d_copies_2d(0, None, None, None, None, None, None, None) == _lib.MKX_OK
    one = lambda t, v: (t * 1)(v)  # noqa: E731
    bad = [  # (dst, dpitch, src, spitch, width, height): a null pointer, width past a pitch, no rows
        (0, 64, 0x1000, 64, 64, 1), (0x1000, 32, 0x2000, 64, 64, 1), (0x1000, 64, 0x2000, 32, 64, 1),
        (0x1000, 64, 0x2000, 64, 64, 0)]
    for d, dp, s_, sp, w, h in bad:  # rejected before any copy is enqueued
        assert lib.mkx_h2d_copies_2d(1, one(C.c_void_p, d), one(C.c_size_t, dp), one(C.c_void_p, s_), one(C.c_size_t, sp),
                                     one(C.c_size_t, w), one(C.c_size_t, h), None) == _lib.MKX_ERR_INVALID_ARG


def test_readiness_values_never_repeat_consecutively():
    """``run_from_host`` tells its launch which readiness-word value marks this call's K/V: it must
    differ from the zero the words start at and from the previous call's value, across the wrap."""
    from reki_megakernel_b200.mk_expert import READY_PERIOD, ready_value
    seqs = [1, 2, 3, READY_PERIOD - 1, READY_PERIOD, READY_PERIOD + 1, READY_PERIOD + 2, 2 * READY_PERIOD + 1]
    vals = [ready_value(s) for s in seqs]
    assert vals[:3] == [1, 2, 3] and vals[4:7] == [READY_PERIOD, 1, 2]
    assert all(1 <= v <= READY_PERIOD < 2 ** 31 for v in vals)
    for s in [1, READY_PERIOD - 1, READY_PERIOD, READY_PERIOD + 1, 5 * READY_PERIOD]:
        assert ready_value(s + 1) != ready_value(s)


def test_traced_profiling_build_loads_on_request():
    """``_lib.use_traced_build()`` before the first load selects the profiling variant of the library
    (``libmkx_trace.so``), which exports the same entry points; after a load it refuses."""
    from reki_megakernel_b200 import _lib
    from reki_megakernel_b200 import build as B
    if B.stale(B.TRACE_LIB):
        try:
            B.nvcc()
        except RuntimeError:
            pytest.skip("no traced build and no nvcc")
    code = "from reki_megakernel_b200 import _lib; _lib.use_traced_build(); _lib.load(); print(_lib.lib_path().name)"
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=ROOT, timeout=600)
    assert r.returncode == 0, r.stderr
    assert r.stdout.split()[0] == "libmkx_trace.so"
    nm = shutil.which("nm")
    if nm:
        out = subprocess.run([nm, "-D", "--defined-only", str(B.TRACE_LIB)], capture_output=True, text=True).stdout
        assert set(declared_symbols()) <= set(re.findall(r"\b(mkx_[a-z0-9_]+)\b", out))
    _lib.load()
    with pytest.raises(RuntimeError):
        _lib.use_traced_build()
