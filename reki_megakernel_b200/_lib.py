"""ctypes binding of ``libmkx.so`` (declarations in ``include/mkx.h``, ``include/mkx_prepare.h``,
``include/mkx_mods.h`` and ``include/mkx_batch.h``).

The library is built in-tree by ``reki_megakernel_b200.build``. There is no fallback: if the
library is missing or does not load, importing this module raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

from . import build as _build

MAX_LAYERS = 16

MKX_OK, MKX_ERR_INVALID_ARG, MKX_ERR_UNSUPPORTED, MKX_ERR_CUDA, MKX_ERR_DEVICE, MKX_ERR_RESOURCES = range(6)
STATUS_NAMES = {0: "OK", 1: "INVALID_ARG", 2: "UNSUPPORTED", 3: "CUDA", 4: "DEVICE", 5: "RESOURCES"}

# Exported entry points and their ctypes signatures (restype, argtypes).
P = C.c_void_p


class Dims(C.Structure):
    _fields_ = [("L", C.c_int), ("H", C.c_int), ("NH", C.c_int), ("HD", C.c_int), ("I", C.c_int),
                ("A", C.c_int), ("eps", C.c_float), ("qk_eps", C.c_float), ("max_rows", C.c_int),
                ("grid", C.c_int)]


class Weights(C.Structure):
    _fields_ = [(n, P) for n in ("wqkv", "wo", "wqca", "woca", "wg", "wu", "wd", "qn", "kn", "qcan",
                                 "win", "bin", "wout", "bout")]


class StepInputs(C.Structure):
    _fields_ = [("x_in", P), ("x_out", P), ("mods", P), ("mods_fp32", C.c_int), ("dt", P),
                ("memk", P * MAX_LAYERS), ("memv", P * MAX_LAYERS), ("mem_rows", C.c_int),
                ("mem_row_stride", C.c_int), ("cu_kv", P),
                ("kca", P * MAX_LAYERS), ("vca", P * MAX_LAYERS), ("ca_rows", C.c_int), ("ca_row_stride", C.c_int),
                ("cu_src", P),
                ("sa_cos", P), ("sa_sin", P), ("ca_cos", P), ("ca_sin", P),
                ("T", C.c_int), ("n_steps", C.c_int), ("action_dim", C.c_int), ("trace_h", P), ("prof", P),
                ("kv_ready", P), ("kv_ready_value", C.c_int)]


class PackedWeights(C.Structure):
    _fields_ = [("w", P * 6), ("nrm", P), ("tailw", P), ("wout", P)]


class BatchInputs(C.Structure):
    _fields_ = [("x_in", P), ("x_out", P), ("mods", P), ("dt", P), ("memk", P), ("memv", P), ("kv_start", P),
                ("mem_rows", C.c_int), ("kca", P), ("vca", P), ("src_rows", P), ("ca_rows", C.c_int),
                ("sa_cos", P), ("sa_sin", P), ("ca_cos", P), ("ca_sin", P), ("B", C.c_int), ("T", C.c_int),
                ("n_steps", C.c_int), ("action_dim", C.c_int)]


class RegisterInputs(C.Structure):
    _fields_ = [("reg_in", P), ("memk", P), ("memv", P), ("kv_start", P), ("mem_rows", C.c_int), ("kca", P),
                ("vca", P), ("src_rows", P), ("ca_rows", C.c_int), ("sa_cos", P), ("sa_sin", P), ("ca_cos", P),
                ("ca_sin", P), ("R", C.c_int)]


class PrepDims(C.Structure):
    _fields_ = [("L", C.c_int), ("H", C.c_int), ("NH", C.c_int), ("HD", C.c_int), ("src_dim", C.c_int),
                ("eps", C.c_float)]


class ModsDims(C.Structure):
    _fields_ = [("H", C.c_int), ("L", C.c_int), ("tdim", C.c_int), ("sdim", C.c_int)]


SIGNATURES = {
    "mkx_create": (C.c_int, [C.POINTER(Dims), C.POINTER(Weights), C.c_int, C.POINTER(P)]),
    "mkx_run": (C.c_int, [P, C.POINTER(StepInputs), P]),
    "mkx_sync_points": (C.c_int, [P, C.c_int]),
    "mkx_last_error": (C.c_int, [P, C.POINTER(C.c_int), C.POINTER(C.c_longlong)]),
    "mkx_clear_error": (C.c_int, [P]),
    "mkx_set_timeout_ns": (C.c_int, [P, C.c_ulonglong]),
    "mkx_set_fault_injection": (C.c_int, [P, C.c_int]),
    "mkx_set_launch_sequence": (C.c_int, [P, C.c_uint]),
    "mkx_launch_shape": (C.c_int, [P, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "mkx_run_static": (C.c_int, [C.POINTER(Dims), C.POINTER(PackedWeights), C.POINTER(StepInputs), P, P]),
    "mkx_last_cuda_error": (C.c_char_p, []),
    "mkx_h2d_copies": (C.c_int, [C.c_int, P, P, P, P]),
    "mkx_h2d_copies_2d": (C.c_int, [C.c_int, P, P, P, P, P, P, P]),
    "mkx_destroy": (None, [P]),
    "mkx_batch_create": (C.c_int, [C.POINTER(Dims), C.POINTER(Weights), C.c_int, C.c_int, C.POINTER(P)]),
    "mkx_batch_run": (C.c_int, [P, C.POINTER(BatchInputs), P]),
    "mkx_batch_register_pass": (C.c_int, [P, C.POINTER(RegisterInputs), P]),
    "mkx_batch_last_error": (C.c_int, [P, C.POINTER(C.c_int)]),
    "mkx_batch_launches": (C.c_int, [P, C.c_int, C.c_int, C.c_int]),
    "mkx_batch_last_cuda_error": (C.c_char_p, []),
    "mkx_batch_copy_state": (C.c_int, [P, C.c_int, P, C.c_size_t]),
    "mkx_batch_destroy": (None, [P]),
    "mkx_prep_create": (C.c_int, [C.POINTER(PrepDims), P, P, C.c_int, C.POINTER(P)]),
    "mkx_prep_run": (C.c_int, [P, P, C.c_int, P, P, P, P, C.c_int, P]),
    "mkx_prep_last_error": (C.c_int, [P, C.POINTER(C.c_int)]),
    "mkx_prep_destroy": (None, [P]),
    "mkx_mods_create": (C.c_int, [C.POINTER(ModsDims), P, P, P, P, C.c_int, C.POINTER(P)]),
    "mkx_mods_run": (C.c_int, [P, C.c_int, P, P, P, P]),
    "mkx_mods_width": (C.c_int, [P]),
    "mkx_mods_input": (C.c_int, [P, P, P]),
    "mkx_mods_last_error": (C.c_int, [P, C.POINTER(C.c_int)]),
    "mkx_mods_destroy": (None, [P]),
}

_LIB = None


_TRACED = False


def lib_path() -> Path:
    return _build.TRACE_LIB if _TRACED else _build.LIB


def use_traced_build() -> None:
    """Make ``load`` use the sub-stage-traced profiling variant (``libmkx_trace.so``) instead of
    ``libmkx.so``. Must be called before the first ``load`` in the process."""
    global _TRACED
    if _LIB is not None:
        raise RuntimeError("the CUDA library is already loaded")
    _TRACED = True


def load(build_if_missing: bool = True) -> C.CDLL:
    """Load (building first if missing or stale and nvcc exists) the CUDA library."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = _build.TRACE_LIB if _TRACED else _build.LIB
    if build_if_missing:
        try:
            if _build.stale(path):
                _build.build(traced=_TRACED)
        except RuntimeError:
            if not path.exists():
                raise
    if not path.exists():
        raise ImportError(f"{path} is missing: run `python -m reki_megakernel_b200.build` (needs nvcc)")
    lib = C.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


class MkxError(RuntimeError):
    def __init__(self, where: str, status: int, detail: str = ""):
        self.status = status
        super().__init__(f"{where} failed: {STATUS_NAMES.get(status, status)}" + (f" ({detail})" if detail else ""))


def check(status: int, where: str) -> None:
    if status != MKX_OK:
        detail = ""
        if status == MKX_ERR_CUDA:
            fn = load().mkx_batch_last_cuda_error if where.startswith("mkx_batch") else load().mkx_last_cuda_error
            detail = (fn() or b"").decode(errors="replace")
        raise MkxError(where, status, detail)
