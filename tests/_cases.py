"""Shared test configurations (mirrors of ``tests/golden/make_golden.py``'s CONFIGS) and helpers."""
import json

import numpy as np
import torch

from reki_megakernel_b200.synthetic import ExpertDims, make_inputs, make_weights

# max / mean |d| on the real action dims of the normalized chunk
TOL_MAX = 1e-2
TOL_MEAN = 1.5e-3


def load_golden(path):
    z = np.load(path)
    cfg = json.loads(str(z["config"]))
    return z, cfg


def golden_case(path):
    """(dims, weights (CPU), inputs (CPU, poisoned), fixture) regenerated from a golden file's seeds."""
    z, cfg = load_golden(path)
    dims = ExpertDims(**cfg["dims"])
    return dims, make_weights(dims, seed=0), make_inputs(dims, poison=True, **cfg["inputs"]), z


def bf16_from_u16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).float()


def chunk_err(a: torch.Tensor, b: torch.Tensor, adim: int):
    d = (a[..., :adim].float().cpu() - b[..., :adim].float().cpu()).abs()
    return float(d.max()), float(d.mean())

from pathlib import Path  # noqa: E402

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"
GOLDEN_FILES = {name: GOLDEN_DIR / f"ref_{name}.npz" for name in ("layer", "small", "full")}
