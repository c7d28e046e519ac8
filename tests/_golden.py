"""Loads the golden fixtures of tests/golden (reference outputs on fixed inputs)."""
from __future__ import annotations

import glob
import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# The reference's own op-test tolerance (tests/python/test_*.py: ATOL, RTOL = 1e-3, 1e-2).
ATOL, RTOL = 1e-3, 1e-2

TENSOR_KEYS = {"q", "k", "v", "out", "k_cache", "v_cache", "x", "w", "cos", "sin", "w1", "w3"}


def names(op: str) -> list[str]:
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, op + "__*.npz")))


def load(name: str) -> dict:
    """Returns a dict of torch CPU tensors (fp16/bf16/int32) and python scalars."""
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    dtype = str(z["dtype"])
    out = {"dtype": dtype}
    for key in z.files:
        if key == "dtype":
            continue
        a = z[key]
        if key in TENSOR_KEYS:
            if dtype == "bf16":
                out[key] = torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
            else:
                out[key] = torch.from_numpy(a.copy())
        elif a.dtype == np.int32:
            out[key] = torch.from_numpy(a.copy())
        else:
            out[key] = a.item() if a.shape == () else a
    return out


def to_f32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def torch_dtype(name: str):
    return torch.bfloat16 if name == "bf16" else torch.float16
