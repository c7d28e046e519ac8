"""Loads the golden fixtures of tests/golden (reference outputs on fixed inputs)."""
from __future__ import annotations

import glob
import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# The reference's own op-test tolerance (tests/python/test_*.py: ATOL, RTOL = 1e-3, 1e-2),
# stated for fp16. bf16 keeps 8 significant bits instead of fp16's 11, so one rounding of
# a value near 1 (P before P@V, the output itself) is 2^-8 instead of 2^-11: for bf16 the
# absolute tolerance is scaled by that factor of 8 (rounded up to 1e-2).
ATOL, RTOL = 1e-3, 1e-2
BF16_ATOL, BF16_RTOL = 1e-2, 1e-2


def tol(dtype) -> dict:
    """allclose tolerance for an I/O dtype ("fp16"/"bf16" or a torch dtype)."""
    if dtype in ("bf16", torch.bfloat16):
        return dict(atol=BF16_ATOL, rtol=BF16_RTOL)
    return dict(atol=ATOL, rtol=RTOL)


def assert_doubled_exactly(a: torch.Tensor, b: torch.Tensor):
    """b == 2*a exactly wherever a is a normal number of its dtype.

    Doubling commutes with round-to-nearest except in the subnormal range (below 2^-14 in
    fp16), where the rounding grid does not scale; there b may differ by one subnormal step.
    """
    a2 = a.float() * 2
    bf = b.float()
    tiny = torch.finfo(a.dtype).tiny
    normal = a.float().abs() >= tiny  # a itself was rounded on the normal grid
    bad = (a2 != bf) & normal
    assert int(bad.sum()) == 0, f"{int(bad.sum())} normal values not doubled exactly"
    # Where a is subnormal, a and b were rounded on different grids: one fp16 subnormal step
    # (doubled) bounds the difference.
    sub_step = 2 * tiny * torch.finfo(a.dtype).eps
    assert float((a2 - bf)[~normal].abs().max().item() if (~normal).any() else 0.0) <= sub_step

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
