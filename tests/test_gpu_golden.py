"""CUDA kernels vs the reference's own outputs (golden fixtures), at the reference's
tolerance (atol 1e-3, rtol 1e-2; tests/python/test_*.py)."""
import pytest
import torch

import tritonllmcompiler_b200 as T
from tests import _golden as G

pytestmark = pytest.mark.gpu


def _close(out: torch.Tensor, ref: torch.Tensor):
    t = G.tol(ref.dtype)
    out = out.float().cpu()
    ref = ref.float()
    err = (out - ref).abs().max().item() if out.numel() else 0.0
    assert torch.allclose(out, ref, equal_nan=True, **t), f"max abs err {err}"


@pytest.mark.parametrize("name", G.names("flash"))
def test_flash_golden(cuda_device, name):
    c = G.load(name)
    out = T.flash_attention(c["q"].cuda(), c["k"].cuda(), c["v"].cuda(), causal=bool(c["causal"]),
                            sm_scale=float(c["sm_scale"]))
    _close(out, c["out"])


@pytest.mark.parametrize("name", G.names("paged"))
def test_paged_golden(cuda_device, name):
    c = G.load(name)
    out = T.paged_attention(c["q"].cuda(), c["k_cache"].cuda(), c["v_cache"].cuda(),
                            c["block_tables"].cuda(), c["context_lens"].cuda(),
                            block_size=int(c["block_size"]), sm_scale=float(c["sm_scale"]))
    _close(out, c["out"])


@pytest.mark.parametrize("name", G.names("rmsnorm_rope"))
def test_rmsnorm_rope_golden(cuda_device, name):
    c = G.load(name)
    out = T.rmsnorm_rope(c["x"].cuda(), c["w"].cuda(), c["cos"].cuda(), c["sin"].cuda(), float(c["eps"]))
    _close(out, c["out"])


@pytest.mark.parametrize("name", G.names("swiglu"))
def test_swiglu_golden(cuda_device, name):
    c = G.load(name)
    out = T.swiglu(c["x"].cuda(), c["w1"].cuda(), c["w3"].cuda())
    _close(out, c["out"])


def test_no_device_errors_recorded(cuda_device):
    from tritonllmcompiler_b200 import _lib

    torch.cuda.synchronize()
    assert _lib.debug_status() == 0
