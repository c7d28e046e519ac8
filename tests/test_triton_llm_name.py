"""The reference's own import lines resolve to the B200 kernels.

The reference's callers import ``triton_llm`` and ``triton_llm.ops.<op>``
(tests/python/test_*.py:4, python/triton_llm/__init__.py:2-8, ops/__init__.py:2-7). The
``triton_llm`` package of this repository serves those names from ``tritonllmcompiler_b200``
with no ``sys.modules`` patching, and brings in neither an oracle nor the reference's
``triton_llm.reference``.
"""
import importlib
import subprocess
import sys

import pytest
import torch

from tests import _golden as G
from tests.conftest import ROOT

OPS = ["flash_attention", "paged_attention", "rmsnorm_rope", "swiglu"]


def test_import_lines_resolve_to_the_b200_ops():
    import triton_llm
    import triton_llm.ops

    import tritonllmcompiler_b200 as T

    assert triton_llm.__version__ == "0.2.0"
    assert sorted(triton_llm.__all__) == OPS and sorted(triton_llm.ops.__all__) == OPS
    for op in OPS:
        mod = importlib.import_module(f"triton_llm.ops.{op}")
        fn = getattr(mod, op)
        assert fn is getattr(T, op) is getattr(triton_llm, op) is getattr(triton_llm.ops, op)
        assert fn.__module__ == f"tritonllmcompiler_b200.ops.{op}"


def test_import_pulls_in_no_oracle_and_no_reference_oracles():
    code = ("import sys; from triton_llm.ops.swiglu import swiglu; "
            "from triton_llm.ops.flash_attention import flash_attention; "
            "import triton_llm; "
            "bad = [m for m in sys.modules if m == 'oracle' or m.startswith('oracle.') "
            "or m.startswith('triton_llm.reference') or m.startswith('tests')]; "
            "print(triton_llm.__file__); assert not bad, bad")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip().startswith(ROOT)
    with pytest.raises(ModuleNotFoundError):
        importlib.import_module("triton_llm.reference")


def _close(out, ref):
    out, ref = out.float().cpu(), ref.float()
    assert torch.allclose(out, ref, equal_nan=True, **G.tol(ref.dtype)), (out - ref).abs().max()


@pytest.mark.gpu
@pytest.mark.parametrize("name", [n for n in G.names("flash") if "reftest" in n])
def test_reference_flash_case_through_triton_llm(cuda_device, name):
    from triton_llm.ops.flash_attention import flash_attention

    c = G.load(name)
    out = flash_attention(c["q"].cuda(), c["k"].cuda(), c["v"].cuda(), causal=bool(c["causal"]),
                          sm_scale=float(c["sm_scale"]))
    _close(out, c["out"])


@pytest.mark.gpu
def test_reference_paged_case_through_triton_llm(cuda_device):
    from triton_llm.ops.paged_attention import paged_attention

    c = G.load("paged__reftest")
    out = paged_attention(c["q"].cuda(), c["k_cache"].cuda(), c["v_cache"].cuda(),
                          c["block_tables"].cuda(), c["context_lens"].cuda(),
                          block_size=int(c["block_size"]), sm_scale=float(c["sm_scale"]))
    _close(out, c["out"])


@pytest.mark.gpu
def test_reference_rmsnorm_rope_case_through_triton_llm(cuda_device):
    from triton_llm.ops.rmsnorm_rope import rmsnorm_rope

    c = G.load("rmsnorm_rope__reftest")
    out = rmsnorm_rope(c["x"].cuda(), c["w"].cuda(), c["cos"].cuda(), c["sin"].cuda(), float(c["eps"]))
    _close(out, c["out"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", [n for n in G.names("swiglu") if "reftest" in n])
def test_reference_swiglu_case_through_triton_llm(cuda_device, name):
    from triton_llm.ops.swiglu import swiglu

    c = G.load(name)
    out = swiglu(c["x"].cuda(), c["w1"].cuda(), c["w3"].cuda())
    _close(out, c["out"])
