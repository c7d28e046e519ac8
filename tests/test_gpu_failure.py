"""Failure detection on the GPU without a fault: a bounded wait that runs out is reported
through the device status word and the context stays usable."""
import pytest
import torch

import tritonllmcompiler_b200 as T
from tritonllmcompiler_b200 import _lib

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports(cuda_device):
    lib = _lib.load()
    torch.cuda.synchronize()
    assert _lib.debug_status() == 0
    _lib.check(lib.tllm_selftest_bounded_wait(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert _lib.debug_status() == 0x17F
    assert _lib.debug_status() == 0
    # The context is still usable: run an operator and check it against torch.
    x = torch.randn(64, 64, device="cuda").half()
    w = (torch.randn(64, 64, device="cuda") / 8).half()
    out = T.swiglu(x, w, w)
    g = x.float() @ w.float()
    ref = torch.nn.functional.silu(g) * g
    assert torch.allclose(out.float(), ref, atol=1e-2, rtol=1e-2)
