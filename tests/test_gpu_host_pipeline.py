"""SwiGLU on pinned host operands with pipelined transfers: bit-identical to ``swiglu`` on the
device (the same kernel computes every output tile)."""
import pytest
import torch

import tritonllmcompiler_b200 as T
from tritonllmcompiler_b200.ops.host_pipeline import SwigluHostPipeline, swiglu_from_host

pytestmark = pytest.mark.gpu


def _host(shape, g, scale=1.0):
    return (torch.randn(shape, generator=g) * scale).half().pin_memory()


@pytest.mark.parametrize("m,n,k,chunks", [(256, 1000, 512, 3), (130, 384, 96, 8), (64, 128, 64, 1),
                                          (512, 2048, 1024, 16)])
def test_host_pipeline_matches_device_swiglu(cuda_device, m, n, k, chunks):
    g = torch.Generator().manual_seed(m + n + k)
    x, w1, w3 = _host((m, k), g), _host((k, n), g, k ** -0.5), _host((k, n), g, k ** -0.5)
    out = swiglu_from_host(x, w1, w3, chunks=chunks)
    torch.cuda.synchronize()
    ref = T.swiglu(x.cuda(), w1.cuda(), w3.cuda()).cpu()
    assert out.is_pinned() and torch.equal(out, ref)


def test_host_pipeline_reuse_and_full_size(cuda_device):
    # The Llama-3-8B MLP shape, twice through one pipeline (buffers and events reused).
    M, K, N = 4096, 4096, 14336
    g = torch.Generator().manual_seed(5)
    x, w1, w3 = _host((M, K), g), _host((K, N), g, K ** -0.5), _host((K, N), g, K ** -0.5)
    pipe = SwigluHostPipeline(M, N, K, torch.float16, "cuda", chunks=8)
    out = torch.empty((M, N), dtype=torch.float16).pin_memory()
    ref = T.swiglu(x.cuda(), w1.cuda(), w3.cuda()).cpu()
    for _ in range(2):
        out.zero_()
        pipe(x, w1, w3, out)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)


def test_host_pipeline_rejects_pageable_memory(cuda_device):
    x = torch.zeros(64, 64, dtype=torch.float16)
    with pytest.raises(AssertionError):
        swiglu_from_host(x, x, x)
