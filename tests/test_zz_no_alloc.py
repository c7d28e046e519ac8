"""The allocation-free paged decode entry point, called through the C ABI.

tllm_paged_attn_decode_noalloc serves callers that cannot allocate device memory (engines
that reserve all device memory at start-up, foreign-language hosts with no device
allocator): it keeps its split-KV partials in a fixed array inside the library instead of a
caller-provided workspace. These tests compare it with the workspace-taking entry point,
tllm_paged_attn_decode, on two calls in a row (the second with different lengths, so
leftovers of the first call in the shared array would show), and check the size limit.
This file sorts last so a failure here comes after every other test has run.
"""
import ctypes

import pytest
import torch

from tests import _golden as G
from tritonllmcompiler_b200 import _lib

pytestmark = pytest.mark.gpu


def _case(seed, lens, b=None, h=8, d=128, bs=16):
    g = torch.Generator().manual_seed(seed)
    b = len(lens) if b is None else b
    nb = [(n + bs - 1) // bs for n in lens]
    pool = sum(nb) + 2
    perm = torch.randperm(pool, generator=g)
    bt = torch.zeros(b, max(nb) + 1, dtype=torch.int32)
    pos = 0
    for i, n in enumerate(nb):
        bt[i, :n] = perm[pos:pos + n].to(torch.int32)
        pos += n
    kc = torch.randn(pool, bs, h, d, generator=g).half().cuda()
    vc = torch.randn(pool, bs, h, d, generator=g).half().cuda()
    q = torch.randn(b, h, 1, d, generator=g).half().cuda()
    return q, kc, vc, bt.cuda(), torch.tensor(lens, dtype=torch.int32).cuda(), bs


def _with_workspace(lib, q, kc, vc, bt, cl, bs):
    """Reference result from the existing entry point with a torch-allocated workspace."""
    b, h, _, d = q.shape
    out = torch.empty_like(q)
    ws_bytes = lib.tllm_paged_attn_workspace_size(b, h, d, bs, bt.shape[1])
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    _lib.check(lib.tllm_paged_attn_decode(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), cl.data_ptr(), out.data_ptr(),
        ws.data_ptr(), ws_bytes, b, h, d, bs, bt.shape[1], kc.shape[0],
        _lib.strides(q), _lib.strides(kc), _lib.strides(vc), _lib.strides(bt), _lib.strides(out),
        d ** -0.5, 0, torch.cuda.current_stream().cuda_stream))
    return out, ws_bytes


def _no_alloc(lib, q, kc, vc, bt, cl, bs):
    b, h, _, d = q.shape
    out = torch.empty_like(q)  # outputs are still the caller's
    rc = lib.tllm_paged_attn_decode_noalloc(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), cl.data_ptr(), out.data_ptr(),
        b, h, d, bs, bt.shape[1], kc.shape[0],
        _lib.strides(q), _lib.strides(kc), _lib.strides(vc), _lib.strides(bt), _lib.strides(out),
        d ** -0.5, 0, torch.cuda.current_stream().cuda_stream)
    return rc, out


def test_no_alloc_matches_workspace_entry_point_on_two_calls(cuda_device):
    lib = _lib.load()
    cases = [_case(101, [3000, 17, 2049, 512, 4096, 1, 700, 1500]),
             _case(202, [64, 5000, 333, 1024, 2, 4097, 128, 999])]
    for q, kc, vc, bt, cl, bs in cases:
        ref, ws_bytes = _with_workspace(lib, q, kc, vc, bt, cl, bs)
        assert ws_bytes > 0, "the case must use split-KV scratch"
        assert ws_bytes <= 32 << 20
        rc, out = _no_alloc(lib, q, kc, vc, bt, cl, bs)
        _lib.check(rc)
        torch.cuda.synchronize()
        # Both entry points plan the same splits and run the same kernels in the same order,
        # so anything short of bit equality means stale or misplaced scratch.
        assert torch.equal(out, ref)
        assert torch.allclose(out.float(), ref.float(), **G.tol(out.dtype))


def test_no_alloc_rejects_problems_beyond_its_array(cuda_device):
    lib = _lib.load()
    b, h, d, bs, max_blocks = 512, 64, 128, 16, 2048
    need = lib.tllm_paged_attn_workspace_size(b, h, d, bs, max_blocks)
    assert need > (32 << 20)
    s4 = (ctypes.c_int64 * 4)(1, 1, 1, 1)
    s4c = (ctypes.c_int64 * 4)(bs * h * d, h * d, d, 1)
    s2 = (ctypes.c_int64 * 2)(max_blocks, 1)
    rc = lib.tllm_paged_attn_decode_noalloc(16, 16, 16, 16, 16, 16, b, h, d, bs, max_blocks, 8,
                                            s4, s4c, s4c, s2, s4, 0.1, 0, None)
    assert rc == 3
    assert b"fixed" in lib.tllm_last_error()


def test_no_alloc_rejects_bad_dimensions_before_sizing(cuda_device):
    """A negative batch or an unsupported head dim is an argument error, not a scratch overflow."""
    lib = _lib.load()
    s4 = (ctypes.c_int64 * 4)(1, 1, 1, 1)
    s4c = (ctypes.c_int64 * 4)(16 * 8 * 128, 8 * 128, 128, 1)
    s2 = (ctypes.c_int64 * 2)(4, 1)
    for b, h, d, bs in [(-1, 8, 128, 16), (4, -3, 128, 16), (4, 8, 96, 16), (4, 8, 128, 8)]:
        rc = lib.tllm_paged_attn_decode_noalloc(16, 16, 16, 16, 16, 16, b, h, d, bs, 4, 8,
                                                s4, s4c, s4c, s2, s4, 0.1, 0, None)
        assert rc == 1, (b, h, d, bs)
