"""SwiGLU on operands that live in pinned host memory, with the PCIe transfers pipelined.

The reference's ``swiglu`` (python/triton_llm/ops/swiglu.py:54-76) takes device tensors; a
caller whose x, w1, w3 are in host memory copies them over, runs it and copies the result
back, one step after the other. Here the weights are split into column blocks: block c's
columns of w1 and w3 are copied host -> device (one 2-D DMA request each) on a copy stream,
block c's GEMM (the same ``tllm_swiglu`` kernel on column slices, ldb = N) runs on a compute
stream as soon as they have arrived, and block c's output columns go device -> host on a
third stream, so the upload of block c+1, the kernel on block c and the download of block
c-1 overlap. The result is bit-identical to ``swiglu`` (every output tile is computed by the
same kernel with the same K order).
"""
from __future__ import annotations

import torch

from tritonllmcompiler_b200 import _lib

_TILE_N = 128  # the kernel's output tile width


def _equal_blocks(n: int, chunks: int):
    cols = -(-n // max(chunks, 1))          # ceil(n / chunks)
    per = -(-cols // _TILE_N) * _TILE_N      # rounded up to whole tiles
    out, c0 = [], 0
    while c0 < n:
        c1 = min(n, c0 + per)
        out.append((c0, c1))
        c0 = c1
    return out


def _blocks(n: int, chunks: int):
    """Column blocks [c0, c1), boundaries on tile multiples: the last block is about a quarter
    of the others, because its kernel and its download are the part of the step that no
    upload overlaps (4 % faster end to end than equal blocks at N = 14336, 8 blocks)."""
    last = -(-(n // max(4 * chunks, 1)) // _TILE_N) * _TILE_N
    start = (n - last) // _TILE_N * _TILE_N  # the last block starts on a tile boundary
    if chunks <= 1 or start <= 0:
        return _equal_blocks(n, chunks)
    return _equal_blocks(start, chunks - 1) + [(start, n)]


class SwigluHostPipeline:
    """Device buffers, streams and events for ``swiglu`` of [M, K] x [K, N] operands held in
    pinned host memory; reuse one instance for repeated calls of the same shape."""

    def __init__(self, m: int, n: int, k: int, dtype: torch.dtype = torch.float16,
                 device: torch.device | str | None = None, chunks: int = 8):
        assert dtype in _lib.DTYPE_CODES and m > 0 and n > 0 and k > 0
        self.m, self.n, self.k, self.dtype = m, n, k, dtype
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.blocks = _blocks(n, chunks)
        with torch.cuda.device(self.device):
            self.dx = torch.empty((m, k), dtype=dtype, device=self.device)
            self.d1 = torch.empty((k, n), dtype=dtype, device=self.device)
            self.d3 = torch.empty((k, n), dtype=dtype, device=self.device)
            self.dout = torch.empty((m, n), dtype=dtype, device=self.device)
            self.s_in = torch.cuda.Stream(self.device)
            self.s_comp = torch.cuda.Stream(self.device)
            self.s_out = torch.cuda.Stream(self.device)
            self.ev_in = [torch.cuda.Event() for _ in self.blocks]
            self.ev_done = [torch.cuda.Event() for _ in self.blocks]
            # Recorded on s_out at the end of every call: the next call's uploads and kernels
            # wait for it, so they never overwrite buffers the previous call still reads, even
            # when the caller switches streams between calls.
            self.ev_end = torch.cuda.Event()
            self.ev_end.record(self.s_out)

    def __call__(self, x: torch.Tensor, w1: torch.Tensor, w3: torch.Tensor,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        """x [M, K], w1/w3 [K, N], out [M, N]: contiguous pinned host tensors. Enqueued after
        the current stream's work; the current stream waits for the result (read out after
        synchronising)."""
        m, n, k, dt = self.m, self.n, self.k, self.dtype
        for t, shape in ((x, (m, k)), (w1, (k, n)), (w3, (k, n))):
            assert not t.is_cuda and t.is_pinned() and t.is_contiguous()
            assert tuple(t.shape) == shape and t.dtype == dt
        if out is None:
            out = torch.empty((m, n), dtype=dt, pin_memory=True)
        assert not out.is_cuda and out.is_pinned() and out.is_contiguous()
        assert tuple(out.shape) == (m, n) and out.dtype == dt
        lib = _lib.load()
        es = self.dx.element_size()
        code = _lib.DTYPE_CODES[dt]
        with torch.cuda.device(self.device):
            cur = torch.cuda.current_stream(self.device)
            for s in (self.s_in, self.s_comp, self.s_out):
                s.wait_stream(cur)
                s.wait_event(self.ev_end)
            sin, scomp, sout = (s.cuda_stream for s in (self.s_in, self.s_comp, self.s_out))
            # host -> device: x, then the weight blocks in order
            _lib.check(lib.tllm_copy2d_async(self.dx.data_ptr(), k * es, x.data_ptr(), k * es,
                                             k * es, m, sin))
            for (c0, c1), ev in zip(self.blocks, self.ev_in):
                for dst, src in ((self.d1, w1), (self.d3, w3)):
                    _lib.check(lib.tllm_copy2d_async(dst.data_ptr() + c0 * es, n * es,
                                                     src.data_ptr() + c0 * es, n * es,
                                                     (c1 - c0) * es, k, sin))
                ev.record(self.s_in)
            # the kernel on each block once it is on the device
            for (c0, c1), ev, done in zip(self.blocks, self.ev_in, self.ev_done):
                self.s_comp.wait_event(ev)
                _lib.check(lib.tllm_swiglu(
                    self.dx.data_ptr(), self.d1.data_ptr() + c0 * es, self.d3.data_ptr() + c0 * es,
                    self.dout.data_ptr() + c0 * es, m, c1 - c0, k, k, n, n, n, code, scomp))
                done.record(self.s_comp)
            # device -> host: each block's output columns
            for (c0, c1), done in zip(self.blocks, self.ev_done):
                self.s_out.wait_event(done)
                _lib.check(lib.tllm_copy2d_async(out.data_ptr() + c0 * es, n * es,
                                                 self.dout.data_ptr() + c0 * es, n * es,
                                                 (c1 - c0) * es, m, sout))
            self.ev_end.record(self.s_out)
            cur.wait_stream(self.s_out)
        return out


_PIPELINES: dict = {}


def swiglu_from_host(x: torch.Tensor, w1: torch.Tensor, w3: torch.Tensor,
                     out: torch.Tensor | None = None, *, chunks: int = 8,
                     device: torch.device | str | None = None) -> torch.Tensor:
    """silu(x @ w1) * (x @ w3) for pinned host tensors x [M, K], w1/w3 [K, N]; returns a pinned
    host [M, N] tensor (``out`` if given), complete once the current stream is synchronised.
    Device buffers are cached per (shape, dtype, device, chunks)."""
    m, k = x.shape
    n = w1.shape[1]
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    key = (m, n, k, x.dtype, dev, chunks)
    p = _PIPELINES.get(key)
    if p is None:
        p = _PIPELINES[key] = SwigluHostPipeline(m, n, k, x.dtype, dev, chunks)
    return p(x, w1, w3, out)
