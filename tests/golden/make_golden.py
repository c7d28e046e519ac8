"""Generates the golden fixtures in this directory from the reference's own oracle functions.

Run in a checkout where xdlhzdh/TritonLLMCompiler is present (read-only is fine):

    python tests/golden/make_golden.py path/to/TritonLLMCompiler

It imports ``triton_llm.reference`` from ``<reference>/python`` (CPU only: those functions
are plain PyTorch), builds the cases of the reference's op tests (tests/python/test_*.py:
same seeds and shapes, generated on the CPU) plus the CUDA known-answer patterns
(tests/cuda/rmsnorm_rope_correctness.cu:11-17, tests/cuda/swiglu_correctness.cu:13-17) and a
few edge cases, and stores inputs and the reference's outputs as ``<op>__<case>.npz``.
fp16 tensors are stored as float16, bf16 tensors as their uint16 bit patterns. The fixtures
are committed, so the tests never need the reference at run time.
"""
from __future__ import annotations

import math
import os
import sys
import zlib

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(root: str):
    sys.path.insert(0, os.path.join(root, "python"))
    from triton_llm.reference.flash_attention import flash_attention_ref
    from triton_llm.reference.norm_rope import rmsnorm_rope_ref
    from triton_llm.reference.paged_attention import paged_attention_ref
    from triton_llm.reference.swiglu import swiglu_ref

    return flash_attention_ref, paged_attention_ref, rmsnorm_rope_ref, swiglu_ref


def _np(t: torch.Tensor):
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float16:
        return t.numpy()
    return t.numpy()


def _save(name: str, dtype: torch.dtype, tensors: dict, scalars: dict):
    arrays = {k: _np(v) for k, v in tensors.items()}
    arrays["dtype"] = np.array("bf16" if dtype == torch.bfloat16 else "fp16")
    for k, v in scalars.items():
        arrays[k] = np.array(v)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrays)


def _rope_cos_sin(seqlen: int, dim: int, dtype=torch.float16):
    # tests/python/test_rmsnorm_rope.py:11-16
    pos = torch.arange(seqlen, dtype=torch.float32)
    inv_freq = 1.0 / (10000 ** (torch.arange(0, dim, 2).float() / dim))
    freqs = torch.outer(pos, inv_freq)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def main(root: str):
    fa_ref, pa_ref, rr_ref, sw_ref = _import_reference(root)
    torch.set_num_threads(4)

    # ---------------- flash_attention ----------------
    # tests/python/test_flash_attention.py:10-21 (seed 0, B1 H2 D64, S in {64,128}).
    for seqlen in (64, 128):
        for causal in (False, True):
            torch.manual_seed(0)
            q = torch.randn(1, 2, seqlen, 64, dtype=torch.float16)
            k = torch.randn(1, 2, seqlen, 64, dtype=torch.float16)
            v = torch.randn(1, 2, seqlen, 64, dtype=torch.float16)
            out = fa_ref(q, k, v, causal=causal)
            _save(f"flash__reftest_s{seqlen}_{'causal' if causal else 'full'}", torch.float16,
                  dict(q=q, k=k, v=v, out=out), dict(causal=causal, sm_scale=64 ** -0.5))
    # Edge cases: Sq != Sk (both directions), ragged tiles, every head dim, bf16.
    edge = [
        ("sq100_sk160_causal", 1, 2, 100, 160, 128, True, torch.float16, None),
        ("sq100_sk160_full", 2, 1, 100, 160, 128, False, torch.float16, None),
        ("sq200_sk72_causal", 1, 2, 200, 72, 64, True, torch.float16, None),
        ("d16_s130_causal", 1, 2, 130, 130, 16, True, torch.float16, None),
        ("d32_s256_full", 1, 2, 256, 256, 32, False, torch.float16, 0.3),
        ("d128_s300_causal_bf16", 1, 1, 300, 300, 128, True, torch.bfloat16, None),
    ]
    for name, b, h, sq, sk, d, causal, dt, scale in edge:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
        q = torch.randn(b, h, sq, d, generator=g).to(dt)
        k = torch.randn(b, h, sk, d, generator=g).to(dt)
        v = torch.randn(b, h, sk, d, generator=g).to(dt)
        out = fa_ref(q, k, v, causal=causal, sm_scale=scale)
        _save(f"flash__{name}", dt, dict(q=q, k=k, v=v, out=out),
              dict(causal=causal, sm_scale=scale if scale is not None else d ** -0.5))

    # ---------------- paged_attention ----------------
    # tests/python/test_paged_attention.py:11-24 (seed 1, identity block table).
    torch.manual_seed(1)
    b, h, d, bs = 2, 2, 64, 16
    context_lens = torch.tensor([40, 24], dtype=torch.int32)
    max_blocks = 4
    num_blocks = b * max_blocks
    k_cache = torch.randn(num_blocks, bs, h, d, dtype=torch.float16)
    v_cache = torch.randn(num_blocks, bs, h, d, dtype=torch.float16)
    block_tables = torch.arange(num_blocks, dtype=torch.int32).reshape(b, max_blocks)
    q = torch.randn(b, h, 1, d, dtype=torch.float16)
    out = pa_ref(q, k_cache, v_cache, block_tables, context_lens, block_size=bs)
    _save("paged__reftest", torch.float16,
          dict(q=q, k_cache=k_cache, v_cache=v_cache, block_tables=block_tables,
               context_lens=context_lens, out=out), dict(block_size=bs, sm_scale=d ** -0.5))
    # Permuted pool, lengths off block boundaries and below one block, several block sizes.
    cases = [
        ("perm_bs16_d128", 5, 2, 128, 16, [1, 15, 16, 17, 300], torch.float16),
        ("perm_bs32_d64", 3, 2, 64, 32, [33, 64, 400], torch.float16),
        ("perm_bs64_d32_bf16", 3, 2, 32, 64, [5, 128, 129], torch.bfloat16),
        ("perm_bs16_d16", 2, 3, 16, 16, [1000, 7], torch.float16),
    ]
    for name, b, h, d, bs, lens, dt in cases:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
        lens_t = torch.tensor(lens, dtype=torch.int32)
        nb = [(n + bs - 1) // bs for n in lens]
        pool = sum(nb) + 3  # a few blocks nobody references
        perm = torch.randperm(pool, generator=g)
        width = max(nb) + 2  # padding columns that must never be read
        bt = torch.full((b, width), 0, dtype=torch.int32)
        pos = 0
        for i, n in enumerate(nb):
            bt[i, :n] = perm[pos:pos + n].to(torch.int32)
            pos += n
        kc = torch.randn(pool, bs, h, d, generator=g).to(dt)
        vc = torch.randn(pool, bs, h, d, generator=g).to(dt)
        qq = torch.randn(b, h, 1, d, generator=g).to(dt)
        out = pa_ref(qq, kc, vc, bt, lens_t, block_size=bs)
        _save(f"paged__{name}", dt,
              dict(q=qq, k_cache=kc, v_cache=vc, block_tables=bt, context_lens=lens_t, out=out),
              dict(block_size=bs, sm_scale=d ** -0.5))

    # ---------------- rmsnorm_rope ----------------
    # tests/python/test_rmsnorm_rope.py:19-28 (seed 2, B2 S16 H4 D64, w ~ N(0,1)).
    torch.manual_seed(2)
    b, s, h, d = 2, 16, 4, 64
    x = torch.randn(b, s, h, d, dtype=torch.float16)
    w = torch.randn(d, dtype=torch.float16)
    cos, sin = _rope_cos_sin(s, d)
    out = rr_ref(x, w, cos, sin)
    _save("rmsnorm_rope__reftest", torch.float16, dict(x=x, w=w, cos=cos, sin=sin, out=out),
          dict(eps=1e-6))
    # tests/cuda/rmsnorm_rope_correctness.cu:9-17 known-answer pattern (fp16-rounded inputs).
    B, S, H, D = 1, 8, 2, 64
    xi = torch.tensor([((i % 9) - 4) * 0.1 for i in range(B * S * H * D)], dtype=torch.float32)
    x = xi.reshape(B, S, H, D).to(torch.float16)
    w = torch.ones(D, dtype=torch.float16)
    sd = torch.tensor([[0.01 * (si + i) for i in range(D)] for si in range(S)], dtype=torch.float32)
    cos, sin = torch.cos(sd).to(torch.float16), torch.sin(sd).to(torch.float16)
    out = rr_ref(x, w, cos, sin)
    _save("rmsnorm_rope__cuda_pattern", torch.float16, dict(x=x, w=w, cos=cos, sin=sin, out=out),
          dict(eps=1e-6))
    for name, (b, s, h, d), dt in [("d128", (2, 33, 3, 128), torch.float16),
                                   ("d16", (3, 5, 2, 16), torch.float16),
                                   ("d32_bf16", (2, 7, 5, 32), torch.bfloat16)]:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
        x = torch.randn(b, s, h, d, generator=g).to(dt)
        w = (1 + 0.1 * torch.randn(d, generator=g)).to(dt)
        cos, sin = _rope_cos_sin(s, d, dt)
        out = rr_ref(x, w, cos, sin)
        _save(f"rmsnorm_rope__{name}", dt, dict(x=x, w=w, cos=cos, sin=sin, out=out), dict(eps=1e-6))

    # ---------------- swiglu ----------------
    # tests/python/test_swiglu.py:10-19 (seed 3, w ~ N(0,1)).
    for m, n, k in [(64, 64, 64), (128, 256, 64)]:
        torch.manual_seed(3)
        x = torch.randn(m, k, dtype=torch.float16)
        w1 = torch.randn(k, n, dtype=torch.float16)
        w3 = torch.randn(k, n, dtype=torch.float16)
        out = sw_ref(x, w1, w3)
        _save(f"swiglu__reftest_{m}x{n}x{k}", torch.float16, dict(x=x, w1=w1, w3=w3, out=out), {})
    # tests/cuda/swiglu_correctness.cu:13-17 known-answer pattern.
    M = N = K = 64
    x = torch.tensor([((i % 7) - 3) * 0.1 for i in range(M * K)]).reshape(M, K).to(torch.float16)
    w1 = torch.tensor([((i % 5) - 2) * 0.05 for i in range(K * N)]).reshape(K, N).to(torch.float16)
    w3 = torch.tensor([((i % 3) - 1) * 0.05 for i in range(K * N)]).reshape(K, N).to(torch.float16)
    out = sw_ref(x, w1, w3)
    _save("swiglu__cuda_pattern", torch.float16, dict(x=x, w1=w1, w3=w3, out=out), {})
    for name, (m, n, k), dt in [("ragged_100x72x40", (100, 72, 40), torch.float16),
                                ("multi_tile_260x264x136", (260, 264, 136), torch.float16),
                                ("bf16_256x128x128", (256, 128, 128), torch.bfloat16),
                                ("odd_k_33x24x13", (33, 24, 13), torch.float16)]:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
        x = torch.randn(m, k, generator=g).to(dt)
        w1 = (torch.randn(k, n, generator=g) / math.sqrt(k)).to(dt)
        w3 = (torch.randn(k, n, generator=g) / math.sqrt(k)).to(dt)
        out = sw_ref(x, w1, w3)
        _save(f"swiglu__{name}", dt, dict(x=x, w1=w1, w3=w3, out=out), {})


if __name__ == "__main__":
    # The reference checkout is given explicitly: the first argument, or TRITON_LLM_REFERENCE.
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("TRITON_LLM_REFERENCE")
    if not ref_root:
        sys.exit("usage: make_golden.py <reference checkout> (or set TRITON_LLM_REFERENCE)")
    main(ref_root)
