"""Parity at the benchmark configurations (full sizes), checked on sampled rows, heads and
sequences against the numpy oracle, and the multi-GPU partitions emulated on one GPU.

Inputs follow the configuration recipes (seeded normal data; weights N(0, 1/K); RoPE base
10000; context lengths U[lo, hi]). The oracle is run on the CPU on the sampled slices only,
so each case finishes in seconds; tolerance as in the other parity tests.
"""
import math

import numpy as np
import pytest
import torch

import tritonllmcompiler_b200 as T
from oracle import ops_oracle as O
from tests import _golden as G
from tritonllmcompiler_b200 import sharded as S

pytestmark = pytest.mark.gpu


def _close(got, ref):
    got = got.float().cpu().numpy() if torch.is_tensor(got) else got
    err = float(np.nanmax(np.abs(got - ref))) if got.size else 0.0
    assert np.allclose(got, ref, equal_nan=True, **G.tol("fp16")), f"max abs err {err}"


def _f(t):
    return t.float().cpu().numpy()


def _gpu_randn(shape, seed, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda") * scale).half()


def _rope(s, d):
    pos = torch.arange(s, dtype=torch.float32)
    inv = 1.0 / (10000 ** (torch.arange(0, d, 2).float() / d))
    emb = torch.cat([torch.outer(pos, inv)] * 2, dim=-1)
    return emb.cos().half(), emb.sin().half()


def test_cfg_rmsnorm_rope_2x128x8x64(cuda_device):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(2, 128, 8, 64, generator=g).half()
    w = (1 + 0.1 * torch.randn(64, generator=g)).half()
    cos, sin = _rope(128, 64)
    out = T.rmsnorm_rope(x.cuda(), w.cuda(), cos.cuda(), sin.cuda(), 1e-6)
    _close(out, O.rmsnorm_rope(_f(x), _f(w), _f(cos), _f(sin), 1e-6))


def test_cfg_rmsnorm_rope_bandwidth_variant(cuda_device):
    x = _gpu_randn((16, 4096, 32, 128), 5)
    w = (1 + 0.1 * torch.randn(128, generator=torch.Generator().manual_seed(5))).half().cuda()
    cos, sin = _rope(4096, 128)
    out = T.rmsnorm_rope(x, w, cos.cuda(), sin.cuda())
    for b, s in [(0, 0), (7, 4095), (15, 1234)]:
        ref = O.rmsnorm_rope(_f(x[b:b + 1, s:s + 1]), _f(w), _f(cos[s:s + 1]), _f(sin[s:s + 1]))
        _close(out[b:b + 1, s:s + 1], ref)


def _swiglu_sampled(m, k, n, seed, rows):
    x = _gpu_randn((m, k), seed)
    w1 = _gpu_randn((k, n), seed + 1, 1 / math.sqrt(k))
    w3 = _gpu_randn((k, n), seed + 2, 1 / math.sqrt(k))
    out = T.swiglu(x, w1, w3)
    idx = torch.tensor(rows)
    ref = O.swiglu(_f(x[idx]), _f(w1), _f(w3))
    _close(out[idx.cuda()], ref)
    return x, w1, w3, out


def test_cfg_swiglu_llama3_8b(cuda_device):
    rows = [0, 1, 127, 128, 2047, 4095] + list(range(1000, 1040))
    _swiglu_sampled(4096, 4096, 14336, 1, rows)


def test_cfg_swiglu_llama3_70b_and_column_shards(cuda_device):
    m, k, n = 8192, 8192, 28672
    x, w1, w3, out = _swiglu_sampled(m, k, n, 4, [0, 4095, 8191] + list(range(300, 316)))
    # The column shards of the 8-way split, computed one at a time, reassemble exactly.
    for r in (0, 3, 7):
        n0, n1 = S.column_range(n, r, 8)
        part = T.swiglu(x, w1[:, n0:n1].contiguous(), w3[:, n0:n1].contiguous())
        assert torch.equal(part, out[:, n0:n1])


def _flash_heads(b, h, s, d, causal, seed, heads):
    q = _gpu_randn((b, h, s, d), seed)
    k = _gpu_randn((b, h, s, d), seed + 1)
    v = _gpu_randn((b, h, s, d), seed + 2)
    out = T.flash_attention(q, k, v, causal=causal, sm_scale=1 / math.sqrt(d))
    for bi, hi in heads:
        ref = O.flash_attention(_f(q[bi:bi + 1, hi:hi + 1]), _f(k[bi:bi + 1, hi:hi + 1]),
                                _f(v[bi:bi + 1, hi:hi + 1]), causal=causal, sm_scale=1 / math.sqrt(d))
        _close(out[bi:bi + 1, hi:hi + 1], ref)
    return q, k, v, out


def test_cfg_flash_causal_4x32x4096(cuda_device):
    _flash_heads(4, 32, 4096, 128, True, 2, [(0, 0), (3, 31), (2, 17)])


def test_cfg_flash_full_4x32x1024(cuda_device):
    _flash_heads(4, 32, 1024, 128, False, 12, [(0, 5), (1, 0), (3, 31), (2, 9)])


def test_cfg_flash_causal_70b_and_head_shards(cuda_device):
    q, k, v, out = _flash_heads(8, 64, 8192, 128, True, 20, [(0, 0), (7, 63)])
    # Head shards of the 8-way split give the same bits as the full launch.
    for r in (0, 5):
        h0, h1 = S.head_range(64, r, 8)
        part = S.flash_attention_head_sharded(q[:, h0:h1].contiguous(), k[:, h0:h1].contiguous(),
                                              v[:, h0:h1].contiguous(), causal=True,
                                              sm_scale=1 / math.sqrt(128))
        assert torch.equal(part, out[:, h0:h1])


def _paged_cfg(batch, heads, d, bs, lo, hi, seed):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(lo, hi + 1, (batch,), dtype=torch.int32, generator=g)
    nb = [(int(n) + bs - 1) // bs for n in lens]
    pool = sum(nb)
    perm = torch.randperm(pool, generator=g)
    bt = torch.zeros(batch, max(nb), dtype=torch.int32)
    pos = 0
    for i, n in enumerate(nb):
        bt[i, :n] = perm[pos:pos + n].to(torch.int32)
        pos += n
    kc = _gpu_randn((pool, bs, heads, d), seed + 1)
    vc = _gpu_randn((pool, bs, heads, d), seed + 2)
    q = _gpu_randn((batch, heads, 1, d), seed + 3)
    return q, kc, vc, bt, lens


def _paged_check(q, kc, vc, bt, lens, bs, seqs, out):
    for s in seqs:
        n = (int(lens[s]) + bs - 1) // bs
        blocks = bt[s, :n].long()
        kl = kc[blocks.cuda()]
        vl = vc[blocks.cuda()]
        local_bt = torch.arange(n, dtype=torch.int32)[None]
        ref = O.paged_attention(_f(q[s:s + 1]), _f(kl), _f(vl), local_bt.numpy(),
                                lens[s:s + 1].numpy(), block_size=bs)
        _close(out[s:s + 1], ref)


def test_cfg_paged_decode_b64(cuda_device):
    q, kc, vc, bt, lens = _paged_cfg(64, 32, 128, 16, 512, 8192, 3)
    out = T.paged_attention(q, kc, vc, bt.cuda(), lens.cuda(), block_size=16)
    _paged_check(q, kc, vc, bt, lens, 16, [0, 1, 17, 31, 42, 63], out)


def test_cfg_paged_70b_batch_shard(cuda_device):
    """One rank's share of the 70B decode configuration (B256 H64 D128 block 32, lengths
    U[1024,32768]), re-indexed into a local pool, against the oracle and a global launch."""
    batch, heads, d, bs = 256, 64, 128, 32
    g = torch.Generator().manual_seed(4)
    lens = torch.randint(1024, 32769, (batch,), dtype=torch.int32, generator=g)
    parts = S.partition_sequences(lens.tolist(), 8, "tokens")
    mine = parts[0]
    # Build only this rank's cache: its sequences, a permuted local pool.
    nb = [(int(lens[s]) + bs - 1) // bs for s in mine]
    pool = sum(nb)
    perm = torch.randperm(pool, generator=g)
    bt = torch.zeros(len(mine), max(nb), dtype=torch.int32)
    pos = 0
    for i, n in enumerate(nb):
        bt[i, :n] = perm[pos:pos + n].to(torch.int32)
        pos += n
    kc = _gpu_randn((pool, bs, heads, d), 41)
    vc = _gpu_randn((pool, bs, heads, d), 42)
    q = _gpu_randn((len(mine), heads, 1, d), 43)
    ll = lens[mine]
    out = T.paged_attention(q, kc, vc, bt.cuda(), ll.cuda(), block_size=bs)
    _paged_check(q, kc, vc, bt, ll, bs, [0, len(mine) - 1, len(mine) // 2], out)
    # Localising a sub-batch into its own pool gives the same result.
    sub = [0, 3, 5]
    ids, lbt, lcl = S.localize_blocks(bt, ll, sub, bs)
    out2 = T.paged_attention(q[sub], kc[ids.cuda()], vc[ids.cuda()], lbt.cuda(), lcl.cuda(), block_size=bs)
    assert torch.allclose(out2.float(), out[sub].float(), **G.tol("fp16"))
