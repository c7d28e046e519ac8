"""CUDA kernels vs the numpy oracle on seeded inputs, plus exact size-independent properties.

Tolerance: the reference's op tolerance, atol 1e-3 and rtol 1e-2 (tests/python/test_*.py).
"""
import math

import numpy as np
import pytest
import torch

import tritonllmcompiler_b200 as T
from oracle import ops_oracle as O
from tests import _golden as G

pytestmark = pytest.mark.gpu


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def _dt(name):
    return torch.bfloat16 if name == "bf16" else torch.float16


def _f32(t):
    return t.float().cpu().numpy()


def _assert_close(out, ref_np):
    got = out.float().cpu().numpy()
    assert got.shape == ref_np.shape
    err = np.nanmax(np.abs(got - ref_np)) if got.size else 0.0
    assert np.allclose(got, ref_np, equal_nan=True, **G.tol(out.dtype)), f"max abs err {err}"


# ----------------------------------------------------------------------------- rmsnorm_rope
def _rope(s, d, dt):
    pos = torch.arange(s, dtype=torch.float32)
    inv = 1.0 / (10000 ** (torch.arange(0, d, 2).float() / d))
    emb = torch.cat([torch.outer(pos, inv)] * 2, dim=-1)
    return emb.cos().to(dt), emb.sin().to(dt)


@pytest.mark.parametrize("shape,dt", [((2, 128, 8, 64), "fp16"), ((1, 7, 3, 128), "fp16"),
                                      ((3, 9, 5, 16), "bf16"), ((4, 64, 8, 32), "bf16"),
                                      ((2, 1, 1, 128), "fp16")])
def test_rmsnorm_rope_random(cuda_device, shape, dt):
    b, s, h, d = shape
    g = _gen(10 + d)
    x = torch.randn(shape, generator=g).to(_dt(dt))
    w = (1 + 0.1 * torch.randn(d, generator=g)).to(_dt(dt))
    cos, sin = _rope(s, d, _dt(dt))
    out = T.rmsnorm_rope(x.cuda(), w.cuda(), cos.cuda(), sin.cuda())
    _assert_close(out, O.rmsnorm_rope(_f32(x), _f32(w), _f32(cos), _f32(sin), dtype=dt))


def test_rmsnorm_rope_noncontiguous(cuda_device):
    g = _gen(11)
    base = torch.randn(2, 6, 5, 64, generator=g).half()  # [B, H, S, D] storage
    x = base.permute(0, 2, 1, 3)  # [B, S, H, D] view, unit inner stride (vector path)
    w = torch.randn(64, generator=g).half()
    cos, sin = _rope(5, 64, torch.float16)
    out = T.rmsnorm_rope(x.cuda(), w.cuda(), cos.cuda(), sin.cuda())
    _assert_close(out, O.rmsnorm_rope(_f32(x), _f32(w), _f32(cos), _f32(sin)))
    # Inner stride 2 (general-stride path).
    wide = torch.randn(2, 5, 3, 128, generator=g).half()
    x2 = wide[..., ::2]
    cos2, sin2 = _rope(5, 64, torch.float16)
    out2 = T.rmsnorm_rope(x2.cuda(), w.cuda(), cos2.cuda(), sin2.cuda())
    _assert_close(out2, O.rmsnorm_rope(_f32(x2), _f32(w), _f32(cos2), _f32(sin2)))


def test_rmsnorm_rope_head_permutation_is_exact(cuda_device):
    """Rows are independent: permuting heads (and batches) permutes the output bit-for-bit."""
    g = _gen(12)
    x = torch.randn(4, 256, 8, 128, generator=g).half().cuda()
    w = (1 + 0.1 * torch.randn(128, generator=g)).half().cuda()
    cos, sin = _rope(256, 128, torch.float16)
    cos, sin = cos.cuda(), sin.cuda()
    a = T.rmsnorm_rope(x, w, cos, sin)
    hp = torch.randperm(8, generator=g).cuda()
    bp = torch.randperm(4, generator=g).cuda()
    b = T.rmsnorm_rope(x[bp][:, :, hp].contiguous(), w, cos, sin)
    assert torch.equal(a[bp][:, :, hp], b)


# ----------------------------------------------------------------------------- swiglu
@pytest.mark.parametrize("m,n,k,dt", [(128, 128, 64, "fp16"), (256, 384, 512, "fp16"),
                                      (129, 136, 72, "fp16"), (1, 8, 8, "fp16"),
                                      (300, 1000, 1032, "bf16"), (40, 24, 13, "fp16"),
                                      (1024, 2048, 1024, "bf16")])
def test_swiglu_random(cuda_device, m, n, k, dt):
    g = _gen(m * 7 + n * 3 + k)
    x = torch.randn(m, k, generator=g).to(_dt(dt))
    w1 = (torch.randn(k, n, generator=g) / math.sqrt(k)).to(_dt(dt))
    w3 = (torch.randn(k, n, generator=g) / math.sqrt(k)).to(_dt(dt))
    out = T.swiglu(x.cuda(), w1.cuda(), w3.cuda())
    _assert_close(out, O.swiglu(_f32(x), _f32(w1), _f32(w3), dtype=dt))


@pytest.mark.parametrize("m,n,k,dt", [(256, 128, 64, "fp16"), (300, 256, 1000, "bf16"),
                                      (1000, 640, 520, "fp16"), (4096, 1024, 4096, "fp16")])
def test_swiglu_kernel_variants_agree(cuda_device, m, n, k, dt):
    """The CTA-pair kernel (tcgen05.mma.cta_group::2, two SMs per 256 x 128 tile) and the
    one-CTA kernel accumulate every output element in the same K order: bit-identical."""
    from tritonllmcompiler_b200 import _lib

    g = _gen(m + n + k)
    x = torch.randn(m, k, generator=g).to(_dt(dt)).cuda()
    w1 = (torch.randn(k, n, generator=g) / math.sqrt(k)).to(_dt(dt)).cuda()
    w3 = (torch.randn(k, n, generator=g) / math.sqrt(k)).to(_dt(dt)).cuda()
    outs = []
    for variant in (1, 2):
        o = torch.empty(m, n, dtype=x.dtype, device="cuda")
        _lib.check(_lib.load().tllm_swiglu_variant(
            x.data_ptr(), w1.data_ptr(), w3.data_ptr(), o.data_ptr(), m, n, k, k, n, n, n,
            _lib.DTYPE_CODES[x.dtype], variant, torch.cuda.current_stream().cuda_stream))
        outs.append(o)
    assert torch.equal(outs[0], outs[1])
    _assert_close(outs[1], O.swiglu(_f32(x.cpu()), _f32(w1.cpu()), _f32(w3.cpu()), dtype=dt))
    assert _lib.debug_status() == 0


def test_swiglu_strided_inputs(cuda_device):
    g = _gen(21)
    big = torch.randn(200, 264, generator=g).half()
    x = big[:, 8:200]  # lda = 264 > K = 192 (TMA path)
    w1 = (torch.randn(192, 136, generator=g) / 14).half()
    w3 = (torch.randn(192, 136, generator=g) / 14).half()
    out = T.swiglu(x.cuda(), w1.cuda(), w3.cuda())
    _assert_close(out, O.swiglu(_f32(x), _f32(w1), _f32(w3)))
    xt = torch.randn(192, 200, generator=g).half().t()  # column-major x -> copied
    out = T.swiglu(xt.cuda(), w1.cuda(), w3.cuda())
    _assert_close(out, O.swiglu(_f32(xt), _f32(w1), _f32(w3)))


def test_swiglu_zero_k(cuda_device):
    x = torch.empty(5, 0, dtype=torch.float16, device="cuda")
    w = torch.empty(0, 16, dtype=torch.float16, device="cuda")
    out = T.swiglu(x, w, w)
    assert out.shape == (5, 16) and torch.count_nonzero(out) == 0


def _no_subnormals(t):
    """Zero the fp16 subnormals: the doubling properties below hold for normal operands."""
    return t.masked_fill(t.abs() < torch.finfo(t.dtype).tiny, 0)


def test_swiglu_linearity_in_w3_is_exact(cuda_device):
    g = _gen(22)
    x = torch.randn(512, 1024, generator=g).half().cuda()
    w1 = (torch.randn(1024, 768, generator=g) / 32).half().cuda()
    w3 = _no_subnormals((torch.randn(1024, 768, generator=g) / 32).half().cuda())
    a = T.swiglu(x, w1, w3)
    b = T.swiglu(x, w1, w3 * 2)
    G.assert_doubled_exactly(a, b)


# ----------------------------------------------------------------------------- flash
@pytest.mark.parametrize("b,h,sq,sk,d,causal,dt", [
    (1, 2, 128, 128, 128, False, "fp16"),
    (1, 2, 128, 128, 128, True, "fp16"),
    (2, 3, 384, 384, 128, True, "fp16"),
    (1, 2, 257, 257, 64, True, "fp16"),
    (1, 2, 100, 700, 128, False, "bf16"),
    (1, 1, 700, 100, 64, True, "fp16"),
    (2, 2, 333, 333, 32, True, "bf16"),
    (1, 3, 200, 517, 16, False, "fp16"),
    (1, 1, 1, 1, 128, True, "fp16"),
])
def test_flash_random(cuda_device, b, h, sq, sk, d, causal, dt):
    g = _gen(b * 1000 + sq + sk + d)
    q = torch.randn(b, h, sq, d, generator=g).to(_dt(dt))
    k = torch.randn(b, h, sk, d, generator=g).to(_dt(dt))
    v = torch.randn(b, h, sk, d, generator=g).to(_dt(dt))
    out = T.flash_attention(q.cuda(), k.cuda(), v.cuda(), causal=causal)
    _assert_close(out, O.flash_attention(_f32(q), _f32(k), _f32(v), causal=causal, dtype=dt))


def test_flash_noncontiguous_and_scale(cuda_device):
    g = _gen(31)
    base = torch.randn(2, 300, 4, 64, generator=g).half()  # [B, S, H, D] storage
    q = base.permute(0, 2, 1, 3)  # [B, H, S, D] view with TMA-compatible strides
    k = torch.randn(2, 4, 300, 64, generator=g).half()
    v = torch.randn(2, 4, 300, 64, generator=g).half()
    out = T.flash_attention(q.cuda(), k.cuda(), v.cuda(), causal=True, sm_scale=0.05)
    _assert_close(out, O.flash_attention(_f32(q), _f32(k), _f32(v), causal=True, sm_scale=0.05))
    assert out.is_contiguous()


@pytest.mark.parametrize("causal", [False, True])
def test_flash_empty_keys_is_nan(cuda_device, causal):
    # Sk = 0 (torch hands the library null pointers for empty k/v): 0/0 in every row, as the
    # reference kernel gives.
    q = torch.randn(1, 2, 100, 64, generator=_gen(40)).half().cuda()
    k = torch.empty(1, 2, 0, 64, dtype=torch.float16, device="cuda")
    out = T.flash_attention(q, k, k, causal=causal)
    assert out.shape == q.shape and torch.isnan(out).all()


def test_flash_value_scaling_is_exact(cuda_device):
    g = _gen(32)
    q = torch.randn(2, 4, 1024, 128, generator=g).half().cuda()
    k = torch.randn(2, 4, 1024, 128, generator=g).half().cuda()
    v = _no_subnormals(torch.randn(2, 4, 1024, 128, generator=g).half().cuda())
    a = T.flash_attention(q, k, v, causal=True)
    b = T.flash_attention(q, k, v * 2, causal=True)
    G.assert_doubled_exactly(a, b)


# ----------------------------------------------------------------------------- paged
def _paged_case(seed, b, h, d, bs, lens, dt, extra_cols=2):
    g = _gen(seed)
    nb = [(n + bs - 1) // bs for n in lens]
    pool = sum(nb) + 5
    perm = torch.randperm(pool, generator=g)
    bt = torch.zeros(b, max(nb) + extra_cols, dtype=torch.int32)
    pos = 0
    for i, n in enumerate(nb):
        bt[i, :n] = perm[pos:pos + n].to(torch.int32)
        pos += n
    kc = torch.randn(pool, bs, h, d, generator=g).to(_dt(dt))
    vc = torch.randn(pool, bs, h, d, generator=g).to(_dt(dt))
    q = torch.randn(b, h, 1, d, generator=g).to(_dt(dt))
    return q, kc, vc, bt, torch.tensor(lens, dtype=torch.int32)


@pytest.mark.parametrize("b,h,d,bs,lens,dt", [
    (4, 8, 128, 16, [512, 8192, 1000, 17], "fp16"),
    (3, 4, 64, 32, [5000, 31, 33], "bf16"),
    (2, 2, 32, 64, [64, 65], "fp16"),
    (6, 2, 16, 16, [1, 2, 3, 4, 5, 2049], "fp16"),
    (1, 32, 128, 16, [4100], "fp16"),
])
def test_paged_random(cuda_device, b, h, d, bs, lens, dt):
    q, kc, vc, bt, cl = _paged_case(b * 31 + d + bs, b, h, d, bs, lens, dt)
    out = T.paged_attention(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), cl.cuda(), block_size=bs)
    ref = O.paged_attention(_f32(q), _f32(kc), _f32(vc), bt.numpy(), cl.numpy(), block_size=bs, dtype=dt)
    _assert_close(out, ref)


def test_paged_pool_permutation_is_exact(cuda_device):
    """Relabelling the physical blocks (cache rows and table entries alike) changes nothing."""
    q, kc, vc, bt, cl = _paged_case(41, 8, 8, 128, 16, [3000, 100, 7, 4096, 512, 1, 999, 2048], "fp16")
    pool = kc.shape[0]
    perm = torch.randperm(pool, generator=_gen(42))
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(pool)
    a = T.paged_attention(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), cl.cuda(), block_size=16)
    b = T.paged_attention(q.cuda(), kc[perm].cuda(), vc[perm].cuda(), inv[bt.long()].to(torch.int32).cuda(),
                          cl.cuda(), block_size=16)
    assert torch.equal(a, b)


def test_paged_zero_length_is_nan_like_reference_kernel(cuda_device):
    q, kc, vc, bt, cl = _paged_case(43, 2, 2, 64, 16, [0, 20], "fp16")
    out = T.paged_attention(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), cl.cuda(), block_size=16)
    assert torch.isnan(out[0].float()).all()
    ref = O.paged_attention(_f32(q[1:]), _f32(kc), _f32(vc), bt[1:].numpy(), cl[1:].numpy(), block_size=16)
    _assert_close(out[1:], ref)


def test_paged_out_of_range_table_entry_is_clamped_and_reported(cuda_device):
    from tritonllmcompiler_b200 import _lib

    q, kc, vc, bt, cl = _paged_case(44, 1, 2, 64, 16, [40], "fp16")
    torch.cuda.synchronize()
    assert _lib.debug_status() == 0
    bt[0, 1] = kc.shape[0] + 100  # outside the pool: the kernel clamps it, never reads there
    T.paged_attention(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), cl.cuda(), block_size=16)
    torch.cuda.synchronize()
    assert _lib.debug_status() == 0x200
    assert _lib.debug_status() == 0  # reading clears it


def test_paged_int64_metadata_and_strided_q(cuda_device):
    q, kc, vc, bt, cl = _paged_case(45, 3, 4, 128, 16, [100, 200, 300], "fp16")
    qw = torch.randn(3, 4, 2, 128).half()
    qw[:, :, 0] = q[:, :, 0]
    qs = qw[:, :, :1]  # non-contiguous q view
    out = T.paged_attention(qs.cuda(), kc.cuda(), vc.cuda(), bt.long().cuda(), cl.long().cuda(), block_size=16)
    ref = O.paged_attention(_f32(q), _f32(kc), _f32(vc), bt.numpy(), cl.numpy(), block_size=16)
    _assert_close(out, ref)


@pytest.mark.parametrize("b,h,s,d,causal", [(2, 4, 1000, 128, True), (1, 4, 384, 64, False),
                                            (1, 2, 300, 32, True), (1, 2, 257, 16, False),
                                            (4, 64, 2048, 128, True), (2, 32, 1536, 64, False)])
def test_flash_kernel_variants_agree(cuda_device, b, h, s, d, causal):
    """The two-tile kernel (work stealing, the default), the single-tile kernel, the two-tile
    kernel with one item per CTA and the two-tile kernel with P in shared memory agree; work
    stealing changes only which CTA computes an item, and P holds the same values in TMEM or in
    shared memory, so variants 0, 2 and 3 match bit for bit."""
    from tritonllmcompiler_b200 import _lib

    g = _gen(s + d)
    q, k, v = (torch.randn(b, h, s, d, generator=g).half().cuda() for _ in range(3))
    outs = []
    for variant in (0, 1, 2, 3):
        o = torch.empty_like(q)
        _lib.check(_lib.load().tllm_flash_attn_fwd_variant(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), b, h, s, s, d,
            _lib.strides(q), _lib.strides(k), _lib.strides(v), _lib.strides(o),
            d ** -0.5, int(causal), 0, variant, torch.cuda.current_stream().cuda_stream))
        outs.append(o)
    for o in outs[1:]:
        assert torch.allclose(outs[0].float(), o.float(), **G.tol(torch.float16))
    assert torch.equal(outs[0], outs[2])
    assert torch.equal(outs[0], outs[3])
    assert _lib.debug_status() == 0
