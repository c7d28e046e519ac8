"""The FP8 attention oracle and its error bound, and the host-side e4m3 packing, on the CPU."""
import numpy as np
import torch

from oracle import fp8_attn_oracle as F
from oracle import ops_oracle as O
from tritonllmcompiler_b200.ops.flash_fp8 import quantize_qkv_e4m3, transpose_v_e4m3


def _e4m3(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.float8_e4m3fn).float().numpy()


def test_oracle_is_the_reference_definition_on_dequantized_inputs():
    g = np.random.default_rng(0)
    q8, k8, v8 = (_e4m3(g.standard_normal((1, 2, 33, 64)) * 4) for _ in range(3))
    for causal in (False, True):
        got = F.flash_attention_fp8(q8, k8, v8, 0.5, 0.25, 2.0, causal=causal)
        ref = O.flash_attention(q8 * 0.5, k8 * 0.25, v8 * 2.0, causal=causal, dtype="fp32")
        np.testing.assert_array_equal(got, ref)


def test_bound_covers_e4m3_probabilities():
    # Rounding the probabilities to e4m3 (relative to the row max, the worst case for the
    # subnormal range) stays within the bound the GPU test uses.
    g = np.random.default_rng(1)
    for causal in (False, True):
        q8, k8, v8 = (_e4m3(g.standard_normal((1, 1, 200, 64)) * 8) for _ in range(3))
        s = 1.0 / 8
        q, k, v = q8 * s, k8 * s, v8 * s
        sc = (q @ np.swapaxes(k, -1, -2)) * np.float32(64 ** -0.5)
        if causal:
            sc = np.where(np.triu(np.ones(sc.shape[-2:], bool), 1), -np.inf, sc)
        p = np.exp2((sc - sc.max(-1, keepdims=True)) * np.log2(np.e)).astype(np.float32)
        sim = (_e4m3(p) @ v) / p.sum(-1, keepdims=True)
        ref = F.flash_attention_fp8(q8, k8, v8, s, s, s, causal=causal)
        bound = F.error_bound(q8, k8, v8, s, s, s, causal=causal)
        tol = bound + 2.0 ** -9 * np.abs(v).max() + 1e-6
        assert np.all(np.abs(sim - ref) <= tol)
        # and the bound is not vacuous: the e4m3 error is a sizeable fraction of it
        assert np.abs(sim - ref).max() > 0.05 * bound.max()


def test_quantize_and_transposed_v_layout():
    g = torch.Generator().manual_seed(2)
    q, k, v = (torch.randn(2, 3, 37, 64, generator=g) for _ in range(3))
    q8, k8, vt8, sq, sk, sv = quantize_qkv_e4m3(q, k, v)
    assert q8.dtype == torch.float8_e4m3fn and vt8.shape == (2, 3, 64, 37)
    assert vt8.stride(-1) == 1 and all(x % 16 == 0 for x in vt8.stride()[:-1])
    v8 = vt8.transpose(-1, -2)
    for t, t8, sc in ((q, q8, sq), (k, k8, sk), (v, v8, sv)):
        err = (t - t8.float() * sc).abs()
        assert torch.all(err <= 2.0 ** -4 * t.abs() + 2.0 ** -9 * sc)
    # the padding past the keys is zero
    base = vt8.view(torch.uint8).as_strided((2, 3, 64, 48), vt8.stride())
    assert torch.all(base[..., 37:] == 0)
    # repacking an already transposed tensor is the identity
    assert torch.equal(transpose_v_e4m3(v8).view(torch.uint8), vt8.view(torch.uint8))
