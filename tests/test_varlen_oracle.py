"""The packed (variable-length) attention oracle against the reference-pinned dense oracle,
and the C entry point's argument checks (CPU only)."""
import ctypes

import numpy as np

from oracle import ops_oracle as O
from oracle import varlen_oracle as V
from tritonllmcompiler_b200 import _lib


def _h(rng, *shape):
    return O.round_to(rng.standard_normal(shape).astype(np.float32), "fp16")


def test_equal_lengths_match_the_dense_oracle():
    rng = np.random.default_rng(0)
    B, H, S, D = 3, 2, 37, 32
    q, k, v = (_h(rng, B, H, S, D) for _ in range(3))
    cu = np.arange(B + 1) * S
    pack = lambda t: np.transpose(t, (0, 2, 1, 3)).reshape(B * S, H, D)  # noqa: E731
    for causal in (False, True):
        dense = O.flash_attention(q, k, v, causal=causal)
        got = V.flash_attention_varlen(pack(q), pack(k), pack(v), cu, cu, causal=causal)
        np.testing.assert_array_equal(got, pack(dense))


def test_gqa_and_ragged_lengths_are_per_sequence():
    rng = np.random.default_rng(1)
    lq, lk = [5, 0, 70, 1], [9, 3, 70, 40]
    H, Hkv, D = 4, 2, 16
    cq, ck = np.cumsum([0] + lq), np.cumsum([0] + lk)
    q, k, v = _h(rng, cq[-1], H, D), _h(rng, ck[-1], Hkv, D), _h(rng, ck[-1], Hkv, D)
    got = V.flash_attention_varlen(q, k, v, cq, ck)
    for b in range(4):
        if lq[b] == 0:
            continue
        for h in range(H):
            qs = q[cq[b]:cq[b + 1], h][None, None]
            ks = k[ck[b]:ck[b + 1], h // 2][None, None]
            vs = v[ck[b]:ck[b + 1], h // 2][None, None]
            np.testing.assert_array_equal(got[cq[b]:cq[b + 1], h], O.flash_attention(qs, ks, vs)[0, 0])


def test_entry_point_validates_without_a_gpu():
    lib = _lib.load()
    s = (ctypes.c_int64 * 3)(8, 8, 1)
    rc = lib.tllm_flash_attn_varlen_fwd(16, 16, 16, 16, 16, 16, 2, 6, 4, 10, 10, 5, 5, 64, s, s, s,
                                        s, 0.1, 0, 0, None)
    assert rc != 0 and b"do not group" in lib.tllm_last_error()
    rc = lib.tllm_flash_attn_varlen_fwd(16, 16, 16, 16, 16, 16, 2, 4, 4, 10, 10, 5, 5, 48, s, s, s,
                                        s, 0.1, 0, 0, None)
    assert rc != 0 and b"head dim 48" in lib.tllm_last_error()
    assert lib.tllm_flash_attn_varlen_fwd(None, None, None, None, None, None, 0, 4, 4, 0, 0, 0, 0,
                                          64, s, s, s, s, 0.1, 0, 0, None) == 0
