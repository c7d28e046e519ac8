"""The paged-KV oracle (append, fused append+RoPE, multi-token GQA attention) agrees with the
reference-pinned oracle functions it is built from (CPU only)."""
import ctypes

import numpy as np

from oracle import ops_oracle as O
from oracle import paged_kv_oracle as P
from tritonllmcompiler_b200 import _lib


def _h(rng, *shape):
    return O.round_to(rng.standard_normal(shape).astype(np.float32), "fp16")


def _tables(rng, lens, bs, extra=0):
    nb = [(n + bs - 1) // bs for n in lens]
    pool = sum(nb) + extra
    perm = rng.permutation(pool)
    bt = np.zeros((len(lens), max(nb) if nb else 1), np.int32)
    i = 0
    for b, n in enumerate(nb):
        bt[b, :n] = perm[i:i + n]
        i += n
    return bt, pool


def _gather(cache, bt, b, n, bs):
    nblk = (n + bs - 1) // bs
    return cache[bt[b, :nblk]].reshape(-1, *cache.shape[2:])[:n]


def test_append_then_gather_returns_the_new_tokens():
    rng = np.random.default_rng(0)
    bs, h, d = 16, 3, 32
    start = np.array([0, 5, 31], np.int32)
    T = 20
    bt, pool = _tables(rng, [s + T for s in start], bs)
    kc = _h(rng, pool, bs, h, d)
    vc = _h(rng, pool, bs, h, d)
    kn, vn = _h(rng, 3, T, h, d), _h(rng, 3, T, h, d)
    n_new = np.array([20, 7, 0], np.int32)
    k2, v2 = P.paged_kv_append(kn, vn, kc, vc, bt, start, n_new, block_size=bs)
    for b in range(3):
        n = int(n_new[b])
        got = _gather(k2, bt, b, int(start[b]) + n, bs)
        np.testing.assert_array_equal(got[start[b]:], kn[b, :n])
        np.testing.assert_array_equal(_gather(v2, bt, b, int(start[b]) + n, bs)[start[b]:], vn[b, :n])
        # tokens before start_pos are untouched
        np.testing.assert_array_equal(got[:start[b]], _gather(kc, bt, b, int(start[b]), bs))


def test_append_rope_rotates_k_at_absolute_positions():
    rng = np.random.default_rng(1)
    bs, h, d, T = 16, 2, 64, 6
    start = np.array([3, 40], np.int32)
    bt, pool = _tables(rng, [s + T for s in start], bs)
    kc = np.zeros((pool, bs, h, d), np.float32)
    vc = np.zeros_like(kc)
    kn, vn = _h(rng, 2, T, h, d), _h(rng, 2, T, h, d)
    w = O.round_to(1 + 0.1 * rng.standard_normal(d).astype(np.float32), "fp16")
    cos = O.round_to(np.cos(rng.standard_normal((64, d))).astype(np.float32), "fp16")
    sin = O.round_to(np.sin(rng.standard_normal((64, d))).astype(np.float32), "fp16")
    k2, v2 = P.paged_kv_append_rope(kn, vn, w, cos, sin, kc, vc, bt, start, block_size=bs)
    for b in range(2):
        pos = start[b] + np.arange(T)
        want = O.rmsnorm_rope(kn[b:b + 1], w, cos[pos], sin[pos], dtype="fp16")[0]
        np.testing.assert_array_equal(_gather(k2, bt, b, int(start[b]) + T, bs)[start[b]:], want)
        np.testing.assert_array_equal(_gather(v2, bt, b, int(start[b]) + T, bs)[start[b]:], vn[b])


def test_prefill_with_one_token_and_equal_heads_is_the_reference_decode():
    rng = np.random.default_rng(2)
    bs, h, d = 16, 4, 32
    lens = np.array([1, 17, 64, 100], np.int32)
    bt, pool = _tables(rng, lens, bs, extra=3)
    kc, vc = _h(rng, pool, bs, h, d), _h(rng, pool, bs, h, d)
    q = _h(rng, 4, h, 1, d)
    a = P.paged_attention_prefill(q, kc, vc, bt, lens, block_size=bs)
    b = O.paged_attention(q, kc, vc, bt, lens, block_size=bs)
    np.testing.assert_allclose(a, b, rtol=0, atol=1e-3)


def test_prefill_of_a_whole_sequence_is_causal_flash_attention():
    rng = np.random.default_rng(3)
    bs, h, d, n = 16, 2, 32, 45
    bt, pool = _tables(rng, [n], bs)
    kc, vc = _h(rng, pool, bs, h, d), _h(rng, pool, bs, h, d)
    q = _h(rng, 1, h, n, d)
    got = P.paged_attention_prefill(q, kc, vc, bt, np.array([n]), block_size=bs, causal=True)
    k = np.transpose(_gather(kc, bt, 0, n, bs), (1, 0, 2))[None]
    v = np.transpose(_gather(vc, bt, 0, n, bs), (1, 0, 2))[None]
    want = O.flash_attention(q, k, v, causal=True)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-3)


def test_prefill_gqa_reads_the_shared_kv_head():
    rng = np.random.default_rng(4)
    bs, hkv, g, d, sq = 16, 2, 3, 32, 4
    lens = np.array([9, 33], np.int32)
    bt, pool = _tables(rng, lens, bs)
    kc, vc = _h(rng, pool, bs, hkv, d), _h(rng, pool, bs, hkv, d)
    q = _h(rng, 2, hkv * g, sq, d)
    got = P.paged_attention_prefill(q, kc, vc, bt, lens, block_size=bs)
    for hq in range(hkv * g):
        kvh = hq // g
        one = P.paged_attention_prefill(q[:, hq:hq + 1], kc[:, :, kvh:kvh + 1],
                                        vc[:, :, kvh:kvh + 1], bt, lens, block_size=bs)
        np.testing.assert_array_equal(got[:, hq:hq + 1], one)


def test_prefill_query_without_visible_keys_is_nan():
    rng = np.random.default_rng(5)
    bt, pool = _tables(rng, [2], 16)
    kc = vc = _h(rng, pool, 16, 1, 16)
    q = _h(rng, 1, 1, 4, 16)
    out = P.paged_attention_prefill(q, kc, vc, bt, np.array([2]), block_size=16)
    # queries 0 and 1 sit at positions -2 and -1: nothing visible
    assert np.isnan(out[0, 0, :2]).all() and np.isfinite(out[0, 0, 2:]).all()


def _arr(*v):
    return (ctypes.c_int64 * len(v))(*v)


def test_append_entry_points_validate_arguments_without_a_gpu():
    lib = _lib.load()
    s = _arr(8, 8, 8, 1)
    rc = lib.tllm_paged_kv_append(8, 8, 8, 8, 8, 8, None, 1, 1, 1, 48, 16, 1, 1, s, s, s, s,
                                  _arr(1, 1), 0, None)
    assert rc != 0 and b"head dim 48" in lib.tllm_last_error()
    rc = lib.tllm_paged_kv_append_rope(16, 16, None, None, None, 1, 8, 8, 16, 16, 8, 8, None, 1,
                                       1, 1, 64, 16, 1, 1, s, s, s, s, _arr(1, 1), 1e-6, 0, None)
    assert rc != 0 and b"weight/cos/sin" in lib.tllm_last_error()
    # nothing to do: no error, no CUDA call
    assert lib.tllm_paged_kv_append(None, None, None, None, None, None, None, 0, 4, 2, 64, 16, 1,
                                    1, s, s, s, s, _arr(1, 1), 0, None) == 0
