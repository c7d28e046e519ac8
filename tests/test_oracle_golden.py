"""Pins the numpy oracle to the reference's own outputs (golden fixtures; CPU only)."""
import numpy as np
import pytest

from oracle import ops_oracle as O
from tests import _golden as G


def _ulp_close(got: np.ndarray, want: np.ndarray, dtype: str, max_bad_frac: float = 0.0):
    """got == want except for rare one-ulp differences from fp32 summation order."""
    assert got.shape == want.shape
    tol = np.abs(want) * (2.0 ** -10 if dtype == "fp16" else 2.0 ** -7) + 1e-6
    bad = np.abs(got - want) > tol
    assert bad.mean() <= max_bad_frac, f"{bad.sum()} of {bad.size} beyond one ulp"
    assert np.allclose(got, want, atol=G.ATOL, rtol=G.RTOL)


@pytest.mark.parametrize("name", G.names("flash"))
def test_flash_oracle_matches_reference(name):
    c = G.load(name)
    got = O.flash_attention(G.to_f32(c["q"]), G.to_f32(c["k"]), G.to_f32(c["v"]),
                            causal=bool(c["causal"]), sm_scale=float(c["sm_scale"]), dtype=c["dtype"])
    _ulp_close(got, G.to_f32(c["out"]), c["dtype"], 1e-3)


@pytest.mark.parametrize("name", G.names("paged"))
def test_paged_oracle_matches_reference(name):
    c = G.load(name)
    got = O.paged_attention(G.to_f32(c["q"]), G.to_f32(c["k_cache"]), G.to_f32(c["v_cache"]),
                            c["block_tables"].numpy(), c["context_lens"].numpy(),
                            block_size=int(c["block_size"]), sm_scale=float(c["sm_scale"]),
                            dtype=c["dtype"])
    _ulp_close(got, G.to_f32(c["out"]), c["dtype"], 1e-3)


@pytest.mark.parametrize("name", G.names("rmsnorm_rope"))
def test_rmsnorm_rope_oracle_matches_reference(name):
    c = G.load(name)
    got = O.rmsnorm_rope(G.to_f32(c["x"]), G.to_f32(c["w"]), G.to_f32(c["cos"]), G.to_f32(c["sin"]),
                         float(c["eps"]), dtype=c["dtype"])
    _ulp_close(got, G.to_f32(c["out"]), c["dtype"], 1e-2)


@pytest.mark.parametrize("name", G.names("swiglu"))
def test_swiglu_oracle_matches_reference(name):
    c = G.load(name)
    got = O.swiglu(G.to_f32(c["x"]), G.to_f32(c["w1"]), G.to_f32(c["w3"]), dtype=c["dtype"])
    _ulp_close(got, G.to_f32(c["out"]), c["dtype"], 1e-3)


def test_round_to_bf16_is_round_nearest_even():
    import torch

    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 100
    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(O.round_to(x, "bf16"), want)
    assert np.array_equal(O.bf16_bits_to_f32(O.f32_to_bf16_bits(want)), want)


def test_oracle_detects_a_planted_error():
    """A deliberately wrong oracle variant (scale off by 1%) must fail the golden check."""
    c = G.load("flash__reftest_s128_causal")
    got = O.flash_attention(G.to_f32(c["q"]), G.to_f32(c["k"]), G.to_f32(c["v"]),
                            causal=True, sm_scale=float(c["sm_scale"]) * 1.01, dtype="fp16")
    with pytest.raises(AssertionError):
        _ulp_close(got, G.to_f32(c["out"]), "fp16", 1e-3)
