"""The oracle's correctly rounded router logits (CPU).

The logit of (token, expert) is the model-dtype rounding (nearest, ties to
even) of the exact dot product.  These tests pin the integer rounding helper
against torch's own conversions and the fp64 + bound + integer-fallback scheme
against cases where plain fp64 accumulation rounds the wrong way.
"""
from fractions import Fraction

import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo

DTYPES = [torch.bfloat16, torch.float16]


@pytest.mark.parametrize("dtype", DTYPES)
def test_round_scaled_int_matches_torch(dtype):
    rng = np.random.default_rng(5)
    vals = np.concatenate([rng.standard_normal(2000) * 10.0 ** rng.integers(-6, 4, 2000),
                           [2.0 ** -133, 3 * 2.0 ** -134, 2.0 ** -24, 2.0 ** -25 * 3, 65504.0]])
    for v in vals:
        n = int(np.ldexp(v, 400))                  # v is exactly n * 2^-400
        got = mo.round_scaled_int(n, -400, dtype)
        want = torch.tensor(v, dtype=torch.float64).to(dtype).item()
        assert got == want, (v, got, want)


def test_round_scaled_int_ties_to_even():
    bf = torch.bfloat16
    one = 1 << 100
    assert mo.round_scaled_int(one + (one >> 8), -100, bf) == 1.0                  # 1 + 2^-8 -> 1
    assert mo.round_scaled_int(one + 3 * (one >> 8), -100, bf) == 1.0 + 2.0 ** -6  # odd neighbour -> up
    assert mo.round_scaled_int(-(one + (one >> 8)), -100, bf) == -1.0


@pytest.mark.parametrize("dtype", DTYPES)
def test_exact_dot_round_against_fractions(dtype):
    rng = np.random.default_rng(11)
    for _ in range(20):
        a = torch.from_numpy(rng.standard_normal(64)).to(dtype).double().numpy()
        b = torch.from_numpy(rng.standard_normal(64) * 0.02).to(dtype).double().numpy()
        exact = sum(Fraction(x) * Fraction(y) for x, y in zip(a, b))
        # correctly rounded: compare with the neighbours of the result
        got = mo.exact_dot_round(a, b, dtype)
        gf = Fraction(got)
        up = Fraction(torch.tensor(got, dtype=dtype).view(torch.int16).add(1 if got >= 0 else -1)
                      .view(dtype).double().item()) if got != 0 else None
        assert abs(exact - gf) <= abs(exact - up) if up is not None else True


def test_cancellation_case_fp64_alone_is_wrong():
    """Products 2^60, 1, -2^60, 2^-9: the exact sum 1 + 2^-9 is a bf16 tie and
    rounds to 1.0; fp64 accumulation loses the 1 and gives 2^-9."""
    bf = torch.bfloat16
    h = torch.tensor([[2.0 ** 40, 1.0, -2.0 ** 40, 2.0 ** -9, 0, 0, 0, 0]], dtype=torch.float64).to(bf)
    w = torch.tensor([[2.0 ** 20, 1.0, 2.0 ** 20, 1.0, 0, 0, 0, 0],
                      [1.0, 0, 0, 0, 0, 0, 0, 0]], dtype=torch.float64).to(bf)
    acc = 0.0                                      # left-to-right fp64 accumulation
    for x, y in zip(h[0].double().tolist(), w[0].double().tolist()):
        acc += x * y
    assert mo.round_f64(np.array([acc]), bf)[0].item() == 2.0 ** -9
    lg = mo.router_logits(h, w)
    assert lg[0, 0].item() == 1.0
    assert lg[0, 1].item() == 2.0 ** 40


def test_exact_logits_equal_fp64_rounding_on_generic_data():
    rng = np.random.default_rng(3)
    h = torch.from_numpy(rng.standard_normal((8, 512))).to(torch.bfloat16)
    w = torch.from_numpy(rng.standard_normal((64, 512)) * 0.02).to(torch.bfloat16)
    lg = mo.router_logits(h, w)
    ref = mo.round_f64(h.double().numpy() @ w.double().numpy().T, torch.bfloat16)
    assert torch.equal(lg.view(torch.int16), ref.view(torch.int16))
