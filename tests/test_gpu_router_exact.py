"""Router logits on the device are the correctly rounded exact dot products.

Crafted rows make the fp32 TwoSum bound inconclusive (products 2^30, 1, -2^30,
2^-9: the running sum loses the 1 and the exact value is a bf16 tie), so the
kernels must take their exact integer path; rows of zeros and mirrored rows
produce exact ties, +0 and -0 logits for the top-k order.  Every case is
compared bit for bit with the oracle (fp64 + bound + integer fallback).
"""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo
from tarfa_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tarfa_b200 import build
    build.build()


def crafted(T, E, H, dtype, seed=0):
    """Tokens and router rows with cancellation, exact ties and signed zeros."""
    rng = np.random.default_rng(seed)
    h = rng.standard_normal((T, H))
    w = rng.standard_normal((E, H)) * 0.02
    small = 2.0 ** -9 if dtype == torch.bfloat16 else 2.0 ** -11
    for t in range(T):
        sgn = -1.0 if t % 2 else 1.0
        h[t, :4] = [sgn * 2.0 ** 15, sgn, -sgn * 2.0 ** 15, sgn * small]
    for e in range(0, E, 4):     # exact sum 1 + small (tie, to even: 1.0)
        w[e] = 0.0
        w[e, :4] = [2.0 ** 15, 1.0, 2.0 ** 15, 1.0]
    for e in range(1, E, 8):     # exact sum 1 + 3 small (tie, to even: up)
        w[e] = 0.0
        w[e, :4] = [2.0 ** 15, 1.0, 2.0 ** 15, 3.0]
    for e in range(2, E, 8):     # exact zero: +0 and -0 candidates
        w[e] = 0.0
    ht = torch.from_numpy(h).to(dtype)
    wt = torch.from_numpy(w).to(dtype)
    return ht, wt


def _check(h, w, k, bias=None):
    idx_o, w_o, lg_o = mo.router_topk(h, w, k, bias)
    idx, wt, lg = ops.router_topk(h.to(DEV), w.to(DEV), k, None if bias is None else bias.to(DEV),
                                  return_logits=True)
    torch.cuda.synchronize()
    assert torch.equal(lg.cpu().to(h.dtype).view(torch.int16), lg_o.view(torch.int16)), \
        "logits differ from the correctly rounded values"
    assert torch.equal(idx.cpu(), idx_o)
    assert torch.allclose(wt.cpu(), w_o, rtol=2e-6, atol=0)
    return lg_o


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T", [1, 3, 16])
def test_decode_router_exact_on_crafted_rows(dtype, T):
    h, w = crafted(T, 64, 256, dtype, seed=T)
    lg = _check(h, w, 8)
    # the crafted rows did hit the ties the fp32 sum alone rounds the wrong way
    assert (lg[0, 0::4].float() == 1.0).all()
    assert (lg[0, 1::8].float() == (1.0 + 2.0 ** -7 if dtype == torch.bfloat16 else 1.0 + 2.0 ** -9)).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T", [256, 64])
def test_prefill_router_exact_on_crafted_rows(dtype, T):
    # 48 tokens or more with 128 experts take the tensor-core logits + fix-up
    # route (64: half of one 128-row tile)
    h, w = crafted(T, 128, 512, dtype, seed=9)
    _check(h, w, 8)


def test_topk_tie_order_and_signed_zero():
    T, E, H = 4, 32, 64
    h = torch.zeros((T, H))
    h[:, 0] = torch.tensor([1.0, -1.0, 0.0, 2.0])
    w = torch.zeros((E, H))
    w[::3, 0] = 0.5          # many equal logits
    w[1::3, 0] = -0.0        # +0 / -0 logits mixed with zeros
    _check(h.to(torch.bfloat16), w.to(torch.bfloat16), 8)
