"""GPU parity of the tcgen05 grouped-GEMM (batched / prefill) path against the
CPU oracle (the reference's T > 1 branch, fused_int4.py:227-248).

Bars: top-k indices bit-exact; model-dtype outputs max|err| <= 2^-7 * max|ref|
and cosine >= 0.99999 (``gpu_helpers``).
"""
import pytest
import torch

from gpu_helpers import assert_close
from oracle import moe_oracle as mo
from tarfa_b200 import ops
from tarfa_b200 import synthetic as syn

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tarfa_b200 import build
    build.build()
    ops.device_status(clear=True)
    ops.set_gemm_min_tokens(1)          # force the GEMM path for every dense call here
    yield
    ops.set_gemm_min_tokens(64)
    torch.cuda.synchronize()
    assert ops.device_status() == 0, "a kernel raised a device status bit (timeout / bad id)"


SMALL = syn.LayerShape(hidden=256, experts=16, inter=128, shared_inter=128)


@pytest.mark.parametrize("T", [2, 37, 300])
def test_gemm_experts_small(T):
    s = SMALL
    gu, dn = syn.layer_cpu(3, 0, s)
    h = syn.tokens_cpu(3, T, s)
    idx, w, _ = mo.router_topk(h, syn.router_cpu(3, 0, s), 8)
    ref = mo.experts_exact(h, idx, w, lambda e: (gu[e], dn[e]), s.experts)
    out = ops.experts_forward(h.to(DEV), idx.to(DEV), w.to(DEV),
                              ops.ExpertWeights(gu.to(DEV), dn.to(DEV)))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert_close(out, ref, f"gemm experts T={T}")


@pytest.mark.parametrize("shape,T", [(syn.L0, 64), (syn.L0, 133), (SMALL, 17)])
def test_gemm_moe_layer(shape, T):
    s = shape
    seed = 5
    h = syn.tokens_cpu(seed, T, s)
    w_r = syn.router_cpu(seed, 0, s)
    sh = syn.shared_cpu(seed, 0, s)
    gu, dn = syn.layer_cpu(seed, 0, s)
    idx_o, w_o, _ = mo.router_topk(h, w_r, 8)
    ref = mo.experts_exact(h, idx_o, w_o, lambda e: (gu[e], dn[e]), s.experts) + \
        mo.shared_expert(h, *sh)
    out, idx, _ = ops.moe_layer(h.to(DEV), w_r.to(DEV), ops.ExpertWeights(gu.to(DEV), dn.to(DEV)),
                                ops.SharedWeights(*[t.to(DEV) for t in sh]), return_routing=True)
    torch.cuda.synchronize()
    assert torch.equal(idx.cpu(), idx_o)
    assert_close(out, ref, f"gemm moe_layer T={T}")


@pytest.fixture(scope="module")
def l1_layer():
    return syn.layer_device(0, syn.L1, DEV)


def _l1_ref(L, h, bias):
    s = syn.L1
    w_r = L["router"].cpu()
    sh = [L[k].cpu() for k in ("sh_gate", "sh_up", "sh_down", "sh_gate_w")]
    idx_o, w_o, _ = mo.router_topk(h, w_r, 8, bias)
    cache = {}

    def get(e):
        if e not in cache:
            cache[e] = (L["gate_up"][e].cpu(), L["down"][e].cpu())
        return cache[e]
    ref = mo.experts_exact(h, idx_o, w_o, get, s.experts) + mo.shared_expert(h, *sh)
    return idx_o, ref


@pytest.mark.parametrize("T,zipf", [(512, False), (4096, True)])
def test_gemm_config_prefill(l1_layer, T, zipf):
    """Config 1 layer at batched / prefill sizes; 4096 tokens with the Zipf(1.1)
    per-expert router bias (config 3: uneven segments, some experts empty)."""
    L = l1_layer
    h = syn.tokens_cpu(9, T, syn.L1, stream=5)
    bias = torch.from_numpy(syn.zipf_bias(0, syn.L1.experts)).to(torch.bfloat16) if zipf else None
    idx_o, ref = _l1_ref(L, h, bias)
    out, idx, _ = ops.moe_layer(h.to(DEV), L["router"], ops.ExpertWeights(L["gate_up"], L["down"]),
                                ops.SharedWeights(L["sh_gate"], L["sh_up"], L["sh_down"], L["sh_gate_w"]),
                                bias=None if bias is None else bias.to(DEV), return_routing=True)
    torch.cuda.synchronize()
    assert torch.equal(idx.cpu(), idx_o)
    if zipf:
        counts = torch.bincount(idx_o.flatten(), minlength=syn.L1.experts)
        assert int((counts == 0).sum()) > 0 and int(counts.max()) > 4 * int(counts.float().mean())
    assert_close(out, ref, f"config1 prefill T={T}")
