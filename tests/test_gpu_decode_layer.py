"""GPU parity of the decode layer (router, in-GEMV routing, expert GEMVs,
combine) against the CPU oracle, on dense and int4 experts, across workspace
reuse and graph replay.

Bars: top-k indices bit-exact; outputs max|err| <= 2^-7 * max|ref| and cosine
>= 0.99999 (``gpu_helpers``).
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
    yield
    torch.cuda.synchronize()
    assert ops.device_status() == 0, "a kernel raised a device status bit (timeout / bad id)"


@pytest.fixture(scope="module")
def l1():
    return syn.layer_device(0, syn.L1, DEV)


def _shared(L):
    return ops.SharedWeights(L["sh_gate"], L["sh_up"], L["sh_down"], L["sh_gate_w"])


@pytest.mark.parametrize("T", [1, 2, 7, 9, 16])
def test_decode_layer_vs_oracle(l1, T):
    L = l1
    h = syn.tokens_cpu(21, T, syn.L1, stream=2)
    w = ops.ExpertWeights(L["gate_up"], L["down"])
    out, idx, wts = ops.moe_layer(h.to(DEV), L["router"], w, _shared(L), return_routing=True)
    torch.cuda.synchronize()
    idx_o, w_o, _ = mo.router_topk(h, L["router"].cpu(), 8)
    assert torch.equal(idx.cpu(), idx_o)
    torch.testing.assert_close(wts.cpu(), w_o, rtol=2e-6, atol=0)
    ref = mo.experts_exact(h, idx_o, w_o, lambda e: (L["gate_up"][e].cpu(), L["down"][e].cpu()),
                           syn.L1.experts) + mo.shared_expert(h, *[L[k].cpu() for k in
                                                                   ("sh_gate", "sh_up", "sh_down", "sh_gate_w")])
    assert_close(out, ref, f"decode layer vs oracle T={T}")


@pytest.mark.parametrize("T,group", [(1, 128), (4, 128), (16, 128), (1, 0), (3, 0)])
def test_int4_layer(T, group):
    """Fast mode through the whole layer: int4 routed experts + bf16 shared expert."""
    s = syn.LayerShape(hidden=1024, experts=64, inter=512, shared_inter=256)
    dtype = torch.bfloat16
    seed = 30 + T
    q = [syn.q4_expert_reflayout(seed, e, s, dtype) for e in range(s.experts)]
    gq = torch.stack([x[0] for x in q]).view(torch.int32)
    dq = torch.stack([x[2] for x in q]).view(torch.int32)
    if group == 0:
        gs = torch.stack([x[1] for x in q])
        ds = torch.stack([x[3] for x in q])
    else:
        g = torch.Generator().manual_seed(seed)
        gs = (torch.rand(s.experts, 2 * s.inter, s.hidden // group, generator=g) * 0.004 + 0.001).to(dtype)
        ds = (torch.rand(s.experts, s.hidden, s.inter // group, generator=g) * 0.004 + 0.001).to(dtype)
    h = syn.tokens_cpu(seed, T, s)
    w_r = syn.router_cpu(seed, 0, s)
    sh = syn.shared_cpu(seed, 0, s)
    idx_o, w_o, _ = mo.router_topk(h, w_r, 8)

    def get_q4(e):
        return (gq[e].view(torch.uint8), gs[e], dq[e].view(torch.uint8), ds[e])
    ref = mo.experts_int4(h, idx_o, w_o, get_q4, s.experts, group or None) + mo.shared_expert(h, *sh)
    wts = ops.ExpertWeights(gq.to(DEV), dq.to(DEV), "int4", gs.to(DEV), ds.to(DEV), group)
    out, idx, _ = ops.moe_layer(h.to(DEV), w_r.to(DEV), wts, ops.SharedWeights(*[t.to(DEV) for t in sh]),
                                return_routing=True)
    torch.cuda.synchronize()
    assert torch.equal(idx.cpu(), idx_o)
    assert_close(out, ref, f"int4 layer T={T} group={group}")


def test_layer_reuses_workspace_across_calls(l1):
    """Back-to-back layer calls and an interleaved experts_forward on the shared
    workspace: the zero-at-rest counters must survive every sequence."""
    L = l1
    w = ops.ExpertWeights(L["gate_up"], L["down"])
    h = syn.tokens_cpu(3, 4, syn.L1).to(DEV)
    first = ops.moe_layer(h, L["router"], w, _shared(L))
    for _ in range(3):
        idx = torch.randint(0, 256, (2, 8), device=DEV)
        ops.experts_forward(h[:2].contiguous(), idx, torch.full((2, 8), 0.125, device=DEV), w)
        again = ops.moe_layer(h, L["router"], w, _shared(L))
        torch.cuda.synchronize()
        assert torch.equal(first, again)


def test_layer_graph_replay(l1):
    L = l1
    w = ops.ExpertWeights(L["gate_up"], L["down"])
    h = syn.tokens_cpu(4, 1, syn.L1).to(DEV)
    plan = ops.MoePlan(h.clone(), L["router"], w, _shared(L))
    g = plan.capture()
    ref = ops.moe_layer(h, L["router"], w, _shared(L))
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(plan.out, ref)
