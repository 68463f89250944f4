"""Streaming tier fed from a JNF v1 store (tarfa_b200/jnf.py) on the GPU.

A layer written to a JNF tree and placed with ``StreamingExpertTier.load_layer_jnf``
(resident experts into HBM slots, the rest read straight into pinned host memory,
each expert's SHA-256 checked) must give the same layer output, bit for bit, as
the same experts held resident, including routes that hit streamed experts."""
import pytest
import torch

from tarfa_b200 import jnf, ops
from tarfa_b200 import synthetic as syn

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_tier_from_jnf_equals_resident(tmp_path):
    from tarfa_b200.streaming import StreamingExpertTier
    s = syn.LayerShape(hidden=256, experts=8, inter=128, shared_inter=128)
    L = syn.layer_device(5, s, DEV)
    jnf.write_layer(tmp_path, 0, L["gate_up"], L["down"])
    store = jnf.JnfStore(tmp_path)
    tier = StreamingExpertTier(n_layers=1, experts=8, hidden=256, inter=128, resident=3, staging=5,
                               device=DEV)
    tier.load_layer_jnf(0, store)
    assert tier.host_bytes() == 5 * 3 * 256 * 128 * 2
    shared = ops.SharedWeights(L["sh_gate"], L["sh_up"], L["sh_down"], L["sh_gate_w"])
    full = ops.ExpertWeights(L["gate_up"], L["down"])
    gen = torch.Generator(device=DEV).manual_seed(11)
    for T in (1, 4):
        h = torch.randn((T, s.hidden), generator=gen, device=DEV).to(torch.bfloat16)
        ref, idx, _ = ops.moe_layer(h, L["router"], full, shared, top_k=4, return_routing=True)
        w = tier.weights_for(0, idx.flatten().tolist())
        out = ops.moe_layer(h, L["router"], w, shared, top_k=4)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"T={T}"
    assert tier.stats()["misses"] > 0
