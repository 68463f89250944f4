"""Generate golden vectors by running the REFERENCE on the CPU (this container only).

Run:  python tests/golden/make_golden.py --ref /path/to/tarfa-checkout
      (or set TARFA_REF to that path; one of the two is required)

It imports the reference's own routed-experts closure
(``tarfa/engine/fused_int4.py:148-262``, ``TarfaFused._install_streamed_experts``)
and the ``transformers`` 5.5.0 ``Qwen3_5MoeSparseMoeBlock`` it is installed
into, feeds them seeded synthetic weights (``tarfa_b200.synthetic``) and stores
inputs that are not regenerable plus every output, as ``.npz`` under
``tests/golden/``.  Expert weights are not stored: they are regenerated from the
seed, and SHA-256 digests of a few of them are stored to catch generator drift.

Recipe (the reference needs ``accelerate``, which is not installed here, only
for ``init_empty_weights`` in ``layered.py:10``): stub that module, put
``tarfa/engine`` on ``sys.path``, import ``fused_int4`` with ``BF16=1``, and
replace its ``read_bf16`` (the NVMe transport, ``exact_bf16.py:126``) by a
lookup into the synthetic weights.  The int4 prefill branch gets the same
treatment through ``_read_experts`` (``channel_q4.py:39-50``).
"""
from __future__ import annotations

import argparse
import contextlib
import hashlib
import json
import os
import sys
import types
from types import SimpleNamespace

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from tarfa_b200 import synthetic as syn  # noqa: E402


def _load_reference(ref_root: str):
    import transformers  # noqa: F401  (must come before the accelerate stub)
    import huggingface_hub  # noqa: F401
    acc = types.ModuleType("accelerate")
    acc.init_empty_weights = contextlib.nullcontext
    sys.modules.setdefault("accelerate", acc)
    os.environ["BF16"] = "1"
    os.environ["JTOPK"] = "8"
    sys.path.insert(0, os.path.join(ref_root, "tarfa", "engine"))
    import fused_int4
    import channel_q4
    import moe_kernel
    return fused_int4, channel_q4, moe_kernel


def _np(t: torch.Tensor) -> np.ndarray:
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(_np(t).tobytes()).hexdigest()[:16]


def _block(shape: syn.LayerShape, seed: int, dtype, experts_needed=None):
    from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeSparseMoeBlock
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig
    cfg = Qwen3_5MoeTextConfig(hidden_size=shape.hidden, num_experts=shape.experts,
                               moe_intermediate_size=shape.inter,
                               shared_expert_intermediate_size=shape.shared_inter,
                               num_experts_per_tok=shape.top_k)
    with torch.device("meta"):
        blk = Qwen3_5MoeSparseMoeBlock(cfg)
    blk = blk.to_empty(device="cpu").to(dtype)
    with torch.no_grad():
        blk.gate.weight.copy_(syn.router_cpu(seed, 0, shape, dtype))
        g, u, d, w = syn.shared_cpu(seed, 0, shape, dtype)
        blk.shared_expert.gate_proj.weight.copy_(g)
        blk.shared_expert.up_proj.weight.copy_(u)
        blk.shared_expert.down_proj.weight.copy_(d)
        blk.shared_expert_gate.weight.copy_(w)
    cache = {}

    def get(e):
        if e not in cache:
            cache[e] = syn.expert_cpu(seed, 0, e, shape, dtype)
        return cache[e]
    return blk, get


def _install(fused_int4, blk, get, dtype):
    fused_int4.read_bf16 = lambda layer, experts, device, d, use_ram_cache=False: {
        e: get(e) for e in experts}
    eng = SimpleNamespace(device="cpu", dtype=dtype, nL=1)
    fused_int4.TarfaFused._install_streamed_experts(eng, blk.experts, "model.layers.0.")


def case_exact(fi, name, shape, seed, T, dtype=torch.bfloat16, sentinel=False, jtopk=8,
               token_stream=0):
    blk, get = _block(shape, seed, dtype)
    _install(fi, blk, get, dtype)
    fi.JTOPK = jtopk
    h = syn.tokens_cpu(seed, T, shape, dtype, stream=token_stream)
    with torch.no_grad():
        lg_full, w, idx = blk.gate(h)
        # the block's router output (this is what the closure receives)
        idx_in, w_in = idx.clone(), w.clone()
        if sentinel:
            idx_in[0, 3] = shape.experts          # skip sentinel (fused_int4.py:167)
        routed = blk.experts(h, idx_in, w_in)
        shared = torch.nn.functional.sigmoid(blk.shared_expert_gate(h)) * blk.shared_expert(h)
        block = blk(h.view(1, T, shape.hidden)).view(T, shape.hidden) if not sentinel else routed + shared
        lg = torch.nn.functional.linear(h, blk.gate.weight)
    fi.JTOPK = 8
    hit = sorted({int(e) for e in idx_in.flatten().tolist() if int(e) < shape.experts})
    digests = {str(e): [_sha(get(e)[0]), _sha(get(e)[1])] for e in hit[:3]}
    arrays = dict(h=_np(h), top_idx=idx_in.numpy(), top_w=w_in.numpy(), logits=_np(lg),
                  probs=lg_full.numpy(), routed=_np(routed), shared=_np(shared), block=_np(block))
    meta = dict(kind="exact", name=name, shape=shape.__dict__, seed=seed, T=T,
                dtype=str(dtype).replace("torch.", ""), sentinel=sentinel, jtopk=jtopk,
                token_stream=token_stream, digests=digests,
                router_digest=_sha(blk.gate.weight))
    return name, arrays, meta


def case_int4_dequant(cq, name, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    packed = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, generator=g)
    scale = (torch.randn(N, generator=g) * 0.02).to(torch.float16)
    deq = cq.dequant_int4(packed, scale)
    return name, dict(packed=packed.numpy(), scale=_np(scale), deq=_np(deq)), dict(
        kind="dequant", name=name, N=N, K=K, seed=seed)


def case_int4_prefill(fi, name, shape, seed, T, dtype=torch.float16):
    """The reference's int4 T>1 branch (fused_int4.py:249-261), fp16 engine dtype
    (the reference's default; with a bf16 engine its fp16*bf16 dequant promotes
    to fp32 and ``F.linear`` rejects the mix)."""
    blk, _ = _block(shape, seed, dtype)
    fi.BF16 = False
    q4 = {e: syn.q4_expert_reflayout(seed, e, shape, torch.float16) for e in range(shape.experts)}
    names = ("gate_up_q", "gate_up_s", "down_q", "down_s")

    def fake_read(path, experts):
        parts = {e: {nm: bytearray(_np(q4[e][i]).tobytes()) if q4[e][i].dtype != torch.uint8
                     else bytearray(q4[e][i].numpy().tobytes()) for i, nm in enumerate(names)}
                 for e in experts}
        meta = {nm: (0, 0, tuple(q4[0][i].shape), q4[0][i].dtype) for i, nm in enumerate(names)}
        return parts, meta
    fi._read_experts = fake_read
    eng = SimpleNamespace(device="cpu", dtype=dtype, nL=1)
    fi.TarfaFused._install_streamed_experts(eng, blk.experts, "model.layers.0.")
    h = syn.tokens_cpu(seed, T, shape, dtype)
    with torch.no_grad():
        _, w, idx = blk.gate(h)
        routed = blk.experts(h, idx, w)
    fi.BF16 = True
    return name, dict(h=_np(h), top_idx=idx.numpy(), top_w=w.numpy(), routed=_np(routed)), dict(
        kind="int4_prefill", name=name, shape=shape.__dict__, seed=seed, T=T,
        dtype=str(dtype).replace("torch.", ""))


def case_int4_ref_ffn(mk, name, shape, seed, dtype=torch.float16):
    """``moe_kernel._ref_ffn`` (moe_kernel.py:117-125): fp32 dequant reference of
    the fused int4 decode, on 8 reference-layout experts."""
    g = torch.Generator().manual_seed(seed)
    E, H, I = 8, shape.hidden, shape.inter
    gq = torch.randint(0, 256, (E, 2 * I, H // 2), dtype=torch.uint8, generator=g)
    dq = torch.randint(0, 256, (E, H, I // 2), dtype=torch.uint8, generator=g)
    gs = (torch.randn(E, 2 * I, generator=g) * 0.02).to(dtype)
    ds = (torch.randn(E, H, generator=g) * 0.02).to(dtype)
    x = (torch.randn(H, generator=g) * 0.5).to(dtype)
    rw = torch.softmax(torch.randn(E, generator=g), 0)
    ref = mk._ref_ffn(x, gq, gs, dq, ds, rw)
    return name, dict(gq=gq.numpy(), gs=_np(gs), dq=dq.numpy(), ds=_np(ds), x=_np(x),
                      rw=rw.numpy(), ref=ref.numpy()), dict(
        kind="int4_ref_ffn", name=name, shape=shape.__dict__, seed=seed,
        dtype=str(dtype).replace("torch.", ""))


def case_router_stats(name, shape, seed, T):
    """The literal HF router at a realistic token count, for tie statistics."""
    w_r = syn.router_cpu(seed, 0, shape)
    h = syn.tokens_cpu(seed, T, shape, stream=7)
    lg = torch.nn.functional.linear(h, w_r)
    p = torch.softmax(lg, dtype=torch.float, dim=-1)
    v, i = torch.topk(p, shape.top_k, dim=-1)
    v = v / v.sum(-1, keepdim=True)
    return name, dict(h=_np(h), logits=_np(lg), top_idx=i.numpy(), top_w=v.numpy()), dict(
        kind="router", name=name, shape=shape.__dict__, seed=seed, T=T,
        router_digest=_sha(w_r))


SMALL = syn.LayerShape(hidden=256, experts=16, inter=128, shared_inter=128)
SMALL_ODD = syn.LayerShape(hidden=512, experts=40, inter=192, shared_inter=64)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("TARFA_REF"),
                    help="root of a tarfa checkout (default: $TARFA_REF)")
    a = ap.parse_args()
    if not a.ref:
        ap.error("give the reference checkout with --ref or TARFA_REF")
    if not os.path.isdir(os.path.join(a.ref, "tarfa", "engine")):
        ap.error(f"{a.ref} has no tarfa/engine: not a tarfa checkout")
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    fi, cq, mk = _load_reference(a.ref)
    cases = []
    cases.append(case_exact(fi, "small_t1", SMALL, 1, 1))
    cases.append(case_exact(fi, "small_t3", SMALL, 2, 3))
    cases.append(case_exact(fi, "small_t37", SMALL, 3, 37))
    cases.append(case_exact(fi, "small_t1_sentinel", SMALL, 4, 1, sentinel=True))
    cases.append(case_exact(fi, "small_t5_jtopk5", SMALL, 5, 5, jtopk=5))
    cases.append(case_exact(fi, "small_t1_jtopk5", SMALL, 6, 1, jtopk=5))
    cases.append(case_exact(fi, "small_t4_f16", SMALL, 7, 4, dtype=torch.float16))
    cases.append(case_exact(fi, "small_t1_f16", SMALL, 8, 1, dtype=torch.float16))
    cases.append(case_exact(fi, "odd_t9", SMALL_ODD, 9, 9))
    cases.append(case_exact(fi, "c0_t4", syn.L0, 0, 4))
    cases.append(case_exact(fi, "c0_t1", syn.L0, 0, 1))
    cases.append(case_exact(fi, "c1_t1", syn.L1, 0, 1))
    cases.append(case_exact(fi, "c1_t4", syn.L1, 0, 4))
    cases.append(case_int4_dequant(cq, "dequant_ref_layout", 96, 256, 11))
    cases.append(case_int4_prefill(fi, "int4_prefill_small_t6", SMALL, 12, 6))
    cases.append(case_int4_ref_ffn(mk, "int4_ref_ffn_small", SMALL, 13))
    cases.append(case_router_stats("router_c1_t256", syn.L1, 0, 256))
    index = {}
    for name, arrays, meta in cases:
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
        index[name] = meta
        print(name, {k: v.shape for k, v in arrays.items()})
    with open(os.path.join(HERE, "index.json"), "w") as f:
        json.dump(index, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
