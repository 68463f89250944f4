"""Expert parallelism over NVLink peer memory (``tarfa_b200_ep_moe_layer``).

One GPU: a one-rank group (the only box is the rank's own) must equal the
single-GPU layer bit for bit -- outputs, ids and weights -- eagerly and
replayed from a CUDA graph, for dense and int4 experts.  A group whose second
rank never runs must end both of its waits with TARFA_DEV_WAIT_TIMEOUT (the
waits are bounded) and leave the device usable.  Two or more GPUs: one
process per GPU; every rank's output equals the single-GPU layer on the same
tokens bit for bit, for eager calls, CUDA-graph replays, dense and int4, with
whole experts per rank (tp=1) and with pairs of ranks sharing experts by halves
(tp=2, whose two fp32 partials are added in the single-GPU GEMV's order).
"""
import ctypes as C
import os
import socket
import time
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu

S_ARGS = dict(hidden=1024, experts=64, inter=512, shared_inter=256)


def _q4(w, group):
    """Quantise an expert stack [E, N, K] with the library's own quantiser."""
    from tarfa_b200 import ops
    E, N, K = w.shape
    packed, scale = ops.quantize_int4(w.reshape(E * N, K).contiguous(), group)
    return packed.view(E, N, K // 8), scale.view(E, N, K // group)


def _layer(dev, kind):
    from tarfa_b200 import ops
    from tarfa_b200 import synthetic as syn
    s = syn.LayerShape(**S_ARGS)
    L = syn.layer_device(3, s, dev)
    shared = ops.SharedWeights(L["sh_gate"], L["sh_up"], L["sh_down"], L["sh_gate_w"])
    if kind == "dense":
        full = ops.ExpertWeights(L["gate_up"], L["down"])
    else:
        gq, gs = _q4(L["gate_up"], 128)
        dq, ds = _q4(L["down"], 128)
        full = ops.ExpertWeights(gq, dq, "int4", gs, ds, 128)
    return s, L, full, shared


def _slice(full, e0, e1):
    from tarfa_b200 import ops
    if full.kind == "dense":
        return ops.ExpertWeights(full.gate_up[e0:e1].contiguous(), full.down[e0:e1].contiguous())
    return ops.ExpertWeights(full.gate_up[e0:e1].contiguous(), full.down[e0:e1].contiguous(), "int4",
                             full.gate_up_scale[e0:e1].contiguous(),
                             full.down_scale[e0:e1].contiguous(), full.group)


class _CGroup:
    """A group built directly on the C ABI from boxes of this process."""

    def __init__(self, s, full, shared, router, boxes, rank, max_tokens, world):
        from tarfa_b200 import _capi as api
        from tarfa_b200 import ops
        self.api, self.ops = api, ops
        self.L = api.lib()
        E, I = full.dims(s.hidden)
        self.dims = (s.hidden, s.experts, I, s.shared_inter, 8)
        self.mine = _slice(full, rank * (s.experts // world), (rank + 1) * (s.experts // world))
        self.wc = self.mine.c_struct()
        self.sc = shared.c_struct()
        self.router = router
        arr = (C.c_void_p * api.EP_MAX_RANKS)(*boxes)
        self.group = api.EpGroup(world, rank, max_tokens, 1, 0, arr)
        shape = ops._shape(max_tokens, s.hidden, s.experts, I, s.shared_inter, 8, torch.bfloat16)
        n = self.L.tarfa_b200_ep_workspace_size(C.byref(shape), world, max_tokens)
        self.ws = torch.zeros(n, dtype=torch.uint8, device=router.device)

    def __call__(self, h, out, idx, wt):
        H, E, I, Is, K = self.dims
        shape = self.ops._shape(h.shape[0], H, E, I, Is, K, h.dtype)
        p = self.ops._ptr
        self.api.check(self.L.tarfa_b200_ep_moe_layer(
            C.byref(shape), p(h), p(self.router), None, C.byref(self.wc), C.byref(self.sc),
            C.byref(self.group), p(out), p(idx), p(wt), p(self.ws), self.ws.numel(),
            self.ops._stream(h.device)))


def _alloc_box(s, world, max_tokens):
    from tarfa_b200 import _capi as api
    from tarfa_b200 import ops
    L = api.lib()
    shape = ops._shape(max_tokens, s.hidden, s.experts, s.inter, s.shared_inter, 8, torch.bfloat16)
    n = L.tarfa_b200_ep_box_bytes(C.byref(shape), world, max_tokens)
    box = C.c_void_p()
    api.check(L.tarfa_b200_ep_box_alloc(n, C.byref(box), None))
    return box


@pytest.mark.parametrize("kind", ["dense", "int4"])
def test_ep_one_rank_equals_layer(kind):
    from tarfa_b200 import _capi as api
    from tarfa_b200 import ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    s, L, full, shared = _layer(dev, kind)
    box = _alloc_box(s, 1, 16)
    try:
        ep = _CGroup(s, full, shared, L["router"], [box.value], 0, 16, 1)
        gen = torch.Generator(device=dev).manual_seed(7)
        for T in ((1, 3, 16) if kind == "dense" else (1, 4)):
            for rep in range(2):   # the step counter advances between calls
                h = torch.randn((T, s.hidden), generator=gen, device=dev).to(torch.bfloat16)
                out = torch.empty_like(h)
                idx = torch.empty((T, 8), dtype=torch.int64, device=dev)
                wt = torch.empty((T, 8), dtype=torch.float32, device=dev)
                ep(h, out, idx, wt)
                ref, ridx, rw = ops.moe_layer(h, L["router"], full, shared, return_routing=True)
                torch.cuda.synchronize()
                assert ops.device_status() == 0
                assert torch.equal(idx, ridx), f"{kind} T={T}: routing differs"
                assert torch.equal(wt, rw), f"{kind} T={T}: routing weights differ"
                assert torch.equal(out, ref), f"{kind} T={T}: output differs"
        # CUDA graph replays: one step per replay
        static_h = torch.randn((1, s.hidden), generator=gen, device=dev).to(torch.bfloat16)
        out = torch.empty_like(static_h)
        idx = torch.empty((1, 8), dtype=torch.int64, device=dev)
        wt = torch.empty((1, 8), dtype=torch.float32, device=dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ep(static_h, out, idx, wt)
        for _ in range(3):
            static_h.copy_(torch.randn((1, s.hidden), generator=gen, device=dev).to(torch.bfloat16))
            g.replay()
            ref = ops.moe_layer(static_h, L["router"], full, shared)
            torch.cuda.synchronize()
            assert torch.equal(out, ref), f"{kind}: graph replay differs"
        assert ops.device_status() == 0
        del g
    finally:
        torch.cuda.synchronize()
        api.check(api.lib().tarfa_b200_ep_box_free(box))


def test_ep_missing_peer_times_out():
    """Rank 1 of a two-rank group never runs: both waits of rank 0 (the
    exchange and the combine) give up after their bound, raise the status and
    the next layer call on the device works."""
    from tarfa_b200 import _capi as api
    from tarfa_b200 import ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    s, L, full, shared = _layer(dev, "dense")
    ops.device_status(clear=True)
    boxes = [_alloc_box(s, 2, 4), _alloc_box(s, 2, 4)]   # the second one stands for the absent peer
    try:
        ep = _CGroup(s, full, shared, L["router"], [b.value for b in boxes], 0, 4, 2)
        h = torch.randn((1, s.hidden), device=dev).to(torch.bfloat16)
        out = torch.empty_like(h)
        idx = torch.empty((1, 8), dtype=torch.int64, device=dev)
        wt = torch.empty((1, 8), dtype=torch.float32, device=dev)
        t0 = time.time()
        ep(h, out, idx, wt)
        torch.cuda.synchronize()
        dt = time.time() - t0
        st = ops.device_status(clear=True)
        assert st & api.DEV_WAIT_TIMEOUT, f"status {st}: the missing peer was not detected"
        assert dt < 60, f"waits took {dt:.1f} s"
        ref = ops.moe_layer(h, L["router"], full, shared)
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        assert torch.isfinite(ref.float()).all()
    finally:
        torch.cuda.synchronize()
        for b in boxes:
            api.check(api.lib().tarfa_b200_ep_box_free(b))


@pytest.mark.parametrize("T", [50, 64])
def test_ep_one_rank_tensor_core_router(T):
    """From 48 tokens (128 or more experts) the expert-parallel layer takes its
    logits from the tensor-core router and its exact fix-up; the exchange then
    tops-k them and clears the fix-up counter.  Two calls in a row equal the
    single-GPU layer on the expert GEMVs (routing, weights and output)."""
    from tarfa_b200 import _capi as api
    from tarfa_b200 import ops
    from tarfa_b200 import synthetic as syn
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    s = syn.LayerShape(hidden=1024, experts=128, inter=256, shared_inter=256)
    L = syn.layer_device(5, s, dev)
    full = ops.ExpertWeights(L["gate_up"], L["down"])
    shared = ops.SharedWeights(L["sh_gate"], L["sh_up"], L["sh_down"], L["sh_gate_w"])
    box = _alloc_box(s, 1, 64)
    ops.set_gemm_min_tokens(1 << 30)   # the EP layer's experts run on the GEMV kernels
    try:
        ep = _CGroup(s, full, shared, L["router"], [box.value], 0, 64, 1)
        gen = torch.Generator(device=dev).manual_seed(T)
        for rep in range(2):
            h = torch.randn((T, s.hidden), generator=gen, device=dev).to(torch.bfloat16)
            out = torch.empty_like(h)
            idx = torch.empty((T, 8), dtype=torch.int64, device=dev)
            wt = torch.empty((T, 8), dtype=torch.float32, device=dev)
            ep(h, out, idx, wt)
            ref, ridx, rw = ops.moe_layer(h, L["router"], full, shared, return_routing=True)
            torch.cuda.synchronize()
            assert ops.device_status() == 0
            assert torch.equal(idx, ridx), f"T={T} call {rep}: routing differs"
            assert torch.equal(wt, rw), f"T={T} call {rep}: routing weights differ"
            assert torch.equal(out, ref), f"T={T} call {rep}: output differs"
    finally:
        ops.set_gemm_min_tokens(64)
        torch.cuda.synchronize()
        api.check(api.lib().tarfa_b200_ep_box_free(box))


def _check_ep_stack(dev, rank):
    """A small expert-parallel stack (collective): every layer's output equals
    the single-GPU layer's on the same input, and so do the greedy tokens."""
    from tarfa_b200 import ops, synthetic as syn
    from tarfa_b200.stack import ExpertParallelStack, lm_head_argmax, rms_norm
    ss = syn.LayerShape(hidden=256, experts=16, inter=128, shared_inter=128)
    st = ExpertParallelStack(ss, 3, 512, dev, seed=9, max_tokens=8)
    try:
        for T in (1, 5):
            tok = (torch.arange(T, device=dev) * 31 + 7 * rank) % 512
            rec = []
            nxt = st.step(tok, record=rec)
            h = st.embed.index_select(0, tok)
            for l in range(3):
                w_r, full_l, sh = st.full_layer(l)
                x = rms_norm(h, st.layers[l]["norm"])
                assert torch.equal(x, rec[l][0]), f"rank {rank} T={T} layer {l}: input differs"
                y = ops.moe_layer(x, w_r, full_l, sh)
                assert torch.equal(y, rec[l][1]), f"rank {rank} T={T} layer {l}: output differs"
                h = h + y
            ref = lm_head_argmax(rms_norm(h, st.final_norm), st.lm_head)
            assert torch.equal(ref, nxt), f"rank {rank} T={T}: greedy tokens differ"
        assert ops.device_status() == 0
    finally:
        torch.cuda.synchronize()
        st.close()


def test_ep_stack_one_rank_equals_layers():
    """The expert-parallel stack in a one-rank group (gloo for the handle
    exchange): layer for layer the single-GPU layer."""
    import torch.distributed as dist
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if dist.is_initialized():
        pytest.skip("a process group is already initialised in this process")
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0,
                            world_size=1)
    try:
        _check_ep_stack(dev, 0)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _worker(rank, world, port, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=dev)
        from tarfa_b200 import ops
        from tarfa_b200.ep import EPShard, PeerExpertParallelMoE, shard_experts
        cases = [(k, tp) for k in ("dense", "int4") for tp in ((1, 2) if world % 2 == 0 else (1,))]
        for kind, tp in cases:
            s, L, full, shared = _layer(dev, kind)
            mine = shard_experts(full, rank, world, tp)
            ep = PeerExpertParallelMoE(EPShard(L["router"], mine, shared, s.experts), max_tokens=16,
                                       tp=tp)
            gen = torch.Generator(device=dev).manual_seed(100 + rank)
            for T in ((1, 3, 16) if kind == "dense" else (1, 4)):
                h = torch.randn((T, s.hidden), generator=gen, device=dev).to(torch.bfloat16)
                out, idx, wt = ep.forward(h, return_routing=True)
                ref, ridx, rw = ops.moe_layer(h, L["router"], full, shared, return_routing=True)
                torch.cuda.synchronize()
                assert ops.device_status() == 0, f"rank {rank}: device status set"
                assert torch.equal(idx, ridx), f"rank {rank} {kind} tp={tp} T={T}: routing differs"
                assert torch.equal(out, ref), f"rank {rank} {kind} tp={tp} T={T}: output differs"
            static_h = torch.randn((1, s.hidden), generator=gen, device=dev).to(torch.bfloat16)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                static_out = ep.forward(static_h)
            for _ in range(3):   # the same replay count on every rank
                static_h.copy_(torch.randn((1, s.hidden), generator=gen, device=dev).to(torch.bfloat16))
                g.replay()
                ref = ops.moe_layer(static_h, L["router"], full, shared)
                torch.cuda.synchronize()
                assert torch.equal(static_out, ref), f"rank {rank} {kind} tp={tp}: graph replay differs"
            del g
            assert ops.device_status() == 0
            ep.close()
        _check_ep_stack(dev, rank)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put((rank, traceback.format_exc()))


def test_ep_peer_memory_matches_single_gpu():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 or more GPUs")
    import torch.multiprocessing as mp
    world = min(4, torch.cuda.device_count())
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        if p.is_alive():
            p.kill()
            raise AssertionError("an EP rank did not finish")
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs)
