"""Expert parallelism on 2+ B200s over NCCL (child processes, one per GPU).

Each rank holds E/N experts, the replicated router and shared expert, and its
own tokens.  Its EP output must match the single-GPU layer on the same tokens
(indices identical, outputs within the project tolerance), for the
variable-split exchange and for the fixed-block exchange replayed from a CUDA
graph.  Skipped on a box with one GPU.
"""
import os
import socket
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu

S_ARGS = dict(hidden=1024, experts=64, inter=512, shared_inter=256)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        from gpu_helpers import assert_close
        from tarfa_b200 import ops
        from tarfa_b200 import synthetic as syn
        from tarfa_b200.ep import EPShard, ExpertParallelMoE
        dev = torch.device("cuda", rank)
        s = syn.LayerShape(**S_ARGS)
        L = syn.layer_device(3, s, dev)                 # same seed on every rank: same layer
        per = s.experts // world
        mine = ops.ExpertWeights(L["gate_up"][rank * per:(rank + 1) * per].contiguous(),
                                 L["down"][rank * per:(rank + 1) * per].contiguous())
        shared = ops.SharedWeights(L["sh_gate"], L["sh_up"], L["sh_down"], L["sh_gate_w"])
        full = ops.ExpertWeights(L["gate_up"], L["down"])
        ep = ExpertParallelMoE(EPShard(L["router"], mine, shared, s.experts))
        gen = torch.Generator(device=dev).manual_seed(100 + rank)
        for T in (1, 3, 16):
            h = torch.randn((T, s.hidden), generator=gen, device=dev).to(torch.bfloat16)
            ref, ridx, _ = ops.moe_layer(h, L["router"], full, shared, return_routing=True)
            for fwd in (ep.forward, ep.forward_padded):
                out, idx, _ = fwd(h, return_routing=True)
                torch.cuda.synchronize()
                assert torch.equal(idx, ridx), f"rank {rank} T={T}: routing differs"
                assert_close(out, ref, f"rank {rank} T={T} {fwd.__name__}")
        # fixed-block exchange captured in a CUDA graph
        h = torch.randn((1, s.hidden), generator=gen, device=dev).to(torch.bfloat16)
        static_h = h.clone()
        ep.forward_padded(static_h)                       # warm-up (allocations, NCCL setup)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            static_out = ep.forward_padded(static_h)
        g.replay()
        torch.cuda.synchronize()
        ref = ops.moe_layer(h, L["router"], full, shared)
        assert_close(static_out, ref, f"rank {rank} graph replay")
        del g
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put((rank, traceback.format_exc()))


def test_ep_nccl_matches_single_gpu():
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
