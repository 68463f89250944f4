"""Expert-parallel exchange logic on CPU ``gloo`` ranks (world size 2).

The dispatch / combine code of ``tarfa_b200.ep`` runs unchanged; only its
compute steps come from the CPU oracle.  Each rank's output must match the
single-rank oracle block on that rank's tokens (indices identical, outputs
within the project tolerance).  A second test makes one rank drop out before
the exchange and checks that the other rank fails with an error instead of
hanging.
"""
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from oracle import moe_oracle as mo
from tarfa_b200 import synthetic as syn

S = syn.LayerShape(hidden=256, experts=16, inter=128, shared_inter=128)
SEED = 7


class OracleBackend:
    """CPU stand-in for the CUDA kernels (test only)."""

    def router_topk(self, h, w_r, k, bias=None):
        idx, w, _ = mo.router_topk(h, w_r, k, bias)
        return idx, w

    def permute(self, idx, E):
        seg, tok, slot = mo.permute(idx.numpy(), E)
        R = idx.numel()
        pt = np.full(R, -1, np.int32)
        ps = np.full(R, -1, np.int32)
        pt[:len(tok)] = tok
        ps[:len(slot)] = slot
        return torch.from_numpy(seg), torch.from_numpy(pt), torch.from_numpy(ps)

    def expert_rows(self, x, local_ids, weights):
        gu, dn = weights
        out = torch.zeros_like(x)
        for r in range(x.shape[0]):
            e = int(local_ids[r])
            if e >= gu.shape[0]:                       # skip id (padding row)
                continue
            g, u = F.linear(x[r], gu[e]).chunk(2, dim=-1)
            out[r] = F.linear(F.silu(g) * u, dn[e])
        return out

    def shared_expert(self, h, shared):
        return mo.shared_expert(h, *shared)

    def combine_routes(self, y_routes, idx, w, E, shared_gated):
        T, K = idx.shape
        out = torch.zeros((T, y_routes.shape[1]), dtype=y_routes.dtype)
        for t in range(T):
            if T == 1:
                acc = torch.zeros_like(out[t])
                for k in range(K):                     # router order, w rounded first
                    acc = acc + w[t, k] * y_routes[t * K + k]
            else:
                acc = torch.zeros_like(out[t])
                for k in sorted(range(K), key=lambda k: (int(idx[t, k]), k)):
                    acc = acc + (y_routes[t * K + k].float() * w[t, k]).to(acc.dtype)
            out[t] = acc
        return out + shared_gated


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, T, mode, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        from datetime import timedelta
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        from tarfa_b200.ep import EPShard, ExpertParallelMoE
        gu, dn = syn.layer_cpu(SEED, 0, S)
        per = S.experts // world
        sh = syn.shared_cpu(SEED, 0, S)
        shard = EPShard(router=syn.router_cpu(SEED, 0, S),
                        experts=(gu[rank * per:(rank + 1) * per], dn[rank * per:(rank + 1) * per]),
                        shared=sh, num_experts=S.experts)
        ep = ExpertParallelMoE(shard, backend=OracleBackend())
        h = syn.tokens_cpu(SEED, T, S, stream=100 + rank)
        if mode == "dropout" and rank == 1:
            return                                    # leaves before the exchange
        fwd = ep.forward_padded if mode == "padded" else ep.forward
        out, idx, w = fwd(h, return_routing=True)
        ref, idx_o, w_o, _ = mo.moe_block_exact(h, syn.router_cpu(SEED, 0, S),
                                                 lambda e: (gu[e], dn[e]), S.experts, sh)
        assert torch.equal(idx, idx_o), "routing differs from the single-rank oracle"
        err = (out.float() - ref.float()).abs().max().item()
        assert err <= 2 ** -7 * ref.float().abs().max().item(), err
        cos = F.cosine_similarity(out.flatten().double(), ref.flatten().double(), dim=0).item()
        assert cos >= 0.99999, cos
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put((rank, traceback.format_exc()))


def _run(world, T, mode):
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T, mode, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            raise AssertionError("an EP rank hung past the test timeout")
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    return errs


@pytest.mark.parametrize("T,mode", [(1, "normal"), (5, "normal"), (1, "padded"), (4, "padded")])
def test_ep_two_ranks_match_single_rank_oracle(T, mode):
    errs = _run(2, T, mode)
    assert not errs, errs


def test_ep_rank_dropout_fails_fast_instead_of_hanging():
    errs = _run(2, 3, "dropout")
    # rank 0 must report an error (collective timeout / peer gone), never hang
    assert any(r == 0 for r, _ in errs), errs
