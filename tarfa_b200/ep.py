"""Expert-parallel MoE layer over ``torch.distributed`` (NCCL over NVLink on B200s).

The reference runs on one GPU and streams experts from NVMe; on 2/4/8 B200s
the experts of a layer are instead sharded and kept resident: rank ``g`` of
``N`` owns experts ``[g*E/N, (g+1)*E/N)``.  Router and shared expert are
replicated, tokens are sharded (each rank brings its own batch).  Per layer:

1. route locally (``tarfa_b200_router_topk``, the reference router's arithmetic);
2. sort the routes by expert id (``tarfa_b200_permute``: expert ascending, then
   k-slot, then token -- the reference's segment order); experts are sharded in
   contiguous id ranges, so that order is also grouped by owner rank;
3. exchange per-peer route counts, then token rows and expert ids, with
   ``all_to_all_single`` (NCCL all-to-all over NVLink);
4. each rank runs its experts on the rows it received (``experts_forward`` with
   one route of weight 1 per row, which returns the expert output itself);
5. send the outputs back with the reverse all-to-all;
6. combine per token in the reference order with the locally computed gated
   shared expert (``tarfa_b200_combine_routes``).

Every rank takes the same collective steps in the same order.  The compute
steps go through a backend object, so the same exchange logic runs on CPU
``gloo`` ranks in tests with an oracle-backed backend.  Exact (dense) experts
only: the fused int4 decode keeps fp32 expert outputs across the combine, which
this exchange does not carry.
"""
from __future__ import annotations

import dataclasses

import torch
import torch.distributed as dist

from . import ops


class CudaBackend:
    """The CUDA kernels (C ABI) as the EP compute backend."""

    def router_topk(self, h, w_r, k, bias=None):
        return ops.router_topk(h, w_r, k, bias)

    def permute(self, idx, E):
        return ops.permute(idx, E)

    def expert_rows(self, x, local_ids, weights):
        if x.shape[0] == 0:
            return torch.empty_like(x)
        ones = torch.ones((x.shape[0], 1), dtype=torch.float32, device=x.device)
        return ops.experts_forward(x, local_ids.view(-1, 1), ones, weights)

    def shared_expert(self, h, shared):
        return ops.shared_expert(h, shared) if shared is not None else None

    def combine_routes(self, y_routes, idx, w, E, shared_gated):
        return ops.combine_routes(y_routes, idx, w, E, shared_gated)


@dataclasses.dataclass
class EPShard:
    """This rank's part of one layer."""
    router: torch.Tensor                 # [E, H], replicated
    experts: ops.ExpertWeights | object  # this rank's experts, local index 0..E/N-1
    shared: ops.SharedWeights | object | None
    num_experts: int
    top_k: int = 8
    bias: torch.Tensor | None = None


class ExpertParallelMoE:
    def __init__(self, shard: EPShard, group=None, backend=None):
        self.s = shard
        self.group = group
        self.backend = backend or CudaBackend()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        E = shard.num_experts
        if E % self.world:
            raise ValueError(f"{E} experts do not shard evenly over {self.world} ranks")
        self.e_per = E // self.world
        self.e0 = self.rank * self.e_per

    def owner(self, e: int) -> int:
        return e // self.e_per

    def forward_padded(self, h: torch.Tensor, return_routing: bool = False):
        """Decode-sized exchange with fixed block sizes: every peer block holds
        T*K rows (unused rows carry expert id -1 and are skipped), so no route
        count ever crosses to the host and the whole step can be captured in a
        CUDA graph (NCCL collectives are capturable).  Same results as forward().
        """
        b, s = self.backend, self.s
        T, H = h.shape
        K, E, N = s.top_k, s.num_experts, self.world
        dev = h.device
        RB = T * K                                      # rows per peer block
        idx, w = b.router_topk(h, s.router, K, s.bias)
        seg, perm_tok, perm_slot = b.permute(idx, E)
        seg = seg.to(dev, torch.int64)
        i = torch.arange(RB, device=dev)
        valid = i < seg[E]
        ptok = torch.where(valid, perm_tok.long(), torch.zeros_like(i))
        pslot = torch.where(valid, perm_slot.long(), torch.zeros_like(i))
        e = idx[ptok, pslot]
        g = torch.div(e, self.e_per, rounding_mode="floor")
        bounds = seg[torch.arange(N, device=dev) * self.e_per]
        dest = torch.where(valid, g * RB + (i - bounds[g]), torch.full_like(i, N * RB))
        x_send = torch.zeros((N * RB + 1, H), dtype=h.dtype, device=dev)
        e_send = torch.full((N * RB + 1,), -1, dtype=torch.int64, device=dev)
        x_send.index_copy_(0, dest, h.index_select(0, ptok))
        e_send.index_copy_(0, dest, torch.where(valid, e, torch.full_like(e, -1)))
        x_send, e_send = x_send[:N * RB], e_send[:N * RB]
        x_recv = torch.empty_like(x_send)
        e_recv = torch.empty_like(e_send)
        dist.all_to_all_single(x_recv, x_send, group=self.group)
        dist.all_to_all_single(e_recv, e_send, group=self.group)
        local = torch.where(e_recv >= 0, e_recv - self.e0, torch.full_like(e_recv, self.e_per))
        y_recv = b.expert_rows(x_recv, local, s.experts)
        y_back = torch.empty_like(y_recv)
        dist.all_to_all_single(y_back, y_recv, group=self.group)
        y_routes = torch.zeros((T * K + 1, H), dtype=h.dtype, device=dev)
        rpos = torch.where(valid, ptok * K + pslot, torch.full_like(i, T * K))
        y_routes.index_copy_(0, rpos, y_back.index_select(0, torch.clamp(dest, max=N * RB - 1)))
        shared_gated = b.shared_expert(h, s.shared)
        out = b.combine_routes(y_routes[:T * K], idx, w, E, shared_gated)
        return (out, idx, w) if return_routing else out

    def forward(self, h: torch.Tensor, return_routing: bool = False):
        b, s = self.backend, self.s
        T, H = h.shape
        K, E, N = s.top_k, s.num_experts, self.world
        dev = h.device
        idx, w = b.router_topk(h, s.router, K, s.bias)
        seg, perm_tok, perm_slot = b.permute(idx, E)
        seg_h = seg.to("cpu", torch.int64)
        R = int(seg_h[-1])
        bounds = [int(seg_h[g * self.e_per]) for g in range(N)] + [R]
        send_counts = [bounds[g + 1] - bounds[g] for g in range(N)]
        # ---- exchange counts, rows and expert ids ------------------------------
        sc = torch.tensor(send_counts, dtype=torch.int64, device=dev)
        rc = torch.empty_like(sc)
        dist.all_to_all_single(rc, sc, group=self.group)
        recv_counts = [int(x) for x in rc.cpu()]
        ptok = perm_tok[:R].long()
        pslot = perm_slot[:R].long()
        x_send = h.index_select(0, ptok)
        e_send = idx[ptok, pslot].to(torch.int64)
        x_recv = torch.empty((sum(recv_counts), H), dtype=h.dtype, device=dev)
        e_recv = torch.empty((sum(recv_counts),), dtype=torch.int64, device=dev)
        dist.all_to_all_single(x_recv, x_send, recv_counts, send_counts, group=self.group)
        dist.all_to_all_single(e_recv, e_send, recv_counts, send_counts, group=self.group)
        # ---- local experts on the received rows --------------------------------
        y_recv = b.expert_rows(x_recv, e_recv - self.e0, s.experts)
        # ---- outputs back to the token owners, then combine --------------------
        y_back = torch.empty((R, H), dtype=h.dtype, device=dev)
        dist.all_to_all_single(y_back, y_recv, send_counts, recv_counts, group=self.group)
        y_routes = torch.zeros((T * K, H), dtype=h.dtype, device=dev)
        y_routes.index_copy_(0, ptok * K + pslot, y_back)
        shared_gated = b.shared_expert(h, s.shared)
        out = b.combine_routes(y_routes, idx, w, E, shared_gated)
        return (out, idx, w) if return_routing else out
