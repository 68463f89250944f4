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

:class:`PeerExpertParallelMoE` is the B200 path: the same sharding, but the
dispatch and the return are stores into the peers' HBM from inside the
library's kernels (``tarfa_b200_ep_moe_layer``; NVLink peer memory mapped with
CUDA IPC), with sequence-numbered flags and bounded waits instead of
collectives, so a decode step is six kernels and no NCCL call.  Dense and int4
experts; every rank brings the same number of tokens per step.
"""
from __future__ import annotations

import ctypes as C
import copy
import dataclasses

import torch
import torch.distributed as dist

from . import _capi as api
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


def shard_experts(full: ops.ExpertWeights, rank: int, world: int, tp: int = 1) -> ops.ExpertWeights:
    """This rank's part of a layer's experts for :class:`PeerExpertParallelMoE`.

    tp = 1: experts ``[rank*E/N, (rank+1)*E/N)`` whole.  tp = 2: ranks ``2p`` and
    ``2p+1`` share experts ``[p*2E/N, (p+1)*2E/N)``; rank ``2p+h`` keeps half ``h``
    of each one's intermediate dimension (gate and up rows ``[h*I/2, (h+1)*I/2)``,
    the same down columns), as contiguous copies.
    """
    E = full.gate_up.shape[0]
    groups = world // tp
    e0, e1 = (rank // tp) * (E // groups), (rank // tp + 1) * (E // groups)

    def rows(t, h):   # gate and up rows of half h: t [E, 2I, ...]
        n = t.shape[1] // 2
        a = t[e0:e1, h * n // tp:(h + 1) * n // tp]
        b = t[e0:e1, n + h * n // tp:n + (h + 1) * n // tp]
        return torch.cat([a, b], dim=1).contiguous()

    def cols(t, h):   # down columns of half h: t [E, H, K']
        k = t.shape[2]
        return t[e0:e1, :, h * k // tp:(h + 1) * k // tp].contiguous()

    h = rank % tp
    if full.kind == "dense":
        return ops.ExpertWeights(rows(full.gate_up, h), cols(full.down, h))
    return ops.ExpertWeights(rows(full.gate_up, h), cols(full.down, h), "int4",
                             rows(full.gate_up_scale, h), cols(full.down_scale, h), full.group)


class PeerExpertParallelMoE:
    """Expert-parallel layer over NVLink peer memory (one process per GPU).

    Same results as :class:`ExpertParallelMoE` (router and shared expert
    replicated; with ``tp=1`` rank ``g`` owns experts ``[g*E/N, (g+1)*E/N)``,
    with ``tp=2`` pairs of ranks share their experts by halves, which evens out
    the pairs' load: :func:`shard_experts` cuts a rank's part), but a step is
    one call of ``tarfa_b200_ep_moe_layer``: the kernels store the
    routed token rows into the owners' boxes and the expert outputs back into
    the sources' boxes, so no collective runs on the data path.  Construction
    and :meth:`close` are collective (they exchange the IPC handles and
    barrier).  Every rank must call :meth:`forward` the same number of times
    with the same token count; the calls can be captured in a CUDA graph.
    """

    def __init__(self, shard: EPShard, group=None, max_tokens: int = 16, tp: int = 1):
        self.s = shard
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > api.EP_MAX_RANKS:
            raise ValueError(f"peer-memory EP supports at most {api.EP_MAX_RANKS} ranks")
        E, K = shard.num_experts, shard.top_k
        if tp not in (1, 2) or self.world % tp:
            raise ValueError(f"tp {tp} must be 1, or 2 with an even number of ranks")
        groups = self.world // tp
        if E % groups:
            raise ValueError(f"{E} experts do not shard evenly over {groups} rank groups")
        w_r = shard.router
        ops._need_cuda(w_r, shard.bias)
        H = w_r.shape[1]
        self.dtype = w_r.dtype
        E_loc, I_loc = ops._check_weights(shard.experts, H, self.dtype)
        if E_loc != E // groups:
            raise ValueError(f"rank holds {E_loc} experts, expected {E // groups}")
        I = I_loc * tp
        self.tp = tp
        Is = shard.shared.gate_proj.shape[0] if shard.shared is not None else 0
        self.dims = (H, E, I, Is, K)
        self.max_tokens = int(max_tokens)
        self.device = w_r.device
        L = api.lib()
        full = ops._shape(self.max_tokens, H, E, I, Is, K, self.dtype)
        box_bytes = L.tarfa_b200_ep_box_bytes(C.byref(full), self.world, self.max_tokens)
        ws_bytes = L.tarfa_b200_ep_workspace_size(C.byref(full), self.world, self.max_tokens)
        self.ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=self.device)
        self._box = C.c_void_p()
        handle = (C.c_uint8 * api.EP_IPC_HANDLE_BYTES)()
        with torch.cuda.device(self.device):
            api.check(L.tarfa_b200_ep_box_alloc(box_bytes, C.byref(self._box), handle))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._peers = []
        boxes = []
        with torch.cuda.device(self.device):
            for r, hb in enumerate(handles):
                if r == self.rank:
                    boxes.append(self._box.value)
                    continue
                p = C.c_void_p()
                buf = (C.c_uint8 * api.EP_IPC_HANDLE_BYTES).from_buffer_copy(hb)
                api.check(L.tarfa_b200_ep_box_open(buf, C.byref(p)))
                self._peers.append(p)
                boxes.append(p.value)
        arr = (C.c_void_p * api.EP_MAX_RANKS)(*boxes)
        self._group = api.EpGroup(self.world, self.rank, self.max_tokens, tp, 0, arr)
        self._wc = shard.experts.c_struct()
        self._sc = shard.shared.c_struct() if shard.shared is not None else None
        self._fn = L.tarfa_b200_ep_moe_layer
        dist.barrier(group)   # every box is mapped everywhere before the first store

    def forward(self, h: torch.Tensor, return_routing: bool = False,
                out: torch.Tensor | None = None):
        ops._need_cuda(h, out)
        T, H = h.shape
        H0, E, I, Is, K = self.dims
        if H != H0 or h.dtype != self.dtype:
            raise RuntimeError("hidden states do not match the layer")
        if not 1 <= T <= self.max_tokens:
            raise RuntimeError(f"{T} tokens not in [1, max_tokens={self.max_tokens}]")
        if out is None:
            out = torch.empty_like(h)
        idx = torch.empty((T, K), dtype=torch.int64, device=h.device) if return_routing else None
        wt = torch.empty((T, K), dtype=torch.float32, device=h.device) if return_routing else None
        shape = ops._shape(T, H, E, I, Is, K, h.dtype)
        api.check(self._fn(C.byref(shape), ops._ptr(h), ops._ptr(self.s.router), ops._ptr(self.s.bias),
                           C.byref(self._wc), C.byref(self._sc) if self._sc is not None else None,
                           C.byref(self._group), ops._ptr(out), ops._ptr(idx), ops._ptr(wt),
                           ops._ptr(self.ws), self.ws.numel(), ops._stream(h.device)))
        return (out, idx, wt) if return_routing else out

    __call__ = forward

    def bind(self, shard: EPShard) -> "PeerExpertParallelMoE":
        """This group (boxes, workspace, step counter) with another layer's
        weights of the same shapes: the layers of a stack share one group and
        run in order on one stream.  Not collective; every rank binds the same
        layers and calls them in the same order.  The bound layer is released
        with this one (its own ``close`` does nothing)."""
        H, E, I, Is, K = self.dims
        if shard.num_experts != E or shard.top_k != K or tuple(shard.router.shape) != (E, H):
            raise ValueError("bound layer's router does not match the group's layer")
        ops._need_cuda(shard.router, shard.bias)
        E_loc, I_loc = ops._check_weights(shard.experts, H, self.dtype)
        if E_loc != E // (self.world // self.tp) or I_loc * self.tp != I:
            raise ValueError("bound layer's experts do not match the group's layer")
        Is_b = shard.shared.gate_proj.shape[0] if shard.shared is not None else 0
        if Is_b != Is:
            raise ValueError("bound layer's shared expert does not match the group's layer")
        b = copy.copy(self)
        b.s = shard
        b._wc = shard.experts.c_struct()
        b._sc = shard.shared.c_struct() if shard.shared is not None else None
        b._bound = True
        return b

    def close(self):
        """Collective: unmap the peers' boxes, then free this rank's own."""
        if getattr(self, "_bound", False) or self._box is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        L = api.lib()
        with torch.cuda.device(self.device):
            for p in self._peers:
                api.check(L.tarfa_b200_ep_box_close(p))
            self._peers = []
            dist.barrier(self.group)
            api.check(L.tarfa_b200_ep_box_free(self._box))
        self._box = None
