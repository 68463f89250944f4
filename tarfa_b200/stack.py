"""Synthetic MoE-only decoder stack for whole-model measurements.

``n_layers`` x (``h = h + MoE(RMSNorm(h))``) between an embedding and an LM
head with greedy argmax: the MoE path of the reference's decoder layer
(``modeling_qwen3_5_moe.py:828-870``: post-attention RMSNorm, sparse MoE block,
residual) with attention left out; the reference takes its final logits in fp32
(``serve.py:128-132``), this stack in fp64 (below).  Weights are synthetic, regenerable per (layer, expert)
(``tarfa_b200.synthetic``); the routed experts come from a
``StreamingExpertTier`` (resident + pinned-host streaming) or are all resident.

RMSNorm follows ``Qwen3_5MoeRMSNorm`` (modeling_qwen3_5_moe.py:795-808),
``x * rsqrt(mean(x^2) + eps) * (1 + w)`` rounded to the model dtype, but in
fp64 with the squares summed by a fixed pairwise tree of elementwise adds:
IEEE additions, division and square root in a fixed order give the CUDA stack
and the CPU oracle stack the same bits (a library reduction would depend on its
order and on the device's rsqrt).  The LM head is fp64 (its argmax is the
greedy token; summation order moves its logits by ~1e-16 relative).  These two are the synthetic skeleton around
the MoE blocks, not part of the path under test.
"""
from __future__ import annotations

import torch

from . import ops
from . import synthetic as syn
from .streaming import StreamingExpertTier


def _tree_sum(v: torch.Tensor) -> torch.Tensor:
    """Sum over the last dimension by a fixed pairwise tree of elementwise adds
    (halves while even, then left to right): the same additions in the same
    order on every device."""
    while v.shape[-1] > 1 and v.shape[-1] % 2 == 0:
        n = v.shape[-1] // 2
        v = v[..., :n] + v[..., n:]
    acc = v[..., :1]
    for j in range(1, v.shape[-1]):
        acc = acc + v[..., j:j + 1]
    return acc


def rms_norm_host(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """The stack's RMSNorm as torch operations (any device): the reference
    statement of ``tarfa_b200_rms_norm``."""
    xd = x.double()
    r = 1.0 / torch.sqrt(_tree_sum(xd * xd) / x.shape[-1] + eps)
    return (xd * r * (1.0 + w.double())).to(torch.float32).to(x.dtype)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """One kernel on the GPU (``ops.rms_norm``), torch operations on the CPU;
    the same bits either way."""
    return ops.rms_norm(x, w, eps) if x.is_cuda else rms_norm_host(x, w, eps)


def lm_head_argmax(h: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Greedy token: argmax of the fp64 logits h @ w.T (``w`` in the model dtype
    or already in fp64)."""
    return (h.double() @ w.double().t()).argmax(-1)


class SyntheticStack:
    def __init__(self, shape: syn.LayerShape, n_layers: int, vocab: int, device, seed: int = 0,
                 resident: int | None = None, staging: int = 64, dtype=torch.bfloat16):
        self.s, self.n, self.V = shape, n_layers, vocab
        self.device = torch.device(device)
        self.dtype = dtype
        g = torch.Generator(device=self.device).manual_seed(syn._mix(seed, 0xE5))

        def n(shape_, std):
            t = torch.empty(shape_, dtype=torch.float32, device=self.device)
            t.normal_(0.0, std, generator=g)
            return t.to(dtype)

        self.embed = n((vocab, shape.hidden), 1.0)
        self.lm_head = n((vocab, shape.hidden), 0.02)
        self.final_norm = n((shape.hidden,), 0.1)
        R = shape.experts if resident is None else resident
        self.tier = StreamingExpertTier(n_layers, shape.experts, shape.hidden, shape.inter, R,
                                        max(1, staging), self.device, dtype)
        self.layers = []
        for l in range(n_layers):
            L = syn.layer_device(syn._mix(seed, l), shape, self.device, dtype)
            self.tier.load_layer(l, L["gate_up"], L["down"])
            self.layers.append({
                "norm": n((shape.hidden,), 0.1), "router": L["router"],
                "shared": ops.SharedWeights(L["sh_gate"], L["sh_up"], L["sh_down"], L["sh_gate_w"]),
            })
            del L
        self._prev = [None] * n_layers

    def expert_cpu(self, l: int, e: int):
        """(gate_up, down) of expert ``e`` of layer ``l`` on the CPU (for the oracle)."""
        return self.tier.expert_cpu(l, e)

    def layer_weights_cpu(self, l: int):
        """(gate_up, down) of all experts of layer l, on the CPU (for the oracle)."""
        R = self.tier.R
        gu = torch.empty((self.s.experts, 2 * self.s.inter, self.s.hidden), dtype=self.dtype)
        dn = torch.empty((self.s.experts, self.s.hidden, self.s.inter), dtype=self.dtype)
        if R:
            gu[:R] = self.tier.gate_up[l * R:(l + 1) * R].cpu()
            dn[:R] = self.tier.down[l * R:(l + 1) * R].cpu()
        if R < self.s.experts:
            gu[R:] = self.tier.host_gu[l]
            dn[R:] = self.tier.host_dn[l]
        return gu, dn

    @torch.no_grad()
    def step(self, tokens: torch.Tensor, prefetch="pipe") -> torch.Tensor:
        """One decode step for a batch of token ids -> next token ids (greedy).

        ``prefetch``: which of the next layer's experts to start copying while
        this layer computes.  "pipe": the ones the next layer used for the
        previous step (the reference's PIPE prediction, fused_int4.py:206-224).
        "pregate": the next layer's router applied to this layer's input (its
        ids come back with this layer's, in one host read); the residual stream
        changes little per layer, so it mostly names the next layer's experts.
        None: no prefetch.  The prediction only moves copies earlier: each
        layer still routes exactly and stages whatever it misses."""
        h = self.embed.index_select(0, tokens.to(self.device))
        for l, layer in enumerate(self.layers):
            x = rms_norm(h, layer["norm"])
            idx, _ = ops.router_topk(x, layer["router"], self.s.top_k)
            pregate = prefetch == "pregate" and l + 1 < self.n
            if pregate:
                nidx, _ = ops.router_topk(x, self.layers[l + 1]["router"], self.s.top_k)
                both = torch.cat([idx.view(-1), nidx.view(-1)]).tolist()   # one host read
                k = idx.numel()
                ids, pred = sorted(set(both[:k])), sorted(set(both[k:]))
            else:
                ids = sorted(set(idx.view(-1).tolist()))   # routed ids on the host (fused_int4.py:166)
            weights = self.tier.weights_for(l, ids)
            if pregate:
                self.tier.prefetch(l + 1, pred)
            elif prefetch and l + 1 < self.n and self._prev[l + 1] is not None:
                self.tier.prefetch(l + 1, self._prev[l + 1])   # PIPE-style prediction
            self._prev[l] = ids
            # the whole block over the staged experts (the router again: exact, so
            # the same routes); the same arithmetic as the expert-parallel stack's
            # layers, which equal this layer bit for bit
            h = h + ops.moe_layer(x, layer["router"], weights, layer["shared"], self.s.top_k)
        return lm_head_argmax(rms_norm(h, self.final_norm), self.lm_head)


class ExpertParallelStack:
    """The synthetic stack run expert-parallel over the ranks of ``group`` (one
    process per GPU): the same model as :class:`SyntheticStack` built from the
    same seed.  The embedding, norms, routers, shared experts and LM head are
    replicated; rank ``r`` of ``N`` keeps experts ``[r*E/N, (r+1)*E/N)`` of
    every layer resident.  Each MoE block is one call of the peer-memory
    expert-parallel layer (``tarfa_b200_ep_moe_layer``); all layers share one
    peer group (its boxes, workspace and step counter).

    Construction and :meth:`close` are collective.  Every rank steps with its
    own tokens, the same count on every rank, at most ``max_tokens``."""

    def __init__(self, shape: syn.LayerShape, n_layers: int, vocab: int, device, seed: int = 0,
                 group=None, max_tokens: int = 64, dtype=torch.bfloat16):
        import torch.distributed as dist
        from .ep import EPShard, PeerExpertParallelMoE
        self.s, self.n, self.V = shape, n_layers, vocab
        self.device = torch.device(device)
        self.dtype = dtype
        self.seed = seed
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        E = shape.experts
        if E % world:
            raise ValueError(f"{E} experts do not shard evenly over {world} ranks")
        e0, e1 = rank * E // world, (rank + 1) * E // world
        g = torch.Generator(device=self.device).manual_seed(syn._mix(seed, 0xE5))

        def n(shape_, std):   # same draws, in the same order, as SyntheticStack
            t = torch.empty(shape_, dtype=torch.float32, device=self.device)
            t.normal_(0.0, std, generator=g)
            return t.to(dtype)

        self.embed = n((vocab, shape.hidden), 1.0)
        self.lm_head = n((vocab, shape.hidden), 0.02)
        self.final_norm = n((shape.hidden,), 0.1)
        self.layers = []
        for l in range(n_layers):
            L = syn.layer_device(syn._mix(seed, l), shape, self.device, dtype)
            mine = ops.ExpertWeights(L["gate_up"][e0:e1].clone(), L["down"][e0:e1].clone())
            shared = ops.SharedWeights(L["sh_gate"], L["sh_up"], L["sh_down"], L["sh_gate_w"])
            shard = EPShard(L["router"], mine, shared, E, shape.top_k)
            del L
            self.layers.append({"norm": n((shape.hidden,), 0.1), "shard": shard})
        self._head64 = self.lm_head.double()   # converted once, not every step
        self._group = PeerExpertParallelMoE(self.layers[0]["shard"], group, max_tokens)
        self.moe = [self._group] + [self._group.bind(x["shard"]) for x in self.layers[1:]]

    def full_layer(self, l: int):
        """All experts of layer ``l`` (regenerated from the seed) as single-GPU
        weights, with its router and shared expert: (router, experts, shared)."""
        L = syn.layer_device(syn._mix(self.seed, l), self.s, self.device, self.dtype)
        sh = self.layers[l]["shard"]
        return sh.router, ops.ExpertWeights(L["gate_up"], L["down"]), sh.shared

    @torch.no_grad()
    def step(self, tokens: torch.Tensor, record: list | None = None) -> torch.Tensor:
        """One decode step of this rank's tokens -> next token ids (greedy).
        ``record``: if given, gets each layer's (MoE input, MoE output)."""
        h = self.embed.index_select(0, tokens.to(self.device))
        for l, layer in enumerate(self.layers):
            x = rms_norm(h, layer["norm"])
            y = self.moe[l](x)
            if record is not None:
                record.append((x, y))
            h = h + y
        return lm_head_argmax(rms_norm(h, self.final_norm), self._head64)

    def close(self):
        """Collective: releases the peer group."""
        if self._group is not None:
            self._group.close()
            self._group = None
