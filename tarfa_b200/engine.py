"""The drop-in engine: the reference's routed-compute interface, on B200 kernels.

``TarfaB200._install_streamed_experts(experts, pre)`` has the signature and the
effect of the reference's ``TarfaFused._install_streamed_experts``
(``tarfa/engine/fused_int4.py:148-262``, base ``channel.py:40``): it binds
``experts.forward(hidden_states, top_k_index, top_k_weights) -> [T, H]`` on the
``transformers`` experts module of one MoE block, shadowing its class-level
forward (``transformers/integrations/moe.py:508-511``).  The caller — the
``Qwen3_5MoeSparseMoeBlock.forward`` of ``modeling_qwen3_5_moe.py:781-792`` —
is unchanged.

Mode selection keeps the reference's environment semantics
(``fused_int4.py:17,63``, ``cli.py:28-34``): ``BF16=1`` (``tarfa serve``) is the
exact path over dense experts, anything else (``tarfa start-fast``) the int4
fast path; ``JTOPK`` (default 8 = no truncation) keeps the top-``JTOPK``
routes and renormalises.

``install_moe_block(block, pre)`` additionally replaces the whole block's
forward with the fused device op (router + experts + shared expert).
"""
from __future__ import annotations

import os
import re
import threading
import types

import torch

from . import ops
from .residency import ExpertStore


def _env_bf16() -> bool:
    return os.environ.get("BF16", "0") == "1"


def _env_jtopk() -> int:
    return int(os.environ.get("JTOPK", "8"))


class TarfaB200:
    """Engine object the reference's model skeleton calls into.

    Attributes the reference's closures read from the engine: ``device``,
    ``dtype``, ``nL`` (``fused_int4.py:152-153``).
    """

    def __init__(self, store: ExpertStore, nL: int, device=None, dtype=None,
                 bf16: bool | None = None, jtopk: int | None = None):
        self.store = store
        self.device = torch.device(device) if device is not None else store.device
        self.dtype = dtype if dtype is not None else store.dtype
        self.nL = nL
        self.bf16 = _env_bf16() if bf16 is None else bf16
        self.jtopk = _env_jtopk() if jtopk is None else jtopk
        self._tlock = threading.Lock()
        self._tstat = {"moe_calls": 0, "prefill_moe_calls": 0, "decode_moe_calls": 0}

    @property
    def kind(self) -> str:
        return "dense" if self.bf16 else "int4"

    # -- telemetry (fused_int4.py:97-109, counters only: no host sync) ---------
    def telemetry(self, reset: bool = False) -> dict:
        with self._tlock:
            out = dict(self._tstat)
            if reset:
                for k in self._tstat:
                    self._tstat[k] = 0
        return out

    def _count(self, T: int):
        with self._tlock:
            self._tstat["moe_calls"] += 1
            self._tstat["decode_moe_calls" if T == 1 else "prefill_moe_calls"] += 1

    @staticmethod
    def _layer_of(pre: str) -> int:
        return int(re.search(r"layers\.(\d+)\.", pre).group(1))   # fused_int4.py:149

    def _truncate(self, idx: torch.Tensor, w: torch.Tensor):
        """fused_int4.py:157-160 (a no-op at the default JTOPK=8)."""
        if w.shape[-1] <= self.jtopk:
            return idx, w
        tv, ti = w.topk(self.jtopk, dim=-1)
        return torch.gather(idx, -1, ti).contiguous(), (tv / tv.sum(dim=-1, keepdim=True)).contiguous()

    def _install_streamed_experts(self, experts, pre: str):
        eng = self
        layer = self._layer_of(pre)

        def forward(self, hidden_states, top_k_index, top_k_weights):
            top_k_index, top_k_weights = eng._truncate(top_k_index, top_k_weights)
            w = eng.store.layer_weights(layer, eng.kind)
            eng._count(hidden_states.shape[0])
            return ops.experts_forward(hidden_states.contiguous(), top_k_index.contiguous(),
                                       top_k_weights.to(torch.float32).contiguous(), w)

        experts.forward = types.MethodType(forward, experts)

    def install_moe_block(self, block, pre: str):
        """Replace ``Qwen3_5MoeSparseMoeBlock.forward`` by the fused layer op.

        The block keeps its router / shared-expert parameters; they are read
        from it on every call (views, no copies).
        """
        eng = self
        layer = self._layer_of(pre)
        if self.jtopk < block.gate.top_k:
            raise RuntimeError("the fused block op routes top-k natively; use "
                               "_install_streamed_experts for JTOPK truncation")

        def forward(self, hidden_states):
            B, S, H = hidden_states.shape
            h = hidden_states.reshape(-1, H).contiguous()
            sh = ops.SharedWeights(self.shared_expert.gate_proj.weight,
                                   self.shared_expert.up_proj.weight,
                                   self.shared_expert.down_proj.weight,
                                   self.shared_expert_gate.weight)
            eng._count(h.shape[0])
            y = ops.moe_layer(h, self.gate.weight, eng.store.layer_weights(layer, eng.kind), sh,
                              top_k=self.gate.top_k)
            return y.reshape(B, S, H)

        block.forward = types.MethodType(forward, block)
