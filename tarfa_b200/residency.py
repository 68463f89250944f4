"""Expert residency: the VRAM tier of the routed experts.

Mirrors the reference's residency interface
``read_bf16(layer, experts, device, dtype, use_ram_cache=False) -> {e: (gate_up, down)}``
(``tarfa/engine/exact_bf16.py:126-161``) and its ``stats(reset)``
(``exact_bf16.py:68-75``).  On a B200 the full layer is resident in HBM as one
stacked tensor per projection (``gate_up [E, 2I, H]``, ``down [E, H, I]``), so a
read is a view, not a transfer; the kernels index the stacks directly.

The reference returns from ``read_bf16`` only after ``torch.cuda.synchronize``
(``exact_bf16.py:186``); here nothing is copied, so no synchronisation is
needed and the views are valid immediately.
"""
from __future__ import annotations

import threading

import torch

from .ops import ExpertWeights


class ExpertStore:
    """Per-layer resident expert stacks, dense (exact mode) and/or int4 (fast mode)."""

    def __init__(self, device="cuda", dtype=torch.bfloat16):
        self.device = torch.device(device)
        self.dtype = dtype
        self._dense: dict[int, ExpertWeights] = {}
        self._int4: dict[int, ExpertWeights] = {}
        self._lock = threading.Lock()
        self._stat = {"calls": 0, "experts": 0, "bytes": 0, "read_seconds": 0.0,
                      "h2d_seconds": 0.0, "prefetch_calls": 0, "prefetch_bytes": 0}

    # -- population -----------------------------------------------------------
    def put_layer(self, layer: int, gate_up: torch.Tensor, down: torch.Tensor):
        """Make layer ``layer``'s dense experts resident (copied to the device once)."""
        gu = gate_up.to(self.device, self.dtype).contiguous()
        dn = down.to(self.device, self.dtype).contiguous()
        self._dense[layer] = ExpertWeights(gu, dn, "dense")

    def put_layer_int4(self, layer: int, gate_up_q, gate_up_s, down_q, down_s, group: int):
        """Make layer ``layer``'s int4 experts resident (scales cast to the model dtype,
        as the reference does on load, ``fused_int4.py:139-141``)."""
        dev = self.device
        self._int4[layer] = ExpertWeights(
            gate_up_q.to(dev).contiguous(), down_q.to(dev).contiguous(), "int4",
            gate_up_s.to(dev, self.dtype).contiguous(), down_s.to(dev, self.dtype).contiguous(),
            int(group))

    def has_layer(self, layer: int, kind: str = "dense") -> bool:
        return layer in (self._dense if kind == "dense" else self._int4)

    def layer_weights(self, layer: int, kind: str = "dense") -> ExpertWeights:
        table = self._dense if kind == "dense" else self._int4
        try:
            return table[layer]
        except KeyError:
            raise RuntimeError(f"layer {layer} has no resident {kind} experts") from None

    # -- the reference's residency interface ------------------------------------
    def read_bf16(self, layer: int, experts, device=None, dtype=None, use_ram_cache=False):
        """``{e: (gate_up[2I, H], down[H, I])}`` for the requested experts (views)."""
        w = self.layer_weights(layer, "dense")
        if dtype is not None and dtype != w.gate_up.dtype:
            raise RuntimeError(f"resident experts are {w.gate_up.dtype}, asked for {dtype}")
        out = {int(e): (w.gate_up[int(e)], w.down[int(e)]) for e in experts}
        with self._lock:
            self._stat["calls"] += 1
            self._stat["experts"] += len(out)
        return out

    def stats(self, reset: bool = False) -> dict:
        with self._lock:
            out = dict(self._stat)
            if reset:
                for k in self._stat:
                    self._stat[k] = 0.0 if k.endswith("seconds") else 0
        out["read_GBps"] = 0.0
        return out

    def resident_bytes(self) -> int:
        n = 0
        for table in (self._dense, self._int4):
            for w in table.values():
                for t in (w.gate_up, w.down, w.gate_up_scale, w.down_scale):
                    if t is not None:
                        n += t.numel() * t.element_size()
        return n
