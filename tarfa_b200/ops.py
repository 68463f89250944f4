"""Torch-tensor wrappers over the C ABI (device memory and streams come from torch).

Each wrapper checks shapes, dtypes, devices and contiguity, passes raw device
pointers plus the current CUDA stream to ``libtarfa_b200.so`` and raises
``RuntimeError`` (``TarfaError``) on a non-zero return.  Nothing here computes
on the CPU: a CPU tensor is an error, and a missing library is an error.

Scratch: every device gets one zero-filled workspace buffer, grown on demand;
the kernels return its counters to zero, so consecutive calls on one stream
can share it.  Callers that launch on several streams at once must pass their
own ``workspace`` tensors.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import threading

import torch

from . import _capi as api

_DT = {torch.bfloat16: api.TARFA_BF16, torch.float16: api.TARFA_F16}
_ws_lock = threading.Lock()
_ws: dict[int, torch.Tensor] = {}


def _ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else C.c_void_p(0)


def _stream(device) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _need_cuda(*ts):
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("tarfa_b200 ops take CUDA tensors only (no CPU path)")
        if not t.is_contiguous():
            raise RuntimeError("tarfa_b200 ops take contiguous tensors")


def workspace(nbytes: int, device) -> torch.Tensor:
    """Shared zero-filled scratch of at least ``nbytes`` on ``device``."""
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    with _ws_lock:
        buf = _ws.get(idx)
        if buf is None or buf.numel() < nbytes:
            if buf is not None:
                torch.cuda.current_stream(dev).synchronize()
            buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
            _ws[idx] = buf
        return buf


def _shape(T, H, E, I, Is, K, dtype) -> api.MoeShape:
    if dtype not in _DT:
        raise RuntimeError(f"unsupported dtype {dtype}; bf16 or fp16")
    return api.MoeShape(T, H, E, I, Is, K, _DT[dtype])


@dataclasses.dataclass
class ExpertWeights:
    """Routed-expert weights of one layer, resident on the device.

    kind ``"dense"``: ``gate_up [E, 2I, H]``, ``down [E, H, I]`` in the model dtype.
    kind ``"int4"``: ``gate_up`` int32 ``[E, 2I, H/8]`` (or uint8 ``[E, 2I, H/2]``),
    ``down`` int32 ``[E, H, I/8]``, scales in the model dtype ``[E, N, K/group]``
    (``group`` > 0) or ``[E, N]`` (``group == 0``, the reference's per-row layout).
    ``expert_slot`` (optional int32 ``[E]``): expert ``e`` is stored at index
    ``expert_slot[e]`` of the stacks (used by a streaming tier).
    """
    gate_up: torch.Tensor
    down: torch.Tensor
    kind: str = "dense"
    gate_up_scale: torch.Tensor | None = None
    down_scale: torch.Tensor | None = None
    group: int = 0
    expert_slot: torch.Tensor | None = None

    def c_struct(self) -> api.MoeWeights:
        _need_cuda(self.gate_up, self.down, self.gate_up_scale, self.down_scale, self.expert_slot)
        kind = api.TARFA_W_INT4 if self.kind == "int4" else api.TARFA_W_DENSE
        if self.expert_slot is not None and self.expert_slot.dtype != torch.int32:
            raise RuntimeError("expert_slot must be int32")
        return api.MoeWeights(kind, int(self.group), _ptr(self.gate_up), _ptr(self.gate_up_scale),
                              _ptr(self.down), _ptr(self.down_scale), _ptr(self.expert_slot),
                              self.slots() if self.expert_slot is not None else 0)

    def dims(self, H: int):
        """(E, I): with an ``expert_slot`` table, E is its length (the layer's
        experts; the stacks hold any number of slots), else the stacks' depth."""
        E = self.expert_slot.numel() if self.expert_slot is not None else self.gate_up.shape[0]
        I = self.gate_up.shape[1] // 2
        return E, I

    def slots(self) -> int:
        """Depth of the weight stacks (slots the kernels may read)."""
        return self.gate_up.shape[0]


@dataclasses.dataclass
class SharedWeights:
    """Shared expert (``Qwen3_5MoeMLP``) and its sigmoid gate, model dtype."""
    gate_proj: torch.Tensor   # [Is, H]
    up_proj: torch.Tensor     # [Is, H]
    down_proj: torch.Tensor   # [H, Is]
    gate_weight: torch.Tensor  # [1, H]

    def c_struct(self) -> api.SharedExpert:
        _need_cuda(self.gate_proj, self.up_proj, self.down_proj, self.gate_weight)
        return api.SharedExpert(_ptr(self.gate_proj), _ptr(self.up_proj), _ptr(self.down_proj),
                                _ptr(self.gate_weight))


def _check_weights(w: ExpertWeights, H: int, dtype):
    E, I = w.dims(H)
    S = w.slots()
    if w.expert_slot is not None and (w.expert_slot.dtype != torch.int32 or
                                      w.expert_slot.device != w.gate_up.device):
        raise RuntimeError("expert_slot must be an int32 tensor on the weights' device")
    if w.kind == "dense":
        if w.gate_up.dtype != dtype or w.down.dtype != dtype:
            raise RuntimeError("dense expert weights must be in the activation dtype")
        if tuple(w.gate_up.shape) != (S, 2 * I, H) or tuple(w.down.shape) != (S, H, I):
            raise RuntimeError(f"expert weight shapes {tuple(w.gate_up.shape)} / "
                               f"{tuple(w.down.shape)} do not match H={H}")
    elif w.kind == "int4":
        for t, (n, k) in ((w.gate_up, (2 * I, H)), (w.down, (H, I))):
            if t.dtype not in (torch.int32, torch.uint8):
                raise RuntimeError("int4 weights must be int32 or uint8 packed")
            if t.shape[0] != S or t.shape[1] != n or t.numel() * t.element_size() != S * n * k // 2:
                raise RuntimeError("int4 weight shape mismatch")
        for s, n, k in ((w.gate_up_scale, 2 * I, H), (w.down_scale, H, I)):
            if s is None or s.dtype != dtype:
                raise RuntimeError("int4 scales must be given in the activation dtype")
            want = S * n * (k // w.group if w.group else 1)
            if s.numel() != want:
                raise RuntimeError(f"int4 scale has {s.numel()} elements, expected {want}")
    else:
        raise RuntimeError(f"unknown weight kind {w.kind}")
    return E, I


def router_topk(h: torch.Tensor, w_r: torch.Tensor, top_k: int, bias: torch.Tensor | None = None,
                return_logits: bool = False):
    """``Qwen3_5MoeTopKRouter.forward`` on the device: ``(top_k_index int64, top_k_weights fp32)``.

    Logits are correctly rounded model-dtype values of ``h @ w_r.T`` (+ ``bias``);
    equal values are ordered as the reference's ``torch.topk`` orders them on
    the CPU.
    """
    _need_cuda(h, w_r, bias)
    T, H = h.shape
    E = w_r.shape[0]
    if w_r.shape[1] != H or w_r.dtype != h.dtype or (bias is not None and bias.dtype != h.dtype):
        raise RuntimeError("router weight / bias must match hidden size and dtype")
    shape = _shape(T, H, E, 32, 0, top_k, h.dtype)
    idx = torch.empty((T, top_k), dtype=torch.int64, device=h.device)
    w = torch.empty((T, top_k), dtype=torch.float32, device=h.device)
    lg = torch.empty((T, E), dtype=torch.float32, device=h.device) if return_logits else None
    L = api.lib()
    nbytes = L.tarfa_b200_workspace_size(C.byref(shape), api.OP_ROUTER)
    ws = workspace(nbytes, h.device)
    api.check(L.tarfa_b200_router_topk(C.byref(shape), _ptr(h), _ptr(w_r), _ptr(bias), _ptr(idx),
                                       _ptr(w), _ptr(lg), _ptr(ws), ws.numel(), _stream(h.device)))
    return (idx, w, lg) if return_logits else (idx, w)


def permute(top_idx: torch.Tensor, num_experts: int):
    """Expert-sorted route order: ``(seg_offsets[E+1], perm_token[R], perm_slot[R])`` int32."""
    _need_cuda(top_idx)
    if top_idx.dtype != torch.int64:
        raise RuntimeError("top_idx must be int64")
    T, K = top_idx.shape
    shape = _shape(T, 32, num_experts, 32, 0, K, torch.bfloat16)
    dev = top_idx.device
    seg = torch.zeros(num_experts + 1, dtype=torch.int32, device=dev)
    tok = torch.empty(T * K, dtype=torch.int32, device=dev)
    slot = torch.empty(T * K, dtype=torch.int32, device=dev)
    L = api.lib()
    ws = workspace(L.tarfa_b200_workspace_size(C.byref(shape), api.OP_PERMUTE), dev)
    api.check(L.tarfa_b200_permute(C.byref(shape), _ptr(top_idx), _ptr(seg), _ptr(tok), _ptr(slot),
                                   _ptr(ws), ws.numel(), _stream(dev)))
    return seg, tok, slot


def experts_forward(h: torch.Tensor, top_idx: torch.Tensor, top_w: torch.Tensor,
                    weights: ExpertWeights, out: torch.Tensor | None = None) -> torch.Tensor:
    """The routed-experts closure: ``experts.forward(h, top_k_index, top_k_weights)``."""
    _need_cuda(h, top_idx, top_w, out)
    T, H = h.shape
    if top_idx.dtype != torch.int64 or top_w.dtype != torch.float32 or top_idx.shape != top_w.shape:
        raise RuntimeError("top_k_index int64 and top_k_weights fp32 of one shape [T, K]")
    E, I = _check_weights(weights, H, h.dtype)
    K = top_idx.shape[1]
    if out is None:
        out = torch.empty_like(h)
    shape = _shape(T, H, E, I, 0, K, h.dtype)
    L = api.lib()
    ws = workspace(L.tarfa_b200_workspace_size(C.byref(shape), api.OP_EXPERTS), h.device)
    wc = weights.c_struct()
    api.check(L.tarfa_b200_experts_forward(C.byref(shape), _ptr(h), _ptr(top_idx), _ptr(top_w),
                                           C.byref(wc), _ptr(out), _ptr(ws), ws.numel(),
                                           _stream(h.device)))
    return out


def moe_layer(h: torch.Tensor, w_r: torch.Tensor, weights: ExpertWeights,
              shared: SharedWeights | None, top_k: int = 8, bias: torch.Tensor | None = None,
              return_routing: bool = False, out: torch.Tensor | None = None):
    """``Qwen3_5MoeSparseMoeBlock.forward`` (router + routed experts + gated shared expert)."""
    _need_cuda(h, w_r, bias, out)
    T, H = h.shape
    E, I = _check_weights(weights, H, h.dtype)
    if w_r.shape != (E, H) or w_r.dtype != h.dtype:
        raise RuntimeError("router weight must be [E, H] in the activation dtype")
    Is = shared.gate_proj.shape[0] if shared is not None else 0
    if out is None:
        out = torch.empty_like(h)
    idx = torch.empty((T, top_k), dtype=torch.int64, device=h.device) if return_routing else None
    wt = torch.empty((T, top_k), dtype=torch.float32, device=h.device) if return_routing else None
    shape = _shape(T, H, E, I, Is, top_k, h.dtype)
    L = api.lib()
    ws = workspace(L.tarfa_b200_workspace_size(C.byref(shape), api.OP_MOE_LAYER), h.device)
    wc = weights.c_struct()
    sc = shared.c_struct() if shared is not None else None
    api.check(L.tarfa_b200_moe_layer(C.byref(shape), _ptr(h), _ptr(w_r), _ptr(bias), C.byref(wc),
                                     C.byref(sc) if sc is not None else None, _ptr(out), _ptr(idx),
                                     _ptr(wt), _ptr(ws), ws.numel(), _stream(h.device)))
    return (out, idx, wt) if return_routing else out


def shared_expert(h: torch.Tensor, shared: SharedWeights, out: torch.Tensor | None = None):
    """``sigmoid(shared_expert_gate(h)) * shared_expert(h)`` alone, ``[T, H]``."""
    _need_cuda(h, out)
    T, H = h.shape
    Is = shared.gate_proj.shape[0]
    if out is None:
        out = torch.empty_like(h)
    shape = _shape(T, H, 1, 32, Is, 1, h.dtype)
    L = api.lib()
    ws = workspace(L.tarfa_b200_workspace_size(C.byref(shape), api.OP_SHARED), h.device)
    sc = shared.c_struct()
    api.check(L.tarfa_b200_shared_expert(C.byref(shape), _ptr(h), C.byref(sc), _ptr(out), _ptr(ws),
                                         ws.numel(), _stream(h.device)))
    return out


def combine_routes(y_routes: torch.Tensor, top_idx: torch.Tensor, top_w: torch.Tensor,
                   num_experts: int, shared_gated: torch.Tensor | None = None,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """Reference-order combine of per-route expert outputs ``y_routes [T*K, H]``."""
    _need_cuda(y_routes, top_idx, top_w, shared_gated, out)
    T, K = top_idx.shape
    H = y_routes.shape[1]
    if y_routes.shape[0] != T * K or top_idx.dtype != torch.int64 or top_w.dtype != torch.float32:
        raise RuntimeError("y_routes [T*K, H], top_idx int64 [T, K], top_w fp32 [T, K]")
    if out is None:
        out = torch.empty((T, H), dtype=y_routes.dtype, device=y_routes.device)
    shape = _shape(T, H, num_experts, 32, 0, K, y_routes.dtype)
    api.check(api.lib().tarfa_b200_combine_routes(C.byref(shape), _ptr(y_routes), _ptr(top_idx),
                                                  _ptr(top_w), _ptr(shared_gated), _ptr(out),
                                                  _stream(y_routes.device)))
    return out


class MoePlan:
    """A prepared ``moe_layer`` call on fixed device buffers.

    Shapes, pointers and the C structs are built once; :meth:`run` is a single
    foreign call (a few microseconds of host time), and :meth:`capture`
    records the layer's kernels into a CUDA graph so a decode step replays
    them with no host launch work at all.  The plan owns a private workspace,
    so plans may run on different streams.  Inputs are read from ``self.h``
    (copy new tokens into it), the result lands in ``self.out``.
    """

    def __init__(self, h: torch.Tensor, w_r: torch.Tensor, weights: ExpertWeights,
                 shared: SharedWeights | None, top_k: int = 8, bias: torch.Tensor | None = None,
                 return_routing: bool = False):
        _need_cuda(h, w_r, bias)
        T, H = h.shape
        E, I = _check_weights(weights, H, h.dtype)
        if w_r.shape != (E, H) or w_r.dtype != h.dtype:
            raise RuntimeError("router weight must be [E, H] in the activation dtype")
        Is = shared.gate_proj.shape[0] if shared is not None else 0
        self.h, self.w_r, self.bias, self.weights, self.shared = h, w_r, bias, weights, shared
        self.out = torch.empty_like(h)
        dev = h.device
        self.top_idx = torch.empty((T, top_k), dtype=torch.int64, device=dev) if return_routing else None
        self.top_w = torch.empty((T, top_k), dtype=torch.float32, device=dev) if return_routing else None
        self._shape = _shape(T, H, E, I, Is, top_k, h.dtype)
        L = api.lib()
        n = L.tarfa_b200_workspace_size(C.byref(self._shape), api.OP_MOE_LAYER)
        self.ws = torch.zeros(n, dtype=torch.uint8, device=dev)
        self._wc = weights.c_struct()
        self._sc = shared.c_struct() if shared is not None else None
        self._fn = L.tarfa_b200_moe_layer
        self._args = (C.byref(self._shape), _ptr(h), _ptr(w_r), _ptr(bias), C.byref(self._wc),
                      C.byref(self._sc) if self._sc is not None else None, _ptr(self.out),
                      _ptr(self.top_idx), _ptr(self.top_w), _ptr(self.ws), C.c_size_t(n))
        self.device = dev

    def run(self) -> torch.Tensor:
        api.check(self._fn(*self._args, C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)))
        return self.out

    def capture(self, host_in: torch.Tensor | None = None,
                host_out: torch.Tensor | None = None) -> torch.cuda.CUDAGraph:
        """Record the layer into a CUDA graph (after one eager warm-up run).

        With ``host_in`` / ``host_out`` (pinned host tensors shaped like
        ``h`` / ``out``) the graph also copies the tokens in from ``host_in``
        and the result out to ``host_out`` (kernel copies over the host link up
        to 1 MiB, ``stage_copy``; the copy engine above): a serving step is then
        one replay, the copies back to back with the kernels, after which the host reads
        ``host_out`` once the stream (or an event recorded after the replay)
        has completed.
        """
        for t, ref, name in ((host_in, self.h, "host_in"), (host_out, self.out, "host_out")):
            if t is not None and (t.device.type != "cpu" or not t.is_pinned() or
                                  t.shape != ref.shape or t.dtype != ref.dtype):
                raise RuntimeError(f"{name} must be a pinned host tensor shaped like the plan's {name[5:]}")
        self.run()
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            if host_in is not None:
                _host_copy(self.h, host_in)
            self.run()
            if host_out is not None:
                _host_copy(host_out, self.out)
        return g


_STAGE_COPY_MAX = 1 << 20


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """RMSNorm of the synthetic stack (``tarfa_b200_rms_norm``): fp64 with a
    fixed pairwise tree for the sum of squares, rounded through fp32 to the
    model dtype; bit-identical to :func:`tarfa_b200.stack.rms_norm_host`."""
    _need_cuda(x, w)
    if x.dtype not in _DT or w.dtype != x.dtype or w.numel() != x.shape[-1]:
        raise RuntimeError("rms_norm: x [..., H] and w [H] in one model dtype")
    x = x.contiguous()
    w = w.contiguous()
    out = torch.empty_like(x)
    H = x.shape[-1]
    api.check(api.lib().tarfa_b200_rms_norm(_ptr(x), _ptr(w), x.numel() // H, H, float(eps), _DT[x.dtype],
                                            _ptr(out), _stream(x.device)))
    return out


def stage_copy(dst: torch.Tensor, src: torch.Tensor) -> None:
    """Kernel copy between device memory and pinned host memory (same shape and
    dtype, contiguous) on the current stream: for small transfers, faster than
    the copy engine (``tarfa_b200_stage_copy``)."""
    if dst.shape != src.shape or dst.dtype != src.dtype or not (dst.is_contiguous() and src.is_contiguous()):
        raise RuntimeError("stage_copy: dst and src must be contiguous with the same shape and dtype")
    dev = dst.device if dst.is_cuda else src.device
    api.check(api.lib().tarfa_b200_stage_copy(_ptr(dst), _ptr(src), dst.numel() * dst.element_size(),
                                              _stream(dev)))


def _host_copy(dst: torch.Tensor, src: torch.Tensor) -> None:
    nbytes = dst.numel() * dst.element_size()
    if nbytes <= _STAGE_COPY_MAX and nbytes % 16 == 0:
        stage_copy(dst, src)
    else:
        dst.copy_(src, non_blocking=True)


def dequant_int4(packed: torch.Tensor, scale: torch.Tensor, group: int = 0) -> torch.Tensor:
    """``channel_q4.dequant_int4`` on the device (group 0 = one scale per row)."""
    _need_cuda(packed, scale)
    N = packed.shape[0]
    K = packed.numel() * packed.element_size() * 2 // N
    out = torch.empty((N, K), dtype=scale.dtype, device=packed.device)
    api.check(api.lib().tarfa_b200_dequant_int4(_ptr(packed), _ptr(scale), N, K, group,
                                                _DT[scale.dtype], _ptr(out), _stream(packed.device)))
    return out


def quantize_int4(w: torch.Tensor, group: int = 128):
    """Symmetric int4 quantisation of bf16 ``w [N, K]`` -> (int32 ``[N, K/8]``, bf16 ``[N, K/group]``)."""
    _need_cuda(w)
    if w.dtype != torch.bfloat16:
        raise RuntimeError("quantize_int4 takes bf16 weights")
    N, K = w.shape[-2], w.shape[-1]
    lead = w.shape[:-2]
    rows = w.numel() // K
    packed = torch.empty((*lead, N, K // 8), dtype=torch.int32, device=w.device)
    scale = torch.empty((*lead, N, K // group), dtype=torch.bfloat16, device=w.device)
    api.check(api.lib().tarfa_b200_quantize_int4(_ptr(w), rows, K, group, _ptr(packed), _ptr(scale),
                                                 _stream(w.device)))
    return packed, scale


def set_gemm_min_tokens(tokens: int) -> None:
    """Dense layers with at least ``tokens`` tokens take the tcgen05 grouped-GEMM
    path; fewer take the tensor-core GEMV path (process-wide, default 64)."""
    api.check(api.lib().tarfa_b200_set_gemm_min_tokens(int(tokens)))


def set_decode_routing_max_tokens(tokens: int) -> None:
    """``moe_layer`` runs batches of 1..``tokens`` (<= 16) as one chain of
    programmatic dependent launches; 0 launches the kernels one after the
    other (process-wide, default 16)."""
    api.check(api.lib().tarfa_b200_set_decode_routing_max_tokens(int(tokens)))


def set_stage_events(events) -> None:
    """Record ``events[i]`` (``torch.cuda.Event``) at layer stage boundary ``i``
    (0 start, 1 router/permute, 2 gate_up, 3 down, 4 combine) on this thread;
    ``None`` or ``[]`` turns it off.  Each event must have been recorded once."""
    events = list(events or [])
    arr = (C.c_void_p * max(1, len(events)))(*[C.c_void_p(e.cuda_event) for e in events])
    api.check(api.lib().tarfa_b200_set_stage_events(arr, len(events)))


def device_status(clear: bool = False) -> int:
    """Error bits raised by kernels on the current device (``DEV_*`` in ``_capi``)."""
    v = C.c_uint32(0)
    api.check(api.lib().tarfa_b200_device_status(C.byref(v), int(clear),
                                                 _stream(torch.cuda.current_device())))
    return v.value
