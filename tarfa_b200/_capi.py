"""ctypes binding of the C ABI declared in ``include/tarfa_b200.h``.

The library is loaded from the package's ``_lib/`` directory; there is no
fallback: if it is missing, :func:`lib` raises.  Structures mirror the C
structs field by field.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

from . import build as _build

ABI_VERSION = 2

TARFA_OK, TARFA_ERR_INVALID, TARFA_ERR_UNSUPPORTED, TARFA_ERR_WORKSPACE, TARFA_ERR_CUDA = range(5)
TARFA_BF16, TARFA_F16 = 0, 1
TARFA_W_DENSE, TARFA_W_INT4 = 0, 1
OP_EXPERTS, OP_MOE_LAYER, OP_ROUTER, OP_PERMUTE, OP_SHARED = 0, 1, 2, 3, 4
DEV_BAD_EXPERT_ID, DEV_WAIT_TIMEOUT = 1, 2


class MoeShape(C.Structure):
    _fields_ = [("tokens", C.c_int64), ("hidden", C.c_int64), ("experts", C.c_int64),
                ("inter", C.c_int64), ("shared_inter", C.c_int64), ("top_k", C.c_int32),
                ("dtype", C.c_int32)]


class MoeWeights(C.Structure):
    _fields_ = [("kind", C.c_int32), ("group", C.c_int32), ("gate_up", C.c_void_p),
                ("gate_up_scale", C.c_void_p), ("down", C.c_void_p),
                ("down_scale", C.c_void_p), ("expert_slot", C.c_void_p), ("slots", C.c_int64)]


class SharedExpert(C.Structure):
    _fields_ = [("gate_proj", C.c_void_p), ("up_proj", C.c_void_p), ("down_proj", C.c_void_p),
                ("gate_weight", C.c_void_p)]


EP_MAX_RANKS = 8
EP_IPC_HANDLE_BYTES = 64


class EpGroup(C.Structure):
    _fields_ = [("world", C.c_int32), ("rank", C.c_int32), ("max_tokens", C.c_int64),
                ("tp", C.c_int32), ("reserved", C.c_int32), ("boxes", C.c_void_p * EP_MAX_RANKS)]


# name -> (restype, argtypes); every symbol include/tarfa_b200.h declares
_P = C.c_void_p
SIGNATURES = {
    "tarfa_b200_abi_version": (C.c_int, []),
    "tarfa_b200_last_error": (C.c_char_p, []),
    "tarfa_b200_workspace_size": (C.c_size_t, [C.POINTER(MoeShape), C.c_int32]),
    "tarfa_b200_experts_forward": (C.c_int, [C.POINTER(MoeShape), _P, _P, _P,
                                             C.POINTER(MoeWeights), _P, _P, C.c_size_t, _P]),
    "tarfa_b200_moe_layer": (C.c_int, [C.POINTER(MoeShape), _P, _P, _P, C.POINTER(MoeWeights),
                                       C.POINTER(SharedExpert), _P, _P, _P, _P, C.c_size_t, _P]),
    "tarfa_b200_moe_layer_noalloc": (C.c_int, [C.POINTER(MoeShape), _P, _P, _P,
                                               C.POINTER(MoeWeights), C.POINTER(SharedExpert),
                                               _P, _P, _P, _P]),
    "tarfa_b200_router_topk": (C.c_int, [C.POINTER(MoeShape), _P, _P, _P, _P, _P, _P, _P,
                                         C.c_size_t, _P]),
    "tarfa_b200_permute": (C.c_int, [C.POINTER(MoeShape), _P, _P, _P, _P, _P, C.c_size_t, _P]),
    "tarfa_b200_dequant_int4": (C.c_int, [_P, _P, C.c_int64, C.c_int64, C.c_int32, C.c_int32,
                                          _P, _P]),
    "tarfa_b200_quantize_int4": (C.c_int, [_P, C.c_int64, C.c_int64, C.c_int32, _P, _P, _P]),
    "tarfa_b200_device_status": (C.c_int, [C.POINTER(C.c_uint32), C.c_int32, _P]),
    "tarfa_b200_set_stage_events": (C.c_int, [C.POINTER(C.c_void_p), C.c_int32]),
    "tarfa_b200_set_gemm_min_tokens": (C.c_int, [C.c_int64]),
    "tarfa_b200_shared_expert": (C.c_int, [C.POINTER(MoeShape), _P, C.POINTER(SharedExpert), _P, _P,
                                           C.c_size_t, _P]),
    "tarfa_b200_combine_routes": (C.c_int, [C.POINTER(MoeShape), _P, _P, _P, _P, _P, _P]),
    "tarfa_b200_set_decode_routing_max_tokens": (C.c_int, [C.c_int64]),
    "tarfa_b200_stage_copy": (C.c_int, [_P, _P, C.c_size_t, _P]),
    "tarfa_b200_rms_norm": (C.c_int, [_P, _P, C.c_int64, C.c_int64, C.c_double, C.c_int32, _P, _P]),
    "tarfa_b200_ep_box_bytes": (C.c_size_t, [C.POINTER(MoeShape), C.c_int32, C.c_int64]),
    "tarfa_b200_ep_workspace_size": (C.c_size_t, [C.POINTER(MoeShape), C.c_int32, C.c_int64]),
    "tarfa_b200_ep_box_alloc": (C.c_int, [C.c_size_t, C.POINTER(C.c_void_p), _P]),
    "tarfa_b200_ep_box_open": (C.c_int, [_P, C.POINTER(C.c_void_p)]),
    "tarfa_b200_ep_box_close": (C.c_int, [_P]),
    "tarfa_b200_ep_box_free": (C.c_int, [_P]),
    "tarfa_b200_ep_moe_layer": (C.c_int, [C.POINTER(MoeShape), _P, _P, _P, C.POINTER(MoeWeights),
                                          C.POINTER(SharedExpert), C.POINTER(EpGroup), _P, _P, _P,
                                          _P, C.c_size_t, _P]),
}

_lock = threading.Lock()
_lib = None


def lib_path() -> str:
    return _build.LIB


def lib() -> C.CDLL:
    """Load (once) the CUDA extension; raises if it is absent or stale-ABI."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not os.path.exists(path):
            raise RuntimeError(
                f"tarfa_b200 CUDA extension not built ({path} missing); run "
                "`python -m tarfa_b200.build` — there is no CPU fallback")
        L = C.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        if L.tarfa_b200_abi_version() != ABI_VERSION:
            raise RuntimeError("tarfa_b200 ABI version mismatch; rebuild the extension")
        _lib = L
    return _lib


class TarfaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"tarfa_b200 error {code}: {msg}")
        self.code = code


def check(rc: int) -> None:
    if rc != TARFA_OK:
        raise TarfaError(rc, lib().tarfa_b200_last_error().decode(errors="replace"))
