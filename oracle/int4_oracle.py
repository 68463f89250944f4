"""CPU ORACLE for the int4 weight formats — test infrastructure, never the product.

Byte/integer work in numpy.  Two layouts share one packing: nibble ``j`` of
32-bit little-endian word ``i`` holds column ``8*i + j`` (low nibble first).
Byte-wise that is exactly the reference's ``uint8 [N, K/2]`` layout, low nibble
= even column (``tarfa/engine/moe_kernel.py:10-14``, ``channel_q4.py:10-14``).

* reference layout: one scale per output row (group = K), fp16 on disk, cast to
  the model dtype on load (``fused_int4.py:139-141``);
* group-128 layout: one bf16 scale per 128 columns of a row.

Dequantisation ``w = (nib - 8) * s`` rounded once to the scale dtype is the
reference's ``dequant_int4`` (channel_q4.py:10-14) and is pinned bit-exactly
against it by ``tests/golden``.

The quantiser is not shipped by the reference (its int4 files are produced
outside the repository, ``channel_q4.py:6``), so ``quantize_int4`` below is this
project's own statement of "symmetric int4, scale = max|w| / 7 per group":
``s = bf16_rne(max|w| / 7)``, ``q = clamp(rint(w / s), -7, 7) + 8`` (fp32 IEEE
division, round-half-even), ``q = 8`` for an all-zero group.  Parity of the
quantiser is against this statement only ("quantiser parity unpinned").
"""
from __future__ import annotations

import numpy as np


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(f: np.ndarray) -> np.ndarray:
    u = np.asarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return np.where(np.isnan(np.asarray(f, np.float32)), 0x7FC0, r).astype(np.uint16)


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    """``uint8 [N, K/2]`` or ``int32 [N, K/8]`` -> ``uint8 [N, K]`` nibble values."""
    b = np.ascontiguousarray(packed).view(np.uint8)
    N = b.shape[0]
    b = b.reshape(N, -1)
    out = np.empty((N, b.shape[1] * 2), dtype=np.uint8)
    out[:, 0::2] = b & 0xF
    out[:, 1::2] = b >> 4
    return out


def pack_nibbles(q: np.ndarray) -> np.ndarray:
    """``uint8 [N, K]`` nibble values -> ``int32 [N, K/8]`` (byte-identical to u8 [N, K/2])."""
    q = np.asarray(q, dtype=np.uint8)
    N, K = q.shape
    assert K % 8 == 0
    b = (q[:, 0::2] & 0xF) | ((q[:, 1::2] & 0xF) << 4)
    return np.ascontiguousarray(b).view(np.int32).reshape(N, K // 8)


def dequant(packed: np.ndarray, scale_bits: np.ndarray, group: int, dtype: str) -> np.ndarray:
    """Dequantised weights as bit patterns (uint16) of ``dtype`` ('bf16' | 'f16').

    ``scale_bits``: uint16 bit patterns ``[N]`` (group = K) or ``[N, K/group]``.
    """
    q = unpack_nibbles(packed).astype(np.int32) - 8
    N, K = q.shape
    sb = np.asarray(scale_bits, dtype=np.uint16)
    if sb.ndim == 1:
        sb = sb[:, None]
        group = K
    if dtype == "bf16":
        s = bf16_bits_to_f32(sb)
    else:
        s = sb.view(np.float16).astype(np.float32)
    s = np.repeat(s, group, axis=1)[:, :K]
    prod = q.astype(np.float32) * s          # exact: |q| <= 8, s has <= 11 significant bits
    if dtype == "bf16":
        return f32_to_bf16_bits(prod)
    return prod.astype(np.float16).view(np.uint16)


def quantize_int4(w_bits: np.ndarray, group: int = 128):
    """bf16 weights (uint16 bits ``[N, K]``) -> (int32 packed ``[N, K/8]``, bf16 scale bits ``[N, K/group]``)."""
    w = bf16_bits_to_f32(w_bits)
    N, K = w.shape
    assert K % group == 0 and group % 8 == 0
    wg = w.reshape(N, K // group, group)
    amax = np.abs(wg).max(axis=-1)
    s_bits = f32_to_bf16_bits((amax / np.float32(7.0)).astype(np.float32))
    s = bf16_bits_to_f32(s_bits)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = np.rint((wg / s[..., None]).astype(np.float32))
    r = np.where(s[..., None] == 0, 0, r)
    q = (np.clip(r, -7, 7) + 8).astype(np.uint8).reshape(N, K)
    return pack_nibbles(q), s_bits
