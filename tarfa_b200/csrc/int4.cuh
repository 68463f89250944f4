// int4 weight format kernels: dequantise (test / prefill helper) and quantise.
//
// Packing: nibble j of 32-bit word i of a row is column 8*i + j (low nibble
// first) == the reference's uint8 [N, K/2] layout (moe_kernel.py:10-14).
#pragma once
#include "common.cuh"

namespace tarfa {

// channel_q4.dequant_int4 (channel_q4.py:10-14): (nibble - 8) * scale, one RNE
// to the model dtype.  One thread per 32-bit word (8 outputs, one 16-byte store).
template <typename T>
__global__ void dequant_int4_kernel(const uint32_t* packed, const T* scale, int64_t rows,
                                    int64_t cols, int group, T* out) {
  const int64_t words = cols / 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * words) return;
  const int64_t n = i / words, wi = i % words;
  const uint32_t w = packed[i];
  const int64_t gi = group ? (wi * 8) / group : 0;
  const int64_t gpr = group ? cols / group : 1;
  const float s = Elem<T>::to_f(scale[n * gpr + gi]);
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float lo = (float)((int)((w >> (8 * j)) & 0xF) - 8);
    const float hi = (float)((int)((w >> (8 * j + 4)) & 0xF) - 8);
    const T a = Elem<T>::from_f(lo * s), b = Elem<T>::from_f(hi * s);   // exact products
    o[j] = uint32_t(*reinterpret_cast<const uint16_t*>(&a)) |
           (uint32_t(*reinterpret_cast<const uint16_t*>(&b)) << 16);
  }
  reinterpret_cast<uint4*>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
}

// Symmetric int4 quantisation, one warp per (row, group):
//   s = bf16_rne(max|w| / 7);  q = clamp(rint(w / s), -7, 7) + 8;  q = 8 if s == 0.
// group is a multiple of 128 and at most 1024.
__global__ void quantize_int4_kernel(const __nv_bfloat16* w, int64_t rows, int64_t cols,
                                     int group, uint32_t* packed, __nv_bfloat16* scale) {
  const int lane = threadIdx.x & 31;
  const int64_t gid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t gpr = cols / group;
  if (gid >= rows * gpr) return;
  const int64_t n = gid / gpr, gj = gid % gpr;
  const __nv_bfloat16* src = w + n * cols + gj * group;
  const int blocks = group / 128;   // each 128-column block: lane owns 4 consecutive columns
  float amax = 0.f;
  for (int b = 0; b < blocks; ++b) {
    const uint2 v = *reinterpret_cast<const uint2*>(src + b * 128 + lane * 4);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
    for (int q = 0; q < 4; ++q) amax = fmaxf(amax, fabsf(__bfloat162float(e[q])));
  }
#pragma unroll
  for (int d = 16; d; d >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, d));
  const __nv_bfloat16 sb = __float2bfloat16_rn(__fdiv_rn(amax, 7.0f));
  const float s = __bfloat162float(sb);
  if (lane == 0) scale[n * gpr + gj] = sb;
  for (int b = 0; b < blocks; ++b) {
    const uint2 v = *reinterpret_cast<const uint2*>(src + b * 128 + lane * 4);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
    uint32_t nib = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      int qi = 8;
      if (s != 0.f) {
        const float r = rintf(__fdiv_rn(__bfloat162float(e[q]), s));
        qi = (int)fminf(fmaxf(r, -7.f), 7.f) + 8;
      }
      nib |= (uint32_t)qi << (4 * q);
    }
    const uint32_t other = __shfl_down_sync(0xffffffffu, nib, 1);
    if ((lane & 1) == 0)
      packed[(n * cols + gj * group + b * 128) / 8 + lane / 2] = nib | (other << 16);
  }
}

}  // namespace tarfa
