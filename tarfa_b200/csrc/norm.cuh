// RMSNorm of the synthetic decoder stack's skeleton (the part around the MoE
// blocks; not the routed-MoE path).
//
//   out = bf16(f32((x * r) * (1 + w))),   r = 1 / sqrt(S / H + eps)
//
// in fp64, S = sum of x^2 over the row by a fixed pairwise tree: while the
// length is even, element i += element i + len/2; then left to right.  Every
// step is one IEEE fp64 operation in a fixed order (explicit _rn intrinsics,
// no contraction into FMAs), so the result equals the same tree evaluated by
// any IEEE implementation, the host's included.  One CTA per row; the squares
// sit in shared memory (8 bytes per column).
#pragma once
#include "common.cuh"

namespace tarfa {

template <typename T>
__global__ void __launch_bounds__(256) rms_norm_tree_kernel(const T* x, const T* w, T* out, int H,
                                                            double eps) {
  extern __shared__ double sq[];
  __shared__ double s_r;
  const T* xr = x + (int64_t)blockIdx.x * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const double d = (double)Elem<T>::to_f(xr[i]);
    sq[i] = __dmul_rn(d, d);
  }
  __syncthreads();
  int n = H;
  while (n > 1 && (n & 1) == 0) {
    const int h = n >> 1;
    for (int i = threadIdx.x; i < h; i += blockDim.x) sq[i] = __dadd_rn(sq[i], sq[i + h]);
    __syncthreads();
    n = h;
  }
  if (threadIdx.x == 0) {
    double acc = sq[0];
    for (int j = 1; j < n; ++j) acc = __dadd_rn(acc, sq[j]);
    s_r = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(acc, (double)H), eps)));
  }
  __syncthreads();
  const double r = s_r;
  T* orow = out + (int64_t)blockIdx.x * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const double d = (double)Elem<T>::to_f(xr[i]);
    const double g = __dadd_rn(1.0, (double)Elem<T>::to_f(w[i]));
    orow[i] = Elem<T>::from_f(__double2float_rn(__dmul_rn(__dmul_rn(d, r), g)));
  }
}

}  // namespace tarfa
