// Shared device helpers for the tarfa_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define TARFA_DEVI __device__ __forceinline__

// Phase marks for timing probes built outside the library (no-ops here).
#ifndef TARFA_PHASE
#define TARFA_PHASE(i)
#endif

namespace tarfa {

// ---------------------------------------------------------------------------
// element types: the model dtype is bf16 or fp16 (activations, dense weights,
// int4 scales).  Traits give the conversions and the int4 "magic" constants.
// ---------------------------------------------------------------------------
template <typename T> struct Elem;

template <> struct Elem<__nv_bfloat16> {
  static constexpr int kId = 0;
  TARFA_DEVI static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  TARFA_DEVI static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  TARFA_DEVI static float bits_to_f(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }
  TARFA_DEVI static uint16_t to_bits(float v) { return __bfloat16_as_ushort(__float2bfloat16_rn(v)); }
  // bf16 0x4300 = 128.0 with a 7-bit mantissa: 0x4300 | q == 128 + q exactly
  static constexpr uint32_t kMagic = 0x43004300u;
  static constexpr uint32_t kMagicMinus8 = 0x43084308u;  // 136.0 in both halves
};

template <> struct Elem<__half> {
  static constexpr int kId = 1;
  TARFA_DEVI static float to_f(__half v) { return __half2float(v); }
  TARFA_DEVI static __half from_f(float v) { return __float2half_rn(v); }
  TARFA_DEVI static float bits_to_f(uint16_t b) { return __half2float(__ushort_as_half(b)); }
  TARFA_DEVI static uint16_t to_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }
  // fp16 0x6400 = 1024.0 with a 10-bit mantissa: 0x6400 | q == 1024 + q exactly
  static constexpr uint32_t kMagic = 0x64006400u;
  static constexpr uint32_t kMagicMinus8 = 0x64086408u;  // 1032.0 in both halves
};

// Round a value through the model dtype (the "F.linear output is bf16" points).
template <typename T> TARFA_DEVI float rnd(float v) { return Elem<T>::to_f(Elem<T>::from_f(v)); }

// fp64 -> fp32 rounding to odd: truncate, then set the sticky bit if inexact.
// A later round-to-nearest-even to bf16/fp16 is then one correct rounding of
// the fp64 value (the fp32 carries >= 2 more bits than the target).
TARFA_DEVI float f64_to_f32_odd(double d) {
  float f = __double2float_rz(d);
  if ((double)f != d) f = __int_as_float(__float_as_int(f) | 1);
  return f;
}

template <typename T> TARFA_DEVI T round_from_f64(double d) { return Elem<T>::from_f(f64_to_f32_odd(d)); }

// The activation of Qwen3.5-MoE experts (hidden_act = "silu"), in fp32 with an
// IEEE division, as torch's silu kernel evaluates it: x / (1 + exp(-x)).
TARFA_DEVI float silu_f(float x) { return __fdiv_rn(x, 1.0f + expf(-x)); }
TARFA_DEVI float sigmoid_f(float x) { return __fdiv_rn(1.0f, 1.0f + expf(-x)); }

// ---------------------------------------------------------------------------
// memory helpers
// ---------------------------------------------------------------------------
// Streaming 128-bit load of weights read once: bypass L1 allocation.
TARFA_DEVI uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// 128-bit load of small reused operands (activations): cached in L1.
TARFA_DEVI uint4 ld_cached(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ---------------------------------------------------------------------------
// warp-level tensor-core MMA (m16n8k16, fp32 accumulate).
// Fragment layout (PTX ISA, mma.m16n8k16 .bf16/.f16), g = lane/4, c = lane%4:
//   A: a0 (row g,   k 2c..2c+1)   a1 (row g+8, k 2c..2c+1)
//      a2 (row g,   k 2c+8..2c+9) a3 (row g+8, k 2c+8..2c+9)
//   B: b0 (k 2c..2c+1, col g)     b1 (k 2c+8..2c+9, col g)
//   D: d0 (row g, col 2c) d1 (row g, col 2c+1) d2 (row g+8, col 2c) d3 (row g+8, col 2c+1)
// ---------------------------------------------------------------------------
template <typename T> struct Mma;

template <> struct Mma<__nv_bfloat16> {
  TARFA_DEVI static void run(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  // (q - 8) for two packed "128 + q" halves: (128 + q) * 1 - 136, exact.
  // Written as a bf16x2 fused multiply-add (a native instruction since sm_80).
  TARFA_DEVI static uint32_t sub_magic(uint32_t v) {
    uint32_t r;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;"
        : "=r"(r)
        : "r"(v), "r"(0x3F803F80u), "r"(Elem<__nv_bfloat16>::kMagicMinus8 | 0x80008000u));
    return r;
  }
  // one correctly rounded product per half
  TARFA_DEVI static uint32_t mul2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(0x80008000u));
    return r;
  }
};

template <> struct Mma<__half> {
  TARFA_DEVI static void run(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  TARFA_DEVI static uint32_t sub_magic(uint32_t v) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(Elem<__half>::kMagicMinus8));
    return r;
  }
  TARFA_DEVI static uint32_t mul2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
};

// Dequantise nibbles s and s+4 of word w into one packed pair (q-8, q'-8).
template <typename T> TARFA_DEVI uint32_t nib_pair(uint32_t w, int s) {
  uint32_t v = ((w >> (4 * s)) & 0x000F000Fu) | Elem<T>::kMagic;
  return Mma<T>::sub_magic(v);
}

// ---------------------------------------------------------------------------
// device status word (error flags raised by kernels; read by the host API)
// ---------------------------------------------------------------------------
constexpr unsigned kStatusBadExpert = 1u;    // TARFA_DEV_BAD_EXPERT_ID
constexpr unsigned kStatusWaitTimeout = 2u;  // TARFA_DEV_WAIT_TIMEOUT

// kModeExact: dense weights, the exact path's rounding points
//   (fused_int4.py:191-194 and 240-244).
// kModeInt4Fused: int4, the fused decode kernel's arithmetic
//   (moe_kernel.py:27-104: scale folded after the dot, fp32 intermediates).
// kModeInt4Dequant: int4 dequantised to the model dtype, then the exact path
//   (fused_int4.py:254-260 with channel_q4.py:10-14).
enum GemvMode { kModeExact = 0, kModeInt4Fused = 1, kModeInt4Dequant = 2 };

// Programmatic dependent launch.  launch_dependents lets the next kernel of the
// stream (launched with programmatic stream serialization) be scheduled before
// this one ends; grid_dep_wait blocks until the previous kernel has completed
// and its memory is visible.  Both are no-ops without the launch attribute.
TARFA_DEVI void grid_dep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
TARFA_DEVI void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

TARFA_DEVI void raise_status(unsigned* status, unsigned bit) {
  if (status) atomicOr(status, bit);
}

}  // namespace tarfa
