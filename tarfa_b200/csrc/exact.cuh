// Correctly rounded dot products of model-dtype vectors without fp64 arithmetic.
//
// The router's logit is the model-dtype rounding (nearest, ties to even) of
// the exact dot product h . w_e (the definition the oracle uses).  The kernels
// accumulate in fp32 only (an fp64 accumulation costs a conversion and an add
// per product; the 16-token decode router with the scheme below, and a new
// work split, runs in half the time of the fp64 one):
//
// fast path   Products of two bf16 / fp16 values are exact in fp32 (at most
//             22 significant bits).  They are summed with TwoSum (Knuth), which
//             returns the rounded sum s and its exact error e; the errors are
//             summed into c, and sum|e| into a.  The exact dot product is then
//             s + sum(e) with |sum(e) - c| <= gamma_D * sum|e| (D = additions on
//             the longest path of the summation tree).  If rounding both ends of
//             [s + c - B, s + c + B] gives the same value, that value is the
//             correctly rounded result (rounding is monotonic).  B is about
//             2^-17 of sum|e| ~ 2^-41 of the logit, so this fails for ~1e-7 of
//             all logits, and for exact ties reached through rounded sums.
//             The check runs in fp32 (exact_round).
// slow path   An exact integer sum: every product is m_w * m_x * 2^(e_w + e_x)
//             with integer significands; a 576-bit two's complement
//             fixed-point accumulator (LSB 2^-266, the smallest product of two
//             subnormal bf16 values) holds any sum of up to 2^16 products
//             exactly.  The result is rounded from the integer.
#pragma once
#include "common.cuh"

namespace tarfa {

// TwoSum accumulator: s + (exact sum of the errors) == exact sum of the terms.
struct ExactAcc {
  float s, c, a;   // rounded sum, sum of TwoSum errors, sum of |errors|
};

TARFA_DEVI ExactAcc exact_zero() { return ExactAcc{0.f, 0.f, 0.f}; }

TARFA_DEVI void exact_add(ExactAcc& x, float p) {
  const float t = __fadd_rn(x.s, p);
  const float z = __fsub_rn(t, x.s);
  const float e = __fadd_rn(__fsub_rn(x.s, __fsub_rn(t, z)), __fsub_rn(p, z));
  x.s = t;
  x.c = __fadd_rn(x.c, e);
  x.a = __fadd_rn(x.a, fabsf(e));
}

TARFA_DEVI void exact_merge(ExactAcc& x, const ExactAcc& y) {
  exact_add(x, y.s);
  x.c = __fadd_rn(x.c, y.c);
  x.a = __fadd_rn(x.a, y.a);
}

// Accumulate the 8 products of two 16-byte chunks of model-dtype values.
template <typename T>
TARFA_DEVI void exact_chunk(ExactAcc& x, const uint4& wv, const uint4& hv) {
  const T* wp = reinterpret_cast<const T*>(&wv);
  const T* hp = reinterpret_cast<const T*>(&hv);
#pragma unroll
  for (int q = 0; q < 8; ++q)
    exact_add(x, __fmul_rn(Elem<T>::to_f(wp[q]), Elem<T>::to_f(hp[q])));
}

// Warp all-reduce of the accumulators (xor butterfly; every lane ends with the total).
TARFA_DEVI void exact_warp_reduce(ExactAcc& x) {
#pragma unroll
  for (int d = 16; d; d >>= 1) {
    ExactAcc y;
    y.s = __shfl_xor_sync(0xffffffffu, x.s, d);
    y.c = __shfl_xor_sync(0xffffffffu, x.c, d);
    y.a = __shfl_xor_sync(0xffffffffu, x.a, d);
    exact_merge(x, y);
  }
}

// Correct rounding from a reduced accumulator, in fp32 only.  depth = the
// longest chain of additions into c (terms per lane + 2 per merge level).
// f + g == s + c exactly (TwoSum); v = the model-dtype rounding of f.  The
// exact dot product lies within B of f + g; when both rounding midpoints
// around v are farther than B from f + g, v is its correct rounding.
// (mu - f and f - md are exact: f lies between the midpoints, within a factor
// of two of each.)  Returns false when that does not decide, or when v is zero
// (sign undecided: +0 for an exact zero) or not finite; the exact slow path
// then decides.
template <typename T>
TARFA_DEVI bool exact_round(const ExactAcc& x, int depth, float* out) {
  const float f = __fadd_rn(x.s, x.c);
  const float z = __fsub_rn(f, x.s);
  const float g = __fadd_rn(__fsub_rn(x.s, __fsub_rn(f, z)), __fsub_rn(x.c, z));
  const float v = Elem<T>::to_f(Elem<T>::from_f(f));
  *out = v;
  if (!isfinite(f)) return true;                 // inf / nan inputs: nothing to decide
  if (v == 0.f || !isfinite(v)) return false;
  // gamma_D / (1 - gamma_D) <= 1.02 * D * 2^-24 covers the sum of the errors and
  // its own rounding; 2^-126 covers products that underflowed fp32
  const float B = fmaf(1.02f * (float)depth * 0x1p-24f, x.a, 0x1p-126f);
  const uint16_t b = Elem<T>::to_bits(v);
  const float vu = Elem<T>::bits_to_f((uint16_t)(v > 0.f ? b + 1 : b - 1));   // next larger
  const float vd = Elem<T>::bits_to_f((uint16_t)(v > 0.f ? b - 1 : b + 1));   // next smaller
  const float mu = 0.5f * (v + vu), md = 0.5f * (v + vd);                     // exact
  const float du = __fsub_rn(__fsub_rn(mu, f), g);
  const float dd = __fadd_rn(__fsub_rn(f, md), g);
  return du > B && dd > B;
}

// ---------------------------------------------------------------------------
// slow path: exact integer accumulation
// ---------------------------------------------------------------------------
constexpr int kLimbs = 18;          // 576-bit accumulator, value = N * 2^-266
constexpr int kFixExp = -266;

// Model-dtype bits -> (negative, integer significand, exponent); value = m * 2^e.
template <typename T>
TARFA_DEVI bool decode_bits(uint16_t u, bool& neg, uint32_t& m, int& e) {
  neg = (u >> 15) != 0;
  if (Elem<T>::kId == 0) {   // bf16: 8 exponent bits, 7 fraction bits
    const int E = (u >> 7) & 0xFF;
    const uint32_t f = u & 0x7F;
    if (E == 0xFF) return false;
    m = E ? (f | 0x80u) : f;
    e = E ? E - 134 : -133;
  } else {                   // fp16: 5 exponent bits, 10 fraction bits
    const int E = (u >> 10) & 0x1F;
    const uint32_t f = u & 0x3FF;
    if (E == 0x1F) return false;
    m = E ? (f | 0x400u) : f;
    e = E ? E - 25 : -24;
  }
  return true;
}

// acc += (neg ? -1 : 1) * M * 2^off  (off in bits from the accumulator LSB)
TARFA_DEVI void limbs_add(uint32_t (&acc)[kLimbs], bool neg, uint32_t M, int off) {
  const uint64_t v = (uint64_t)M << (off & 31);
  const int li = off >> 5;
  const uint32_t lo = (uint32_t)v, hi = (uint32_t)(v >> 32);
  uint32_t carry = 0;
#pragma unroll
  for (int i = 0; i < kLimbs; ++i) {
    const uint32_t add = i == li ? lo : (i == li + 1 ? hi : 0u);
    if (!neg) {
      const uint64_t t = (uint64_t)acc[i] + add + carry;
      acc[i] = (uint32_t)t;
      carry = (uint32_t)(t >> 32);
    } else {
      const uint64_t t = (uint64_t)acc[i] - add - carry;
      acc[i] = (uint32_t)t;
      carry = (uint32_t)(t >> 63);
    }
  }
}

TARFA_DEVI void limbs_add_full(uint32_t (&acc)[kLimbs], const uint32_t (&b)[kLimbs]) {
  uint32_t carry = 0;
#pragma unroll
  for (int i = 0; i < kLimbs; ++i) {
    const uint64_t t = (uint64_t)acc[i] + b[i] + carry;
    acc[i] = (uint32_t)t;
    carry = (uint32_t)(t >> 32);
  }
}

// Round the exact value N * 2^-266 to the model dtype (nearest, ties to even).
template <typename T>
TARFA_DEVI float limbs_round(uint32_t (&acc)[kLimbs]) {
  const bool neg = (acc[kLimbs - 1] >> 31) != 0;
  if (neg) {   // magnitude: two's complement negation
    uint32_t carry = 1;
#pragma unroll
    for (int i = 0; i < kLimbs; ++i) {
      const uint64_t t = (uint64_t)(~acc[i]) + carry;
      acc[i] = (uint32_t)t;
      carry = (uint32_t)(t >> 32);
    }
  }
  int top = -1;
#pragma unroll
  for (int i = 0; i < kLimbs; ++i)
    if (acc[i]) top = 32 * i + 31 - __clz(acc[i]);
  if (top < 0) return 0.f;
  constexpr int p = Elem<T>::kId == 0 ? 8 : 11;            // significant bits
  constexpr int lsb_min = (Elem<T>::kId == 0 ? -133 : -24) - kFixExp;
  const int lsb = max(top - p + 1, lsb_min);
  auto bit = [&](int i) -> uint32_t {
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < kLimbs; ++j)
      if (j == (i >> 5)) w = acc[j];
    return (w >> (i & 31)) & 1u;
  };
  uint32_t q = 0;
  for (int i = top; i >= lsb; --i) q = (q << 1) | bit(i);
  const uint32_t rbit = bit(lsb - 1);
  bool sticky = false;
  const int sb = lsb - 1;   // bits strictly below sb
#pragma unroll
  for (int j = 0; j < kLimbs; ++j) {
    const int lo = 32 * j;
    if (lo + 32 <= sb) sticky |= acc[j] != 0;
    else if (lo < sb) sticky |= (acc[j] & ((1u << (sb - lo)) - 1u)) != 0;
  }
  if (rbit && (sticky || (q & 1u))) ++q;
  const float v = ldexpf((float)q, lsb + kFixExp);
  return neg ? -v : v;
}

// Exact, correctly rounded dot product of two H-element model-dtype vectors by
// one warp (all lanes return the value).  H a multiple of 8, 16-byte aligned.
template <typename T>
__device__ __noinline__ float warp_exact_dot(const T* a, const T* b, int H) {
  const int lane = threadIdx.x & 31;
  uint32_t acc[kLimbs];
#pragma unroll
  for (int i = 0; i < kLimbs; ++i) acc[i] = 0u;
  bool finite = true;
  for (int ch = lane; ch < H / 8; ch += 32) {
    const uint4 av = ld_cached(a + ch * 8), bv = ld_cached(b + ch * 8);
    const uint16_t* ap = reinterpret_cast<const uint16_t*>(&av);
    const uint16_t* bp = reinterpret_cast<const uint16_t*>(&bv);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      bool na, nb;
      uint32_t ma, mb;
      int ea, eb;
      finite &= decode_bits<T>(ap[q], na, ma, ea);
      finite &= decode_bits<T>(bp[q], nb, mb, eb);
      const uint32_t M = ma * mb;
      if (finite && M) limbs_add(acc, na != nb, M, ea + eb - kFixExp);
    }
  }
#pragma unroll
  for (int d = 16; d; d >>= 1) {
    uint32_t o[kLimbs];
#pragma unroll
    for (int i = 0; i < kLimbs; ++i) o[i] = __shfl_xor_sync(0xffffffffu, acc[i], d);
    limbs_add_full(acc, o);
  }
  if (!__all_sync(0xffffffffu, finite)) return __int_as_float(0x7fc00000);
  return limbs_round<T>(acc);
}

// Finish a warp's two accumulators into the correctly rounded value; lane 0
// decides for the warp (lanes may differ in c after the butterfly).  chains =
// terms in the longer per-lane chain.  Falls back to the exact integer sum.
template <typename T>
TARFA_DEVI float exact_finish(ExactAcc x0, const ExactAcc& x1, int chains, const T* a, const T* b,
                              int H) {
  exact_merge(x0, x1);
  exact_warp_reduce(x0);
  float v = 0.f;
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = exact_round<T>(x0, chains + 2 + 10, &v);
  ok = __shfl_sync(0xffffffffu, ok, 0);
  v = __shfl_sync(0xffffffffu, v, 0);
  if (!ok) v = warp_exact_dot<T>(a, b, H);
  return v;
}

// Correctly rounded a . b (H elements, both from memory) by one warp.  The
// chunks are loaded four per lane at a time, so a 3072-element dot makes three
// round trips to memory, not twelve.
template <typename T>
TARFA_DEVI float warp_dot_exact(const T* a, const T* b, int H) {
  const int lane = threadIdx.x & 31;
  const int nch = H / 8;
  ExactAcc x0 = exact_zero(), x1 = exact_zero();
  for (int c0 = lane; c0 < nch; c0 += 4 * 32) {
    uint4 av[4], bv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int ch = c0 + 32 * i;
      av[i] = ch < nch ? ld_cached(a + ch * 8) : make_uint4(0, 0, 0, 0);
      bv[i] = ch < nch ? ld_cached(b + ch * 8) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (c0 + 32 * i >= nch) break;
      if (i & 1) exact_chunk<T>(x1, av[i], bv[i]);
      else exact_chunk<T>(x0, av[i], bv[i]);
    }
  }
  const int per_lane = (nch + 31) / 32;
  return exact_finish<T>(x0, x1, 8 * ((per_lane + 1) / 2), a, b, H);
}

// Correctly rounded w . x for a weight row held in registers (16-byte chunk j
// of lane l is chunk l + 32 j of the row); wrow is the row in memory, for the
// slow path.
template <typename T, int MAXC>
TARFA_DEVI float row_dot_exact(const uint4 (&wv)[MAXC], const T* wrow, const T* xrow, int H) {
  const int lane = threadIdx.x & 31, nch = H / 8;
  ExactAcc x0 = exact_zero(), x1 = exact_zero();
#pragma unroll
  for (int j = 0; j < MAXC; ++j) {
    const int ch = lane + 32 * j;
    if (ch < nch) {
      const uint4 xv = ld_cached(xrow + ch * 8);
      if (j & 1) exact_chunk<T>(x1, wv[j], xv);
      else exact_chunk<T>(x0, wv[j], xv);
    }
  }
  return exact_finish<T>(x0, x1, 8 * ((MAXC + 1) / 2), wrow, xrow, H);
}

}  // namespace tarfa
