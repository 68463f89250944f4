// Fused decode layer: one persistent cooperative launch runs the whole MoE
// block for a decode batch (T <= 16 tokens):
//
//   phase 0  router logits (exact, fp64-accumulated)  ||  shared-expert gate/up
//            (the shared expert does not depend on the routing, so its weights
//            stream while the router's are read)
//   barrier  (grid-wide, bounded spin)
//   phase 1  every CTA computes the top-k and the expert-sorted unit table for
//            all tokens itself, from the logits in L2, into shared memory
//   phase 2  routed gate/up + SiLU*mul; afterwards each CTA prefetches into L2
//            the down-projection rows it will read in phase 3
//   barrier
//   phase 3  down projections (routed + shared); per 16-row output block a
//            completion counter elects the CTA that finishes the block last to
//            combine it (routing-weighted sum in the reference order + gated
//            shared expert), so no third barrier is needed
//
// Arithmetic is identical to the multi-kernel path (router.cuh, gemv.cuh):
// same rounding points, same summation order inside a tile, same combine.
// Every spin-wait is bounded by a clock limit; on timeout the kernel raises
// kStatusWaitTimeout and returns.
#pragma once
#include "common.cuh"
#include "gemv.cuh"
#include "router.cuh"

namespace tarfa {
namespace fused {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxT = 16;
constexpr int kMaxK = 8;
constexpr int kMaxRoutes = kMaxT * kMaxK;
constexpr int kMaxUnits = kMaxRoutes + 1;
constexpr int kKsplitGU = 8;     // warps per gate/up tile
constexpr int kKsplitDN = 8;     // warps per down tile
constexpr long long kSpinCycles = 4000000000ll;   // ~2 s

struct Args {
  int T, H, E, K, I, Is, Imax, group;
  const void* h;
  const void* w_r;
  const void* bias;
  const void* w_sg;
  const void* gate_up;
  const void* down;
  const void* gu_scale;
  const void* dn_scale;
  const int32_t* expert_slot;
  const void* sh_gate;
  const void* sh_up;
  const void* sh_down;
  void* out;
  int64_t* idx_out;
  float* w_out;
  float* logits;       // ws [T, E]
  float* gate_logit;   // ws [T]
  void* act;           // ws [T*K + T, Imax] model dtype
  float* y;            // ws [T*K + T, H]
  unsigned* bar;       // ws [2] {count, generation}; count zero at rest
  unsigned* hb_cnt;    // ws [H/16] completion counters, zero at rest
  unsigned* status;
};

struct Smem {
  int idx[kMaxRoutes];        // top-k ids, [t*K + k]
  float w[kMaxRoutes];        // top-k weights
  int perm_tok[kMaxRoutes + kMaxT];
  int route_row[kMaxRoutes];
  int first[kMaxRoutes];
  UnitDesc units[kMaxUnits];
  int nu;
  int abort;
  int last;
  float red[kWarps * 2 * 4 * 32];   // K-split partial sums (NTB <= 2)
};

TARFA_DEVI bool grid_barrier(unsigned* bar, Smem& s, unsigned* status) {
  __syncthreads();
  if (threadIdx.x == 0) {
    volatile unsigned* gen = bar + 1;
    const unsigned g0 = *gen;
    __threadfence();
    const unsigned prev = atomicAdd(bar, 1u);
    if (prev == gridDim.x - 1) {
      atomicExch(bar, 0u);       // count back to zero before anyone can pass
      __threadfence();
      atomicAdd(bar + 1, 1u);    // release
    } else {
      const long long t0 = clock64();
      while (*gen == g0) {
        if (clock64() - t0 > kSpinCycles) {
          raise_status(status, kStatusWaitTimeout);
          s.abort = 1;
          break;
        }
        __nanosleep(64);
      }
    }
    __threadfence();
  }
  __syncthreads();
  return s.abort == 0;
}

template <int KSPLIT, int NTB>
TARFA_DEVI void group_reduce(float (&acc)[NTB][4], float* red, int grp, int kw, int lane) {
  if (KSPLIT == 1) return;
  float* base = red + grp * KSPLIT * NTB * 4 * 32;
#pragma unroll
  for (int b = 0; b < NTB; ++b)
#pragma unroll
    for (int q = 0; q < 4; ++q) base[(kw * NTB * 4 + b * 4 + q) * 32 + lane] = acc[b][q];
  group_barrier(1 + grp, KSPLIT * 32);
  if (kw == 0) {
#pragma unroll
    for (int b = 0; b < NTB; ++b)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float v = base[(b * 4 + q) * 32 + lane];
#pragma unroll
        for (int w2 = 1; w2 < KSPLIT; ++w2) v += base[(w2 * NTB * 4 + b * 4 + q) * 32 + lane];
        acc[b][q] = v;
      }
  }
  group_barrier(1 + grp, KSPLIT * 32);
}

// x row pointers of one tile's token block group
template <typename T, int NTB>
TARFA_DEVI void token_rows(const char* (&xrow)[NTB], const void* base, int64_t ld, const int* map,
                           int row0, int ntok, int tg, int g) {
#pragma unroll
  for (int b = 0; b < NTB; ++b) {
    const int n = tg * 8 * NTB + b * 8 + g;
    xrow[b] = nullptr;
    if (n < ntok) {
      const int xr = map ? map[row0 + n] : row0 + n;
      xrow[b] = reinterpret_cast<const char*>(static_cast<const T*>(base) + (int64_t)xr * ld);
    }
  }
}

// gate/up tile `tt` (8 intermediate rows) of a unit -> act rows
template <typename T, int MODE, int KSPLIT, int NTB>
TARFA_DEVI void gate_up_tile(const Args& a, Smem& s, const UnitDesc d, bool shared, int tt, int grp,
                             int kw) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const char* rowA;
  const char* rowB;
  const T* scA = nullptr;
  const T* scB = nullptr;
  int K = a.H;
  constexpr bool INT4 = MODE != kModeExact;
  if (!shared) {
    const int slot = a.expert_slot ? a.expert_slot[d.expert] : d.expert;
    const int ra = tt * 8 + g, rb = a.I + tt * 8 + g;
    if (INT4) {
      const char* wb = static_cast<const char*>(a.gate_up) + (int64_t)slot * 2 * a.I * (a.H / 8) * 4;
      rowA = wb + (int64_t)ra * (a.H / 8) * 4;
      rowB = wb + (int64_t)rb * (a.H / 8) * 4;
      const int64_t gpr = a.group ? a.H / a.group : 1;
      const T* sb = static_cast<const T*>(a.gu_scale) + (int64_t)slot * 2 * a.I * gpr;
      scA = sb + ra * gpr;
      scB = sb + rb * gpr;
    } else {
      const T* wb = static_cast<const T*>(a.gate_up) + (int64_t)slot * 2 * a.I * a.H;
      rowA = reinterpret_cast<const char*>(wb + (int64_t)ra * a.H);
      rowB = reinterpret_cast<const char*>(wb + (int64_t)rb * a.H);
    }
  } else {
    rowA = reinterpret_cast<const char*>(static_cast<const T*>(a.sh_gate) + (int64_t)(tt * 8 + g) * a.H);
    rowB = reinterpret_cast<const char*>(static_cast<const T*>(a.sh_up) + (int64_t)(tt * 8 + g) * a.H);
  }
  const int ntok = d.nrows;
  for (int tg = 0; tg * 8 * NTB < ntok; ++tg) {
    float acc[NTB][4];
#pragma unroll
    for (int b = 0; b < NTB; ++b)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[b][q] = 0.f;
    const char* xrow[NTB];
    token_rows<T, NTB>(xrow, a.h, a.H, s.perm_tok, d.row0, ntok, tg, g);
    const bool dense = shared || !INT4;
    const int n_it = K / (dense ? 32 : 128);
    const int i0 = kw * n_it / KSPLIT, i1 = (kw + 1) * n_it / KSPLIT;
    if (dense) gemv_kloop<T, kModeExact, NTB>(rowA, rowB, scA, scB, 0, i0, i1, xrow, acc);
    else gemv_kloop<T, MODE, NTB>(rowA, rowB, scA, scB, a.group, i0, i1, xrow, acc);
    group_reduce<KSPLIT, NTB>(acc, s.red, grp, kw, lane);
    if (kw == 0) {
      float rsa = 1.f, rsb = 1.f;
      if (!shared && MODE == kModeInt4Fused && a.group == 0) {
        rsa = Elem<T>::bits_to_f(reinterpret_cast<const uint16_t*>(scA)[0]);
        rsb = Elem<T>::bits_to_f(reinterpret_cast<const uint16_t*>(scB)[0]);
      }
#pragma unroll
      for (int b = 0; b < NTB; ++b)
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int n = tg * 8 * NTB + b * 8 + 2 * c + q;
          if (n >= ntok) continue;
          const float va = acc[b][q] * rsa, vb = acc[b][2 + q] * rsb;
          const float act = (!shared && MODE == kModeInt4Fused) ? gate_up_act<T, kModeInt4Fused>(va, vb)
                                                               : gate_up_act<T, kModeExact>(va, vb);
          static_cast<T*>(a.act)[(int64_t)(d.row0 + n) * a.Imax + tt * 8 + g] = Elem<T>::from_f(act);
        }
    }
  }
}

// down tile `hb` (16 output rows) of a unit -> y rows
template <typename T, int MODE, int KSPLIT, int NTB>
TARFA_DEVI void down_tile(const Args& a, Smem& s, const UnitDesc d, bool shared, int hb, int grp,
                          int kw) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  constexpr bool INT4 = MODE != kModeExact;
  const char* rowA;
  const char* rowB;
  const T* scA = nullptr;
  const T* scB = nullptr;
  const int K = shared ? a.Is : a.I;
  const int ra = hb * 16 + g, rb = hb * 16 + g + 8;
  if (!shared) {
    const int slot = a.expert_slot ? a.expert_slot[d.expert] : d.expert;
    if (INT4) {
      const char* wb = static_cast<const char*>(a.down) + (int64_t)slot * a.H * (a.I / 8) * 4;
      rowA = wb + (int64_t)ra * (a.I / 8) * 4;
      rowB = wb + (int64_t)rb * (a.I / 8) * 4;
      const int64_t gpr = a.group ? a.I / a.group : 1;
      const T* sb = static_cast<const T*>(a.dn_scale) + (int64_t)slot * a.H * gpr;
      scA = sb + ra * gpr;
      scB = sb + rb * gpr;
    } else {
      const T* wb = static_cast<const T*>(a.down) + (int64_t)slot * a.H * a.I;
      rowA = reinterpret_cast<const char*>(wb + (int64_t)ra * a.I);
      rowB = reinterpret_cast<const char*>(wb + (int64_t)rb * a.I);
    }
  } else {
    rowA = reinterpret_cast<const char*>(static_cast<const T*>(a.sh_down) + (int64_t)ra * a.Is);
    rowB = reinterpret_cast<const char*>(static_cast<const T*>(a.sh_down) + (int64_t)rb * a.Is);
  }
  const int ntok = d.nrows;
  for (int tg = 0; tg * 8 * NTB < ntok; ++tg) {
    float acc[NTB][4];
#pragma unroll
    for (int b = 0; b < NTB; ++b)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[b][q] = 0.f;
    const char* xrow[NTB];
    token_rows<T, NTB>(xrow, a.act, a.Imax, nullptr, d.row0, ntok, tg, g);
    const bool dense = shared || !INT4;
    const int n_it = K / (dense ? 32 : 128);
    const int i0 = kw * n_it / KSPLIT, i1 = (kw + 1) * n_it / KSPLIT;
    if (dense) gemv_kloop<T, kModeExact, NTB>(rowA, rowB, scA, scB, 0, i0, i1, xrow, acc);
    else gemv_kloop<T, MODE, NTB>(rowA, rowB, scA, scB, a.group, i0, i1, xrow, acc);
    group_reduce<KSPLIT, NTB>(acc, s.red, grp, kw, lane);
    if (kw == 0) {
      const bool f32 = !shared && MODE == kModeInt4Fused;
      float rsa = 1.f, rsb = 1.f;
      if (f32 && a.group == 0) {
        rsa = Elem<T>::bits_to_f(reinterpret_cast<const uint16_t*>(scA)[0]);
        rsb = Elem<T>::bits_to_f(reinterpret_cast<const uint16_t*>(scB)[0]);
      }
#pragma unroll
      for (int b = 0; b < NTB; ++b)
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int n = tg * 8 * NTB + b * 8 + 2 * c + q;
          if (n >= ntok) continue;
          float* o = a.y + (int64_t)(d.row0 + n) * a.H + hb * 16 + g;
          const float va = acc[b][q] * rsa, vb = acc[b][2 + q] * rsb;
          o[0] = f32 ? va : rnd<T>(va);
          o[8] = f32 ? vb : rnd<T>(vb);
        }
    }
  }
}

// Combine one 16-row output block for all tokens (same arithmetic as combine_kernel).
template <typename T, int MODE>
TARFA_DEVI void combine_block(const Args& a, const Smem& s, int hb, int tid, int nthr) {
  const int K = a.K;
  for (int i = tid; i < a.T * 16; i += nthr) {
    const int t = i >> 4, h = hb * 16 + (i & 15);
    float acc = 0.f;
    int pe = -1, pk = -1;
    for (int j = 0; j < K; ++j) {
      int k = j;
      if (a.T > 1) {   // ascending expert id
        int be = 0x7fffffff, bk = 0x7fffffff;
        for (int q = 0; q < K; ++q) {
          const int e = s.idx[t * K + q];
          const bool after = e > pe || (e == pe && q > pk);
          const bool before = e < be || (e == be && q < bk);
          if (after && before) { be = e; bk = q; }
        }
        pe = be; pk = bk; k = bk;
      }
      const int r = s.route_row[t * K + k];
      const float yv = __ldcg(a.y + (int64_t)r * a.H + h);
      const float wk = s.w[t * K + k];
      if (MODE == kModeInt4Fused) acc = __fadd_rn(acc, __fmul_rn(yv, wk));
      else if (a.T == 1) acc = rnd<T>(acc + rnd<T>(rnd<T>(wk) * yv));
      else acc = rnd<T>(acc + rnd<T>(__fmul_rn(yv, wk)));
    }
    if (MODE == kModeInt4Fused) acc = rnd<T>(acc);
    if (a.Is) {
      const float sg = rnd<T>(sigmoid_f(__ldcg(a.gate_logit + t)));
      const float sh = __ldcg(a.y + (int64_t)(a.T * K + t) * a.H + h);
      acc = rnd<T>(acc + rnd<T>(sg * sh));
    }
    static_cast<T*>(a.out)[(int64_t)t * a.H + h] = Elem<T>::from_f(acc);
  }
}

template <typename T, int MODE, int NTB>
__global__ void __launch_bounds__(kThreads, 1) decode_layer_kernel(const Args a) {
  __shared__ Smem s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  if (threadIdx.x == 0) { s.abort = 0; s.nu = 0; }
  __syncthreads();
  const int R = a.T * a.K;
  const int nt_sh_gu = a.Is / 8;

  // ---------------- phase 0: router rows || shared gate/up ---------------------
  {
    constexpr int KS = kKsplitGU, NG = kWarps / KS;
    const int grp = warp / KS, kw = warp % KS;
    const int slot = grp * G + blockIdx.x;          // consecutive tiles on different SMs
    if (threadIdx.x < a.T) s.perm_tok[R + threadIdx.x] = threadIdx.x;   // shared rows: token t
    __syncthreads();
    const UnitDesc shd{a.E, R, a.T, 0};
    for (int t = slot; t < nt_sh_gu; t += G * NG) gate_up_tile<T, MODE, KS, NTB>(a, s, shd, true, t, grp, kw);
    // router rows go to the warps of group slots that have no shared tile
    const int busy = nt_sh_gu < G * NG ? nt_sh_gu : G * NG;
    const int nrows = a.E + (a.w_sg ? 1 : 0);
    const int gw = (slot - busy) * KS + kw;        // index among idle warps
    const int nidle = (G * NG - busy) * KS;
    if (slot >= busy && nidle > 0) {
      const int nch = a.H / 8;
      for (int row = gw; row < nrows; row += nidle) {
        const T* wrow = row < a.E ? static_cast<const T*>(a.w_r) + (int64_t)row * a.H
                                  : static_cast<const T*>(a.w_sg);
        for (int t = 0; t < a.T; ++t) {
          const T* xrow = static_cast<const T*>(a.h) + (int64_t)t * a.H;
          double part[4] = {0.0, 0.0, 0.0, 0.0};
          for (int ch = lane; ch < nch; ch += 32) {
            const uint4 wv = ld_stream(wrow + ch * 8);
            const uint4 xv = ld_cached(xrow + ch * 8);
            const T* wp = reinterpret_cast<const T*>(&wv);
            const T* xp = reinterpret_cast<const T*>(&xv);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              part[q & 3] += (double)__fmul_rn(Elem<T>::to_f(wp[q]), Elem<T>::to_f(xp[q]));
          }
          double acc = (part[0] + part[1]) + (part[2] + part[3]);
#pragma unroll
          for (int d = 16; d; d >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, d);
          if (lane == 0) {
            float lgv = Elem<T>::to_f(round_from_f64<T>(acc));
            if (row < a.E) {
              if (a.bias) lgv = rnd<T>(lgv + Elem<T>::to_f(static_cast<const T*>(a.bias)[row]));
              a.logits[(int64_t)t * a.E + row] = lgv;
            } else {
              a.gate_logit[t] = lgv;
            }
          }
        }
      }
    }
  }
  if (!grid_barrier(a.bar, s, a.status)) return;

  // ---------------- phase 1: top-k and unit table, per CTA ----------------------
  for (int t = warp; t < a.T; t += kWarps) {
    int64_t* io = (blockIdx.x == 0 && a.idx_out) ? a.idx_out + (int64_t)t * a.K : nullptr;
    float* wo = (blockIdx.x == 0 && a.w_out) ? a.w_out + (int64_t)t * a.K : nullptr;
    warp_topk(a.logits + (int64_t)t * a.E, a.E, a.K, s.idx + t * a.K, s.w + t * a.K, io, wo);
  }
  __syncthreads();
  for (int r = threadIdx.x; r < R; r += kThreads) {     // route r = k*T + t
    const int t = r % a.T, k = r / a.T;
    const int e = s.idx[t * a.K + k];
    int less = 0, before = 0, same = 0;
    for (int q = 0; q < R; ++q) {
      const int e2 = s.idx[(q % a.T) * a.K + q / a.T];
      less += e2 < e;
      same += e2 == e;
      before += (e2 == e) && (q < r);
    }
    const int row = less + before;
    s.perm_tok[row] = t;
    s.route_row[t * a.K + k] = row;
    s.first[r] = before == 0 ? same : 0;
  }
  __syncthreads();
  for (int r = threadIdx.x; r < R; r += kThreads) {
    if (s.first[r]) {
      const int e = s.idx[(r % a.T) * a.K + r / a.T];
      int u = 0, row0 = 0;
      for (int q = 0; q < R; ++q) {
        const int e2 = s.idx[(q % a.T) * a.K + q / a.T];
        if (s.first[q] && e2 < e) { ++u; row0 += s.first[q]; }
      }
      s.units[u] = UnitDesc{e, row0, s.first[r], 0};
      atomicAdd(&s.nu, 1);
    }
  }
  __syncthreads();
  const int nu = s.nu;
  if (threadIdx.x == 0) s.units[nu] = UnitDesc{a.E, R, a.T, 0};
  __syncthreads();

  // ---------------- phase 2: routed gate/up ------------------------------------
  {
    constexpr int KS = kKsplitGU, NG = kWarps / KS;
    const int grp = warp / KS, kw = warp % KS;
    const int slot = grp * G + blockIdx.x;
    const int tpu = a.I / 8;
    for (int t = slot; t < nu * tpu; t += G * NG)
      gate_up_tile<T, MODE, KS, NTB>(a, s, s.units[t / tpu], false, t % tpu, grp, kw);
  }
  // prefetch this CTA's phase-3 down rows into L2 while the other CTAs finish phase 2
  {
    constexpr int KS = kKsplitDN, NG = kWarps / KS;
    const int hbs = a.H / 16;
    const int ntiles = (nu + (a.Is ? 1 : 0)) * hbs;
    for (int i = threadIdx.x; ; i += kThreads) {
      const int grp = i % NG, n = i / NG;
      const int t = (grp * G + blockIdx.x) + n * G * NG;
      if (t >= ntiles) break;
      const int u = t % (nu + (a.Is ? 1 : 0)), hb = t / (nu + (a.Is ? 1 : 0));
      const UnitDesc d = s.units[u];
      const bool sh = d.expert == a.E;
      const char* p;
      uint32_t bytes;
      if (sh) {
        p = reinterpret_cast<const char*>(static_cast<const T*>(a.sh_down) + (int64_t)hb * 16 * a.Is);
        bytes = 16u * a.Is * sizeof(T);
      } else {
        const int slot = a.expert_slot ? a.expert_slot[d.expert] : d.expert;
        const int64_t rowb = MODE != kModeExact ? (int64_t)(a.I / 8) * 4 : (int64_t)a.I * sizeof(T);
        p = static_cast<const char*>(a.down) + ((int64_t)slot * a.H + hb * 16) * rowb;
        bytes = (uint32_t)(16 * rowb);
      }
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
    }
  }
  if (!grid_barrier(a.bar, s, a.status)) return;

  // ---------------- phase 3: down + per-block combine ---------------------------
  {
    constexpr int KS = kKsplitDN, NG = kWarps / KS;
    const int grp = warp / KS, kw = warp % KS;
    const int slot = grp * G + blockIdx.x;
    const int nun = nu + (a.Is ? 1 : 0);
    const int hbs = a.H / 16;
    __shared__ int s_last[kWarps / kKsplitDN];
    for (int t = slot; t < nun * hbs; t += G * NG) {
      const int u = t % nun, hb = t / nun;
      const UnitDesc d = s.units[u];
      down_tile<T, MODE, KS, NTB>(a, s, d, d.expert == a.E, hb, grp, kw);
      // publish, count, and let the last finisher of the block combine it
      group_barrier(1 + grp, KS * 32);
      if (kw == 0 && lane == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(a.hb_cnt + hb, 1u);
        s_last[grp] = prev == (unsigned)(nun - 1);
        if (s_last[grp]) __threadfence();
      }
      group_barrier(1 + grp, KS * 32);
      if (s_last[grp]) {
        combine_block<T, MODE>(a, s, hb, kw * 32 + lane, KS * 32);
        if (kw == 0 && lane == 0) a.hb_cnt[hb] = 0u;   // leave the counter at rest
      }
    }
  }
}

}  // namespace fused
}  // namespace tarfa
