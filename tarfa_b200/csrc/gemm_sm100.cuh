// Grouped GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Prefill / batched expert products over the permuted token segments
// (fused_int4.py:227-248: per hit expert, gate/up linear, SiLU*mul, down
// linear).  One launch walks every (unit, n-tile, m-tile) of a phase:
//   PHASE 0 (gate_up): D[128 rows, 256] = X[rows, H] . [W_gate(128 rows); W_up(128 rows)]^T,
//            epilogue act = rnd(rnd(silu(rnd(g))) * rnd(u)) -> act[rows, I]
//   PHASE 1 (down):    D[128 rows, 256] = act[rows, I] . W_down(256 rows)^T,
//            epilogue y = rnd(d) -> y[rows, H] (model dtype)
// where a unit is one routed expert with its rows (contiguous in the
// permuted order) or the shared expert with all tokens.
//
// Structure (1 CTA per SM, persistent, static round-robin tile order with the
// m-tile innermost so the CTAs working on one weight tile run together and
// share it through L2):
//   warp 0      TMA producer: A tile 128x64 + two B boxes 128x64 per k-step,
//               4-stage ring (48 KB / stage), 128-byte swizzle, no multicast
//   warp 1      MMA issuer: 4 x tcgen05.mma (M128 N256 K16) per k-step,
//               tcgen05.commit frees the smem stage / publishes the accumulator
//   warp 2      TMEM owner: allocates / frees 512 columns (2 accumulators)
//   warps 4..7  epilogue: tcgen05.ld of their 32-lane quarter, math, stores
// Every mbarrier wait is bounded by a clock limit; on timeout the CTA raises
// kStatusWaitTimeout, the other roles stop, copies and MMAs in flight are
// drained (with their own bounded waits) and TMEM is freed before exit.
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "gemv.cuh"

namespace tarfa {
namespace sm100 {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;            // 16 KB
constexpr int B_BYTES = BN * BK * 2;            // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 48 KB
constexpr int kThreads = 256;
constexpr int kMaxUnits = 1024 + 1;
constexpr uint32_t kTmemCols = 512;
constexpr long long kWaitCycles = 4000000000ll;  // ~2 s at 1.9 GHz

struct __align__(8) Bars {
  uint64_t full[STAGES], empty[STAGES], tfull[2], tempty[2], mma_done;
};

constexpr size_t kSmemBytes = 1024 /*align slack*/ + STAGES * STAGE_BYTES + sizeof(Bars) + 16 +
                              (kMaxUnits + 1) * 4;

struct Params {
  int E, K_r, K_s, N_r, N_s;     // K per unit kind; N_r = I (phase 0) or H (phase 1)
  const int32_t* units;
  const int32_t* expert_slot;
  void* out;
  int64_t ldo;
  unsigned* status;
  uint32_t idesc;
  // phase 2: each output tile is split over ksplit K ranges; split s writes its
  // fp32 partial to out + s * split_stride (elements).  1 elsewhere.
  int ksplit;
  int64_t split_stride;
};

TARFA_DEVI uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

TARFA_DEVI void mbar_init(uint32_t a, uint32_t cnt) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(cnt) : "memory");
}
TARFA_DEVI void mbar_expect_tx(uint32_t a, uint32_t tx) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(tx) : "memory");
}
TARFA_DEVI void mbar_arrive(uint32_t a) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory");
}
TARFA_DEVI bool mbar_try(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(a), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with parity `parity` to complete.  Returns false
// on timeout (which also raises the abort flag) or, if honor_abort, when
// another role has aborted.
TARFA_DEVI bool mbar_wait(uint32_t a, uint32_t parity, volatile int* abort_flag, unsigned* status,
                          bool honor_abort = true) {
  if (mbar_try(a, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try(a, parity)) return true;
    if (honor_abort && *abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort_flag = 1;
      raise_status(status, kStatusWaitTimeout);
      return false;
    }
  }
}

TARFA_DEVI void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// K-major operand tile in the canonical 128-byte-swizzle layout: rows of
// 128 bytes (64 bf16 of K), 8-row atoms 1024 bytes apart (SBO), LBO unused.
TARFA_DEVI uint64_t sdesc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

TARFA_DEVI void umma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
TARFA_DEVI void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
TARFA_DEVI void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
TARFA_DEVI void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

TARFA_DEVI void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
TARFA_DEVI void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// (M=128, N=256) instruction descriptor, K-major A and B, fp32 accumulator.
__host__ __device__ constexpr uint32_t make_idesc(bool bf16) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

struct TileInfo {
  UnitDesc d;
  bool shared;
  int m, n, K;
};

TARFA_DEVI TileInfo decode_tile(int t, const int* prefix, int ntot, const UnitDesc* descs,
                                const Params& p, int nt_r, int nt_s) {
  int lo = 0, hi = ntot;   // prefix[lo] <= t < prefix[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= t) lo = mid;
    else hi = mid;
  }
  TileInfo ti;
  ti.d = descs[lo];
  ti.shared = ti.d.expert == p.E;
  const int mt = (ti.d.nrows + BM - 1) / BM;
  const int local = t - prefix[lo];
  ti.n = local / mt;
  ti.m = local % mt;
  ti.K = ti.shared ? p.K_s : p.K_r;
  (void)nt_r;
  (void)nt_s;
  return ti;
}

template <typename T, int PHASE>
__global__ void __launch_bounds__(kThreads, 1)
grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmS0, const __grid_constant__ CUtensorMap tmS1,
                    const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + STAGES * STAGE_BYTES);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  int* prefix = reinterpret_cast<int*>(tmem_holder + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nu = p.units[0];
  const int ntot = nu + p.units[2];
  const UnitDesc* descs = unit_descs(p.units);
  const int nt_r = PHASE == 0 ? p.N_r / 128 : p.N_r / BN;   // n-tiles per routed unit
  const int nt_s = PHASE == 0 ? p.N_s / 128 : (p.N_s + BN - 1) / BN;   // n-tiles of the shared unit

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&bars->full[s]), 1);
      mbar_init(smem_u32(&bars->empty[s]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&bars->tfull[i]), 1);
      mbar_init(smem_u32(&bars->tempty[i]), 128);
    }
    mbar_init(smem_u32(&bars->mma_done), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (warp == 3) {   // tiles per unit -> exclusive prefix
    const int per = (ntot + 31) / 32;
    const int b0 = min(lane * per, ntot), b1 = min(b0 + per, ntot);
    int s = 0;
    for (int u = b0; u < b1; ++u) {
      const int mt = (descs[u].nrows + BM - 1) / BM;
      s += mt * (descs[u].expert == p.E ? nt_s : nt_r);
    }
    int ps = s;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, ps, d);
      if (lane >= d) ps += x;
    }
    int e = ps - s;
    for (int u = b0; u < b1; ++u) {
      prefix[u] = e;
      const int mt = (descs[u].nrows + BM - 1) / BM;
      e += mt * (descs[u].expert == p.E ? nt_s : nt_r);
    }
    if (lane == 31) prefix[ntot] = ps;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int ksplit = PHASE == 2 ? p.ksplit : 1;
  const int ntiles = prefix[ntot] * ksplit;   // (tile, K range) work items

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------- TMA producer ----------------------------
      int stage = 0;
      uint32_t phase = 0;
      int issued[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const int sp = t % ksplit;
        const TileInfo ti = decode_tile(t / ksplit, prefix, ntot, descs, p, nt_r, nt_s);
        const int slot = ti.shared ? 0 : (p.expert_slot ? p.expert_slot[ti.d.expert] : ti.d.expert);
        const int arow = ti.d.row0 + ti.m * BM;
        const CUtensorMap* b0map;
        const CUtensorMap* b1map;
        int brow0, brow1;
        if (PHASE == 0) {
          if (!ti.shared) {
            b0map = b1map = &tmB;
            brow0 = slot * 2 * p.N_r + ti.n * 128;
            brow1 = brow0 + p.N_r;
          } else {
            b0map = &tmS0;
            b1map = &tmS1;
            brow0 = brow1 = ti.n * 128;
          }
        } else {
          b0map = b1map = ti.shared ? &tmS0 : &tmB;
          brow0 = (ti.shared ? 0 : slot * p.N_r) + ti.n * BN;
          brow1 = brow0 + 128;
        }
        const int nkb = ti.K / BK;
        const int kb0 = sp * nkb / ksplit, kb1 = (sp + 1) * nkb / ksplit;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(smem_u32(&bars->empty[stage]), phase ^ 1u, abort_flag, p.status)) {
            ok = false;
            break;
          }
          const uint32_t full = smem_u32(&bars->full[stage]);
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          mbar_expect_tx(full, STAGE_BYTES);
          tma_load_2d(sa, &tmA, full, kb * BK, arow);
          tma_load_2d(sa + A_BYTES, b0map, full, kb * BK, brow0);
          tma_load_2d(sa + A_BYTES + B_BYTES / 2, b1map, full, kb * BK, brow1);
          issued[stage] = (int)phase;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      // drain: every issued copy has landed before the CTA may exit
      for (int s = 0; s < STAGES; ++s)
        if (issued[s] >= 0)
          mbar_wait(smem_u32(&bars->full[s]), (uint32_t)issued[s], abort_flag, p.status, false);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------- MMA issuer ------------------------------
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++it) {
        const int sp = t % ksplit;
        const TileInfo ti = decode_tile(t / ksplit, prefix, ntot, descs, p, nt_r, nt_s);
        const int acc = it & 1;
        const uint32_t accph = (uint32_t)(it >> 1) & 1u;
        if (!mbar_wait(smem_u32(&bars->tempty[acc]), accph ^ 1u, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        const int nkb = ti.K / BK;
        const int kb0 = sp * nkb / ksplit, kb1 = (sp + 1) * nkb / ksplit;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(smem_u32(&bars->full[stage]), phase, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma(d, sdesc(sa + kk * 32), sdesc(sa + A_BYTES + kk * 32), p.idesc,
                 (kb != kb0 || kk != 0));
          umma_commit(smem_u32(&bars->empty[stage]));
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(smem_u32(&bars->tfull[acc]));
      }
      // drain: all MMAs issued by this thread complete before TMEM is freed
      umma_commit(smem_u32(&bars->mma_done));
      mbar_wait(smem_u32(&bars->mma_done), 0u, abort_flag, p.status, false);
    }
  } else if (warp >= 4) {
    // --------------------------------- epilogue ---------------------------------
    const int q = warp & 3;
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t accph = (uint32_t)(it >> 1) & 1u;
      if (!mbar_wait(smem_u32(&bars->tfull[acc]), accph, abort_flag, p.status)) break;
      tc_fence_after();
      const int sp = t % ksplit;
      const TileInfo ti = decode_tile(t / ksplit, prefix, ntot, descs, p, nt_r, nt_s);
      const int rl = ti.m * BM + q * 32 + lane;
      const bool valid = rl < ti.d.nrows;
      const int64_t orow = ti.d.row0 + rl;
      const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      T* out = static_cast<T*>(p.out);
      if (PHASE == 0) {
#pragma unroll 1
        for (int j0 = 0; j0 < 128; j0 += 16) {
          uint32_t g[16], u[16];
          tmem_ld16(tb + j0, g);
          tmem_ld16(tb + 128 + j0, u);
          tmem_wait_ld();
          if (valid) {
            uint32_t pk[8];
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
              float a2[2];
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const float gr = rnd<T>(__uint_as_float(g[j + h]));
                const float ur = rnd<T>(__uint_as_float(u[j + h]));
                a2[h] = rnd<T>(silu_f(gr)) * ur;   // fused_int4.py:242
              }
              const T lo = Elem<T>::from_f(a2[0]), hi = Elem<T>::from_f(a2[1]);
              pk[j / 2] = uint32_t(*reinterpret_cast<const uint16_t*>(&lo)) |
                          (uint32_t(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
            }
            uint4* dst = reinterpret_cast<uint4*>(out + orow * p.ldo + ti.n * 128 + j0);
            dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          }
        }
      } else if (PHASE == 2) {
        // plain fp32 store (router logits), columns masked at N_s
#pragma unroll 1
        for (int j0 = 0; j0 < BN; j0 += 16) {
          uint32_t v[16];
          tmem_ld16(tb + j0, v);
          tmem_wait_ld();
          const int col0 = ti.n * BN + j0;
          if (valid && col0 < p.N_s) {
            float* dst = static_cast<float*>(p.out) + sp * p.split_stride + orow * p.ldo + col0;
            if (col0 + 16 <= p.N_s) {
              float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                d4[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                    __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
            } else {
              for (int j = 0; j < 16 && col0 + j < p.N_s; ++j) dst[j] = __uint_as_float(v[j]);
            }
          }
        }
      } else {
#pragma unroll 1
        for (int j0 = 0; j0 < BN; j0 += 16) {
          uint32_t v[16];
          tmem_ld16(tb + j0, v);
          tmem_wait_ld();
          if (valid) {
            uint32_t pk[8];
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
              const T lo = Elem<T>::from_f(__uint_as_float(v[j]));
              const T hi = Elem<T>::from_f(__uint_as_float(v[j + 1]));
              pk[j / 2] = uint32_t(*reinterpret_cast<const uint16_t*>(&lo)) |
                          (uint32_t(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
            }
            uint4* dst = reinterpret_cast<uint4*>(out + orow * p.ldo + ti.n * BN + j0);
            dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&bars->tempty[acc]));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// A unit table with one unit covering rows [0, T) (marked as the "shared" unit,
// expert id E), used to run a plain [T, K] x [N, K]^T product through the kernel.
__global__ void single_unit_kernel(int32_t* units, int E, int T) {
  if (threadIdx.x == 0) {
    units[0] = 0;
    units[1] = 0;
    units[2] = 1;
    units[3] = 0;
    reinterpret_cast<UnitDesc*>(units + 4)[0] = UnitDesc{E, 0, T, 0};
  }
}

// X_perm[r] = h[perm_tok[r]] for the routed rows and the shared rows (one warp per row).
template <typename T>
__global__ void gather_rows_kernel(const T* __restrict__ h, const int32_t* __restrict__ perm_tok,
                                   const int32_t* __restrict__ units, int T_, int H,
                                   T* __restrict__ xp) {
  const int rows = units[1] + (units[2] ? T_ : 0);
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += gridDim.x * (blockDim.x >> 5)) {
    const uint4* src = reinterpret_cast<const uint4*>(h + (int64_t)perm_tok[r] * H);
    uint4* dst = reinterpret_cast<uint4*>(xp + (int64_t)r * H);
    for (int v = lane; v < nvec; v += 32) dst[v] = ld_cached(src + v);
  }
}

}  // namespace sm100
}  // namespace tarfa
