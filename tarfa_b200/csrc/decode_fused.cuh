// Fused decode layer: one persistent cooperative launch runs the whole MoE
// block for a decode batch (T <= 16 tokens).
//
// Per CTA (one per SM), 10 warps:
//   warp 0      producer: streams 16-row weight tiles in 1 KB-per-row chunks
//               with cp.async.bulk into an 8-stage shared-memory ring (about
//               130 KB in flight per SM), mbarrier-tracked; it runs ahead
//               across phases, so the down projections are in flight before
//               the second grid barrier releases the consumers
//   warps 1..8  consumers: tensor-core MMA (m16n8k16, fp32 accumulate) from the
//               ring, K split across the 8 warps and reduced in a fixed order
//   warp 9      aux: router rows (phase 0)
//
//   phase 0  router logits (exact, exact.cuh; aux warps) || shared
//            expert gate/up (independent of the routing; producer/consumers)
//   barrier  grid-wide, bounded spin
//   phase 1  every CTA computes the top-k and the expert-sorted unit table for
//            all tokens itself, from the logits in L2, into shared memory; the
//            producer starts streaming as soon as the table is ready
//   phase 2  routed gate/up + SiLU*mul
//   barrier
//   phase 3  down projections (routed + shared); per 16-row output block a
//            completion counter elects the CTA that finishes the block last to
//            combine it (routing-weighted sum in the reference order + gated
//            shared expert) -- no third barrier
//
// Arithmetic is identical to the multi-kernel path (router.cuh, gemv.cuh):
// same rounding points and combine order.  Every wait is bounded by a clock
// limit; on timeout the kernel raises kStatusWaitTimeout, stops issuing work,
// drains its copies in flight and returns.
#pragma once
#include "common.cuh"
#include "gemv.cuh"
#include "router.cuh"

namespace tarfa {
namespace fused {

constexpr int kConsumers = 8;
constexpr int kWarps = 1 + kConsumers + 1;
constexpr int kThreads = 32 * kWarps;                 // 320
constexpr int kAuxWarp = kWarps - 1;
constexpr int kWorkThreads = 32 * (kConsumers + 1);   // consumers + aux (barrier group)
constexpr int kMaxT = 16;
constexpr int kMaxK = 8;
constexpr int kMaxRoutes = kMaxT * kMaxK;
constexpr int kMaxUnits = kMaxRoutes + 1;
constexpr int kStages = 8;
constexpr int kChunkBytes = 1024;                     // per weight row per stage
// Rows are 64 B apart in bank space, so the 16-byte fragment reads of rows g
// and g+1 (lanes 0-7 of one wavefront) fall on disjoint banks.
constexpr int kRowStride = kChunkBytes + 64;
constexpr int kStageBytes = 16 * kRowStride;
constexpr long long kSpinCycles = 4000000000ll;       // ~2 s

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

struct __align__(16) Smem {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  int idx[kMaxRoutes];        // top-k ids, [t*K + k]
  float w[kMaxRoutes];        // top-k weights
  int perm_tok[kMaxRoutes + kMaxT];
  int route_row[kMaxRoutes];
  int first[kMaxRoutes];
  UnitDesc units[kMaxUnits];
  int nu;
  volatile int ready;         // unit table published (producer may stream phase 2/3)
  volatile int abort;
  int last;
  float red[kConsumers * 2 * 4 * 32];   // K-split partial sums (NTB <= 2)
};

constexpr size_t kSmemBytes = 1024 + kStages * kStageBytes + sizeof(Smem);

TARFA_DEVI uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

TARFA_DEVI bool bar_try(uint32_t a, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(a), "r"(parity)
      : "memory");
  return ok != 0;
}

TARFA_DEVI bool bar_wait(uint32_t a, uint32_t parity, Smem& s, unsigned* status, bool honor_abort) {
  if (bar_try(a, parity)) return true;
  const long long t0 = clock64();
  while (!bar_try(a, parity)) {
    if (honor_abort && s.abort) return false;
    if (clock64() - t0 > kSpinCycles) {
      raise_status(status, kStatusWaitTimeout);
      s.abort = 1;
      return false;
    }
  }
  return true;
}

// Grid-wide barrier of the work warps (consumers + aux); the producer is not part of it.
TARFA_DEVI bool grid_barrier(unsigned* bar, Smem& s, unsigned* status) {
  group_barrier(1, kWorkThreads);
  if (threadIdx.x == 32) {
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
  group_barrier(1, kWorkThreads);
  return s.abort == 0;
}

// ---------------------------------------------------------------------------
// work items: 16 weight rows of one unit, streamed chunk by chunk
// ---------------------------------------------------------------------------
enum ItemKind { kSharedGU = 0, kRoutedGU = 1, kDown = 2 };

struct Item {
  int kind;
  UnitDesc d;
  int tt;          // gate/up: 8-pair block; down: 16-row block
  int K;           // reduction length (elements)
  bool int4;       // weights of this item are int4 packed
};

template <int MODE>
TARFA_DEVI Item make_item(const Args& a, const Smem& s, int kind, int t) {
  Item it;
  it.kind = kind;
  it.int4 = false;
  if (kind == kSharedGU) {
    it.d = UnitDesc{a.E, a.T * a.K, a.T, 0};
    it.tt = t;
    it.K = a.H;
  } else if (kind == kRoutedGU) {
    const int tpu = a.I / 8;
    it.d = s.units[t / tpu];
    it.tt = t % tpu;
    it.K = a.H;
    it.int4 = MODE != kModeExact;
  } else {
    const int nun = s.nu + (a.Is ? 1 : 0);
    it.d = s.units[t % nun];
    it.tt = t / nun;
    const bool sh = it.d.expert == a.E;
    it.K = sh ? a.Is : a.I;
    it.int4 = !sh && MODE != kModeExact;
  }
  return it;
}

// byte pointer to weight row r (0..15) of an item, and that row's byte length
template <typename T>
TARFA_DEVI const char* item_row(const Args& a, const Item& it, int r, int64_t* row_bytes) {
  const bool sh = it.d.expert == a.E;
  const int slot = sh ? 0 : (a.expert_slot ? a.expert_slot[it.d.expert] : it.d.expert);
  if (it.kind != kDown) {
    const int i = it.tt * 8 + (r & 7);
    if (sh) {
      *row_bytes = (int64_t)a.H * sizeof(T);
      const T* base = static_cast<const T*>(r < 8 ? a.sh_gate : a.sh_up);
      return reinterpret_cast<const char*>(base + (int64_t)i * a.H);
    }
    const int row = r < 8 ? i : a.I + i;
    if (it.int4) {
      *row_bytes = a.H / 2;
      return static_cast<const char*>(a.gate_up) + ((int64_t)slot * 2 * a.I + row) * (a.H / 2);
    }
    *row_bytes = (int64_t)a.H * sizeof(T);
    return reinterpret_cast<const char*>(static_cast<const T*>(a.gate_up) +
                                         ((int64_t)slot * 2 * a.I + row) * a.H);
  }
  const int hrow = it.tt * 16 + r;
  if (sh) {
    *row_bytes = (int64_t)a.Is * sizeof(T);
    return reinterpret_cast<const char*>(static_cast<const T*>(a.sh_down) + (int64_t)hrow * a.Is);
  }
  if (it.int4) {
    *row_bytes = a.I / 2;
    return static_cast<const char*>(a.down) + ((int64_t)slot * a.H + hrow) * (a.I / 2);
  }
  *row_bytes = (int64_t)a.I * sizeof(T);
  return reinterpret_cast<const char*>(static_cast<const T*>(a.down) + ((int64_t)slot * a.H + hrow) * a.I);
}

// scale row pointer (int4) of fragment row r of an item
template <typename T>
TARFA_DEVI const T* item_scale(const Args& a, const Item& it, int r) {
  const int slot = a.expert_slot ? a.expert_slot[it.d.expert] : it.d.expert;
  if (it.kind != kDown) {
    const int64_t gpr = a.group ? a.H / a.group : 1;
    const int row = r < 8 ? it.tt * 8 + r : a.I + it.tt * 8 + (r - 8);
    return static_cast<const T*>(a.gu_scale) + ((int64_t)slot * 2 * a.I + row) * gpr;
  }
  const int64_t gpr = a.group ? a.I / a.group : 1;
  return static_cast<const T*>(a.dn_scale) + ((int64_t)slot * a.H + it.tt * 16 + r) * gpr;
}

// ---------------------------------------------------------------------------
// producer
// ---------------------------------------------------------------------------
template <typename T>
TARFA_DEVI bool stream_item(const Args& a, Smem& s, uint8_t* ring, const Item& it, int& stage,
                            uint32_t& phase, int (&issued)[kStages]) {
  const char* rows[16];
  int64_t rb = 0;
#pragma unroll
  for (int r = 0; r < 16; ++r) rows[r] = item_row<T>(a, it, r, &rb);
  for (int64_t off = 0; off < rb; off += kChunkBytes) {
    const uint32_t bytes = (uint32_t)(rb - off < kChunkBytes ? rb - off : kChunkBytes);
    if (!bar_wait(saddr(&s.empty[stage]), phase ^ 1u, s, a.status, true)) return false;
    const uint32_t full = saddr(&s.full[stage]);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(full), "r"(16u * bytes)
                 : "memory");
    const uint32_t dst0 = saddr(ring + stage * kStageBytes);
#pragma unroll
    for (int r = 0; r < 16; ++r)
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
          ::"r"(dst0 + r * kRowStride), "l"(rows[r] + off), "r"(bytes), "r"(full)
          : "memory");
    issued[stage] = (int)phase;
    if (++stage == kStages) { stage = 0; phase ^= 1u; }
  }
  return true;
}

// ---------------------------------------------------------------------------
// consumers
// ---------------------------------------------------------------------------
TARFA_DEVI uint4 lds128(uint32_t a) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(a));
  return r;
}

TARFA_DEVI uint4 ld_coherent(const void* p) {   // data written earlier in this launch
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// Consume all chunks of one item; returns false on abort.  acc: this warp's partial.
template <typename T, int MODE, int NTB>
TARFA_DEVI bool consume_item(const Args& a, Smem& s, uint8_t* ring, const Item& it, int& stage,
                             uint32_t& phase, const char* const (&xrow)[NTB], bool x_coherent,
                             float (&acc)[NTB][4], int cw) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int esize = sizeof(T);
  const bool q4 = it.int4;
  const int64_t row_bytes = q4 ? it.K / 2 : (int64_t)it.K * esize;
  const T* scA = nullptr;
  const T* scB = nullptr;
  if (q4) {
    scA = item_scale<T>(a, it, g);
    scB = item_scale<T>(a, it, g + 8);
  }
  for (int64_t off = 0; off < row_bytes; off += kChunkBytes) {
    const int bytes = (int)(row_bytes - off < kChunkBytes ? row_bytes - off : kChunkBytes);
    if (!bar_wait(saddr(&s.full[stage]), phase, s, a.status, true)) return false;
    const uint32_t base = saddr(ring + stage * kStageBytes);
    const uint32_t rA = base + g * kRowStride, rB = base + (g + 8) * kRowStride;
    if (!q4) {
      const int k0 = (int)(off / esize);            // first k of this chunk
      const int n_it = bytes / (32 * esize);        // 32-k iterations in the chunk
      const int i0 = cw * n_it / kConsumers, i1 = (cw + 1) * n_it / kConsumers;
      for (int i = i0; i < i1; ++i) {
        const uint4 wa = lds128(rA + (i * 32 + c * 8) * esize);
        const uint4 wb = lds128(rB + (i * 32 + c * 8) * esize);
        const int64_t xo = ((int64_t)k0 + i * 32 + c * 8) * esize;
#pragma unroll
        for (int b = 0; b < NTB; ++b) {
          uint4 xv = make_uint4(0, 0, 0, 0);
          if (xrow[b]) xv = x_coherent ? ld_coherent(xrow[b] + xo) : ld_cached(xrow[b] + xo);
          Mma<T>::run(acc[b], wa.x, wb.x, wa.y, wb.y, xv.x, xv.y);
          Mma<T>::run(acc[b], wa.z, wb.z, wa.w, wb.w, xv.z, xv.w);
        }
      }
    } else {
      const int k0 = (int)(off * 2);                // 2 k per byte
      const int n_it = bytes / 64;                  // 128-k iterations (64 bytes per row)
      const int i0 = cw * n_it / kConsumers, i1 = (cw + 1) * n_it / kConsumers;
      const bool grp_scale = a.group != 0;
      for (int i = i0; i < i1; ++i) {
        const uint4 qa = lds128(rA + i * 64 + c * 16);
        const uint4 qb = lds128(rB + i * 64 + c * 16);
        const int kk = k0 + i * 128;                 // first k of the iteration
        float sa = 1.f, sb = 1.f;
        uint32_t sa2 = 0, sb2 = 0;
        if (grp_scale || MODE == kModeInt4Dequant) {
          const int gi = grp_scale ? kk / a.group : 0;
          const uint16_t ua = reinterpret_cast<const uint16_t*>(scA)[gi];
          const uint16_t ub = reinterpret_cast<const uint16_t*>(scB)[gi];
          sa = Elem<T>::bits_to_f(ua);
          sb = Elem<T>::bits_to_f(ub);
          sa2 = uint32_t(ua) | (uint32_t(ua) << 16);
          sb2 = uint32_t(ub) | (uint32_t(ub) << 16);
        }
        float part[NTB][4];
#pragma unroll
        for (int b = 0; b < NTB; ++b)
#pragma unroll
          for (int q = 0; q < 4; ++q) part[b][q] = 0.f;
        const uint32_t qaw[4] = {qa.x, qa.y, qa.z, qa.w};
        const uint32_t qbw[4] = {qb.x, qb.y, qb.z, qb.w};
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          uint32_t pa[4], pb[4];
#pragma unroll
          for (int sq = 0; sq < 4; ++sq) {
            pa[sq] = nib_pair<T>(qaw[m], sq);
            pb[sq] = nib_pair<T>(qbw[m], sq);
            if (MODE == kModeInt4Dequant) {
              pa[sq] = Mma<T>::mul2(pa[sq], sa2);
              pb[sq] = Mma<T>::mul2(pb[sq], sb2);
            }
          }
          const int64_t xo = ((int64_t)kk + c * 32 + m * 8) * esize;
#pragma unroll
          for (int b = 0; b < NTB; ++b) {
            uint4 xv = make_uint4(0, 0, 0, 0);
            if (xrow[b]) xv = x_coherent ? ld_coherent(xrow[b] + xo) : ld_cached(xrow[b] + xo);
            const uint32_t x04 = __byte_perm(xv.x, xv.z, 0x5410);
            const uint32_t x15 = __byte_perm(xv.x, xv.z, 0x7632);
            const uint32_t x26 = __byte_perm(xv.y, xv.w, 0x5410);
            const uint32_t x37 = __byte_perm(xv.y, xv.w, 0x7632);
            if (MODE == kModeInt4Fused && grp_scale) {
              Mma<T>::run(part[b], pa[0], pb[0], pa[1], pb[1], x04, x15);
              Mma<T>::run(part[b], pa[2], pb[2], pa[3], pb[3], x26, x37);
            } else {
              Mma<T>::run(acc[b], pa[0], pb[0], pa[1], pb[1], x04, x15);
              Mma<T>::run(acc[b], pa[2], pb[2], pa[3], pb[3], x26, x37);
            }
          }
        }
        if (MODE == kModeInt4Fused && grp_scale) {
#pragma unroll
          for (int b = 0; b < NTB; ++b) {
            acc[b][0] = fmaf(part[b][0], sa, acc[b][0]);
            acc[b][1] = fmaf(part[b][1], sa, acc[b][1]);
            acc[b][2] = fmaf(part[b][2], sb, acc[b][2]);
            acc[b][3] = fmaf(part[b][3], sb, acc[b][3]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(&s.empty[stage])) : "memory");
    if (++stage == kStages) { stage = 0; phase ^= 1u; }
  }
  return true;
}

// Reduce the 8 consumers' partials in a fixed order; consumer 0 gets the sum.
template <int NTB>
TARFA_DEVI void consumer_reduce(float (&acc)[NTB][4], Smem& s, int cw, int lane) {
#pragma unroll
  for (int b = 0; b < NTB; ++b)
#pragma unroll
    for (int q = 0; q < 4; ++q) s.red[(cw * NTB * 4 + b * 4 + q) * 32 + lane] = acc[b][q];
  group_barrier(2, 32 * kConsumers);
  if (cw == 0) {
#pragma unroll
    for (int b = 0; b < NTB; ++b)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float v = s.red[(b * 4 + q) * 32 + lane];
#pragma unroll
        for (int w2 = 1; w2 < kConsumers; ++w2) v += s.red[(w2 * NTB * 4 + b * 4 + q) * 32 + lane];
        acc[b][q] = v;
      }
  }
  group_barrier(2, 32 * kConsumers);
}

template <typename T, int MODE, int NTB>
TARFA_DEVI bool run_item(const Args& a, Smem& s, uint8_t* ring, const Item& it, int& stage,
                         uint32_t& phase, int cw) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int ntok = it.d.nrows;
  const bool is_down = it.kind == kDown;
  // token rows of this lane (one group of NTB token blocks: ntok <= 8 * NTB)
  const char* xrow[NTB];
#pragma unroll
  for (int b = 0; b < NTB; ++b) {
    const int n = b * 8 + g;
    xrow[b] = nullptr;
    if (n < ntok) {
      const int r = it.d.row0 + n;
      xrow[b] = is_down
                    ? reinterpret_cast<const char*>(static_cast<const T*>(a.act) + (int64_t)r * a.Imax)
                    : reinterpret_cast<const char*>(static_cast<const T*>(a.h) + (int64_t)s.perm_tok[r] * a.H);
    }
  }
  float acc[NTB][4];
#pragma unroll
  for (int b = 0; b < NTB; ++b)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[b][q] = 0.f;
  if (!consume_item<T, MODE, NTB>(a, s, ring, it, stage, phase, xrow, is_down, acc, cw)) return false;
  consumer_reduce<NTB>(acc, s, cw, lane);
  if (cw == 0) {
    const bool fused32 = it.int4 && MODE == kModeInt4Fused;
    float rsa = 1.f, rsb = 1.f;
    if (fused32 && a.group == 0) {
      rsa = Elem<T>::bits_to_f(reinterpret_cast<const uint16_t*>(item_scale<T>(a, it, g))[0]);
      rsb = Elem<T>::bits_to_f(reinterpret_cast<const uint16_t*>(item_scale<T>(a, it, g + 8))[0]);
    }
#pragma unroll
    for (int b = 0; b < NTB; ++b)
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int n = b * 8 + 2 * c + q;
        if (n >= ntok) continue;
        const int r = it.d.row0 + n;
        const float va = acc[b][q] * rsa, vb = acc[b][2 + q] * rsb;
        if (!is_down) {
          const float act = fused32 ? gate_up_act<T, kModeInt4Fused>(va, vb)
                                    : gate_up_act<T, kModeExact>(va, vb);
          static_cast<T*>(a.act)[(int64_t)r * a.Imax + it.tt * 8 + g] = Elem<T>::from_f(act);
        } else {
          float* o = a.y + (int64_t)r * a.H + it.tt * 16 + g;
          o[0] = fused32 ? va : rnd<T>(va);
          o[8] = fused32 ? vb : rnd<T>(vb);
        }
      }
  }
  return true;
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
      if (a.T > 1) {   // ascending expert id (index_add_ order)
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

template <typename T, int MAXC>
TARFA_DEVI void router_row(const Args& a, int row) {
  const int lane = threadIdx.x & 31;
  const int nch = a.H / 8;
  const T* wrow = row < a.E ? static_cast<const T*>(a.w_r) + (int64_t)row * a.H
                            : static_cast<const T*>(a.w_sg);
  uint4 wv[MAXC];
#pragma unroll
  for (int j = 0; j < MAXC; ++j) {
    const int ch = lane + 32 * j;
    wv[j] = ch < nch ? ld_stream(wrow + ch * 8) : make_uint4(0, 0, 0, 0);
  }
  for (int t = 0; t < a.T; ++t) {
    const T* xrow = static_cast<const T*>(a.h) + (int64_t)t * a.H;
    float lgv = row_dot_exact<T, MAXC>(wv, wrow, xrow, a.H);
    if (lane == 0) {
      if (row < a.E) {
        if (a.bias) lgv = rnd<T>(lgv + Elem<T>::to_f(static_cast<const T*>(a.bias)[row]));
        a.logits[(int64_t)t * a.E + row] = lgv;
      } else {
        a.gate_logit[t] = lgv;
      }
    }
  }
}

template <typename T, int MODE, int NTB>
__global__ void __launch_bounds__(kThreads, 1) decode_layer_kernel(const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  Smem& s = *reinterpret_cast<Smem*>(ring + kStages * kStageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int R = a.T * a.K;
  const int nt_sh = a.Is / 8;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&s.full[i])) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(&s.empty[i])), "r"(kConsumers)
                   : "memory");
    }
    s.nu = 0;
    s.ready = 0;
    s.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (threadIdx.x < a.T) s.perm_tok[R + threadIdx.x] = threadIdx.x;   // shared rows: token t
  __syncthreads();

  if (warp == 0) {
    // ================================ producer ================================
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued[kStages];
      for (int i = 0; i < kStages; ++i) issued[i] = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < nt_sh && ok; t += G)
        ok = stream_item<T>(a, s, ring, make_item<MODE>(a, s, kSharedGU, t), stage, phase, issued);
      // wait for this CTA's unit table (phase 1), bounded
      if (ok) {
        const long long t0 = clock64();
        while (!s.ready && !s.abort) {
          if (clock64() - t0 > kSpinCycles) {
            raise_status(a.status, kStatusWaitTimeout);
            s.abort = 1;
            break;
          }
          __nanosleep(128);
        }
        ok = !s.abort;
      }
      __threadfence_block();
      if (ok) {
        const int nu = s.nu;
        const int n_gu = nu * (a.I / 8);
        for (int t = blockIdx.x; t < n_gu && ok; t += G)
          ok = stream_item<T>(a, s, ring, make_item<MODE>(a, s, kRoutedGU, t), stage, phase, issued);
        const int n_dn = (nu + (a.Is ? 1 : 0)) * (a.H / 16);
        for (int t = blockIdx.x; t < n_dn && ok; t += G)
          ok = stream_item<T>(a, s, ring, make_item<MODE>(a, s, kDown, t), stage, phase, issued);
      }
      // drain: every issued copy has landed before the CTA may exit
      for (int i = 0; i < kStages; ++i)
        if (issued[i] >= 0) bar_wait(saddr(&s.full[i]), (uint32_t)issued[i], s, a.status, false);
    }
    return;
  }

  // ============================ work warps (1..9) ==============================
  const bool consumer = warp >= 1 && warp <= kConsumers;
  const int cw = warp - 1;
  int stage = 0;
  uint32_t phase = 0;
  // ---- phase 0: shared gate/up (consumers) || router rows (aux) ---------------
  if (consumer) {
    for (int t = blockIdx.x; t < nt_sh; t += G)
      if (!run_item<T, MODE, NTB>(a, s, ring, make_item<MODE>(a, s, kSharedGU, t), stage, phase, cw)) break;
  } else {
    const int nrows = a.E + (a.w_sg ? 1 : 0);
    const int per_lane = (a.H / 8 + 31) / 32;
    for (int row = blockIdx.x; row < nrows; row += G) {
      if (per_lane <= 4) router_row<T, 4>(a, row);
      else if (per_lane <= 8) router_row<T, 8>(a, row);
      else router_row<T, 16>(a, row);          // hidden <= 4096 on this path
    }
  }
  if (!grid_barrier(a.bar, s, a.status)) return;

  // ---- phase 1: top-k and unit table (work warps) -----------------------------
  const int wi = warp - 1;                       // 0..8
  const int tid = threadIdx.x - 32, nthr = kWorkThreads;
  for (int t = wi; t < a.T; t += kConsumers + 1) {
    int64_t* io = (blockIdx.x == 0 && a.idx_out) ? a.idx_out + (int64_t)t * a.K : nullptr;
    float* wo = (blockIdx.x == 0 && a.w_out) ? a.w_out + (int64_t)t * a.K : nullptr;
    warp_topk<T>(a.logits + (int64_t)t * a.E, a.E, a.K, s.idx + t * a.K, s.w + t * a.K, io, wo);
  }
  group_barrier(1, kWorkThreads);
  for (int r = tid; r < R; r += nthr) {     // route r = k*T + t
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
  group_barrier(1, kWorkThreads);
  for (int r = tid; r < R; r += nthr) {
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
  group_barrier(1, kWorkThreads);
  const int nu = s.nu;
  if (tid == 0) {
    s.units[nu] = UnitDesc{a.E, R, a.T, 0};
    __threadfence_block();
    s.ready = 1;                       // the producer may stream phases 2 and 3
  }
  group_barrier(1, kWorkThreads);

  // ---- phase 2: routed gate/up (consumers) ------------------------------------
  if (consumer) {
    const int n_gu = nu * (a.I / 8);
    for (int t = blockIdx.x; t < n_gu; t += G)
      if (!run_item<T, MODE, NTB>(a, s, ring, make_item<MODE>(a, s, kRoutedGU, t), stage, phase, cw)) break;
  }
  if (!grid_barrier(a.bar, s, a.status)) return;

  // ---- phase 3: down + per-block combine (consumers) ---------------------------
  if (consumer) {
    const int nun = nu + (a.Is ? 1 : 0);
    const int n_dn = nun * (a.H / 16);
    for (int t = blockIdx.x; t < n_dn; t += G) {
      const Item it = make_item<MODE>(a, s, kDown, t);
      if (!run_item<T, MODE, NTB>(a, s, ring, it, stage, phase, cw)) break;
      group_barrier(2, 32 * kConsumers);
      if (cw == 0 && lane == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(a.hb_cnt + it.tt, 1u);
        s.last = prev == (unsigned)(nun - 1);
        if (s.last) __threadfence();
      }
      group_barrier(2, 32 * kConsumers);
      if (s.last) {
        combine_block<T, MODE>(a, s, it.tt, cw * 32 + lane, 32 * kConsumers);
        if (cw == 0 && lane == 0) a.hb_cnt[it.tt] = 0u;   // leave the counter at rest
      }
      group_barrier(2, 32 * kConsumers);
    }
  }
}

}  // namespace fused
}  // namespace tarfa
