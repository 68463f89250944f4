// Grouped expert GEMV for decode-shaped batches (few tokens per expert).
//
// One launch computes, for every "unit" (a routed expert with the rows routed
// to it, or the shared expert with all tokens), either
//   phase GATE_UP: act[row, i] = silu(gate_i . x_row) * (up_i . x_row)
//   phase DOWN:    y[row, h]   = down_h . act_row
// with fp32 accumulation on the tensor cores (mma.sync m16n8k16).  The weights
// are the only large operand: each weight element is read from HBM exactly
// once per launch with 128-bit non-allocating loads, so the kernel is bounded
// by HBM bandwidth; the token vectors (<= 16 per expert at decode) are tiny
// and stay in L1/L2.
//
// A tile is 16 weight rows of one unit.  GATE_UP pairs gate row i with up row
// I+i in the same tile (rows 0-7 gate, 8-15 up), so one lane ends up holding
// gate and up of the same (i, token) and applies SiLU*mul in registers.  The K
// dimension of a tile is split across KSPLIT warps and reduced through shared
// memory in a fixed order (deterministic results).
//
// K permutation.  The MMA only needs A and B to agree on which k a lane holds.
// A lane loads 16 contiguous bytes of a weight row and the matching 16 bytes
// of the token vector; both are fed to the same fragment slots, so the dot
// product is unchanged while every load stays 128-bit and coalesced
// (4 lanes read 64 contiguous bytes of a row).  For int4, a 32-bit word holds
// 8 consecutive k; nibbles s and s+4 form one packed (q-8) pair, and the
// token vector is byte-permuted the same way.
#pragma once
#include "common.cuh"
#include "routing.cuh"
#include "combine.cuh"

namespace tarfa {

enum GemvPhase { kGateUp = 0, kDown = 1 };


struct GemvArgs {
  const void* x;             // GATE_UP: hidden [T, ld_x]; DOWN: act [R, ld_x]
  int64_t ld_x;
  const void* x_sh;          // GATE_UP, or null: the shared unit's token rows (else x)
  const int32_t* perm_tok;   // GATE_UP: row -> token; DOWN: unused (row = x row)
  const int32_t* units;
  int which;                 // bit 0: routed units, bit 1: shared unit
  int E;
  const void* w;             // routed weights: GATE_UP gate_up base, DOWN down base
  int64_t w_estride;         // per expert (elements, or 32-bit words for int4)
  int64_t w_rstride;         // per row
  const void* sc;            // int4 scales
  int64_t s_estride, s_rstride;
  int group;                 // int4: 0 = one scale per row, else the group size
  const int32_t* expert_slot;
  int N_r, K_r;              // routed: GATE_UP (I, H); DOWN (H, I)
  const void* sw0;           // shared: GATE_UP gate_proj; DOWN down_proj
  const void* sw1;           // shared: GATE_UP up_proj
  int N_s, K_s;              // shared: GATE_UP (Is, H); DOWN (H, Is)
  void* out;                 // GATE_UP: act (model dtype); DOWN: y (fp32)
  int64_t ld_out;
  unsigned* status;
  // 0: unit table from `units`, written by an earlier kernel (waited for first);
  // 2: shared unit only, at its fixed rows (decode GATE_UP of the dense shared
  //    expert beside int4 routed experts)
  // 3: shared unit first at its fixed rows, then the unit table the previous
  //    kernel writes (decode: the router's last CTA; expert-parallel receive,
  //    ep_p2p.cuh).  The shared tiles need no routing, so they stream while the
  //    previous kernel finishes.
  int route_mode;
  int sh_row0;               // modes 2 / 3: first row and token count of the shared unit
  int sh_rows;
  int add_shared;            // modes 2 / 3: the shared unit takes part
  int raw_out;               // DOWN: the fp32 dot itself, not rounded (a K part of a split expert)
};

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
// Resident CTAs per SM a launch is built for (registers fit it; grids are
// capped at this many per SM).  The int4 kernels of 1-8 tokens fit three in 80
// registers: the int4 loop is latency-bound (dequantisation between each
// batch of loads and its MMAs), so more resident warps hide more of it
// (config-1 layer, T = 1: 45.8 vs 47.9 us per layer).  The dense down GEMV
// measured no better with three.
constexpr int gemv_ctas_per_sm(int mode, int phase, int ntb) {
  return (mode != kModeExact && ntb == 1) ? 3 : 2;
}

TARFA_DEVI void group_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// One warp's share of a 16-row tile: acc[b] += W(rows g, g+8)[k in iterations
// [i0, i1)] . x(token block b).  An iteration is 32 k (dense) or 128 k (int4;
// a scale group spans whole iterations).  xrow[b] is this lane's token row (always a valid row).
// Dense weights are loaded 4 iterations (8 x 16 B per lane) at a time.
template <typename T, int MODE, int NTB>
TARFA_DEVI void gemv_kloop(const char* rowA, const char* rowB, const T* scA, const T* scB,
                           int group, int i0, int i1, const char* const (&xrow)[NTB],
                           float (&acc)[NTB][4]) {
  const int c = (threadIdx.x & 31) & 3;
  if (MODE == kModeExact) {
    constexpr int NB = 4;
    int it = i0;
    for (; it + NB <= i1; it += NB) {
      uint4 wa[NB], wb[NB];
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const int64_t off = ((int64_t)(it + j) * 32 + c * 8) * (int64_t)sizeof(T);
        wa[j] = ld_stream(rowA + off);
        wb[j] = ld_stream(rowB + off);
      }
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const int64_t off = ((int64_t)(it + j) * 32 + c * 8) * (int64_t)sizeof(T);
#pragma unroll
        for (int b = 0; b < NTB; ++b) {
          const uint4 xv = ld_cached(xrow[b] + off);
          Mma<T>::run(acc[b], wa[j].x, wb[j].x, wa[j].y, wb[j].y, xv.x, xv.y);
          Mma<T>::run(acc[b], wa[j].z, wb[j].z, wa[j].w, wb[j].w, xv.z, xv.w);
        }
      }
    }
    for (; it < i1; ++it) {
      const int64_t off = ((int64_t)it * 32 + c * 8) * (int64_t)sizeof(T);
      const uint4 wa = ld_stream(rowA + off), wb = ld_stream(rowB + off);
#pragma unroll
      for (int b = 0; b < NTB; ++b) {
        const uint4 xv = ld_cached(xrow[b] + off);
        Mma<T>::run(acc[b], wa.x, wb.x, wa.y, wb.y, xv.x, xv.y);
        Mma<T>::run(acc[b], wa.z, wb.z, wa.w, wb.w, xv.z, xv.w);
      }
    }
  } else {
    // lane c covers k [32c, 32c+32) of each 128-k iteration
    const bool grp_scale = group != 0;
    const bool need_sc = grp_scale || MODE == kModeInt4Dequant;
    const unsigned short* scA16 = reinterpret_cast<const unsigned short*>(scA);
    const unsigned short* scB16 = reinterpret_cast<const unsigned short*>(scB);
    // scale index of the next iteration: a group spans ipg iterations of 128 k
    // (tracked by a counter; no division in the loop)
    const int ipg = grp_scale ? group >> 7 : 0x7fffffff;
    int g_idx = grp_scale ? i0 / ipg : 0;
    int g_rem = grp_scale ? i0 - g_idx * ipg : 0;
    // iterations whose weights (and scales) are in flight together (three
    // keep the kernel in 80 registers)
    constexpr int NBQ = 3;
    for (int ib = i0; ib < i1; ib += NBQ) {
      uint4 qa_b[NBQ], qb_b[NBQ];
      unsigned short ua_b[NBQ], ub_b[NBQ];
#pragma unroll
      for (int j = 0; j < NBQ; ++j) {
        qa_b[j] = make_uint4(0, 0, 0, 0);
        qb_b[j] = qa_b[j];
        ua_b[j] = ub_b[j] = 0;
        if (ib + j < i1) {
          const int64_t woff = ((int64_t)(ib + j) * 16 + c * 4) * 4;   // bytes
          qa_b[j] = ld_stream(rowA + woff);
          qb_b[j] = ld_stream(rowB + woff);
          if (need_sc) {
            ua_b[j] = __ldg(scA16 + g_idx);
            ub_b[j] = __ldg(scB16 + g_idx);
            if (++g_rem == ipg) {
              g_rem = 0;
              ++g_idx;
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < NBQ; ++j) {
        const int it = ib + j;
        if (it >= i1) break;
        const uint4 qa = qa_b[j], qb = qb_b[j];
        float sa = 1.f, sb = 1.f;
        uint32_t sa2 = 0, sb2 = 0;
        if (need_sc) {
          const uint16_t ua = ua_b[j];
          const uint16_t ub = ub_b[j];
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
          for (int s = 0; s < 4; ++s) {
            pa[s] = nib_pair<T>(qaw[m], s);
            pb[s] = nib_pair<T>(qbw[m], s);
            if (MODE == kModeInt4Dequant) {
              pa[s] = Mma<T>::mul2(pa[s], sa2);
              pb[s] = Mma<T>::mul2(pb[s], sb2);
            }
          }
          const int64_t xoff = ((int64_t)it * 128 + c * 32 + m * 8) * (int64_t)sizeof(T);
#pragma unroll
          for (int b = 0; b < NTB; ++b) {
            const uint4 xv = ld_cached(xrow[b] + xoff);
            // (x0,x4) (x1,x5) (x2,x6) (x3,x7) to match nibble pairs (s, s+4)
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
  }
}

// Epilogue value of one (row, token) pair of a tile, per mode:
// GATE_UP: act from (gate, up); DOWN: y (model-dtype value, or fp32 for the fused int4 decode).
template <typename T, int MODE>
TARFA_DEVI float gate_up_act(float g, float u) {
  if (MODE == kModeInt4Fused) return silu_f(g) * u;          // moe_kernel.py:99-100
  const float gr = rnd<T>(g), ur = rnd<T>(u);                // fused_int4.py:193 / 242
  return rnd<T>(silu_f(gr)) * ur;
}

// A resolved tile: the unit, its 16 weight rows for fragment rows g and g + 8
// (byte pointers) and the int4 scale rows.
struct GemvTile {
  bool shared_unit;
  int tt, K;
  UnitDesc d;
  const char* rowA;
  const char* rowB;
  const void* scA;
  const void* scB;
};

template <typename T, int MODE, int PHASE>
TARFA_DEVI GemvTile gemv_tile(const GemvArgs& a, int tile, int nt_s, int tiles_r,
                              const int32_t* units, int nu, const UnitDesc& fixed_sh, int g) {
  constexpr bool INT4 = MODE != kModeExact;
  GemvTile r;
  r.scA = r.scB = nullptr;
  if (tile >= nt_s) {
    const int u = (tile - nt_s) / tiles_r;
    r.shared_unit = false;
    r.tt = (tile - nt_s) % tiles_r;
    r.d = unit_descs(units)[u];
    const int slot = a.expert_slot ? a.expert_slot[r.d.expert] : r.d.expert;
    r.K = a.K_r;
    const int ra = PHASE == kGateUp ? r.tt * 8 + g : r.tt * 16 + g;
    const int rb = PHASE == kGateUp ? a.N_r + r.tt * 8 + g : r.tt * 16 + g + 8;
    const int64_t esz = INT4 ? 4 : (int64_t)sizeof(T);
    const char* wb = static_cast<const char*>(a.w) + (int64_t)slot * a.w_estride * esz;
    r.rowA = wb + (int64_t)ra * a.w_rstride * esz;
    r.rowB = wb + (int64_t)rb * a.w_rstride * esz;
    if (INT4) {
      const T* sb = static_cast<const T*>(a.sc) + (int64_t)slot * a.s_estride;
      r.scA = sb + (int64_t)ra * a.s_rstride;
      r.scB = sb + (int64_t)rb * a.s_rstride;
    }
  } else {
    r.shared_unit = true;
    r.tt = tile;
    r.d = a.route_mode != 0 ? fixed_sh : unit_descs(units)[nu];
    r.K = a.K_s;
    const T* s0 = static_cast<const T*>(a.sw0);
    if (PHASE == kGateUp) {
      r.rowA = reinterpret_cast<const char*>(s0 + (int64_t)(r.tt * 8 + g) * r.K);
      r.rowB = reinterpret_cast<const char*>(static_cast<const T*>(a.sw1) + (int64_t)(r.tt * 8 + g) * r.K);
    } else {
      r.rowA = reinterpret_cast<const char*>(s0 + (int64_t)(r.tt * 16 + g) * r.K);
      r.rowB = reinterpret_cast<const char*>(s0 + (int64_t)(r.tt * 16 + g + 8) * r.K);
    }
  }
  return r;
}

template <typename T, int MODE, int PHASE, int KSPLIT, int NTB>
__global__ void __launch_bounds__(kGemvThreads, gemv_ctas_per_sm(MODE, PHASE, NTB)) gemv_kernel(const GemvArgs a) {
  constexpr bool INT4 = MODE != kModeExact;
  constexpr int kGroups = kGemvWarps / KSPLIT;              // tiles per CTA step
  constexpr int TR = PHASE == kGateUp ? 8 : 16;             // tile rows per unit index
  __shared__ float red[kGroups][KSPLIT][NTB * 4][32];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int grp = warp / KSPLIT, kw = warp % KSPLIT;
  const int g = lane >> 2, c = lane & 3;

  // Mode 0 releases its dependents only once the kernel before it has
  // completed: the decode chain's combine reads the router's logits before its
  // own wait, so they must be complete when it starts.
  if (a.route_mode != 0) grid_dep_launch_dependents();
  const int32_t* units = a.units;
  const int32_t* const perm_tok = a.perm_tok;
  int nu = -1;          // routed units; unknown until the unit table is there (mode 3)
  bool has_sh;
  if (a.route_mode == 0) {
    grid_dep_wait();
    grid_dep_launch_dependents();
    nu = units[0];
    has_sh = units[2] != 0;
  } else {
    has_sh = a.add_shared != 0;
    if (a.route_mode == 2) nu = 0;
  }
  // the shared unit's rows are fixed when the routing is the router's own top-k
  const UnitDesc fixed_sh{a.E, a.sh_row0, a.sh_rows, 0};
  const int tiles_r = a.N_r / TR, tiles_s = a.N_s / TR;
  // shared-expert tiles first: they need no routing, so they run while the
  // router kernel is still finishing.  The shared expert is never quantised:
  // an int4 kernel runs its tiles with the exact loop and epilogue.
  const int nt_s = ((a.which & 2) && has_sh) ? tiles_s : 0;

  for (int base = blockIdx.x * kGroups;; base += gridDim.x * kGroups) {
    if (nu < 0 && base + kGroups > nt_s) {   // CTA-uniform: first step with a routed tile
      grid_dep_wait();
      nu = units[0];
    }
    const int nt_r = ((a.which & 1) && nu > 0) ? nu * tiles_r : 0;
    const int ntiles = nt_s + nt_r;
    if (base >= ntiles) break;
    const int tile = base + grp;
    if (tile >= ntiles) continue;   // uniform within a warp group; groups sync separately
    const GemvTile tl = gemv_tile<T, MODE, PHASE>(a, tile, nt_s, tiles_r, units, nu, fixed_sh, g);
    const bool shared_unit = tl.shared_unit;
    const int tt = tl.tt, K = tl.K;
    const UnitDesc d = tl.d;
    const char* rowA = tl.rowA;
    const char* rowB = tl.rowB;
    const T* scA = static_cast<const T*>(tl.scA);
    const T* scB = static_cast<const T*>(tl.scB);
    const int ntok = d.nrows;
    const int ntb_groups = (ntok + 8 * NTB - 1) / (8 * NTB);

    for (int tg = 0; tg < ntb_groups; ++tg) {
      float acc[NTB][4];
#pragma unroll
      for (int b = 0; b < NTB; ++b)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[b][q] = 0.f;

      // token vector rows for this lane (B fragment column g of each token
      // block).  Columns past the unit's rows repeat its last row: their MMA
      // outputs are never stored, and the loads need no guard.
      const char* xrow[NTB];
#pragma unroll
      for (int b = 0; b < NTB; ++b) {
        const int n = min(tg * 8 * NTB + b * 8 + g, ntok - 1);
        const int r = d.row0 + n;
        // shared-unit rows hold the tokens in order (perm_tok[row0 + n] == n)
        const int xr = PHASE == kGateUp ? (shared_unit ? n : perm_tok[r]) : r;
        const void* xb = shared_unit && a.x_sh ? a.x_sh : a.x;
        xrow[b] = reinterpret_cast<const char*>(static_cast<const T*>(xb) + (int64_t)xr * a.ld_x);
      }

      if (INT4 && shared_unit) {
        const int n_it = K / 32;
        const int i0 = kw * n_it / KSPLIT, i1 = (kw + 1) * n_it / KSPLIT;
        gemv_kloop<T, kModeExact, NTB>(rowA, rowB, scA, scB, a.group, i0, i1, xrow, acc);
      } else {
        const int n_it = K / (INT4 ? 128 : 32);
        const int i0 = kw * n_it / KSPLIT, i1 = (kw + 1) * n_it / KSPLIT;
        gemv_kloop<T, MODE, NTB>(rowA, rowB, scA, scB, a.group, i0, i1, xrow, acc);
      }

      // -------- cross-warp K reduction (fixed order) ---------------------------
      if (KSPLIT > 1) {
#pragma unroll
        for (int b = 0; b < NTB; ++b)
#pragma unroll
          for (int q = 0; q < 4; ++q) red[grp][kw][b * 4 + q][lane] = acc[b][q];
        group_barrier(1 + grp, KSPLIT * 32);
        if (kw == 0) {
#pragma unroll
          for (int b = 0; b < NTB; ++b)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float s = red[grp][0][b * 4 + q][lane];
#pragma unroll
              for (int w2 = 1; w2 < KSPLIT; ++w2) s += red[grp][w2][b * 4 + q][lane];
              acc[b][q] = s;
            }
        }
        group_barrier(1 + grp, KSPLIT * 32);
      }

      // -------- epilogue --------------------------------------------------------
      if (kw == 0) {
        const bool fused4 = MODE == kModeInt4Fused && !shared_unit;
        float rsa = 1.f, rsb = 1.f;   // per-row int4 scale, folded after the dot
        if (fused4 && a.group == 0) {
          rsa = Elem<T>::bits_to_f(reinterpret_cast<const uint16_t*>(scA)[0]);
          rsb = Elem<T>::bits_to_f(reinterpret_cast<const uint16_t*>(scB)[0]);
        }
#pragma unroll
        for (int b = 0; b < NTB; ++b)
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int n = tg * 8 * NTB + b * 8 + 2 * c + q;
            if (n >= ntok) continue;
            const int r = d.row0 + n;
            const float va = acc[b][q] * rsa;       // row g   (gate / down row g)
            const float vb = acc[b][2 + q] * rsb;   // row g+8 (up   / down row g+8)
            if (PHASE == kGateUp) {
              float act;
              if (fused4) {
                // moe_kernel.py:99-100: silu(g) * u in fp32, one rounding
                act = silu_f(va) * vb;
              } else {
                // fused_int4.py:193 / 242: F.linear output, silu and product each rounded
                const float gr = rnd<T>(va), ur = rnd<T>(vb);
                act = rnd<T>(silu_f(gr)) * ur;
              }
              T* o = static_cast<T*>(a.out) + (int64_t)r * a.ld_out + tt * 8 + g;
              *o = Elem<T>::from_f(act);
            } else {
              float* o = static_cast<float*>(a.out) + (int64_t)r * a.ld_out + tt * 16 + g;
              if (fused4 || a.raw_out) {
                o[0] = va;            // moe_kernel.py:101-102: fp32 per-expert output
                o[8] = vb;
              } else {
                o[0] = rnd<T>(va);    // F.linear(..., dn) output in the model dtype
                o[8] = rnd<T>(vb);
              }
            }
          }
      }
    }
  }
  // a kernel that never waited still completes only after its predecessor, so
  // that the next kernel's wait covers the whole chain
  if (a.route_mode >= 2) grid_dep_wait();
}

}  // namespace tarfa
