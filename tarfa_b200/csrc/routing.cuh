// Routing primitives shared by the router, permute and decode GEMV kernels:
// the unit table, the stable counting-sort permute, and the warp top-k.
//
// Permute (fused_int4.py:228-229, 241): routes r = k*T + t are stably sorted
// by expert id, giving per expert the (k-slot, token) row-major order of
// torch.where(one_hot(idx).permute(2,1,0)[e]).
#pragma once
#include "common.cuh"
#include "topk_ties.cuh"

namespace tarfa {

// Unit table written by the permute stage:
//   hdr[0] routed units, hdr[1] routed rows, hdr[2] has shared unit, hdr[3] shared row0
//   desc[u] = {expert, row0, nrows, 0}; routed units in ascending expert id,
//   the shared unit (expert == E) last.
struct UnitDesc { int expert, row0, nrows, pad; };
TARFA_DEVI const UnitDesc* unit_descs(const int32_t* units) {
  return reinterpret_cast<const UnitDesc*>(units + 4);
}

struct PermuteOut {
  int32_t* seg_offsets;   // [E+1] or null
  int32_t* perm_tok;      // [R_total]: row -> token
  int32_t* perm_slot;     // [T*K] or null: row -> k-slot
  int32_t* route_row;     // [T*K] or null: (t, k) -> row, -1 for a skipped route
  int32_t* units;         // unit table (header + UnitDesc[])
  int32_t* idx32;         // [T*K] or null: int32 copy of the expert ids
};

// Shared-memory ints needed by block_permute.
__host__ __device__ inline size_t permute_smem_ints(int nwarps, int E) {
  return (size_t)nwarps * E + E;
}

// Block-cooperative stable counting sort of T*K routes by expert id.
// Any blockDim that is a multiple of 32; E <= smem budget.
template <typename Idx>
__device__ void block_permute(const Idx* idx, int T, int K, int E, bool add_shared,
                              const PermuteOut& o, int* smem, unsigned* status) {
  const int nw = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = T * K;
  int* wcnt = smem;            // [nw][E] per-warp counts, then running cursors
  int* off = smem + nw * E;    // [E] totals, then segment offsets
  for (int i = threadIdx.x; i < nw * E + E; i += blockDim.x) smem[i] = 0;
  __syncthreads();
  const int r0 = (int)((int64_t)R * warp / nw), r1 = (int)((int64_t)R * (warp + 1) / nw);
  for (int r = r0 + lane; r < r1; r += 32) {
    const int t = r % T, k = r / T;
    const int64_t e = (int64_t)idx[(int64_t)t * K + k];
    if (e >= 0 && e < E) atomicAdd(&wcnt[warp * E + (int)e], 1);
    else if (e != E) raise_status(status, kStatusBadExpert);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int s = 0;
    for (int w = 0; w < nw; ++w) {
      const int cnt = wcnt[w * E + e];
      wcnt[w * E + e] = s;
      s += cnt;
    }
    off[e] = s;
  }
  __syncthreads();
  UnitDesc* descs = reinterpret_cast<UnitDesc*>(o.units + 4);
  if (warp == 0) {
    const int per = (E + 31) / 32;
    const int b0 = min(lane * per, E), b1 = min(b0 + per, E);
    int s = 0, nz = 0;
    for (int e = b0; e < b1; ++e) { s += off[e]; nz += off[e] > 0; }
    int ps = s, pnz = nz;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, ps, d);
      const int y = __shfl_up_sync(0xffffffffu, pnz, d);
      if (lane >= d) { ps += x; pnz += y; }
    }
    int es = ps - s, enz = pnz - nz;
    const int rows = __shfl_sync(0xffffffffu, ps, 31), nunits = __shfl_sync(0xffffffffu, pnz, 31);
    for (int e = b0; e < b1; ++e) {
      const int cnt = off[e];
      if (cnt > 0) { descs[enz] = UnitDesc{e, es, cnt, 0}; ++enz; }
      if (o.seg_offsets) o.seg_offsets[e] = es;
      off[e] = es;
      es += cnt;
    }
    if (lane == 0) {
      if (o.seg_offsets) o.seg_offsets[E] = rows;
      o.units[0] = nunits;
      o.units[1] = rows;
      o.units[2] = add_shared ? 1 : 0;
      o.units[3] = rows;
      if (add_shared) descs[nunits] = UnitDesc{E, rows, T, 0};
    }
  }
  __syncthreads();
  const unsigned lt = (1u << lane) - 1u;
  for (int rb = r0; rb < r1; rb += 32) {
    const int r = rb + lane;
    const bool in = r < r1;
    const int t = in ? r % T : 0, k = in ? r / T : 0;
    const int64_t e64 = in ? (int64_t)idx[(int64_t)t * K + k] : -1;
    const bool routed = in && e64 >= 0 && e64 < E;
    const int e = routed ? (int)e64 : 0;
    if (in && o.idx32) o.idx32[t * K + k] = (int32_t)e64;
    const unsigned peers = __match_any_sync(0xffffffffu, routed ? e : -1 - lane);
    const int rank = __popc(peers & lt);
    const int cur = routed ? wcnt[warp * E + e] : 0;
    __syncwarp();
    if (routed && rank == 0) wcnt[warp * E + e] = cur + __popc(peers);
    __syncwarp();
    if (routed) {
      const int row = off[e] + cur + rank;
      o.perm_tok[row] = t;
      if (o.perm_slot) o.perm_slot[row] = k;
      if (o.route_row) o.route_row[t * K + k] = row;
    } else if (in && o.route_row) {
      o.route_row[t * K + k] = -1;
    }
  }
  __syncthreads();
  const int rows = o.units[1];
  if (add_shared)
    for (int t = threadIdx.x; t < T; t += blockDim.x) o.perm_tok[rows + t] = t;
  if (o.perm_slot)   // rows past the routed ones (skipped routes) are marked -1
    for (int r = rows + threadIdx.x; r < R; r += blockDim.x) {
      o.perm_slot[r] = -1;
      if (!add_shared) o.perm_tok[r] = -1;
    }
}

// ---------------------------------------------------------------------------
// multi-block permute for large batches: the same outputs as block_permute
// ---------------------------------------------------------------------------
// Pass 1: block b counts the experts of routes [b*kPermRoutes, (b+1)*kPermRoutes)
// into hist[b][E].  Pass 2: every block derives, per expert, the start of its
// segment (sum of the totals of smaller ids) plus the routes of that expert in
// earlier blocks, then scatters its routes with stable ranks inside the block
// (per-warp counts, match_any); block 0 also writes the unit table.
constexpr int kPermThreads = 256;
constexpr int kPermRoutes = 2048;

__host__ __device__ inline int perm_blocks(int R) { return (R + kPermRoutes - 1) / kPermRoutes; }

template <typename Idx>
__global__ void __launch_bounds__(kPermThreads) permute_hist_kernel(const Idx* idx, int T, int K, int E,
                                                                    int32_t* hist, PermuteOut o,
                                                                    unsigned* status) {
  extern __shared__ int sh_hist[];
  for (int i = threadIdx.x; i < E; i += blockDim.x) sh_hist[i] = 0;
  __syncthreads();
  const int R = T * K;
  const int r0 = blockIdx.x * kPermRoutes, r1 = min(R, r0 + kPermRoutes);
  for (int r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
    const int t = r % T, k = r / T;
    const int64_t e = (int64_t)idx[(int64_t)t * K + k];
    if (e >= 0 && e < E) atomicAdd(&sh_hist[(int)e], 1);
    else if (e != E) raise_status(status, kStatusBadExpert);
    if (o.idx32) o.idx32[t * K + k] = (int32_t)e;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += blockDim.x) hist[(int64_t)blockIdx.x * E + i] = sh_hist[i];
}

template <typename Idx>
__global__ void __launch_bounds__(kPermThreads) permute_scatter_kernel(const Idx* idx, int T, int K, int E,
                                                                       int add_shared,
                                                                       const int32_t* hist, PermuteOut o) {
  extern __shared__ int sh_sc[];
  const int nw = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* base = sh_sc;            // [E] first row of expert e's routes in this block
  int* tot = sh_sc + E;         // [E] routes of expert e in all blocks
  int* wcnt = sh_sc + 2 * E;    // [nw][E]
  __shared__ int s_rows;
  const int R = T * K, nblk = perm_blocks(R);
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int t_all = 0, t_pre = 0;
    for (int b = 0; b < nblk; ++b) {
      const int c = hist[(int64_t)b * E + e];
      t_all += c;
      if (b < (int)blockIdx.x) t_pre += c;
    }
    base[e] = t_pre;
    tot[e] = t_all;
  }
  for (int i = threadIdx.x; i < nw * E; i += blockDim.x) wcnt[i] = 0;
  __syncthreads();
  UnitDesc* descs = reinterpret_cast<UnitDesc*>(o.units + 4);
  if (warp == 0) {   // segment starts: exclusive prefix of the totals over expert ids
    const int per = (E + 31) / 32;
    const int b0 = min(lane * per, E), b1 = min(b0 + per, E);
    int s = 0, nz = 0;
    for (int e = b0; e < b1; ++e) { s += tot[e]; nz += tot[e] > 0; }
    int ps = s, pnz = nz;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, ps, d);
      const int y = __shfl_up_sync(0xffffffffu, pnz, d);
      if (lane >= d) { ps += x; pnz += y; }
    }
    int es = ps - s, enz = pnz - nz;
    const int rows = __shfl_sync(0xffffffffu, ps, 31), nunits = __shfl_sync(0xffffffffu, pnz, 31);
    const bool pub = blockIdx.x == 0;
    for (int e = b0; e < b1; ++e) {
      const int cnt = tot[e];
      if (pub && cnt > 0) { descs[enz] = UnitDesc{e, es, cnt, 0}; ++enz; }
      if (pub && o.seg_offsets) o.seg_offsets[e] = es;
      base[e] += es;
      es += cnt;
    }
    if (lane == 0) {
      s_rows = rows;
      if (pub) {
        if (o.seg_offsets) o.seg_offsets[E] = rows;
        o.units[0] = nunits;
        o.units[1] = rows;
        o.units[2] = add_shared ? 1 : 0;
        o.units[3] = rows;
        if (add_shared) descs[nunits] = UnitDesc{E, rows, T, 0};
      }
    }
  }
  // this block's routes, split contiguously over the warps (stable order)
  const int rb0 = blockIdx.x * kPermRoutes, rb1 = min(R, rb0 + kPermRoutes);
  const int span = rb1 - rb0;
  const int r0 = rb0 + (int)((int64_t)span * warp / nw), r1 = rb0 + (int)((int64_t)span * (warp + 1) / nw);
  for (int r = r0 + lane; r < r1; r += 32) {
    const int t = r % T, k = r / T;
    const int64_t e = (int64_t)idx[(int64_t)t * K + k];
    if (e >= 0 && e < E) atomicAdd(&wcnt[warp * E + (int)e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {   // per-warp cursors
    int s = base[e];
    for (int w = 0; w < nw; ++w) {
      const int c = wcnt[w * E + e];
      wcnt[w * E + e] = s;
      s += c;
    }
  }
  __syncthreads();
  const unsigned lt = (1u << lane) - 1u;
  for (int rb = r0; rb < r1; rb += 32) {
    const int r = rb + lane;
    const bool in = r < r1;
    const int t = in ? r % T : 0, k = in ? r / T : 0;
    const int64_t e64 = in ? (int64_t)idx[(int64_t)t * K + k] : -1;
    const bool routed = in && e64 >= 0 && e64 < E;
    const int e = routed ? (int)e64 : 0;
    const unsigned peers = __match_any_sync(0xffffffffu, routed ? e : -1 - lane);
    const int rank = __popc(peers & lt);
    const int cur = routed ? wcnt[warp * E + e] : 0;
    __syncwarp();
    if (routed && rank == 0) wcnt[warp * E + e] = cur + __popc(peers);
    __syncwarp();
    if (routed) {
      const int row = cur + rank;
      o.perm_tok[row] = t;
      if (o.perm_slot) o.perm_slot[row] = k;
      if (o.route_row) o.route_row[t * K + k] = row;
    } else if (in && o.route_row) {
      o.route_row[t * K + k] = -1;
    }
  }
  if (blockIdx.x == 0) {   // rows past the routed ones
    __syncthreads();
    const int rows = s_rows;
    if (add_shared)
      for (int t = threadIdx.x; t < T; t += blockDim.x) o.perm_tok[rows + t] = t;
    if (o.perm_slot)
      for (int r = rows + threadIdx.x; r < R; r += blockDim.x) {
        o.perm_slot[r] = -1;
        if (!add_shared) o.perm_tok[r] = -1;
      }
  }
}

// Orderable 32-bit key of a model-dtype logit and its expert id (E <= 65535):
// larger logit first, then smaller id; -0 and +0 compare equal.
template <typename T>
TARFA_DEVI uint32_t topk_key32(float v, int e) {
  uint32_t u = Elem<T>::to_bits(v);
  if ((u & 0x7FFFu) == 0) u = 0;
  u = (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u);
  return (u << 16) | (0xFFFFu - (uint32_t)e);
}

template <typename T>
TARFA_DEVI float key32_value(uint32_t key) {
  uint32_t u = key >> 16;
  u = (u & 0x8000u) ? (u & 0x7FFFu) : (~u & 0xFFFFu);
  return Elem<T>::bits_to_f((uint16_t)u);
}

// Logit spread (max - min) up to which every probability of the token is a
// normal fp32 number, so equal and distinct logits give equal and distinct
// probabilities in the same order.
constexpr float kTieNarrowSpread = 80.f;

// One warp: softmax + top-k over E <= 32 * NPL logits of one token (values in
// the model dtype, held as fp32).  Selection is a warp max-reduction
// (redux.sync) of 32-bit keys per step; only the lane that owned the winner
// rescans its NPL keys (for the largest one below the winner: every larger key
// was taken before).  When two of the top K + 1 values are equal, the ids and
// their order are those of the reference's torch.topk (topk_ties.cuh); tie
// (tie_scratch_ints(E) shared ints of this warp) is its working space.
// pend (optional): a tie strictly inside the top K leaves the set of experts
// as it is, so the reference's order is then left to a later kernel
// (warp_tie_order): the ids come out by (value, id) and *pend is set to 1
// (else 0).  idx_smem (optional) receives the ids as well.
// SMEM_LG: lg is in this CTA's shared memory (else global, read through L2:
// other CTAs of the kernel wrote it).
template <typename T, int NPL, bool SMEM_LG = false>
TARFA_DEVI void warp_topk_n(const float* lg, int E, int K, int32_t* idx32, float* topw,
                            int64_t* idx_out, float* w_out, int32_t* idx_smem, uint32_t* tie,
                            int32_t* pend = nullptr) {
  const int lane = threadIdx.x & 31;
  uint32_t key[NPL];
  uint32_t best = 0, low = 0xffffffffu;
#pragma unroll
  for (int j = 0; j < NPL; ++j) {
    const int e = j * 32 + lane;
    key[j] = e < E ? topk_key32<T>(SMEM_LG ? lg[e] : __ldcg(lg + e), e) : 0u;
    best = max(best, key[j]);
    if (e < E) low = min(low, key[j]);
  }
  const float m = key32_value<T>(__reduce_max_sync(0xffffffffu, best));
  // Probabilities below ~2^-115 may round to equal (or zero) values for
  // different logits: then only the fp32 probabilities give the reference's ties.
  const bool wide = m - key32_value<T>(__reduce_min_sync(0xffffffffu, low)) > kTieNarrowSpread;
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NPL; ++j)
    if (j * 32 + lane < E) s += expf(key32_value<T>(key[j]) - m);
#pragma unroll
  for (int d = 16; d; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);
  TARFA_PHASE(5);
  int my_e = 0;
  float my_v = 0.f;
  uint32_t prev = 0;
  bool tied = false, boundary = false;
  const int rounds = K < E ? K + 1 : K;    // one more to see a tie at the boundary
  for (int k = 0; k < rounds; ++k) {
    const uint32_t kk = __reduce_max_sync(0xffffffffu, best);
    if (k > 0) tied |= (kk >> 16) == (prev >> 16);
    if (k == K) boundary = (kk >> 16) == (prev >> 16);
    prev = kk;
    if (k == K) break;
    const int e = (int)(0xFFFFu - (kk & 0xFFFFu));
    if (lane == k) { my_e = e; my_v = key32_value<T>(kk); }
    if ((e & 31) == lane) {
      best = 0;
#pragma unroll
      for (int j = 0; j < NPL; ++j)
        if (key[j] < kk) best = max(best, key[j]);
    }
  }
  TARFA_PHASE(6);
  const bool defer = pend && tied && !boundary && !wide;
  if (pend && lane == 0) *pend = defer ? 1 : 0;
  if ((tied || wide) && !defer) {
    // the values in sorted order are the same; which ids carry them is not
    TieElem* row = tie_row(tie);
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
      const int e = j * 32 + lane;
      if (e < E)
        row[e] = tie_elem(wide ? __float_as_uint(__fdiv_rn(expf(key32_value<T>(key[j]) - m), s))
                               : key[j] >> 16, e);
    }
    __syncwarp();
    const int id = tie_order_ids(tie, E, K);
    if (lane < K) my_e = id;
  }
  TARFA_PHASE(7);
  // softmax probabilities of the selected (fp32), renormalised over the k
  // (modeling_qwen3_5_moe.py:766-768); K <= 32
  const float p = lane < K ? __fdiv_rn(expf(my_v - m), s) : 0.f;
  float vs = 0.f;
  for (int k = 0; k < K; ++k) vs = __fadd_rn(vs, __shfl_sync(0xffffffffu, p, k));
  if (lane < K) {
    const float w = __fdiv_rn(p, vs);
    idx32[lane] = my_e;
    topw[lane] = w;
    if (idx_out) idx_out[lane] = my_e;
    if (w_out) w_out[lane] = w;
    if (idx_smem) idx_smem[lane] = my_e;
  }
}

// The 32-keys-per-lane variant is not inlined: its registers stay out of the
// callers' hot loops (the decode GEMV inlines the routing).
template <typename T>
__device__ __noinline__ void warp_topk_wide(const float* lg, int E, int K, int32_t* idx32,
                                            float* topw, int64_t* idx_out, float* w_out,
                                            int32_t* idx_smem, uint32_t* tie, int32_t* pend) {
  warp_topk_n<T, 32>(lg, E, K, idx32, topw, idx_out, w_out, idx_smem, tie, pend);
}

// tie: this warp's tie_scratch_ints(E) shared ints; pend: see warp_topk_n.
template <typename T>
TARFA_DEVI void warp_topk(const float* lg, int E, int K, int32_t* idx32, float* topw,
                          int64_t* idx_out, float* w_out, int32_t* idx_smem, uint32_t* tie,
                          int32_t* pend = nullptr) {
  if (E <= 256) warp_topk_n<T, 8>(lg, E, K, idx32, topw, idx_out, w_out, idx_smem, tie, pend);
  else warp_topk_wide<T>(lg, E, K, idx32, topw, idx_out, w_out, idx_smem, tie, pend);
}

// The reference's order of a token whose top K has a tie inside it (warp_topk_n
// deferred it): lane j < K returns the id at place j.  Same logits, same set.
template <typename T, int NPL>
TARFA_DEVI int warp_tie_order_n(const float* lg, int E, int K, uint32_t* tie) {
  const int lane = threadIdx.x & 31;
  TieElem* row = tie_row(tie);
#pragma unroll
  for (int j = 0; j < NPL; ++j) {
    const int e = j * 32 + lane;
    if (e < E) row[e] = tie_elem(topk_key32<T>(__ldcg(lg + e), e) >> 16, e);
  }
  __syncwarp();
  return tie_order_ids(tie, E, K);
}

template <typename T>
TARFA_DEVI int warp_tie_order(const float* lg, int E, int K, uint32_t* tie) {
  return E <= 256 ? warp_tie_order_n<T, 8>(lg, E, K, tie) : warp_tie_order_n<T, 32>(lg, E, K, tie);
}

// Permute for one token whose K routes name K distinct experts (the router's
// own top-k): rows in ascending expert id, one unit per route, shared unit
// last.  Same outputs as block_permute for that case.  One warp.
TARFA_DEVI void warp_permute_one_token(const int32_t* idx, int K, int E, bool add_shared,
                                       const PermuteOut& o) {
  const int lane = threadIdx.x & 31;
  const int e = lane < K ? idx[lane] : 0x7fffffff;
  int rank = 0;
  for (int j = 0; j < K; ++j) rank += __shfl_sync(0xffffffffu, e, j) < e;
  UnitDesc* descs = reinterpret_cast<UnitDesc*>(o.units + 4);
  if (lane < K) {
    descs[rank] = UnitDesc{e, rank, 1, 0};
    o.perm_tok[rank] = 0;
    if (o.perm_slot) o.perm_slot[rank] = lane;
    if (o.route_row) o.route_row[lane] = rank;
    if (o.idx32) o.idx32[lane] = e;
  }
  if (lane == 0) {
    o.units[0] = K;
    o.units[1] = K;
    o.units[2] = add_shared ? 1 : 0;
    o.units[3] = K;
    if (add_shared) {
      descs[K] = UnitDesc{E, K, 1, 0};
      o.perm_tok[K] = 0;
    }
  }
}

}  // namespace tarfa
