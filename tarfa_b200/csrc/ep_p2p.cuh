// Expert parallelism over NVLink peer memory: one process per GPU, the
// dispatch and the return of the routed tokens as stores into the peers' HBM
// from inside this library's kernels (no collective library on the data path).
//
// Every rank owns one "box" in its own HBM, mapped into its peers' address
// spaces with CUDA IPC.  Experts are sharded in contiguous id ranges over
// groups of P ranks (P = 1 or 2): group g = o / P owns experts [g*E/G,
// (g+1)*E/G), G = N/P, and with P = 2 each rank of the pair holds one half of
// every such expert's intermediate dimension (rank o: half o % 2).  A route
// goes to every rank of its expert's group; with P = 2 each returns an fp32
// partial of the down projection and the source adds the two, half 0 first,
// before the rounding: the same sum the single-GPU down GEMV forms from its two
// K halves.  Slot j = t*K + k of a source block is route k of token t; S =
// max_tokens*K slots per block.
//
// Tagged words.  Everything that crosses to another GPU is written as 8-byte
// words (step + 1) << 32 | payload, 16 bytes per store: an aligned 8-byte
// element is written and read whole, so a reader that sees the step's tag in
// a word also sees that step's payload, with no fence and no separate flag.
// (The small-message protocol of NCCL rests on the same property.)  Tags are
// step numbers, so the boxes are never cleared and a CUDA graph can replay the
// step; a rank gets at most one step ahead of a peer, since its next exchange
// waits for every owner's return of this step.
//
// One decode step on rank r:
//   router   logits (router_logits_kernel, the single-GPU router's arithmetic)
//   exchange grid (T, C): top-k per token (warp_topk); the token's rows into
//            the owners' inboxes (x[r][j], two model-dtype values per word)
//            and a metadata word per slot in every owner's block (the local
//            expert id, -1 elsewhere); then every block unpacks a share of
//            this rank's inbox into plain rows of the workspace, polling the
//            tags, while block 0 reads every slot's metadata and sorts the
//            rows by local expert into the unit table of the expert GEMVs
//   experts  gate_up (shared-expert tiles on this rank's own tokens first,
//            they need no exchange) and down over the unpacked rows (gemv.cuh)
//   return   every routed row's fp32 output into its source's box (back[r][j],
//            one value per word); advances this rank's step counter
//   combine  polls the returned words, then the routing-weighted sum in the
//            reference's order plus the gated shared expert.
// Peer memory is only written, with plain stores; every wait is bounded (about
// 2 s at full clock) and raises kStatusWaitTimeout instead of hanging.
#pragma once
#include "common.cuh"
#include "router.cuh"
#include "routing.cuh"

namespace tarfa {
namespace ep {

constexpr int kMaxRanks = 8;                       // TARFA_EP_MAX_RANKS
constexpr long long kSpinCycles = 4000000000ll;    // bounded waits
constexpr int kExchangeThreads = 256;
constexpr int kReturnThreads = 256;

// Box layout (bytes): step counter | x [N*S][H/2] words | meta [N*S] words |
// back [N*S][H] words.
struct Box {
  size_t step, x, meta, back, total;
};

__host__ __device__ inline size_t al256(size_t v) { return (v + 255) & ~size_t(255); }

__host__ __device__ inline Box box_layout(int N, int S, int H) {
  Box b;
  b.step = 0;
  b.x = 256;
  b.meta = b.x + al256((size_t)N * S * (H / 2) * 8);
  b.back = b.meta + al256((size_t)N * S * 8);
  b.total = b.back + al256((size_t)N * S * H * 8);
  return b;
}

struct Args {
  int T, K, H, E, N, rank, S, e_per;   // e_per: experts per group of P ranks
  int tp;                      // P: ranks sharing each expert (1 or 2)
  int mode;                    // GemvMode of the routed experts (combine arithmetic)
  int has_shared;
  void* boxes[kMaxRanks];      // every rank's box in this process's address space
  const float* logits;         // [T, E] router logits (model-dtype values)
  const void* h;               // [T, H] this rank's tokens
  int32_t* idx32;              // [T*K] top-k ids
  float* topw;                 // [T*K] top-k weights
  int64_t* idx_out;            // optional user copies
  float* w_out;
  void* xin;                   // [N*S, H] unpacked inbox rows (model dtype)
  int32_t* local_idx;          // [N*S] inbox row -> local expert (e_per = empty slot)
  int32_t* units;              // unit table of the expert GEMVs
  int32_t* perm_tok;           // [N*S] GEMV row -> inbox row
  unsigned* cur_step;          // the step in flight (written by the exchange)
  const float* y;              // [N*S + T, H] expert outputs (routed rows, then shared)
  const float* gate_logit;     // [T] shared-expert gate logits (has_shared)
  void* out;                   // [T, H]
  unsigned* status;
  unsigned* fx_cnt;            // tensor-core router's fix-up list length: cleared here, or null
};

TARFA_DEVI uint8_t* box_at(const Args& a, int r) { return static_cast<uint8_t*>(a.boxes[r]); }

TARFA_DEVI unsigned read_step(const Args& a, const Box& B) {
  return *reinterpret_cast<const volatile unsigned*>(box_at(a, a.rank) + B.step);
}

// Two tagged words, stored and loaded 16 bytes at a time (two 8-byte elements).
TARFA_DEVI void st_words(unsigned long long* p, unsigned long long w0, unsigned long long w1) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(w0), "l"(w1) : "memory");
}
TARFA_DEVI void st_word(unsigned long long* p, unsigned long long w) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
TARFA_DEVI void ld_words(const unsigned long long* p, unsigned long long& w0, unsigned long long& w1) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p) : "memory");
}
TARFA_DEVI unsigned long long ld_word(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
TARFA_DEVI bool tagged(unsigned long long w, unsigned tag) { return (unsigned)(w >> 32) == tag; }

// Bounded poll of two words until both carry `tag`; false (status raised)
// once the thread's deadline has passed.
TARFA_DEVI bool poll_words(const unsigned long long* p, unsigned tag, unsigned long long& w0,
                           unsigned long long& w1, long long t0, unsigned* status) {
  while (!(tagged(w0, tag) && tagged(w1, tag))) {
    if (clock64() - t0 > kSpinCycles) {
      raise_status(status, kStatusWaitTimeout);
      return false;
    }
    ld_words(p, w0, w1);
  }
  return true;
}

// Sort of the R <= blockDim inbox rows by local expert (ties by row: the order
// block_permute gives) into the unit table, without the per-expert counters:
// each row's rank is the number of rows that sort before it.
TARFA_DEVI void rank_permute(const int32_t* local_idx, int R, int E, int* smem, int32_t* units,
                             int32_t* perm_tok) {
  int* s_v = smem;               // [R] local expert per row
  int* s_sv = smem + R;          // [R] sorted experts
  int* s_row0 = smem + 2 * R;    // [R] unit -> first sorted row
  int* s_wsum = smem + 3 * R;    // [32] per-warp unit starts
  const int i = threadIdx.x, lane = i & 31, warp = i >> 5, nw = (blockDim.x + 31) >> 5;
  int v = E;
  if (i < R) v = s_v[i] = local_idx[i];
  __syncthreads();
  if (i < R) {
    int r = 0;
    for (int j = 0; j < R; ++j) {
      const int vj = s_v[j];
      r += vj < v || (vj == v && j < i);
    }
    s_sv[r] = v;
    perm_tok[r] = i;
  }
  __syncthreads();
  // unit starts: first sorted row of each routed expert; inclusive scan of them
  const int sv = i < R ? s_sv[i] : E;
  const int start = sv < E && (i == 0 || s_sv[i - 1] != sv);
  int incl = start;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int x = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += x;
  }
  if (lane == 31) s_wsum[warp] = incl;
  __syncthreads();
  for (int w = 0; w < warp; ++w) incl += s_wsum[w];
  const int u = incl - 1;
  UnitDesc* descs = reinterpret_cast<UnitDesc*>(units + 4);
  if (start) s_row0[u] = i;
  __syncthreads();
  const bool end = sv < E && (i == R - 1 || s_sv[i + 1] != sv);
  if (end) descs[u] = UnitDesc{sv, s_row0[u], i + 1 - s_row0[u], 0};
  if (i == 0) {
    int nu = 0, rows = 0;
    for (int w = 0; w < nw; ++w) nu += s_wsum[w];
    for (int j = 0; j < R; ++j) rows += s_sv[j] < E;
    units[0] = nu;
    units[1] = rows;
    units[2] = 0;
    units[3] = rows;
  }
}

// Shared-memory ints rank_permute needs.
__host__ __device__ inline int rank_permute_smem_ints(int R) { return 3 * R + 32; }

// Column chunks of one inbox row in the unpack (items = rows x chunks).
__host__ __device__ inline int unpack_chunks(int R, int nblocks, int H) {
  int c = (2 * nblocks + R - 1) / R;
  const int cmax = H / 4 / 64 > 0 ? H / 4 / 64 : 1;   // at least 64 16-byte loads per chunk
  return c < 1 ? 1 : (c > cmax ? cmax : c);
}

// grid (T, C): block (t, c) routes token t and stores column chunk c of its
// rows; block (t, 0) also writes the token's ids, weights and metadata.  Then
// block 0 sorts this rank's inbox and the others unpack it.
template <typename T>
__global__ void __launch_bounds__(kExchangeThreads) exchange_kernel(const Args a) {
  extern __shared__ int ex_smem[];
  __shared__ int32_t s_idx[32];
  __shared__ float s_w[32];
  grid_dep_wait();                       // the router kernel's logits
  // the tensor-core router's fix-up has read its list: leave its counter at zero
  if (a.fx_cnt && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *a.fx_cnt = 0u;
  const Box B = box_layout(a.N, a.S, a.H);
  const unsigned step = read_step(a, B);
  const unsigned tag = step + 1;
  const unsigned long long hi = (unsigned long long)tag << 32;
  const int t = blockIdx.x, K = a.K;
  if ((threadIdx.x >> 5) == 0)   // ex_smem is the tie scratch here, reused after the barrier
    warp_topk<T>(a.logits + (int64_t)t * a.E, a.E, K, s_idx, s_w, nullptr, nullptr, nullptr,
                 reinterpret_cast<uint32_t*>(ex_smem));
  __syncthreads();
  if (blockIdx.y == 0 && threadIdx.x < K) {
    const int j = t * K + threadIdx.x;
    a.idx32[j] = s_idx[threadIdx.x];
    a.topw[j] = s_w[threadIdx.x];
    if (a.idx_out) a.idx_out[j] = s_idx[threadIdx.x];
    if (a.w_out) a.w_out[j] = s_w[threadIdx.x];
  }
  // ---- send: token rows into the owners' inboxes, 4 values per 16-byte store
  const int W = a.H / 4;                 // 16-byte stores per row
  const int w0 = (int)((int64_t)W * blockIdx.y / gridDim.y);
  const int w1 = (int)((int64_t)W * (blockIdx.y + 1) / gridDim.y);
  const int nw = w1 - w0;
  const uint2* src = reinterpret_cast<const uint2*>(static_cast<const T*>(a.h) + (int64_t)t * a.H);
  for (int i = threadIdx.x; i < K * nw; i += blockDim.x) {
    const int k = i / nw, w = w0 + (i - k * nw);
    const int e = s_idx[k];
    if (e < 0 || e >= a.E) continue;
    const uint2 v = __ldg(src + w);
    for (int p = 0; p < a.tp; ++p) {   // every rank of the expert's group
      unsigned long long* dst =
          reinterpret_cast<unsigned long long*>(box_at(a, (e / a.e_per) * a.tp + p) + B.x) +
          ((int64_t)a.rank * a.S + t * K + k) * (a.H / 2) + 2 * w;
      st_words(dst, hi | v.x, hi | v.y);
    }
  }
  if (blockIdx.y == 0) {   // metadata: the local id in the owner's block, -1 in the others
    for (int i = threadIdx.x; i < a.N * K; i += blockDim.x) {
      const int o = i / K, k = i - o * K;
      const int e = s_idx[k];
      const int g = o / a.tp;
      const int v = (e >= 0 && e < a.E && e / a.e_per == g) ? e - g * a.e_per : -1;
      st_word(reinterpret_cast<unsigned long long*>(box_at(a, o) + B.meta) + a.rank * a.S + t * K + k,
              hi | (unsigned)v);
    }
    if (t == 0) {   // slots of tokens this step does not have
      const int per = a.S - a.T * K;
      for (int i = threadIdx.x; i < a.N * per; i += blockDim.x) {
        const int o = i / per, j = a.T * K + (i - o * per);
        st_word(reinterpret_cast<unsigned long long*>(box_at(a, o) + B.meta) + a.rank * a.S + j,
                hi | 0xFFFFFFFFu);
      }
    }
  }
  // Every block of this kernel is resident by now: the GEMV may be scheduled
  // (its shared-expert tiles run while the inbox fills).
  grid_dep_launch_dependents();
  // ---- receive -------------------------------------------------------------
  const int R = a.N * a.S;
  const int nb = gridDim.x * gridDim.y, b = blockIdx.y * gridDim.x + blockIdx.x;
  const unsigned long long* xw = reinterpret_cast<const unsigned long long*>(box_at(a, a.rank) + B.x);
  const unsigned long long* mw = reinterpret_cast<const unsigned long long*>(box_at(a, a.rank) + B.meta);
  const long long t0 = clock64();
  if (b == 0) {
    // block 0 sorts: every slot's metadata word, then the unit table
    for (int i = threadIdx.x; i < R; i += blockDim.x) {
      unsigned long long m = ld_word(mw + i);
      bool ok = true;
      while (!tagged(m, tag)) {
        if (clock64() - t0 > kSpinCycles) {
          raise_status(a.status, kStatusWaitTimeout);
          ok = false;
          break;
        }
        m = ld_word(mw + i);
      }
      const int id = ok ? (int)(unsigned)m : -1;
      a.local_idx[i] = (id >= 0 && id < a.e_per) ? id : a.e_per;
    }
    __syncthreads();
    if (R <= (int)blockDim.x) {
      rank_permute(a.local_idx, R, a.e_per, ex_smem, a.units, a.perm_tok);
    } else {
      const PermuteOut o{nullptr, a.perm_tok, nullptr, nullptr, a.units, nullptr};
      block_permute<int32_t>(a.local_idx, R, 1, a.e_per, false, o, ex_smem, a.status);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      if (a.has_shared) {   // the shared unit: own tokens at rows [R, R + T)
        const int nu = a.units[0];
        a.units[2] = 1;
        a.units[3] = R;
        reinterpret_cast<UnitDesc*>(a.units + 4)[nu] = UnitDesc{a.e_per, R, a.T, 0};
      }
      *a.cur_step = step;   // for the return (which advances the counter) and the combine
    }
    if (nb > 1) return;
    __syncthreads();
  }
  // the other blocks (block 0 too when it is alone) unpack the routed rows:
  // items = slots x column chunks, in rounds of up to blockDim items; every
  // thread polls one item's metadata, then the block unpacks the round's rows
  const int ub = nb > 1 ? b - 1 : 0, unb = nb > 1 ? nb - 1 : 1;
  const int CH = unpack_chunks(R, unb, a.H);
  const int n_items = R * CH;
  const int cwmax = (W + CH - 1) / CH;   // widest column chunk
  for (int base = ub; base < n_items; base += unb * (int)blockDim.x) {
    const int cnt = min((int)blockDim.x, (n_items - base + unb - 1) / unb);
    if ((int)threadIdx.x < cnt) {
      const int slot = (base + threadIdx.x * unb) / CH;
      unsigned long long m = ld_word(mw + slot);
      bool ok = true;
      while (!tagged(m, tag)) {
        if (clock64() - t0 > kSpinCycles) {
          raise_status(a.status, kStatusWaitTimeout);
          ok = false;
          break;
        }
        m = ld_word(mw + slot);
      }
      const int id = ok ? (int)(unsigned)m : -1;
      ex_smem[threadIdx.x] = id >= 0 && id < a.e_per;
    }
    __syncthreads();
    for (int x = threadIdx.x; x < cnt * cwmax; x += blockDim.x) {
      const int li = x / cwmax, dw = x - li * cwmax;
      if (!ex_smem[li]) continue;
      const int item = base + li * unb;
      const int slot = item / CH, c = item - slot * CH;
      const int w = (int)((int64_t)W * c / CH) + dw;
      if (w >= (int)((int64_t)W * (c + 1) / CH)) continue;
      const unsigned long long* p = xw + (int64_t)slot * (a.H / 2) + 2 * w;
      unsigned long long v0, v1;
      ld_words(p, v0, v1);
      poll_words(p, tag, v0, v1, t0, a.status);
      reinterpret_cast<uint2*>(static_cast<T*>(a.xin) + (int64_t)slot * a.H)[w] =
          make_uint2((unsigned)v0, (unsigned)v1);
    }
    __syncthreads();   // ex_smem is reused
  }
}

// Routed rows' fp32 outputs back to their sources, one value per tagged word.
// Grid-stride over rows x groups of 4 columns.
template <typename T>
__global__ void __launch_bounds__(kReturnThreads) return_kernel(const Args a) {
  grid_dep_wait();                       // the down GEMV's outputs
  const Box B = box_layout(a.N, a.S, a.H);
  const unsigned step = *a.cur_step;
  const unsigned long long hi = (unsigned long long)(step + 1) << 32;
  // every exchange block has read the step by now (the exchange has completed)
  if (blockIdx.x == 0 && threadIdx.x == 0)
    *reinterpret_cast<volatile unsigned*>(box_at(a, a.rank) + B.step) = step + 1;
  const int rows = a.units[1];
  const int V = a.H / 4;
  const int64_t n = (int64_t)rows * V;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / V), v = (int)(i - (int64_t)r * V);
    const int q = a.perm_tok[r];
    const int src = q / a.S, j = q - src * a.S;
    const float4 f = __ldcg(reinterpret_cast<const float4*>(a.y + (int64_t)r * a.H) + v);
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(box_at(a, src) + B.back) +
                              ((int64_t)a.rank * a.S + j) * a.H + 4 * v;
    st_words(dst, hi | __float_as_uint(f.x), hi | __float_as_uint(f.y));
    st_words(dst + 2, hi | __float_as_uint(f.z), hi | __float_as_uint(f.w));
  }
}

TARFA_DEVI void ldcg8(const float* p, float (&v)[8]) {
  const float4 x = __ldcg(reinterpret_cast<const float4*>(p));
  const float4 y = __ldcg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w; v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
}

// grid (column blocks, T), one warp per block: the combine of the single-GPU
// layer (combine_token_kernel) over the returned words.  P = 2: a route's
// output is the sum of its two halves' fp32 partials (half 0 first), rounded
// as the single-GPU down GEMV rounds it.
template <typename T, int P>
__global__ void __launch_bounds__(32) combine_kernel(const Args a) {
  __shared__ int s_row[32];
  __shared__ float s_w[32];
  grid_dep_wait();
  const Box B = box_layout(a.N, a.S, a.H);
  const unsigned tag = *a.cur_step + 1;
  const int t = blockIdx.y, K = a.K, lane = threadIdx.x;
  {
    const int e = lane < K ? a.idx32[t * K + lane] : 0x7fffffff;
    int rank = lane;
    if (a.T > 1) {   // ascending expert id (fused_int4.py:241-244); T == 1: router order (:194)
      rank = 0;
      for (int j = 0; j < K; ++j) {
        const int ej = __shfl_sync(0xffffffffu, e, j);
        rank += ej < e || (ej == e && j < lane);
      }
    }
    if (lane < K) {
      const bool valid = e >= 0 && e < a.E;
      s_row[rank] = valid ? (e / a.e_per) * P * a.S + t * K + lane : -1;   // half 0's row
      s_w[rank] = a.topw[t * K + lane];
    }
  }
  __syncwarp();
  const unsigned long long* back =
      reinterpret_cast<const unsigned long long*>(box_at(a, a.rank) + B.back);
  const float sg = a.has_shared ? rnd<T>(sigmoid_f(a.gate_logit[t])) : 0.f;
  const float* shy = a.y + (int64_t)(a.N * a.S + t) * a.H;
  const bool router_order = a.T == 1;
  const long long t0 = clock64();
  for (int c8 = blockIdx.x * 32 + lane; c8 < a.H / 8; c8 += gridDim.x * 32) {
    const int h0 = c8 * 8;
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.f;
    float sv[8];
    if (a.has_shared) ldcg8(shy + h0, sv);   // issued with the routed rows' loads
    constexpr int NB = 8 / P;                // routes' words in flight at a time
    for (int i0 = 0; i0 < K; i0 += NB) {
      unsigned long long wv[NB][P][8];
#pragma unroll
      for (int i = 0; i < NB; ++i) {
        const int r = i0 + i < K ? s_row[i0 + i] : -1;
        if (r >= 0) {
#pragma unroll
          for (int p2 = 0; p2 < P; ++p2) {
            const unsigned long long* p = back + (int64_t)(r + p2 * a.S) * a.H + h0;
#pragma unroll
            for (int q = 0; q < 4; ++q) ld_words(p + 2 * q, wv[i][p2][2 * q], wv[i][p2][2 * q + 1]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < NB; ++i) {
        if (i0 + i >= K) break;
        const int r = s_row[i0 + i];
        if (r < 0) continue;
#pragma unroll
        for (int p2 = 0; p2 < P; ++p2) {
          const unsigned long long* p = back + (int64_t)(r + p2 * a.S) * a.H + h0;
#pragma unroll
          for (int q = 0; q < 4; ++q)
            poll_words(p + 2 * q, tag, wv[i][p2][2 * q], wv[i][p2][2 * q + 1], t0, a.status);
        }
        const float wk = s_w[i0 + i];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float yv = __uint_as_float((unsigned)wv[i][0][q]);
          if (P == 2) {
            yv = __fadd_rn(yv, __uint_as_float((unsigned)wv[i][P - 1][q]));
            if (a.mode != kModeInt4Fused) yv = rnd<T>(yv);
          }
          if (a.mode == kModeInt4Fused) acc[q] = __fadd_rn(acc[q], __fmul_rn(yv, wk));
          else if (router_order) acc[q] = rnd<T>(acc[q] + rnd<T>(rnd<T>(wk) * yv));
          else acc[q] = rnd<T>(acc[q] + rnd<T>(__fmul_rn(yv, wk)));
        }
      }
    }
    if (a.mode == kModeInt4Fused)
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = rnd<T>(acc[q]);
    if (a.has_shared) {
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = rnd<T>(acc[q] + rnd<T>(sg * sv[q]));
    }
    uint4 o;
    T* op = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) op[q] = Elem<T>::from_f(acc[q]);
    *reinterpret_cast<uint4*>(static_cast<T*>(a.out) + (int64_t)t * a.H + h0) = o;
  }
}

}  // namespace ep
}  // namespace tarfa
