// Expert parallelism over NVLink peer memory: one process per GPU, the
// dispatch and the return of the routed tokens as stores into the peers' HBM
// from inside this library's kernels (no collective library on the data path).
//
// Every rank owns one "box" in its own HBM, mapped into its peers' address
// spaces with CUDA IPC.  Experts are sharded in contiguous id ranges: rank o
// owns [o*E/N, (o+1)*E/N).  Slot j = t*K + k of a source block is route k of
// token t; S = max_tokens*K slots per block.  One decode step on rank r:
//   router   logits (router_logits_kernel, the single-GPU router's arithmetic)
//   exchange top-k per token (the router's warp_topk), token rows and local
//            expert ids stored into the owners' inboxes (x[r][j], meta[r][j];
//            -1 in every other owner's block), then flags_in[r] = step + 1 in
//            every box; the last block waits until every rank's flag has
//            arrived here and sorts the N*S inbox rows by local expert
//            (block_permute) into the unit table of the expert GEMVs
//   experts  gate_up (shared-expert tiles on this rank's own tokens first,
//            they need no exchange) and down over the inbox rows (gemv.cuh)
//   return   every routed row's fp32 output stored back into its source's box
//            (back[r][j]), then flags_back[r] = step + 1 in every box
//   combine  waits for every owner's flag, then the routing-weighted sum in the
//            reference's order plus the gated shared expert; the last block
//            advances this rank's step counter.
// A rank gets at most one step ahead of a peer (its next exchange needs every
// owner's return of this step), so the flags are sequence numbers that never
// need resetting, and a CUDA graph can replay the step.  Peer memory is only
// written, with plain 16-byte stores and release stores of the flags; every
// wait is bounded (about 2 s at full clock) and raises kStatusWaitTimeout.
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

// Box layout (bytes): header (step, flags) | x [N*S][H] model dtype |
// meta [N*S] int32 | back [N*S][H] fp32.
struct Box {
  size_t step, flags_in, flags_back, x, meta, back, total;
};

__host__ __device__ inline size_t al256(size_t v) { return (v + 255) & ~size_t(255); }

__host__ __device__ inline Box box_layout(int N, int S, int H, int esz) {
  Box b;
  b.step = 0;
  b.flags_in = 256;
  b.flags_back = 512;
  b.x = 1024;
  b.meta = b.x + al256((size_t)N * S * H * esz);
  b.back = b.meta + al256((size_t)N * S * 4);
  b.total = b.back + al256((size_t)N * S * H * 4);
  return b;
}

struct Args {
  int T, K, H, E, N, rank, S, e_per;
  int mode;                    // GemvMode of the routed experts (combine arithmetic)
  int has_shared;
  void* boxes[kMaxRanks];      // every rank's box in this process's address space
  const float* logits;         // [T, E] router logits (model-dtype values)
  const void* h;               // [T, H] this rank's tokens
  int32_t* idx32;              // [T*K] top-k ids
  float* topw;                 // [T*K] top-k weights
  int64_t* idx_out;            // optional user copies
  float* w_out;
  int32_t* local_idx;          // [N*S] inbox row -> local expert (e_per = empty slot)
  int32_t* units;              // unit table of the expert GEMVs
  int32_t* perm_tok;           // [N*S] GEMV row -> inbox row
  unsigned* counters;          // [3] last-block counters, left at zero
  const float* y;              // [N*S + T, H] expert outputs (routed rows, then shared)
  const float* gate_logit;     // [T] shared-expert gate logits (has_shared)
  void* out;                   // [T, H]
  unsigned* status;
};

TARFA_DEVI uint8_t* box_at(const Args& a, int r) { return static_cast<uint8_t*>(a.boxes[r]); }

TARFA_DEVI unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
TARFA_DEVI void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
TARFA_DEVI unsigned read_step(const Args& a, const Box& B) {
  return *reinterpret_cast<const volatile unsigned*>(box_at(a, a.rank) + B.step);
}

// One thread: wait until flags[0..N) >= want (sequence numbers, wrap-safe);
// false after kSpinCycles, with the status raised.
TARFA_DEVI bool wait_flags(const unsigned* flags, int N, unsigned want, unsigned* status) {
  const long long t0 = clock64();
  for (int i = 0; i < N; ++i) {
    while ((int)(ld_acquire_sys(flags + i) - want) < 0) {
      if (clock64() - t0 > kSpinCycles) {
        raise_status(status, kStatusWaitTimeout);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

// Every thread's stores out, then: is this the grid's last block to get here?
// (The counter is reset by that block, so the kernel leaves it at zero.)
TARFA_DEVI bool last_block(unsigned* counter, int* s_flag) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned nb = gridDim.x * gridDim.y;
    const bool last = atomicAdd(counter, 1u) == nb - 1;
    if (last) {
      *counter = 0u;
      __threadfence();
    }
    *s_flag = last;
  }
  __syncthreads();
  return *s_flag != 0;
}

// grid (T, C): block (t, c) routes token t and stores column chunk c of its
// rows; block (t, 0) also writes the token's ids and weights and its metadata.
template <typename T>
__global__ void __launch_bounds__(kExchangeThreads) exchange_kernel(const Args a) {
  extern __shared__ int ex_smem[];
  __shared__ int32_t s_idx[32];
  __shared__ float s_w[32];
  __shared__ int s_flag;
  grid_dep_launch_dependents();
  grid_dep_wait();                       // the router kernel's logits
  const Box B = box_layout(a.N, a.S, a.H, sizeof(T));
  const unsigned step = read_step(a, B);
  const int t = blockIdx.x, K = a.K;
  const int warp = threadIdx.x >> 5;
  if (warp == 0)
    warp_topk<T>(a.logits + (int64_t)t * a.E, a.E, K, s_idx, s_w, nullptr, nullptr, nullptr);
  __syncthreads();
  if (blockIdx.y == 0 && threadIdx.x < K) {
    const int j = t * K + threadIdx.x;
    a.idx32[j] = s_idx[threadIdx.x];
    a.topw[j] = s_w[threadIdx.x];
    if (a.idx_out) a.idx_out[j] = s_idx[threadIdx.x];
    if (a.w_out) a.w_out[j] = s_w[threadIdx.x];
  }
  // token rows into the owners' inboxes (16-byte stores over NVLink)
  const int V = a.H / 8;
  const int v0 = (int)((int64_t)V * blockIdx.y / gridDim.y);
  const int v1 = (int)((int64_t)V * (blockIdx.y + 1) / gridDim.y);
  const int nv = v1 - v0;
  const uint4* src = reinterpret_cast<const uint4*>(static_cast<const T*>(a.h) + (int64_t)t * a.H);
  for (int i = threadIdx.x; i < K * nv; i += blockDim.x) {
    const int k = i / nv, v = v0 + (i - k * nv);
    const int e = s_idx[k];
    if (e < 0 || e >= a.E) continue;
    uint8_t* ob = box_at(a, e / a.e_per);
    uint4* dst = reinterpret_cast<uint4*>(ob + B.x +
                                          ((int64_t)a.rank * a.S + t * K + k) * a.H * sizeof(T));
    dst[v] = __ldg(src + v);
  }
  // metadata: the local expert id in the owner's block, -1 in every other one
  if (blockIdx.y == 0) {
    for (int i = threadIdx.x; i < a.N * K; i += blockDim.x) {
      const int o = i / K, k = i - o * K;
      const int e = s_idx[k];
      const int v = (e >= 0 && e < a.E && e / a.e_per == o) ? e - o * a.e_per : -1;
      reinterpret_cast<int32_t*>(box_at(a, o) + B.meta)[a.rank * a.S + t * K + k] = v;
    }
    if (t == 0)   // slots of tokens this step does not have
      for (int i = threadIdx.x; i < a.N * (a.S - a.T * K); i += blockDim.x) {
        const int per = a.S - a.T * K;
        const int o = i / per, j = a.T * K + (i - o * per);
        reinterpret_cast<int32_t*>(box_at(a, o) + B.meta)[a.rank * a.S + j] = -1;
      }
  }
  if (!last_block(a.counters + 0, &s_flag)) return;
  // ---- last block: publish, wait for every rank, sort the inbox -----------
  if (threadIdx.x < a.N)
    st_release_sys(reinterpret_cast<unsigned*>(box_at(a, threadIdx.x) + B.flags_in) + a.rank,
                   step + 1);
  if (threadIdx.x == 0)
    s_flag = wait_flags(reinterpret_cast<const unsigned*>(box_at(a, a.rank) + B.flags_in), a.N,
                        step + 1, a.status);
  __syncthreads();
  const bool ok = s_flag != 0;
  const int32_t* meta = reinterpret_cast<const int32_t*>(box_at(a, a.rank) + B.meta);
  const int R = a.N * a.S;
  for (int i = threadIdx.x; i < R; i += blockDim.x) {
    const int v = ok ? __ldcv(meta + i) : -1;
    a.local_idx[i] = (v >= 0 && v < a.e_per) ? v : a.e_per;
  }
  __syncthreads();
  const PermuteOut o{nullptr, a.perm_tok, nullptr, nullptr, a.units, nullptr};
  block_permute<int32_t>(a.local_idx, R, 1, a.e_per, false, o, ex_smem, a.status);
  __syncthreads();
  if (threadIdx.x == 0 && a.has_shared) {   // the shared unit: own tokens at rows [R, R + T)
    const int nu = a.units[0];
    a.units[2] = 1;
    a.units[3] = R;
    reinterpret_cast<UnitDesc*>(a.units + 4)[nu] = UnitDesc{a.e_per, R, a.T, 0};
  }
}

// Routed rows' outputs back to their sources (fp32, 16-byte stores), then the
// flags.  Grid-stride over rows x float4 columns.
template <typename T>
__global__ void __launch_bounds__(kReturnThreads) return_kernel(const Args a) {
  __shared__ int s_flag;
  grid_dep_wait();                       // the down GEMV's outputs
  const Box B = box_layout(a.N, a.S, a.H, sizeof(T));
  const unsigned step = read_step(a, B);
  const int rows = a.units[1];
  const int V = a.H / 4;
  const int64_t n = (int64_t)rows * V;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / V), v = (int)(i - (int64_t)r * V);
    const int q = a.perm_tok[r];
    const int src = q / a.S, j = q - src * a.S;
    const float4 val = __ldcg(reinterpret_cast<const float4*>(a.y + (int64_t)r * a.H) + v);
    float4* dst = reinterpret_cast<float4*>(box_at(a, src) + B.back) +
                  ((int64_t)a.rank * a.S + j) * V + v;
    *dst = val;
  }
  if (!last_block(a.counters + 1, &s_flag)) return;
  if (threadIdx.x < a.N)
    st_release_sys(reinterpret_cast<unsigned*>(box_at(a, threadIdx.x) + B.flags_back) + a.rank,
                   step + 1);
}

TARFA_DEVI void ldcg8(const float* p, float (&v)[8]) {
  const float4 x = __ldcg(reinterpret_cast<const float4*>(p));
  const float4 y = __ldcg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w; v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
}

// grid (column blocks, T), one warp per block: the combine of the single-GPU
// layer (combine_token_kernel) over the returned rows, then the step counter.
template <typename T>
__global__ void __launch_bounds__(32) combine_kernel(const Args a) {
  __shared__ int s_row[32];
  __shared__ float s_w[32];
  __shared__ int s_flag;
  grid_dep_wait();
  const Box B = box_layout(a.N, a.S, a.H, sizeof(T));
  const unsigned step = read_step(a, B);
  const int t = blockIdx.y, K = a.K, lane = threadIdx.x;
  bool ok = true;
  if (lane == 0)
    ok = wait_flags(reinterpret_cast<const unsigned*>(box_at(a, a.rank) + B.flags_back), a.N,
                    step + 1, a.status);
  ok = __shfl_sync(0xffffffffu, ok, 0);
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
      const bool valid = ok && e >= 0 && e < a.E;
      s_row[rank] = valid ? (e / a.e_per) * a.S + t * K + lane : -1;
      s_w[rank] = a.topw[t * K + lane];
    }
  }
  __syncwarp();
  const float* back = reinterpret_cast<const float*>(box_at(a, a.rank) + B.back);
  const float sg = a.has_shared ? rnd<T>(sigmoid_f(a.gate_logit[t])) : 0.f;
  const float* shy = a.y + (int64_t)(a.N * a.S + t) * a.H;
  const bool router_order = a.T == 1;
  for (int c8 = blockIdx.x * 32 + lane; c8 < a.H / 8; c8 += gridDim.x * 32) {
    const int h0 = c8 * 8;
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.f;
    for (int i = 0; i < K; ++i) {
      const int r = s_row[i];
      if (r < 0) continue;
      float yv[8];
      ldcg8(back + (int64_t)r * a.H + h0, yv);
      const float wk = s_w[i];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (a.mode == kModeInt4Fused) acc[q] = __fadd_rn(acc[q], __fmul_rn(yv[q], wk));
        else if (router_order) acc[q] = rnd<T>(acc[q] + rnd<T>(rnd<T>(wk) * yv[q]));
        else acc[q] = rnd<T>(acc[q] + rnd<T>(__fmul_rn(yv[q], wk)));
      }
    }
    if (a.mode == kModeInt4Fused)
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = rnd<T>(acc[q]);
    if (a.has_shared) {
      float sv[8];
      ldcg8(shy + h0, sv);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = rnd<T>(acc[q] + rnd<T>(sg * sv[q]));
    }
    uint4 o;
    T* op = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) op[q] = Elem<T>::from_f(acc[q]);
    *reinterpret_cast<uint4*>(static_cast<T*>(a.out) + (int64_t)t * a.H + h0) = o;
  }
  // every block has read the returned rows: the last one advances the step
  if (last_block(a.counters + 2, &s_flag) && lane == 0)
    *reinterpret_cast<volatile unsigned*>(box_at(a, a.rank) + B.step) = step + 1;
}

}  // namespace ep
}  // namespace tarfa
