// Top-k tie order of the reference's router, on one warp.
//
// The reference selects experts with torch.topk(softmax_fp32(logits), k)
// (transformers modeling_qwen3_5_moe.py:767, in the block that
// tarfa/engine/channel.py:19-30 builds), run on the CPU.  Its comparator looks at
// values only (aten/src/ATen/native/TopKImpl.h, topk_impl_loop).  So when
// probabilities tie, the returned ids and their order come from the C++
// standard-library algorithms it calls, in libstdc++ (GCC 13.3, the compiler of
// torch 2.11.0):
//   * k * 64 <= n: partial_sort (heap select of k, then heap sort);
//   * else: nth_element(k - 1) (introselect: median-of-three pivot swapped
//     into the front, unguarded Hoare partition, heap select after
//     2*floor(log2 n) partitions, insertion sort of <= 3), then sort of the
//     first k - 1 (an insertion sort, which is stable, for k <= 17).
// The values compared here are the model-dtype logits while every probability
// of the token is a normal fp32 number (logit spread up to 80): equal logits then
// give equal probabilities and distinct ones distinct, in the same order.  For a
// wider spread the values are the fp32 probabilities themselves,
// expf(x - max) / sum: tiny ones can round to the same value, or to zero, for
// different logits, and those ties are the reference's too.  CUDA's expf and the
// CPU's can differ by an ulp, which matters only if it moves such a collision.
//
// The warp only takes this path for a token whose top k + 1 logits are not all
// distinct, or whose spread is wide; otherwise the top k by value are the answer.  The Hoare partition runs
// on the whole warp.  Its left scan stops at positions holding a value <= pivot
// (L_1 < L_2 < ...), its right scan at values >= pivot (R_1 > R_2 > ...), and the
// pair (L_m, R_m) is swapped while L_m < R_m.  That is a prefix m <= s, where
// s = #{m : more than m - 1 right stops lie beyond L_m}, and the partition
// point is min(L_{s+1}, R_s) (L_1 when s = 0).  Ballots and population counts
// give every stop's rank, so a partition is one pass over the keys plus one
// over the pairs instead of a serial scan.  The heap steps and the short sorts run on lane 0.
#pragma once
#include "common.cuh"

namespace tarfa {

// Shared-memory ints one warp needs (a multiple of 4; the start must be 8-byte
// aligned): E packed elements, then two lists of E 16-bit positions.
__host__ __device__ inline int tie_scratch_ints(int E) {
  return (2 * E + E + 3) & ~3;
}

// Packed element: a 32-bit orderable value high (larger ranks first), the
// expert id low.
using TieElem = unsigned long long;
TARFA_DEVI uint32_t tie_val(TieElem x) { return (uint32_t)(x >> 32); }
TARFA_DEVI bool tie_before(TieElem x, TieElem y) { return tie_val(x) > tie_val(y); }
TARFA_DEVI TieElem tie_elem(uint32_t value, int id) {
  return ((TieElem)value << 32) | (uint32_t)id;
}

// ---------------------------------------------------------------------------
// one-thread steps (lane 0), on the packed keys in shared memory
// ---------------------------------------------------------------------------
TARFA_DEVI void tie_swap(TieElem* a, int p, int q) {
  const TieElem t = a[p];
  a[p] = a[q];
  a[q] = t;
}

// Median of positions x, y, z into `front`; the comparison sequence decides
// which of equal keys is taken.
TARFA_DEVI void tie_pivot_to_front(TieElem* a, int front, int x, int y, int z) {
  int pick;
  if (tie_before(a[x], a[y]))
    pick = tie_before(a[y], a[z]) ? y : (tie_before(a[x], a[z]) ? z : x);
  else if (tie_before(a[x], a[z]))
    pick = x;
  else if (tie_before(a[y], a[z]))
    pick = z;
  else
    pick = y;
  tie_swap(a, front, pick);
}

// Unguarded Hoare partition of [lo, hi) around the key at piv (< lo).
TARFA_DEVI int tie_hoare(TieElem* a, int lo, int hi, int piv) {
  const uint32_t pv = tie_val(a[piv]);
  for (;;) {
    while (tie_val(a[lo]) > pv) ++lo;
    --hi;
    while (pv > tie_val(a[hi])) --hi;
    if (lo >= hi) return lo;
    tie_swap(a, lo, hi);
    ++lo;
  }
}

TARFA_DEVI int tie_split(TieElem* a, int lo, int hi) {
  tie_pivot_to_front(a, lo, lo + 1, lo + (hi - lo) / 2, hi - 1);
  return tie_hoare(a, lo + 1, hi, lo);
}

// Shift item left from p past every key it ranks before (something stops it).
TARFA_DEVI void tie_walk_left(TieElem* a, int p, TieElem item) {
  while (tie_before(item, a[p - 1])) {
    a[p] = a[p - 1];
    --p;
  }
  a[p] = item;
}

TARFA_DEVI void tie_insertion(TieElem* a, int lo, int hi) {
  for (int p = lo + 1; p < hi; ++p) {
    const TieElem item = a[p];
    if (tie_before(item, a[lo])) {
      for (int q = p; q > lo; --q) a[q] = a[q - 1];
      a[lo] = item;
    } else {
      tie_walk_left(a, p, item);
    }
  }
}

// Heap of [base, base + n) whose top is the key every other ranks before
// (under "ranks before", i.e. the smallest value): sift `item` down from hole.
TARFA_DEVI void tie_sift(TieElem* a, int base, int hole, int n, TieElem item) {
  const int top = hole;
  int child = hole;
  while (child < (n - 1) / 2) {
    child = 2 * (child + 1);
    if (tie_before(a[base + child], a[base + child - 1])) --child;
    a[base + hole] = a[base + child];
    hole = child;
  }
  if ((n & 1) == 0 && child == (n - 2) / 2) {
    child = 2 * (child + 1);
    a[base + hole] = a[base + child - 1];
    hole = child - 1;
  }
  while (hole > top) {
    const int parent = (hole - 1) / 2;
    if (!tie_before(a[base + parent], item)) break;
    a[base + hole] = a[base + parent];
    hole = parent;
  }
  a[base + hole] = item;
}

TARFA_DEVI void tie_heapify(TieElem* a, int lo, int hi) {
  const int n = hi - lo;
  if (n < 2) return;
  for (int parent = (n - 2) / 2; parent >= 0; --parent) tie_sift(a, lo, parent, n, a[lo + parent]);
}

TARFA_DEVI void tie_pop_into(TieElem* a, int lo, int hi, int dst) {
  const TieElem item = a[dst];
  a[dst] = a[lo];
  tie_sift(a, lo, 0, hi - lo, item);
}

TARFA_DEVI void tie_heap_sort(TieElem* a, int lo, int hi) {
  while (hi - lo > 1) {
    --hi;
    tie_pop_into(a, lo, hi, hi);
  }
}

// Introsort of [lo, hi) for the short sorted prefix (k - 1 > 16 only).  The
// ranges it splits are disjoint, so the order they are visited in does not
// change the result: a small stack replaces the recursion.
TARFA_DEVI void tie_sort(TieElem* a, int lo, int hi) {
  if (hi - lo < 2) return;
  int sl[16], sh[16], sb[16];
  int sp = 1;
  sl[0] = lo;
  sh[0] = hi;
  sb[0] = 2 * (31 - __clz(hi - lo));
  while (sp > 0) {
    --sp;
    int l = sl[sp], h = sh[sp], b = sb[sp];
    while (h - l > 16) {
      if (b == 0) {
        tie_heapify(a, l, h);
        tie_heap_sort(a, l, h);
        break;
      }
      --b;
      const int cut = tie_split(a, l, h);
      if (sp < 16) {
        sl[sp] = cut;
        sh[sp] = h;
        sb[sp] = b;
        ++sp;
      }
      h = cut;
    }
  }
  if (hi - lo > 16) {
    tie_insertion(a, lo, lo + 16);
    for (int p = lo + 16; p < hi; ++p) tie_walk_left(a, p, a[p]);
  } else {
    tie_insertion(a, lo, hi);
  }
}

// ---------------------------------------------------------------------------
// warp steps
// ---------------------------------------------------------------------------
// Heap select of [lo, mid) over [lo, hi).  Lane 0 builds the heap; the warp then
// scans 32 keys at a time against the current top.  The top only rises, so a key
// that does not beat the top a chunk starts with never enters; lane 0 inserts the
// others in order, re-checking each against the top of the moment.
TARFA_DEVI void tie_heap_select(TieElem* a, int lo, int mid, int hi) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) tie_heapify(a, lo, mid);
  __syncwarp();
  for (int c = mid; c < hi; c += 32) {
    const TieElem top = a[lo];
    const int p = c + lane;
    const unsigned cand = __ballot_sync(0xffffffffu, p < hi && tie_before(a[p], top));
    if (cand) {
      if (lane == 0) {
        unsigned m = cand;
        while (m) {
          const int q = c + __ffs(m) - 1;
          m &= m - 1;
          if (tie_before(a[q], a[lo])) tie_pop_into(a, lo, mid, q);
        }
      }
    }
    __syncwarp();
  }
}

// nth_element(nth) over [0, E) on the warp.  The loops stay rolled: this runs
// once per tied token in one warp, so its time is mostly instruction fetch,
// and a compact body is fetched once and reused by every partition.
// posL / posR: E 16-bit entries each.
TARFA_DEVI void tie_introselect(TieElem* a, uint16_t* posL, uint16_t* posR, int E, int nth) {
  const int lane = threadIdx.x & 31;
  const unsigned below = (1u << lane) - 1u;
  int lo = 0, hi = E;
  int budget = 2 * (31 - __clz(E));
  while (hi - lo > 3) {
    if (budget == 0) {
      tie_heap_select(a, lo, nth + 1, hi);
      if (lane == 0) tie_swap(a, lo, nth);
      __syncwarp();
      return;
    }
    --budget;
    if (lane == 0) tie_pivot_to_front(a, lo, lo + 1, lo + (hi - lo) / 2, hi - 1);
    __syncwarp();
    const uint32_t pv = tie_val(a[lo]);
    // left stops (value <= pivot) in ascending order into posL; right stops
    // (value >= pivot) also in ascending order, into posR: R_m = posR[nr - m]
    int nl = 0, nr = 0;
#pragma unroll 1
    for (int p0 = lo + 1; p0 < hi; p0 += 32) {
      const int p = p0 + lane;
      const uint32_t v = p < hi ? tie_val(a[p]) : 0u;
      const bool l = p < hi && v <= pv, r = p < hi && v >= pv;
      const unsigned bl = __ballot_sync(0xffffffffu, l), br = __ballot_sync(0xffffffffu, r);
      if (l) posL[nl + __popc(bl & below)] = (uint16_t)p;
      if (r) posR[nr + __popc(br & below)] = (uint16_t)p;
      nl += __popc(bl);
      nr += __popc(br);
    }
    __syncwarp();
    // s: the pairs (L_m, R_m) with L_m < R_m, a prefix of m
    int s = 0;
    const int np = min(nl, nr);
#pragma unroll 1
    for (int j0 = 0; j0 < np; j0 += 32) {
      const int j = j0 + lane;
      const unsigned ok = __ballot_sync(0xffffffffu, j < np && posL[j] < posR[nr - 1 - j]);
      s += __popc(ok);
      if (ok != 0xffffffffu) break;
    }
    int cut;
    if (s == 0) {
      cut = nl > 0 ? (int)posL[0] : hi;   // nl > 0 always: the median guards the scan
    } else {
      cut = posR[nr - s];
      if (nl > s) cut = min(cut, (int)posL[s]);
    }
#pragma unroll 1
    for (int j = lane; j < s; j += 32) tie_swap(a, posL[j], posR[nr - 1 - j]);
    __syncwarp();
    if (cut <= nth) lo = cut;
    else hi = cut;
  }
  if (lane == 0) tie_insertion(a, lo, hi);
  __syncwarp();
}

// The k ids torch.topk returns on the CPU for this row, in its order; lane j < K
// gets id j.  On entry element e of the row (e < E) is at tie_row(scratch)[e]
// (the caller writes it with tie_elem, then __syncwarp); scratch holds
// tie_scratch_ints(E) ints of this warp.  Out of line: only tokens with a tie
// call it, and its registers stay out of the callers' hot loops.
TARFA_DEVI TieElem* tie_row(uint32_t* scratch) { return reinterpret_cast<TieElem*>(scratch); }

static __device__ __noinline__ int tie_order_ids(uint32_t* scratch, int E, int K) {
  const int lane = threadIdx.x & 31;
  TieElem* a = tie_row(scratch);
  uint16_t* posL = reinterpret_cast<uint16_t*>(a + E);
  uint16_t* posR = posL + E;
  int id = 0;
  if (K * 64 <= E) {               // partial_sort
    tie_heap_select(a, 0, K, E);
    if (lane == 0) tie_heap_sort(a, 0, K);
    __syncwarp();
    if (lane < K) id = (int)(a[lane] & 0xFFFFu);
  } else {                         // nth_element, then sort of the first K - 1
    tie_introselect(a, posL, posR, E, K - 1);
    if (K - 1 <= 16) {
      // stable sort by value, descending: the insertion sort's result
      const TieElem mine = lane < K - 1 ? a[lane] : 0ull;
      int rank = 0;
      for (int j = 0; j < K - 1; ++j) {
        const TieElem o = a[j];
        rank += tie_before(o, mine) || (tie_val(o) == tie_val(mine) && j < lane);
      }
      __syncwarp();
      if (lane < K - 1) posL[rank] = (uint16_t)(mine & 0xFFFFu);
      __syncwarp();
      if (lane < K - 1) id = posL[lane];
      else if (lane == K - 1) id = (int)(a[K - 1] & 0xFFFFu);
    } else {
      if (lane == 0) tie_sort(a, 0, K - 1);
      __syncwarp();
      if (lane < K) id = (int)(a[lane] & 0xFFFFu);
    }
  }
  __syncwarp();
  return id;
}

}  // namespace tarfa
