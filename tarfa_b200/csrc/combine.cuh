// Arguments of the combine (routing-weighted sum of the expert outputs plus
// the gated shared expert; router.cuh, combine_token_kernel).
#pragma once
#include "common.cuh"

namespace tarfa {

struct CombineArgs {
  const void* y;           // [R_total, H] expert outputs: fp32 or model dtype (YT)
  const int32_t* route_row;// [T, K]
  const int32_t* idx32;    // [T, K] expert ids (E = skipped)
  const float* w;          // [T, K]
  int T, K, H, E;
  int order_router;        // 1: T == 1 decode branch (router order); 0: ascending expert id
  int mode;                // GemvMode of the routed experts
  const float* gate_logit; // [T] or null: add the gated shared expert
  const int32_t* units;    // unit table: units[3] = first shared-expert row
  void* out;               // [T, H] model dtype
  const int32_t* pend;     // [T] or null: tokens whose tie order the router left open
  const float* logits;     // [T, E] router logits (with pend)
  int64_t* idx_out;        // optional [T, K]: rewritten in the reference's order (with pend)
};

}  // namespace tarfa
