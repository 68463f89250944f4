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
};

}  // namespace tarfa
