// Internal interface between the C ABI (capi.cu) and the tcgen05 grouped GEMM.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace tarfa {

struct PrefillArgs {
  bool bf16;
  int64_t T, H, E, E_store, I, Is;   // E_store: experts in the weight stacks (slots)
  int64_t rows_total;                 // T*K + (Is ? T : 0): rows of x_perm / act / y
  int64_t max_units;                  // bound on the number of units
  const void* hidden;                 // [T, H]
  const int32_t* perm_tok;            // [rows_total]
  const int32_t* units;               // unit table
  const int32_t* expert_slot;         // optional
  const void* gate_up;                // [E_store, 2I, H]
  const void* down;                   // [E_store, H, I]
  const void* sh_gate;                // [Is, H]
  const void* sh_up;                  // [Is, H]
  const void* sh_down;                // [H, Is]
  void* x_perm;                       // scratch [rows_total, H]
  void* act;                          // scratch [rows_total, ld_act]
  int64_t ld_act;
  void* y;                            // out [rows_total, H] model dtype
  unsigned* status;
  int sms;
};

// Router logits h . W_r^T in fp32 on the tensor cores (rounding fixed up by
// the top-k kernel).  units: 8 ints of scratch for a one-unit table.  The K
// range is split ksplit ways (1 <= ksplit <= H / 64); split s writes its fp32
// partial [T, E] at logits + s * T * E.
bool router_gemm_supported(int64_t H, int64_t E);
int router_logits_sm100(bool bf16, const void* h, int64_t T, int64_t H, const void* w_r, int64_t E,
                        int32_t* units, float* logits, int ksplit, unsigned* status, int sms,
                        cudaStream_t st, const char** err);

// True when the tcgen05 path covers this layer shape (dense experts only).
bool prefill_supported(int64_t H, int64_t I, int64_t Is, bool dense);

// gather -> gate_up GEMM (+SiLU*mul) -> down GEMM.  Returns 0 or sets *err.
int prefill_experts_sm100(const PrefillArgs& a, cudaStream_t st, const char** err);

}  // namespace tarfa
