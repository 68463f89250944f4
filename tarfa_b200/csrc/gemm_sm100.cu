// Host side of the tcgen05 grouped GEMM: tensor maps, launch configuration.
// The kernels are in gemm_sm100.cuh; capi.cu calls prefill_experts_sm100().
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "gemm_sm100.cuh"
#include "gemm_sm100.h"

namespace tarfa {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D K-major operand [rows, cols] (cols contiguous), box 64 x box_rows, 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
              bool bf16) {
  EncodeTiledFn fn = encoder();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
            const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, int PHASE>
int launch_phase(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& s0,
                 const CUtensorMap& s1, const sm100::Params& p, int grid, cudaStream_t st,
                 const char** err) {
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(sm100::grouped_gemm_kernel<T, PHASE>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sm100::kSmemBytes) != cudaSuccess) {
      *err = "cudaFuncSetAttribute(grouped_gemm_kernel) failed";
      return 1;
    }
    attr[dev] = true;
  }
  sm100::grouped_gemm_kernel<T, PHASE><<<grid, sm100::kThreads, sm100::kSmemBytes, st>>>(a, b, s0, s1, p);
  if (cudaGetLastError() != cudaSuccess) {
    *err = "grouped_gemm_kernel launch failed";
    return 1;
  }
  return 0;
}

template <typename T>
int run(const PrefillArgs& a, cudaStream_t st, const char** err) {
  const bool bf16 = sizeof(T) == 2 && std::is_same<T, __nv_bfloat16>::value;
  const int64_t Rt = a.rows_total;
  // gather routed + shared rows of the tokens into the permuted order
  {
    const int threads = 256;
    const int grid = a.sms * 4;
    sm100::gather_rows_kernel<T><<<grid, threads, 0, st>>>(
        static_cast<const T*>(a.hidden), a.perm_tok, a.units, (int)a.T, (int)a.H, static_cast<T*>(a.x_perm));
    if (cudaGetLastError() != cudaSuccess) { *err = "gather launch failed"; return 1; }
  }
  CUtensorMap mA, mB, mS0, mS1;
  sm100::Params p{};
  p.E = (int)a.E;
  p.units = a.units;
  p.expert_slot = a.expert_slot;
  p.status = a.status;
  p.idesc = sm100::make_idesc(bf16);
  const int Is = (int)a.Is;
  // ---- phase 0: gate_up + SiLU*mul -> act ------------------------------------
  if (!make_map(&mA, a.x_perm, (uint64_t)Rt, (uint64_t)a.H, 128, bf16) ||
      !make_map(&mB, a.gate_up, (uint64_t)a.E_store * 2 * a.I, (uint64_t)a.H, 128, bf16)) {
    *err = "cuTensorMapEncodeTiled failed (phase 0)";
    return 1;
  }
  mS0 = mB;
  mS1 = mB;
  if (Is) {
    if (!make_map(&mS0, a.sh_gate, (uint64_t)Is, (uint64_t)a.H, 128, bf16) ||
        !make_map(&mS1, a.sh_up, (uint64_t)Is, (uint64_t)a.H, 128, bf16)) {
      *err = "cuTensorMapEncodeTiled failed (shared gate/up)";
      return 1;
    }
  }
  p.K_r = (int)a.H;
  p.K_s = (int)a.H;
  p.N_r = (int)a.I;
  p.N_s = Is;
  p.out = a.act;
  p.ldo = a.ld_act;
  const int64_t mt_bound = (Rt + sm100::BM - 1) / sm100::BM + a.max_units;
  int grid = (int)std::min<int64_t>(a.sms, mt_bound * (a.I / 128 > Is / 128 ? a.I / 128 : Is / 128));
  if (grid < 1) grid = 1;
  if (launch_phase<T, 0>(mA, mB, mS0, mS1, p, grid, st, err)) return 1;
  // ---- phase 1: down -> y (model dtype) ----------------------------------------
  if (!make_map(&mA, a.act, (uint64_t)Rt, (uint64_t)a.ld_act, 128, bf16) ||
      !make_map(&mB, a.down, (uint64_t)a.E_store * a.H, (uint64_t)a.I, 128, bf16)) {
    *err = "cuTensorMapEncodeTiled failed (phase 1)";
    return 1;
  }
  mS0 = mB;
  if (Is && !make_map(&mS0, a.sh_down, (uint64_t)a.H, (uint64_t)Is, 128, bf16)) {
    *err = "cuTensorMapEncodeTiled failed (shared down)";
    return 1;
  }
  mS1 = mS0;
  p.K_r = (int)a.I;
  p.K_s = Is;
  p.N_r = (int)a.H;
  p.N_s = (int)a.H;
  p.out = a.y;
  p.ldo = a.H;
  grid = (int)std::min<int64_t>(a.sms, mt_bound * (a.H / sm100::BN));
  if (grid < 1) grid = 1;
  if (launch_phase<T, 1>(mA, mB, mS0, mS1, p, grid, st, err)) return 1;
  return 0;
}

}  // namespace

bool router_gemm_supported(int64_t H, int64_t E) { return H % 64 == 0 && E % 16 == 0 && E <= 1024; }

int router_logits_sm100(bool bf16, const void* h, int64_t T, int64_t H, const void* w_r, int64_t E,
                        int32_t* units, float* logits, int ksplit, unsigned* status, int sms,
                        cudaStream_t st, const char** err) {
  if (ksplit < 1 || ksplit > H / sm100::BK) {
    *err = "router split out of range";
    return 1;
  }
  if (!encoder()) {
    *err = "cuTensorMapEncodeTiled is not available from the driver";
    return 1;
  }
  sm100::single_unit_kernel<<<1, 32, 0, st>>>(units, (int)E, (int)T);
  if (cudaGetLastError() != cudaSuccess) { *err = "unit table launch failed"; return 1; }
  CUtensorMap mA, mW;
  if (!make_map(&mA, h, (uint64_t)T, (uint64_t)H, 128, bf16) ||
      !make_map(&mW, w_r, (uint64_t)E, (uint64_t)H, 128, bf16)) {
    *err = "cuTensorMapEncodeTiled failed (router)";
    return 1;
  }
  sm100::Params p{};
  p.E = (int)E;
  p.K_r = (int)H;
  p.K_s = (int)H;
  p.N_r = (int)E;
  p.N_s = (int)E;
  p.units = units;
  p.out = logits;
  p.ldo = E;
  p.status = status;
  p.idesc = sm100::make_idesc(bf16);
  p.ksplit = ksplit;
  p.split_stride = T * E;
  const int64_t tiles = ((T + sm100::BM - 1) / sm100::BM) * ((E + sm100::BN - 1) / sm100::BN);
  const int grid = (int)std::min<int64_t>(sms, tiles * ksplit);
  return bf16 ? launch_phase<__nv_bfloat16, 2>(mA, mW, mW, mW, p, grid, st, err)
              : launch_phase<__half, 2>(mA, mW, mW, mW, p, grid, st, err);
}

bool prefill_supported(int64_t H, int64_t I, int64_t Is, bool dense) {
  return dense && H % 256 == 0 && I % 128 == 0 && Is % 128 == 0 && H <= 65536 && I <= 65536;
}

int prefill_experts_sm100(const PrefillArgs& a, cudaStream_t st, const char** err) {
  if (!encoder()) {
    *err = "cuTensorMapEncodeTiled is not available from the driver";
    return 1;
  }
  return a.bf16 ? run<__nv_bfloat16>(a, st, err) : run<__half>(a, st, err);
}

}  // namespace tarfa
