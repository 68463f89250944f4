// C ABI of tarfa_b200: argument checks, workspace layout and launch sequence.
// Declarations and the reference interface each entry point replaces are in
// include/tarfa_b200.h.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <string>
#include <utility>

#include "../../include/tarfa_b200.h"
#include <atomic>

#include "common.cuh"
#include "gemm_sm100.h"
#include "gemv.cuh"
#include "int4.cuh"
#include "router.cuh"
#include "ep_p2p.cuh"
#include "norm.cuh"

using namespace tarfa;

namespace {

thread_local std::string g_last_error;

// stage-boundary events for profiling (tarfa_b200_set_stage_events)
constexpr int kMaxStageEvents = 8;
thread_local cudaEvent_t g_stage_ev[kMaxStageEvents];
thread_local int g_stage_n = 0;

void stage_mark(int i, cudaStream_t st) {
  if (i < g_stage_n && g_stage_ev[i]) cudaEventRecord(g_stage_ev[i], st);
}

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define TARFA_CUDA(call)                                                              \
  do {                                                                                \
    cudaError_t e_ = (call);                                                          \
    if (e_ != cudaSuccess)                                                            \
      return fail(TARFA_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_));    \
  } while (0)

#define TARFA_CHECK(cond, ...)                                                        \
  do {                                                                                \
    if (!(cond)) return fail(TARFA_ERR_INVALID, __VA_ARGS__);                         \
  } while (0)

// ---------------------------------------------------------------------------
// device status word (one per device; kernels atomicOr error bits into it)
// ---------------------------------------------------------------------------
__device__ unsigned g_device_status;

constexpr int kMaxDevices = 64;
std::mutex g_dev_mu;
unsigned* g_status_ptr[kMaxDevices];
int g_sm_count[kMaxDevices];

// Device address of a pointer for kernel access: device memory as is, mapped
// page-locked host memory through its device alias.
int device_alias(const void* p, const void** out) {
  cudaPointerAttributes at{};
  TARFA_CUDA(cudaPointerGetAttributes(&at, p));
  if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) {
    *out = p;
    return TARFA_OK;
  }
  if (at.type == cudaMemoryTypeHost && at.devicePointer) {
    *out = at.devicePointer;
    return TARFA_OK;
  }
  return fail(TARFA_ERR_INVALID, "pointer %p is neither device memory nor mapped page-locked host memory", p);
}

__global__ void stage_copy_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src, size_t n16) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n16) dst[i] = src[i];
}

int device_info(unsigned** status, int* sms) {
  int dev = 0;
  TARFA_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(TARFA_ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_status_ptr[dev]) {
    void* p = nullptr;
    TARFA_CUDA(cudaGetSymbolAddress(&p, g_device_status));
    int n = 0;
    TARFA_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    g_sm_count[dev] = n;
    g_status_ptr[dev] = static_cast<unsigned*>(p);
  }
  *status = g_status_ptr[dev];
  *sms = g_sm_count[dev];
  return TARFA_OK;
}

// ---------------------------------------------------------------------------
// static scratch of tarfa_b200_moe_layer_noalloc: a file-scope device array.
// In host code the symbol is only a host-side stand-in; its device address is
// looked up once per device (with that device current) and cached.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScratchBytes = TARFA_B200_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
void* g_noalloc_ptr[kMaxDevices];

int noalloc_scratch(void** out) {
  int dev = 0;
  TARFA_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(TARFA_ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(TARFA_ERR_CUDA, "cudaGetSymbolAddress(noalloc scratch) failed: %s",
                  cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return TARFA_OK;
}

// ---------------------------------------------------------------------------
// workspace layout
// ---------------------------------------------------------------------------
struct Ws {
  size_t counter, logits, gate_logit, idx32, topw, units, perm_tok, perm_slot, route_row, act, y,
      xperm, bar, hb_cnt, wnorm, lgpart, phist, fxlist, fxcnt, pend;
  size_t total;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

constexpr size_t kZeroHeaderBytes = 2304;   // 16 + 16 + 8192/16*4, rounded to 256
// From here the router logits use the tensor cores (fp32 GEMM, then the exact
// fix-up of logits near a rounding boundary).  Measured on the config-1 router:
// 56 vs 160 us at 64 tokens, 54 vs 88 us at 32 (the exact CUDA-core router
// scales with the tokens).  Smaller batches keep the CUDA-core router and its
// smaller workspace.
constexpr int64_t kRouterGemmMinTokens = 48;
constexpr int kRouterMaxSplit = 8;             // K splits of the tensor-core router GEMM

Ws layout(const tarfa_moe_shape& s, int op) {
  const int64_t T = s.tokens, K = s.top_k, E = s.experts, H = s.hidden;
  const int64_t Is = op == TARFA_OP_MOE_LAYER ? s.shared_inter : 0;
  const int64_t R = T * K;
  const int64_t Rt = R + (Is > 0 ? T : 0);
  const int64_t Umax = (R < E ? R : E) + 1;
  const int64_t Imax = s.inter > Is ? s.inter : Is;
  Ws w{};
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t at = o; o += align256(bytes); return at; };
  // Header shared by every op: counters that every kernel leaves at zero.
  // Identical offsets for all ops, so one workspace can serve any sequence of calls.
  w.counter = 0;
  w.bar = 16;
  w.hb_cnt = 32;   // 8192 / 16 counters at most (hidden <= 8192)
  w.fxcnt = 2096;  // router fix-up list length
  o = kZeroHeaderBytes;
  if (op == TARFA_OP_SHARED) {   // shared expert alone: one unit of T rows
    const int64_t Iss = s.shared_inter;
    w.units = take(8 * 4);
    w.perm_tok = take((T > 0 ? T : 1) * 4);
    w.gate_logit = take(T * 4);
    w.act = take(T * Iss * 2);
    w.y = take(T * H * 4);
    w.total = o;
    return w;
  }
  w.units = take((4 + 4 * Umax) * 4);
  w.idx32 = take(R * 4);
  w.topw = take(R * 4);
  w.route_row = take(R * 4);
  w.perm_tok = take((Rt > 0 ? Rt : 1) * 4);
  w.perm_slot = take(R * 4);
  w.phist = take((size_t)perm_blocks((int)R) * E * 4);   // multi-block permute histograms
  if (op == TARFA_OP_MOE_LAYER || op == TARFA_OP_ROUTER) {
    w.logits = take(T * E * 4);
    w.gate_logit = take(T * 4);
    w.pend = take(T * 4);
    w.wnorm = take(E * 4);
    // fp32 partial logits of the tensor-core router (large batches only)
    if (T >= kRouterGemmMinTokens) {
      w.lgpart = take((size_t)kRouterMaxSplit * T * E * 4);
      w.fxlist = take((size_t)T * (E + 1) * 4);   // logits to recompute exactly
    }
  }
  if (op == TARFA_OP_MOE_LAYER || op == TARFA_OP_EXPERTS) {
    w.act = take(Rt * Imax * 2);
    w.y = take(Rt * H * 4);
    w.xperm = take(Rt * H * 2);
  }
  w.total = o;
  return w;
}

template <typename P> P* at(void* base, size_t off) {
  return reinterpret_cast<P*>(static_cast<char*>(base) + off);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// ---------------------------------------------------------------------------
// shape / weight validation
// ---------------------------------------------------------------------------
int check_shape(const tarfa_moe_shape* s) {
  TARFA_CHECK(s, "null shape");
  TARFA_CHECK(s->tokens >= 0 && s->hidden > 0 && s->experts > 0 && s->inter > 0,
              "bad shape T=%lld H=%lld E=%lld I=%lld", (long long)s->tokens,
              (long long)s->hidden, (long long)s->experts, (long long)s->inter);
  TARFA_CHECK(s->dtype == TARFA_BF16 || s->dtype == TARFA_F16, "dtype %d", s->dtype);
  TARFA_CHECK(s->top_k >= 1 && s->top_k <= 32, "top_k %d not in [1, 32]", s->top_k);
  if (s->experts > 1024) return fail(TARFA_ERR_UNSUPPORTED, "experts %lld > 1024", (long long)s->experts);
  TARFA_CHECK(s->hidden % 32 == 0, "hidden %lld not a multiple of 32", (long long)s->hidden);
  TARFA_CHECK(s->inter % 32 == 0, "inter %lld not a multiple of 32", (long long)s->inter);
  TARFA_CHECK(s->shared_inter >= 0 && s->shared_inter % 32 == 0, "shared_inter %lld",
              (long long)s->shared_inter);
  if (s->hidden > 8192) return fail(TARFA_ERR_UNSUPPORTED, "hidden %lld > 8192", (long long)s->hidden);
  if (s->tokens * s->top_k > (1ll << 30)) return fail(TARFA_ERR_UNSUPPORTED, "too many routes");
  return TARFA_OK;
}

int check_weights(const tarfa_moe_shape* s, const tarfa_moe_weights* w) {
  TARFA_CHECK(w, "null weights");
  TARFA_CHECK(w->gate_up && w->down, "null expert weights");
  TARFA_CHECK(aligned16(w->gate_up) && aligned16(w->down), "expert weights not 16-byte aligned");
  TARFA_CHECK(!w->expert_slot || w->slots >= 1, "expert_slot needs slots (the weight stacks' depth)");
  if (w->kind == TARFA_W_INT4) {
    TARFA_CHECK(w->gate_up_scale && w->down_scale, "int4 weights need scales");
    TARFA_CHECK(s->hidden % 128 == 0 && s->inter % 128 == 0,
                "int4 needs hidden and inter multiples of 128");
    TARFA_CHECK(w->group == 0 || (w->group % 128 == 0 && s->hidden % w->group == 0 &&
                                  s->inter % w->group == 0),
                "int4 group %d must be 0 or a multiple of 128 dividing hidden and inter", w->group);
  } else {
    TARFA_CHECK(w->kind == TARFA_W_DENSE, "weight kind %d", w->kind);
  }
  return TARFA_OK;
}

// Every argument check of the layer entry points, before anything is launched
// or written.
int check_layer_args(const tarfa_moe_shape* shape, const void* hidden, const void* router_weight,
                     const tarfa_moe_weights* weights, const tarfa_shared_expert* shared,
                     const void* out) {
  if (int rc = check_shape(shape)) return rc;
  if (int rc = check_weights(shape, weights)) return rc;
  if (shape->tokens == 0) return TARFA_OK;
  TARFA_CHECK(hidden && router_weight && out, "null argument");
  TARFA_CHECK(aligned16(hidden) && aligned16(router_weight) && aligned16(out),
              "operands not 16-byte aligned");
  TARFA_CHECK(shape->top_k <= shape->experts, "top_k > experts");
  if (shared && shape->shared_inter > 0) {
    TARFA_CHECK(shared->gate_proj && shared->up_proj && shared->down_proj && shared->gate_weight,
                "null shared-expert weight");
    TARFA_CHECK(aligned16(shared->gate_proj) && aligned16(shared->up_proj) &&
                    aligned16(shared->down_proj) && aligned16(shared->gate_weight),
                "shared-expert weights not 16-byte aligned");
  }
  return TARFA_OK;
}

// ---------------------------------------------------------------------------
// launches
// ---------------------------------------------------------------------------
// Launch, optionally as a programmatic dependent of the previous kernel on the
// stream (it may start before that kernel ends and synchronises with
// griddepcontrol.wait).
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     bool pdl, Args&&... args) {
  if (smem > 48 * 1024) {   // above the default dynamic shared-memory limit
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  if (!pdl) {
    kern<<<grid, block, smem, st>>>(std::forward<Args>(args)...);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

template <typename T, int MODE, int PHASE, int KSPLIT, int NTB>
int launch_gemv(const GemvArgs& a, int max_tiles, int sms, cudaStream_t st, bool pdl, int smem) {
  constexpr int groups = kGemvWarps / KSPLIT;
  int grid = (max_tiles + groups - 1) / groups;
  const int cap = gemv_ctas_per_sm(MODE, PHASE, NTB) * sms;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  TARFA_CUDA(launch_k(gemv_kernel<T, MODE, PHASE, KSPLIT, NTB>, dim3(grid), dim3(kGemvThreads),
                      (size_t)smem, st, pdl, a));
  return TARFA_OK;
}

template <typename T, int MODE, int PHASE, int KSPLIT>
int launch_gemv_ntb(const GemvArgs& a, int max_tiles, int T_, int sms, cudaStream_t st,
                    bool pdl = false, int smem = 0) {
  if (T_ <= 8) return launch_gemv<T, MODE, PHASE, KSPLIT, 1>(a, max_tiles, sms, st, pdl, smem);
  return launch_gemv<T, MODE, PHASE, KSPLIT, 2>(a, max_tiles, sms, st, pdl, smem);
}

// Warps sharing one tile's K (the rest of the CTA's warps take other tiles).
// Measured on the config-1 layer with the A/B harness: gate_up 4 and down 2
// beat 8 and 4 (T = 1: 53.3 vs 55.1 us per layer; T = 16: 340 vs 369 us).
constexpr int kKsplitGateUp = 4;
constexpr int kKsplitDown = 2;
// int4 tiles hold a quarter of the bytes of dense ones, so fewer warps share a
// tile's K (the per-tile reduction and epilogue amortise over more data).
// Measured on the config-1 layer (group 128): gate_up split 4 at 1-2 tokens
// (45.8 vs 48.8 us per layer at T = 1 against split 2), 2 from 4 tokens;
// down split 2.

// T_: tokens of the batch (picks the K split, which fixes the fp32 summation
// order); rows: most rows of one unit (picks the token blocks; -1: T_).
constexpr int q4_ksplit(int phase, int T_) { return phase == kGateUp && T_ <= 2 ? 4 : 2; }

template <typename T, int MODE, int PHASE>
int launch_gemv_q4(const GemvArgs& a, int max_tiles, int T_, int sms, cudaStream_t st, bool pdl,
                   int smem, int rows = -1) {
  if (rows < 0) rows = T_;
  if (q4_ksplit(PHASE, T_) == 4)
    return launch_gemv_ntb<T, MODE, PHASE, 4>(a, max_tiles, rows, sms, st, pdl, smem);
  return launch_gemv_ntb<T, MODE, PHASE, 2>(a, max_tiles, rows, sms, st, pdl, smem);
}

// Token count from which dense layers take the tcgen05 grouped-GEMM path
// (tarfa_b200_set_gemm_min_tokens); below it the tensor-core GEMV path.
std::atomic<int64_t> g_gemm_min_tokens{64};

bool use_gemm(const tarfa_moe_shape& s, const tarfa_moe_weights& w, int64_t Is) {
  return w.kind == TARFA_W_DENSE && s.tokens >= g_gemm_min_tokens.load() &&
         prefill_supported(s.hidden, s.inter, Is, true);
}

template <typename T>
// chained: the decode chain (run_decode_layer), every launch a programmatic
// dependent of the previous one.
int run_experts(const tarfa_moe_shape& s, const void* hidden, const tarfa_moe_weights& w,
                const tarfa_shared_expert* sh, const Ws& L, void* ws, void* out,
                unsigned* status, int sms, cudaStream_t st, bool chained = false) {
  const int T_ = (int)s.tokens, K = s.top_k, E = (int)s.experts, H = (int)s.hidden;
  const int I = (int)s.inter, Is = sh ? (int)s.shared_inter : 0;
  const int Imax = I > Is ? I : Is;
  const int R = T_ * K;
  const int Umax = (R < E ? R : E);
  const bool int4 = w.kind == TARFA_W_INT4;
  const int mode = !int4 ? kModeExact : (T_ == 1 ? kModeInt4Fused : kModeInt4Dequant);
  int32_t* units = at<int32_t>(ws, L.units);

  if (use_gemm(s, w, Is)) {   // batched / prefill: tcgen05 grouped GEMM over the segments
    PrefillArgs p{};
    p.bf16 = s.dtype == TARFA_BF16;
    p.T = T_;
    p.H = H;
    p.E = E;
    p.E_store = w.expert_slot ? w.slots : E;   // the TMA maps cover every slot
    p.I = I;
    p.Is = Is;
    p.rows_total = R + (Is ? T_ : 0);
    p.max_units = Umax + 1;
    p.hidden = hidden;
    p.perm_tok = at<int32_t>(ws, L.perm_tok);
    p.units = units;
    p.expert_slot = w.expert_slot;
    p.gate_up = w.gate_up;
    p.down = w.down;
    p.sh_gate = sh ? sh->gate_proj : nullptr;
    p.sh_up = sh ? sh->up_proj : nullptr;
    p.sh_down = sh ? sh->down_proj : nullptr;
    p.x_perm = at<void>(ws, L.xperm);
    p.act = at<void>(ws, L.act);
    p.ld_act = Imax;
    p.y = at<void>(ws, L.y);
    p.status = status;
    p.sms = sms;
    const char* err = nullptr;
    if (prefill_experts_sm100(p, st, &err)) return fail(TARFA_ERR_CUDA, "%s", err ? err : "prefill");
    stage_mark(2, st);
    stage_mark(3, st);
    return TARFA_OK;
  }

  GemvArgs g{};
  g.units = units;
  g.E = E;
  g.expert_slot = w.expert_slot;
  g.status = status;
  // ---- gate_up + SiLU*mul -> act -------------------------------------------
  g.x = hidden;
  g.ld_x = H;
  g.perm_tok = at<int32_t>(ws, L.perm_tok);
  g.N_r = I;
  g.K_r = H;
  g.N_s = Is;
  g.K_s = H;
  g.sw0 = sh ? sh->gate_proj : nullptr;
  g.sw1 = sh ? sh->up_proj : nullptr;
  g.out = at<void>(ws, L.act);
  g.ld_out = Imax;
  g.w = w.gate_up;
  if (int4) {
    g.w_estride = (int64_t)2 * I * H / 8;
    g.w_rstride = H / 8;
    g.sc = w.gate_up_scale;
    g.s_rstride = w.group ? H / w.group : 1;
    g.s_estride = (int64_t)2 * I * g.s_rstride;
    g.group = w.group;
  } else {
    g.w_estride = (int64_t)2 * I * H;
    g.w_rstride = H;
  }
  const int tiles_gu = Umax * (I / 8) + (Is ? Is / 8 : 0);
  // chained: programmatic dependents of the router kernel, whose last CTA
  // writes the unit table; the shared expert's tiles stream meanwhile
  const bool pdl = chained;
  const int smem = 0;
  if (chained) {
    g.route_mode = 3;
    g.sh_row0 = R;
    g.sh_rows = T_;
    g.add_shared = sh != nullptr;
  }
  int rc;
  if (!int4) {
    g.which = 3;
    rc = launch_gemv_ntb<T, kModeExact, kGateUp, kKsplitGateUp>(g, tiles_gu, T_, sms, st, pdl, smem);
  } else {
    // The int4 kernel runs the shared expert's tiles too (first, with the exact
    // loop) when its K split is the dense one's, so the shared expert's fp32
    // summation order is the same as in its own launch.
    const bool with_sh = q4_ksplit(kGateUp, T_) == kKsplitGateUp;
    g.which = with_sh ? 3 : 1;
    rc = mode == kModeInt4Fused
             ? launch_gemv_q4<T, kModeInt4Fused, kGateUp>(g, tiles_gu, T_, sms, st, pdl, smem)
             : launch_gemv_q4<T, kModeInt4Dequant, kGateUp>(g, tiles_gu, T_, sms, st, pdl, smem);
    if (rc == TARFA_OK && Is && !with_sh) {
      GemvArgs gs = g;
      gs.which = 2;
      if (chained) gs.route_mode = 2;   // fixed shared rows, no unit table needed
      rc = launch_gemv_ntb<T, kModeExact, kGateUp, kKsplitGateUp>(gs, Is / 8, T_, sms, st, pdl);
    }
  }
  if (rc) return rc;
  stage_mark(2, st);
  // ---- down -> y -------------------------------------------------------------
  g.x = at<void>(ws, L.act);
  g.ld_x = Imax;
  g.perm_tok = nullptr;
  g.N_r = H;
  g.K_r = I;
  g.N_s = H;
  g.K_s = Is;
  g.sw0 = sh ? sh->down_proj : nullptr;
  g.sw1 = nullptr;
  g.out = at<void>(ws, L.y);
  g.ld_out = H;
  g.w = w.down;
  g.route_mode = 0;   // the unit table is in the workspace now
  if (int4) {
    g.w_estride = (int64_t)H * I / 8;
    g.w_rstride = I / 8;
    g.sc = w.down_scale;
    g.s_rstride = w.group ? I / w.group : 1;
    g.s_estride = (int64_t)H * g.s_rstride;
  } else {
    g.w_estride = (int64_t)H * I;
    g.w_rstride = I;
  }
  const int tiles_dn = (Umax + (Is ? 1 : 0)) * (H / 16);
  if (!int4) {
    g.which = 3;

    rc = launch_gemv_ntb<T, kModeExact, kDown, kKsplitDown>(g, tiles_dn, T_, sms, st, pdl);
  } else {
    const bool with_sh = q4_ksplit(kDown, T_) == kKsplitDown;
    g.which = with_sh ? 3 : 1;
    rc = mode == kModeInt4Fused
             ? launch_gemv_q4<T, kModeInt4Fused, kDown>(g, tiles_dn, T_, sms, st, pdl, 0)
             : launch_gemv_q4<T, kModeInt4Dequant, kDown>(g, tiles_dn, T_, sms, st, pdl, 0);
    if (rc == TARFA_OK && Is && !with_sh) {
      GemvArgs gs = g;
      gs.which = 2;
      rc = launch_gemv_ntb<T, kModeExact, kDown, kKsplitDown>(gs, H / 16, T_, sms, st, pdl);
    }
  }
  if (rc) return rc;
  stage_mark(3, st);
  return TARFA_OK;
}

CombineArgs make_combine_args(const tarfa_moe_shape& s, const Ws& L, void* ws, const float* top_w,
                              bool int4, bool with_shared, void* out) {
  const int T_ = (int)s.tokens;
  CombineArgs c{};
  c.y = at<void>(ws, L.y);
  c.route_row = at<int32_t>(ws, L.route_row);
  c.idx32 = at<int32_t>(ws, L.idx32);
  c.w = top_w;
  c.units = at<int32_t>(ws, L.units);
  c.T = T_;
  c.K = s.top_k;
  c.H = (int)s.hidden;
  c.E = (int)s.experts;
  c.order_router = T_ == 1;
  c.mode = !int4 ? kModeExact : (T_ == 1 ? kModeInt4Fused : kModeInt4Dequant);
  c.gate_logit = with_shared ? at<float>(ws, L.gate_logit) : nullptr;
  c.out = out;
  return c;
}

template <typename T>
// pend / idx_out (decode chain): tokens whose tie order the router left open get
// it here (combine_token_kernel), and their ids are rewritten in idx_out.
int run_combine(const tarfa_moe_shape& s, const Ws& L, void* ws, const float* top_w, bool int4,
                bool with_shared, bool gemm_y, void* out, cudaStream_t st, bool pdl = false,
                bool pend = false, int64_t* idx_out = nullptr) {
  const int T_ = (int)s.tokens, H = (int)s.hidden;
  CombineArgs c = make_combine_args(s, L, ws, top_w, int4, with_shared, out);
  size_t smem = 0;
  if (pend) {
    c.pend = at<int32_t>(ws, L.pend);
    c.logits = at<float>(ws, L.logits);
    c.idx_out = idx_out;
    smem = (size_t)tie_scratch_ints(c.E) * sizeof(int);
  }
  // large batches: one block per token, a thread per 8 columns (up to 512);
  // decode: one-warp blocks, so that the few tokens' columns spread over many
  // SMs (the loads are latency-bound)
  const int threads =
      T_ > 64 ? std::min(kCombineTokenThreads, ((H / 8 + 31) / 32) * 32) : 32;
  const dim3 grid(T_ > 64 ? 1 : (H / 8 + threads - 1) / threads, T_);
  if (gemm_y) TARFA_CUDA(launch_k(combine_token_kernel<T, T>, grid, dim3(threads), smem, st, pdl, c));
  else TARFA_CUDA(launch_k(combine_token_kernel<T, float>, grid, dim3(threads), smem, st, pdl, c));
  TARFA_CUDA(cudaGetLastError());
  stage_mark(4, st);
  return TARFA_OK;
}

int permute_smem_bytes(int nwarps, int E) { return (int)(permute_smem_ints(nwarps, E) * 4); }

template <typename Idx>
int launch_permute(const Idx* idx, int T_, int K, int E, bool add_shared, const PermuteOut& o,
                   int32_t* hist, unsigned* status, cudaStream_t st) {
  const int R = T_ * K;
  if (R > 2 * kPermRoutes) {   // many routes: two passes over many blocks
    const int nblk = perm_blocks(R);
    const int smem_h = E * (int)sizeof(int);
    const int smem_s = (2 + kPermThreads / 32) * E * (int)sizeof(int);
    permute_hist_kernel<Idx><<<nblk, kPermThreads, smem_h, st>>>(idx, T_, K, E, hist, o, status);
    TARFA_CUDA(cudaGetLastError());
    permute_scatter_kernel<Idx><<<nblk, kPermThreads, smem_s, st>>>(idx, T_, K, E, add_shared ? 1 : 0,
                                                                    hist, o);
    TARFA_CUDA(cudaGetLastError());
    return TARFA_OK;
  }
  const int threads = 1024;
  const int smem = permute_smem_bytes(threads / 32, E);
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  TARFA_CUDA(cudaGetDevice(&dev));
  if (!attr_set[dev]) {
    TARFA_CUDA(cudaFuncSetAttribute(permute_kernel<Idx>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    permute_smem_bytes(32, 1024)));
    attr_set[dev] = true;
  }
  permute_kernel<Idx><<<1, threads, smem, st>>>(idx, T_, K, E, add_shared ? 1 : 0, o, status);
  TARFA_CUDA(cudaGetLastError());
  return TARFA_OK;
}

bool use_router_gemm(const tarfa_moe_shape& s) {
  return s.tokens >= kRouterGemmMinTokens && s.experts >= 128 && router_gemm_supported(s.hidden, s.experts);
}

// Exact logits of a batch on the tensor cores: fp32 partial logits (K split),
// row norms of the router for the error window, then the window settles the
// logits it can and lists the rest (and the shared-expert gate row), which are
// recomputed exactly.  Leaves the list counter set: the next kernel that
// reads the logits clears it (topk_kernel, or the expert-parallel exchange).
template <typename T>
int launch_router_logits_tc(const tarfa_moe_shape& s, const void* hidden, const void* w_r,
                            const void* bias, const void* w_sg, const Ws& L, void* ws,
                            float* logits_out, unsigned* status, int sms, cudaStream_t st) {
  const int T_ = (int)s.tokens, H = (int)s.hidden, E = (int)s.experts;
  const char* err = nullptr;
  // split K so that the (tile, K range) work items fill the SMs about twice;
  // shorter fp32 accumulations also narrow the fix-up window (fixup_rel)
  const int64_t tiles = ((T_ + 127) / 128) * ((E + 255) / 256);
  const int ksplit = (int)std::max<int64_t>(
      1, std::min<int64_t>({(int64_t)kRouterMaxSplit, H / 64, 2 * sms / std::max<int64_t>(1, tiles)}));
  if (router_logits_sm100(s.dtype == TARFA_BF16, hidden, T_, H, w_r, E, at<int32_t>(ws, L.units),
                          at<float>(ws, L.lgpart), ksplit, status, sms, st, &err))
    return fail(TARFA_ERR_CUDA, "%s", err ? err : "router logits");
  row_norms_kernel<T><<<(E + 7) / 8, 256, 0, st>>>(static_cast<const T*>(w_r), E, H,
                                                   at<float>(ws, L.wnorm));
  const int grid = (T_ + 7) / 8;
  unsigned* cnt = at<unsigned>(ws, L.fxcnt);
  const T* hT = static_cast<const T*>(hidden);
  const T* bT = static_cast<const T*>(bias);
  fixup_window_kernel<T><<<grid, 256, 0, st>>>(
      at<float>(ws, L.lgpart), ksplit, (int64_t)T_ * E, hT, bT, at<float>(ws, L.wnorm),
      w_sg != nullptr, T_, H, E, at<float>(ws, L.logits), logits_out, at<int32_t>(ws, L.fxlist), cnt);
  fixup_exact_kernel<T><<<sms * 8, 256, 0, st>>>(
      hT, static_cast<const T*>(w_r), static_cast<const T*>(w_sg), bT, H, E,
      at<int32_t>(ws, L.fxlist), cnt, at<float>(ws, L.logits), logits_out, at<float>(ws, L.gate_logit));
  TARFA_CUDA(cudaGetLastError());
  return TARFA_OK;
}

template <typename T>
int launch_router(const tarfa_moe_shape& s, const void* hidden, const void* w_r, const void* bias,
                  const void* w_sg, const Ws& L, void* ws, int64_t* idx_out, float* w_out,
                  float* logits_out, bool permute, bool add_shared, unsigned* status,
                  cudaStream_t st) {
  if (use_router_gemm(s)) {
    // batch: fp32 logits on the tensor cores, exact-rounding fixup + top-k, permute
    unsigned* st_ptr;
    int sms;
    if (int rc = device_info(&st_ptr, &sms)) return rc;
    const int T_ = (int)s.tokens, E = (int)s.experts, K = s.top_k;
    if (int rc = launch_router_logits_tc<T>(s, hidden, w_r, bias, w_sg, L, ws, logits_out, status, sms, st))
      return rc;
    const int grid = (T_ + 7) / 8;
    unsigned* cnt = at<unsigned>(ws, L.fxcnt);
    TARFA_CUDA(launch_k(topk_kernel<T>, dim3(grid), dim3(256),
                        (size_t)8 * tie_scratch_ints(E) * sizeof(int), st, false,
                        at<float>(ws, L.logits), T_, E, K, at<int32_t>(ws, L.idx32),
                        at<float>(ws, L.topw), idx_out, w_out, cnt));
    if (!permute) return TARFA_OK;
    PermuteOut o{nullptr, at<int32_t>(ws, L.perm_tok), at<int32_t>(ws, L.perm_slot),
                 at<int32_t>(ws, L.route_row), at<int32_t>(ws, L.units), nullptr};
    return launch_permute<int32_t>(at<int32_t>(ws, L.idx32), T_, K, E, add_shared, o,
                                   at<int32_t>(ws, L.phist), status, st);
  }
  RouterArgs a{};
  a.h = hidden;
  a.w_r = w_r;
  a.bias = bias;
  a.w_sg = w_sg;
  a.T = (int)s.tokens;
  a.H = (int)s.hidden;
  a.E = (int)s.experts;
  a.K = s.top_k;
  a.logits = at<float>(ws, L.logits);
  a.gate_logit = at<float>(ws, L.gate_logit);
  a.idx32 = at<int32_t>(ws, L.idx32);
  a.topw = at<float>(ws, L.topw);
  a.idx_out = idx_out;
  a.w_out = w_out;
  a.logits_out = logits_out;
  a.counter = at<unsigned>(ws, L.counter);
  a.do_permute = permute;
  a.add_shared = add_shared;
  a.perm = PermuteOut{nullptr, at<int32_t>(ws, L.perm_tok), at<int32_t>(ws, L.perm_slot),
                      at<int32_t>(ws, L.route_row), at<int32_t>(ws, L.units), nullptr};
  a.status = status;
  const int rows = a.E + (w_sg ? 1 : 0);
  const int warps = kRouterThreads / 32;
  unsigned* st_unused;
  int sms;
  if (int rc = device_info(&st_unused, &sms)) return rc;
  // work items = rows x token groups; about two warps' worth per warp slot of one wave
  const int64_t target = 2LL * sms * warps;
  a.tpw = (int)std::max<int64_t>(1, std::min<int64_t>(a.T, ((int64_t)rows * a.T + target - 1) / target));
  const int64_t items = (int64_t)rows * ((a.T + a.tpw - 1) / a.tpw);
  const int grid = (int)((items + warps - 1) / warps);
  const int smem = (router_tie_offset(a.E, a.T * a.K) + warps * tie_scratch_ints(a.E)) *
                   (int)sizeof(int);
  const int per_lane = (a.H / 8 + 31) / 32;
#define TARFA_ROUTER(MC)                                                                  \
  TARFA_CUDA(launch_k(router_kernel<T, MC>, dim3(grid), dim3(kRouterThreads), (size_t)smem, st, \
                      false, a))
  if (per_lane <= 2) TARFA_ROUTER(2);
  else if (per_lane <= 4) TARFA_ROUTER(4);
  else if (per_lane <= 8) TARFA_ROUTER(8);
  else if (per_lane <= 16) TARFA_ROUTER(16);
  else TARFA_ROUTER(32);
#undef TARFA_ROUTER
  return TARFA_OK;
}

}  // namespace

// ===========================================================================
// exported entry points
// ===========================================================================
// Decode batches on the GEMV path run as one chain of programmatic dependents:
// the router kernel (its last CTA routes every token), the gate_up GEMV (shared
// expert first, then the routed tiles once the unit table is there), the down
// GEMV and the combine.
std::atomic<int64_t> g_decode_routing_max_tokens{16};

bool use_decode_routing(const tarfa_moe_shape& s, const tarfa_moe_weights& w) {
  return s.tokens <= g_decode_routing_max_tokens.load() && s.tokens <= 16 &&
         s.tokens * s.top_k <= 128 && s.experts <= 1024 &&
         !use_gemm(s, w, s.shared_inter);
}

// route: the last CTA also runs top-k and permute into the workspace (decode
// chain); idx_out / w_out receive the routing then.
template <typename T>
int launch_router_logits(const tarfa_moe_shape& s, const void* hidden, const void* w_r,
                         const void* bias, const void* w_sg, const Ws& L, void* ws, int sms,
                         cudaStream_t st, bool route = false, int64_t* idx_out = nullptr,
                         float* w_out = nullptr, unsigned* status = nullptr) {
  RouterArgs a{};
  a.route_last = route;
  if (route) {
    a.idx32 = at<int32_t>(ws, L.idx32);
    a.topw = at<float>(ws, L.topw);
    a.idx_out = idx_out;
    a.w_out = w_out;
    a.counter = at<unsigned>(ws, L.counter);
    a.do_permute = 1;
    a.add_shared = w_sg != nullptr;
    a.perm = PermuteOut{nullptr, at<int32_t>(ws, L.perm_tok), at<int32_t>(ws, L.perm_slot),
                        at<int32_t>(ws, L.route_row), at<int32_t>(ws, L.units), nullptr};
    a.status = status;
    a.pend = at<int32_t>(ws, L.pend);   // interior ties: order settled by the combine
  }
  a.h = hidden;
  a.w_r = w_r;
  a.bias = bias;
  a.w_sg = w_sg;
  a.T = (int)s.tokens;
  a.H = (int)s.hidden;
  a.E = (int)s.experts;
  a.K = s.top_k;
  a.logits = at<float>(ws, L.logits);
  a.gate_logit = at<float>(ws, L.gate_logit);
  const int rows = a.E + (w_sg ? 1 : 0);
  constexpr int warps = kRouterThreads / 32;
  if (a.T <= 2) {            // latency: split each row over four warps
    a.wpr = 4;
    a.tpw = 1;
  } else {                   // throughput: a row per warp, tokens grouped
    a.wpr = 1;
    const int64_t target = 2LL * sms * warps;
    a.tpw = (int)std::max<int64_t>(1, std::min<int64_t>(a.T, ((int64_t)rows * a.T + target - 1) / target));
  }
  const int slots = warps / a.wpr;
  const int64_t items = (int64_t)rows * ((a.T + a.tpw - 1) / a.tpw);
  const int grid = (int)((items + slots - 1) / slots);
  const int per_lane = ((a.H / 8 + a.wpr - 1) / a.wpr + 31) / 32;
  const size_t smem =
      route ? (size_t)(router_tie_offset(a.E, a.T * a.K) + warps * tie_scratch_ints(a.E)) * sizeof(int) : 0;
#define TARFA_ROUTER_LOGITS(MC)                                                              \
  TARFA_CUDA(launch_k(router_logits_kernel<T, MC>, dim3(grid), dim3(kRouterThreads), smem, st, \
                      false, a))
  if (per_lane <= 2) TARFA_ROUTER_LOGITS(2);
  else if (per_lane <= 4) TARFA_ROUTER_LOGITS(4);
  else if (per_lane <= 8) TARFA_ROUTER_LOGITS(8);
  else if (per_lane <= 16) TARFA_ROUTER_LOGITS(16);
  else TARFA_ROUTER_LOGITS(32);
#undef TARFA_ROUTER_LOGITS
  return TARFA_OK;
}

template <typename T>
int run_decode_layer(const tarfa_moe_shape& s, const void* hidden, const void* w_r,
                     const void* bias, const tarfa_moe_weights& w, const tarfa_shared_expert* sh,
                     void* out, int64_t* idx_out, float* w_out, const Ws& L, void* ws,
                     unsigned* status, int sms, cudaStream_t st) {
  if (int rc = launch_router_logits<T>(s, hidden, w_r, bias, sh ? sh->gate_weight : nullptr, L, ws,
                                       sms, st, true, idx_out, w_out, status))
    return rc;
  stage_mark(1, st);
  if (int rc = run_experts<T>(s, hidden, w, sh, L, ws, out, status, sms, st, true)) return rc;
  return run_combine<T>(s, L, ws, at<float>(ws, L.topw), w.kind == TARFA_W_INT4, sh != nullptr,
                        false, out, st, true, true, idx_out);
}

// ===========================================================================
// expert parallelism over peer memory (ep_p2p.cuh)
// ===========================================================================

struct EpWs {
  Ws w;
  size_t local_idx, cur_step, xin;
};

// Workspace of one expert-parallel layer, sized for max_tokens (the same
// offsets serve every batch up to it).
EpWs ep_layout(const tarfa_moe_shape& s, int N, int64_t Tmax) {
  const int64_t K = s.top_k, E = s.experts, H = s.hidden;
  const int64_t R = N * Tmax * K;
  const int64_t Imax = std::max<int64_t>(s.inter, s.shared_inter);
  const int64_t Umax = std::min<int64_t>(R, E) + 1;   // any split of the experts over the ranks
  EpWs L{};
  size_t o = kZeroHeaderBytes;
  auto take = [&](size_t b) { size_t at = o; o += align256(b); return at; };
  L.w.fxcnt = 2096;   // header: the router fix-up list length (tensor-core logits)
  L.w.logits = take(Tmax * E * 4);
  L.w.gate_logit = take(Tmax * 4);
  if (Tmax >= kRouterGemmMinTokens) {   // tensor-core router logits for batches
    L.w.wnorm = take(E * 4);
    L.w.lgpart = take((size_t)kRouterMaxSplit * Tmax * E * 4);
    L.w.fxlist = take((size_t)Tmax * (E + 1) * 4);
  }
  L.w.idx32 = take(Tmax * K * 4);
  L.w.topw = take(Tmax * K * 4);
  L.w.units = take((4 + 4 * Umax) * 4);
  L.w.perm_tok = take((R + Tmax) * 4);
  L.local_idx = take(R * 4);
  L.cur_step = take(4);
  L.xin = take(R * H * 2);
  L.w.act = take((R + Tmax) * Imax * 2);
  L.w.y = take((R + Tmax) * H * 4);
  L.w.total = o;
  return L;
}

int check_ep(const tarfa_moe_shape* s, const tarfa_ep_group* g) {
  TARFA_CHECK(g, "null ep group");
  TARFA_CHECK(g->world >= 1 && g->world <= TARFA_EP_MAX_RANKS, "ep world %d not in [1, %d]",
              g->world, TARFA_EP_MAX_RANKS);
  TARFA_CHECK(g->rank >= 0 && g->rank < g->world, "ep rank %d of %d", g->rank, g->world);
  TARFA_CHECK(g->tp == 1 || (g->tp == 2 && g->world % 2 == 0),
              "ep tp %d must be 1, or 2 with an even world (%d)", g->tp, g->world);
  TARFA_CHECK(s->experts % (g->world / g->tp) == 0, "%lld experts do not shard over %d ranks",
              (long long)s->experts, g->world);
  if (g->tp == 2)
    TARFA_CHECK(s->inter % 64 == 0, "ep tp 2 needs inter %lld to split into halves of a multiple of 32",
                (long long)s->inter);
  TARFA_CHECK(g->max_tokens >= 1 && g->max_tokens * s->top_k * g->world <= 8192,
              "ep max_tokens %lld (max_tokens * top_k * world must be <= 8192)",
              (long long)g->max_tokens);
  for (int r = 0; r < g->world; ++r)
    TARFA_CHECK(g->boxes[r] && aligned16(g->boxes[r]), "ep box %d null or not 16-byte aligned", r);
  return TARFA_OK;
}

template <typename T>
int run_ep_layer(const tarfa_moe_shape& s, const void* hidden, const void* w_r, const void* bias,
                 const tarfa_moe_weights& w, const tarfa_shared_expert* sh, const tarfa_ep_group& grp,
                 void* out, int64_t* idx_out, float* w_out, const EpWs& L, void* ws,
                 unsigned* status, int sms, cudaStream_t st) {
  const int N = grp.world, T_ = (int)s.tokens, K = s.top_k, E = (int)s.experts, H = (int)s.hidden;
  const int P = grp.tp;            // ranks sharing each expert (halves of its intermediate dim)
  const int e_per = E / (N / P), S = (int)grp.max_tokens * K, R = N * S;
  const int I = (int)s.inter / P, Is = sh ? (int)s.shared_inter : 0;   // I: this rank's part
  const int Imax = std::max(I, Is);
  const bool int4 = w.kind == TARFA_W_INT4;
  const int mode = !int4 ? kModeExact : (T_ == 1 ? kModeInt4Fused : kModeInt4Dequant);
  // rows an owner can receive: one per token and source for each of its experts
  const int rows_max = std::min(R, N * T_ * K);
  const int units_max = std::min(rows_max, e_per);
  const int rows_unit = N * T_;   // most rows of one unit (token batches of the GEMV)

  stage_mark(0, st);
  // exact logits: the tensor-core router for batches, else the CUDA-core one
  const bool tc_router = use_router_gemm(s) && grp.max_tokens >= kRouterGemmMinTokens;
  if (tc_router) {
    if (int rc = launch_router_logits_tc<T>(s, hidden, w_r, bias, sh ? sh->gate_weight : nullptr, L.w,
                                            ws, nullptr, status, sms, st))
      return rc;
  } else if (int rc = launch_router_logits<T>(s, hidden, w_r, bias, sh ? sh->gate_weight : nullptr, L.w,
                                              ws, sms, st)) {
    return rc;
  }
  stage_mark(1, st);
  ep::Args a{};
  a.fx_cnt = tc_router ? at<unsigned>(ws, L.w.fxcnt) : nullptr;
  a.T = T_;
  a.K = K;
  a.H = H;
  a.E = E;
  a.N = N;
  a.rank = grp.rank;
  a.S = S;
  a.e_per = e_per;
  a.tp = P;
  a.mode = mode;
  a.has_shared = sh != nullptr;
  for (int r = 0; r < N; ++r) a.boxes[r] = grp.boxes[r];
  a.logits = at<float>(ws, L.w.logits);
  a.h = hidden;
  a.idx32 = at<int32_t>(ws, L.w.idx32);
  a.topw = at<float>(ws, L.w.topw);
  a.idx_out = idx_out;
  a.w_out = w_out;
  a.local_idx = at<int32_t>(ws, L.local_idx);
  a.units = at<int32_t>(ws, L.w.units);
  a.perm_tok = at<int32_t>(ws, L.w.perm_tok);
  a.xin = at<void>(ws, L.xin);
  a.cur_step = at<unsigned>(ws, L.cur_step);
  a.y = at<float>(ws, L.w.y);
  a.gate_logit = at<float>(ws, L.w.gate_logit);
  a.out = out;
  a.status = status;
  // 32-64 blocks store the token rows and unpack the inbox; every block tops-k its own token
  const int chunks = std::max(1, std::min(32, 64 / T_));
  const int ex_smem = std::max<int>(
      {ep::kExchangeThreads * (int)sizeof(int),   // the unpack's per-item flags
       R <= ep::kExchangeThreads ? ep::rank_permute_smem_ints(R) * (int)sizeof(int)
                                 : permute_smem_bytes(ep::kExchangeThreads / 32, e_per),
       tie_scratch_ints(E) * (int)sizeof(int)});  // warp 0's top-k tie order
  TARFA_CUDA(launch_k(ep::exchange_kernel<T>, dim3(T_, chunks), dim3(ep::kExchangeThreads),
                      (size_t)ex_smem, st, true, a));

  // ---- local experts over the inbox rows (shared expert on own tokens first)
  GemvArgs g{};
  g.units = a.units;
  g.E = e_per;
  g.expert_slot = w.expert_slot;
  g.status = status;
  g.x = a.xin;
  g.ld_x = H;
  g.x_sh = hidden;
  g.perm_tok = a.perm_tok;
  g.N_r = I;
  g.K_r = H;
  g.N_s = Is;
  g.K_s = H;
  g.sw0 = sh ? sh->gate_proj : nullptr;
  g.sw1 = sh ? sh->up_proj : nullptr;
  g.out = at<void>(ws, L.w.act);
  g.ld_out = Imax;
  g.w = w.gate_up;
  g.route_mode = 3;
  g.sh_row0 = R;
  g.sh_rows = T_;
  g.add_shared = sh != nullptr;
  if (int4) {
    g.w_estride = (int64_t)2 * I * H / 8;
    g.w_rstride = H / 8;
    g.sc = w.gate_up_scale;
    g.s_rstride = w.group ? H / w.group : 1;
    g.s_estride = (int64_t)2 * I * g.s_rstride;
    g.group = w.group;
  } else {
    g.w_estride = (int64_t)2 * I * H;
    g.w_rstride = H;
  }
  int rc;
  if (!int4) {
    g.which = 3;
    rc = launch_gemv_ntb<T, kModeExact, kGateUp, kKsplitGateUp>(
        g, units_max * (I / 8) + Is / 8, rows_unit, sms, st, true);
  } else {
    GemvArgs gs = g;
    g.which = 1;
    rc = mode == kModeInt4Fused
             ? launch_gemv_q4<T, kModeInt4Fused, kGateUp>(g, units_max * (I / 8), T_, sms, st, true, 0, rows_unit)
             : launch_gemv_q4<T, kModeInt4Dequant, kGateUp>(g, units_max * (I / 8), T_, sms, st, true, 0, rows_unit);
    if (rc == TARFA_OK && Is) {
      gs.which = 2;
      rc = launch_gemv_ntb<T, kModeExact, kGateUp, kKsplitGateUp>(gs, Is / 8, T_, sms, st, true);
    }
  }
  if (rc) return rc;
  stage_mark(2, st);
  g.x = at<void>(ws, L.w.act);
  g.ld_x = Imax;
  g.x_sh = nullptr;
  g.perm_tok = nullptr;
  g.N_r = H;
  g.K_r = I;
  g.N_s = H;
  g.K_s = Is;
  g.sw0 = sh ? sh->down_proj : nullptr;
  g.sw1 = nullptr;
  g.out = at<void>(ws, L.w.y);
  g.ld_out = H;
  g.w = w.down;
  g.route_mode = 0;
  if (int4) {
    g.w_estride = (int64_t)H * I / 8;
    g.w_rstride = I / 8;
    g.sc = w.down_scale;
    g.s_rstride = w.group ? I / w.group : 1;
    g.s_estride = (int64_t)H * g.s_rstride;
  } else {
    g.w_estride = (int64_t)H * I;
    g.w_rstride = I;
  }
  if (!int4 && P == 1) {
    g.which = 3;
    rc = launch_gemv_ntb<T, kModeExact, kDown, kKsplitDown>(
        g, (units_max + (Is ? 1 : 0)) * (H / 16), rows_unit, sms, st, true);
  } else {
    // routed experts alone: int4, or the fp32 partial of this rank's half (P = 2:
    // one warp per tile, the same sum as one K half of the single-GPU GEMV)
    g.which = 1;
    g.raw_out = P == 2;
    if (P == 2)
      rc = !int4 ? launch_gemv_ntb<T, kModeExact, kDown, 1>(g, units_max * (H / 16), rows_unit, sms, st, true)
           : mode == kModeInt4Fused
               ? launch_gemv_ntb<T, kModeInt4Fused, kDown, 1>(g, units_max * (H / 16), rows_unit, sms, st, true)
               : launch_gemv_ntb<T, kModeInt4Dequant, kDown, 1>(g, units_max * (H / 16), rows_unit, sms, st, true);
    else
      rc = mode == kModeInt4Fused
               ? launch_gemv_q4<T, kModeInt4Fused, kDown>(g, units_max * (H / 16), T_, sms, st, true, 0, rows_unit)
               : launch_gemv_q4<T, kModeInt4Dequant, kDown>(g, units_max * (H / 16), T_, sms, st, true, 0, rows_unit);
    if (rc == TARFA_OK && Is) {
      GemvArgs gs = g;
      gs.which = 2;
      gs.raw_out = 0;
      rc = launch_gemv_ntb<T, kModeExact, kDown, kKsplitDown>(gs, H / 16, T_, sms, st, true);
    }
  }
  if (rc) return rc;
  stage_mark(3, st);

  // ---- outputs back to their sources, then the combine ----------------------
  const int64_t work = (int64_t)rows_max * (H / 4);
  const int rgrid = (int)std::max<int64_t>(1, std::min<int64_t>(2 * sms, (work + ep::kReturnThreads - 1) /
                                                                           ep::kReturnThreads));
  TARFA_CUDA(launch_k(ep::return_kernel<T>, dim3(rgrid), dim3(ep::kReturnThreads), 0, st, true, a));
  if (P == 2)
    TARFA_CUDA(launch_k(ep::combine_kernel<T, 2>, dim3((H / 8 + 31) / 32, T_), dim3(32), 0, st, true, a));
  else
    TARFA_CUDA(launch_k(ep::combine_kernel<T, 1>, dim3((H / 8 + 31) / 32, T_), dim3(32), 0, st, true, a));
  stage_mark(4, st);
  return TARFA_OK;
}

extern "C" {

int tarfa_b200_abi_version(void) { return TARFA_B200_ABI_VERSION; }

const char* tarfa_b200_last_error(void) { return g_last_error.c_str(); }

size_t tarfa_b200_workspace_size(const tarfa_moe_shape* shape, int32_t op) {
  if (!shape) return 0;
  return layout(*shape, op).total;
}

int tarfa_b200_stage_copy(void* dst, const void* src, size_t bytes, void* stream) {
  TARFA_CHECK(dst && src, "null pointer");
  TARFA_CHECK(aligned16(dst) && aligned16(src) && bytes % 16 == 0,
              "stage_copy needs 16-byte aligned pointers and a multiple of 16 bytes");
  if (bytes == 0) return TARFA_OK;
  const void* d = nullptr;
  const void* sp = nullptr;
  if (int rc = device_alias(dst, &d)) return rc;
  if (int rc = device_alias(src, &sp)) return rc;
  const size_t n16 = bytes / 16;
  const unsigned threads = 256;
  const size_t blocks = (n16 + threads - 1) / threads;
  TARFA_CHECK(blocks <= 0x7fffffffu, "stage_copy of %zu bytes is too large", bytes);
  stage_copy_kernel<<<(unsigned)blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(const_cast<void*>(d)), static_cast<const uint4*>(sp), n16);
  TARFA_CUDA(cudaGetLastError());
  return TARFA_OK;
}

int tarfa_b200_rms_norm(const void* x, const void* w, int64_t rows, int64_t cols, double eps,
                        int32_t dtype, void* out, void* stream) {
  TARFA_CHECK(x && w && out, "null argument");
  TARFA_CHECK(rows >= 0 && rows <= 0x7fffffff && cols > 0 && cols <= 16384,
              "bad shape %lld x %lld (at most 16384 columns)", (long long)rows, (long long)cols);
  if (rows == 0) return TARFA_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t smem = (size_t)cols * sizeof(double);
  if (dtype == TARFA_BF16)
    TARFA_CUDA(launch_k(rms_norm_tree_kernel<__nv_bfloat16>, dim3((unsigned)rows), dim3(256), smem, st,
                        false, static_cast<const __nv_bfloat16*>(x),
                        static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(out),
                        (int)cols, eps));
  else if (dtype == TARFA_F16)
    TARFA_CUDA(launch_k(rms_norm_tree_kernel<__half>, dim3((unsigned)rows), dim3(256), smem, st, false,
                        static_cast<const __half*>(x), static_cast<const __half*>(w),
                        static_cast<__half*>(out), (int)cols, eps));
  else
    return fail(TARFA_ERR_INVALID, "dtype %d", dtype);
  return TARFA_OK;
}

int tarfa_b200_set_decode_routing_max_tokens(int64_t tokens) {
  if (tokens < 0)
    return fail(TARFA_ERR_INVALID, "decode_routing_max_tokens %lld < 0", (long long)tokens);
  g_decode_routing_max_tokens.store(tokens);
  return TARFA_OK;
}

int tarfa_b200_set_gemm_min_tokens(int64_t tokens) {
  if (tokens < 1) return fail(TARFA_ERR_INVALID, "gemm_min_tokens %lld < 1", (long long)tokens);
  g_gemm_min_tokens.store(tokens);
  return TARFA_OK;
}

int tarfa_b200_set_stage_events(void* const* events, int32_t n) {
  if (n < 0 || n > kMaxStageEvents) return fail(TARFA_ERR_INVALID, "stage events %d", n);
  if (n > 0 && !events) return fail(TARFA_ERR_INVALID, "null events");
  for (int i = 0; i < kMaxStageEvents; ++i)
    g_stage_ev[i] = i < n ? static_cast<cudaEvent_t>(events[i]) : nullptr;
  g_stage_n = n;
  return TARFA_OK;
}

int tarfa_b200_device_status(uint32_t* status, int32_t clear, void* stream) {
  unsigned* p = nullptr;
  int sms = 0;
  if (int rc = device_info(&p, &sms)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned v = 0;
  TARFA_CUDA(cudaMemcpyAsync(&v, p, sizeof(v), cudaMemcpyDeviceToHost, st));
  TARFA_CUDA(cudaStreamSynchronize(st));
  if (clear) {
    TARFA_CUDA(cudaMemsetAsync(p, 0, sizeof(unsigned), st));
    TARFA_CUDA(cudaStreamSynchronize(st));
  }
  if (status) *status = v;
  return TARFA_OK;
}

int tarfa_b200_permute(const tarfa_moe_shape* shape, const int64_t* top_idx,
                       int32_t* seg_offsets, int32_t* perm_token, int32_t* perm_slot,
                       void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_shape(shape)) return rc;
  if (shape->tokens == 0) return TARFA_OK;
  TARFA_CHECK(top_idx && perm_token, "null top_idx / perm_token");
  const Ws L = layout(*shape, TARFA_OP_PERMUTE);
  if (workspace_bytes < L.total || !workspace)
    return fail(TARFA_ERR_WORKSPACE, "workspace %zu < %zu bytes", workspace_bytes, L.total);
  unsigned* status;
  int sms;
  if (int rc = device_info(&status, &sms)) return rc;
  PermuteOut o{seg_offsets, perm_token, perm_slot, nullptr, at<int32_t>(workspace, L.units), nullptr};
  return launch_permute<int64_t>(top_idx, (int)shape->tokens, shape->top_k, (int)shape->experts,
                                 false, o, at<int32_t>(workspace, L.phist), status,
                                 static_cast<cudaStream_t>(stream));
}

int tarfa_b200_router_topk(const tarfa_moe_shape* shape, const void* hidden,
                           const void* router_weight, const void* router_bias,
                           int64_t* top_idx, float* top_w, float* logits_out,
                           void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_shape(shape)) return rc;
  if (shape->tokens == 0) return TARFA_OK;
  TARFA_CHECK(hidden && router_weight && top_idx && top_w, "null router argument");
  TARFA_CHECK(aligned16(hidden) && aligned16(router_weight), "router operands not 16-byte aligned");
  TARFA_CHECK(shape->top_k <= shape->experts, "top_k > experts");
  const Ws L = layout(*shape, TARFA_OP_ROUTER);
  if (workspace_bytes < L.total || !workspace)
    return fail(TARFA_ERR_WORKSPACE, "workspace %zu < %zu bytes", workspace_bytes, L.total);
  unsigned* status;
  int sms;
  if (int rc = device_info(&status, &sms)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (shape->dtype == TARFA_BF16)
    return launch_router<__nv_bfloat16>(*shape, hidden, router_weight, router_bias, nullptr, L,
                                        workspace, top_idx, top_w, logits_out, false, false,
                                        status, st);
  return launch_router<__half>(*shape, hidden, router_weight, router_bias, nullptr, L, workspace,
                               top_idx, top_w, logits_out, false, false, status, st);
}

int tarfa_b200_experts_forward(const tarfa_moe_shape* shape, const void* hidden,
                               const int64_t* top_idx, const float* top_w,
                               const tarfa_moe_weights* weights, void* out,
                               void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_shape(shape)) return rc;
  if (int rc = check_weights(shape, weights)) return rc;
  if (shape->tokens == 0) return TARFA_OK;
  TARFA_CHECK(hidden && top_idx && top_w && out, "null argument");
  TARFA_CHECK(aligned16(hidden) && aligned16(out), "hidden / out not 16-byte aligned");
  const Ws L = layout(*shape, TARFA_OP_EXPERTS);
  if (workspace_bytes < L.total || !workspace)
    return fail(TARFA_ERR_WORKSPACE, "workspace %zu < %zu bytes", workspace_bytes, L.total);
  unsigned* status;
  int sms;
  if (int rc = device_info(&status, &sms)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int T_ = (int)shape->tokens, K = shape->top_k, E = (int)shape->experts;
  PermuteOut o{nullptr, at<int32_t>(workspace, L.perm_tok), at<int32_t>(workspace, L.perm_slot),
               at<int32_t>(workspace, L.route_row), at<int32_t>(workspace, L.units),
               at<int32_t>(workspace, L.idx32)};
  stage_mark(0, st);
  if (int rc = launch_permute<int64_t>(top_idx, T_, K, E, false, o, at<int32_t>(workspace, L.phist),
                                      status, st))
    return rc;
  stage_mark(1, st);
  const bool int4 = weights->kind == TARFA_W_INT4;
  int rc;
  if (shape->dtype == TARFA_BF16) {
    rc = run_experts<__nv_bfloat16>(*shape, hidden, *weights, nullptr, L, workspace, out, status, sms, st);
    if (!rc) rc = run_combine<__nv_bfloat16>(*shape, L, workspace, top_w, int4, false, use_gemm(*shape, *weights, 0), out, st);
  } else {
    rc = run_experts<__half>(*shape, hidden, *weights, nullptr, L, workspace, out, status, sms, st);
    if (!rc) rc = run_combine<__half>(*shape, L, workspace, top_w, int4, false, use_gemm(*shape, *weights, 0), out, st);
  }
  return rc;
}

int tarfa_b200_moe_layer(const tarfa_moe_shape* shape, const void* hidden,
                         const void* router_weight, const void* router_bias,
                         const tarfa_moe_weights* weights, const tarfa_shared_expert* shared,
                         void* out, int64_t* top_idx_out, float* top_w_out,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_layer_args(shape, hidden, router_weight, weights, shared, out)) return rc;
  if (shape->tokens == 0) return TARFA_OK;
  const bool has_shared = shared && shape->shared_inter > 0;
  tarfa_moe_shape s = *shape;
  if (!has_shared) s.shared_inter = 0;
  const Ws L = layout(s, TARFA_OP_MOE_LAYER);
  if (workspace_bytes < L.total || !workspace)
    return fail(TARFA_ERR_WORKSPACE, "workspace %zu < %zu bytes", workspace_bytes, L.total);
  unsigned* status;
  int sms;
  if (int rc = device_info(&status, &sms)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool int4 = weights->kind == TARFA_W_INT4;
  const tarfa_shared_expert* sh = has_shared ? shared : nullptr;
  int rc;
  stage_mark(0, st);
  if (use_decode_routing(s, *weights)) {
    return s.dtype == TARFA_BF16
               ? run_decode_layer<__nv_bfloat16>(s, hidden, router_weight, router_bias, *weights,
                                                 sh, out, top_idx_out, top_w_out, L, workspace,
                                                 status, sms, st)
               : run_decode_layer<__half>(s, hidden, router_weight, router_bias, *weights, sh, out,
                                          top_idx_out, top_w_out, L, workspace, status, sms, st);
  }
  if (s.dtype == TARFA_BF16) {
    rc = launch_router<__nv_bfloat16>(s, hidden, router_weight, router_bias,
                                      sh ? sh->gate_weight : nullptr, L, workspace, top_idx_out,
                                      top_w_out, nullptr, true, sh != nullptr, status, st);
    if (!rc) stage_mark(1, st);
    if (!rc) rc = run_experts<__nv_bfloat16>(s, hidden, *weights, sh, L, workspace, out, status, sms, st);
    if (!rc) rc = run_combine<__nv_bfloat16>(s, L, workspace, at<float>(workspace, L.topw), int4, sh != nullptr, use_gemm(s, *weights, s.shared_inter), out, st);
  } else {
    rc = launch_router<__half>(s, hidden, router_weight, router_bias,
                               sh ? sh->gate_weight : nullptr, L, workspace, top_idx_out,
                               top_w_out, nullptr, true, sh != nullptr, status, st);
    if (!rc) stage_mark(1, st);
    if (!rc) rc = run_experts<__half>(s, hidden, *weights, sh, L, workspace, out, status, sms, st);
    if (!rc) rc = run_combine<__half>(s, L, workspace, at<float>(workspace, L.topw), int4, sh != nullptr, use_gemm(s, *weights, s.shared_inter), out, st);
  }
  return rc;
}

int tarfa_b200_shared_expert(const tarfa_moe_shape* shape, const void* hidden,
                             const tarfa_shared_expert* shared, void* out, void* workspace,
                             size_t workspace_bytes, void* stream) {
  if (int rc = check_shape(shape)) return rc;
  if (shape->tokens == 0) return TARFA_OK;
  TARFA_CHECK(shape->shared_inter > 0, "shared_inter must be > 0");
  TARFA_CHECK(hidden && out && shared && shared->gate_proj && shared->up_proj &&
                  shared->down_proj && shared->gate_weight,
              "null argument");
  TARFA_CHECK(aligned16(hidden) && aligned16(shared->gate_proj) && aligned16(shared->up_proj) &&
                  aligned16(shared->down_proj) && aligned16(shared->gate_weight),
              "operands not 16-byte aligned");
  const Ws L = layout(*shape, TARFA_OP_SHARED);
  if (workspace_bytes < L.total || !workspace)
    return fail(TARFA_ERR_WORKSPACE, "workspace %zu < %zu bytes", workspace_bytes, L.total);
  unsigned* status;
  int sms;
  if (int rc = device_info(&status, &sms)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int T_ = (int)shape->tokens, H = (int)shape->hidden, Is = (int)shape->shared_inter;
  GemvArgs g{};
  g.units = at<int32_t>(workspace, L.units);
  g.which = 2;
  g.E = (int)shape->experts;
  g.status = status;
  g.x = hidden;
  g.ld_x = H;
  g.perm_tok = at<int32_t>(workspace, L.perm_tok);
  g.N_s = Is;
  g.K_s = H;
  g.sw0 = shared->gate_proj;
  g.sw1 = shared->up_proj;
  g.out = at<void>(workspace, L.act);
  g.ld_out = Is;
  auto run = [&](auto tag) -> int {
    using T = decltype(tag);
    shared_prep_kernel<T><<<(T_ + 7) / 8, 256, 0, st>>>(
        static_cast<const T*>(hidden), static_cast<const T*>(shared->gate_weight), T_, H,
        at<int32_t>(workspace, L.units), at<int32_t>(workspace, L.perm_tok),
        at<float>(workspace, L.gate_logit));
    TARFA_CUDA(cudaGetLastError());
    if (int rc = launch_gemv_ntb<T, kModeExact, kGateUp, kKsplitGateUp>(g, Is / 8, T_, sms, st)) return rc;
    GemvArgs d = g;
    d.x = at<void>(workspace, L.act);
    d.ld_x = Is;
    d.perm_tok = nullptr;
    d.N_s = H;
    d.K_s = Is;
    d.sw0 = shared->down_proj;
    d.sw1 = nullptr;
    d.out = at<void>(workspace, L.y);
    d.ld_out = H;
    if (int rc = launch_gemv_ntb<T, kModeExact, kDown, kKsplitDown>(d, H / 16, T_, sms, st)) return rc;
    shared_finish_kernel<T><<<dim3((H + 255) / 256, T_), 256, 0, st>>>(
        at<float>(workspace, L.y), at<float>(workspace, L.gate_logit), T_, H, static_cast<T*>(out));
    TARFA_CUDA(cudaGetLastError());
    return TARFA_OK;
  };
  return shape->dtype == TARFA_BF16 ? run(__nv_bfloat16{}) : run(__half{});
}

int tarfa_b200_combine_routes(const tarfa_moe_shape* shape, const void* y_routes,
                              const int64_t* top_idx, const float* top_w,
                              const void* shared_gated, void* out, void* stream) {
  if (int rc = check_shape(shape)) return rc;
  if (shape->tokens == 0) return TARFA_OK;
  TARFA_CHECK(y_routes && top_idx && top_w && out, "null argument");
  const int T_ = (int)shape->tokens, K = shape->top_k, H = (int)shape->hidden, E = (int)shape->experts;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((H + 255) / 256, T_);
  if (shape->dtype == TARFA_BF16)
    combine_routes_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(y_routes), top_idx, top_w,
        static_cast<const __nv_bfloat16*>(shared_gated), T_, K, H, E, static_cast<__nv_bfloat16*>(out));
  else
    combine_routes_kernel<__half><<<grid, 256, 0, st>>>(
        static_cast<const __half*>(y_routes), top_idx, top_w, static_cast<const __half*>(shared_gated),
        T_, K, H, E, static_cast<__half*>(out));
  TARFA_CUDA(cudaGetLastError());
  return TARFA_OK;
}

// The whole layer with the library's own static scratch instead of a
// caller-supplied workspace (see the header for who needs this and the rules).
int tarfa_b200_moe_layer_noalloc(const tarfa_moe_shape* shape, const void* hidden,
                                 const void* router_weight, const void* router_bias,
                                 const tarfa_moe_weights* weights,
                                 const tarfa_shared_expert* shared, void* out,
                                 int64_t* top_idx_out, float* top_w_out, void* stream) {
  // a rejected or empty call leaves the shared scratch untouched
  if (int rc = check_layer_args(shape, hidden, router_weight, weights, shared, out)) return rc;
  if (shape->tokens == 0) return TARFA_OK;
  tarfa_moe_shape s = *shape;
  if (!(shared && shape->shared_inter > 0)) s.shared_inter = 0;
  const Ws L = layout(s, TARFA_OP_MOE_LAYER);
  if (L.total > kNoAllocScratchBytes)
    return fail(TARFA_ERR_UNSUPPORTED,
                "moe_layer_noalloc: this shape needs %zu bytes of scratch; the static scratch "
                "holds %zu bytes (use tarfa_b200_moe_layer with a workspace)",
                L.total, kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the kernels' counters (router completion, grid barrier, per-block completion)
  // must start at zero, whatever the last call left
  TARFA_CUDA(cudaMemsetAsync(scratch, 0, kZeroHeaderBytes, st));
  return tarfa_b200_moe_layer(shape, hidden, router_weight, router_bias, weights, shared, out,
                              top_idx_out, top_w_out, scratch, kNoAllocScratchBytes, stream);
}

int tarfa_b200_dequant_int4(const int32_t* packed, const void* scale, int64_t rows, int64_t cols,
                            int32_t group, int32_t dtype, void* out, void* stream) {
  TARFA_CHECK(packed && scale && out, "null argument");
  TARFA_CHECK(rows >= 0 && cols > 0 && cols % 8 == 0, "bad shape %lld x %lld", (long long)rows,
              (long long)cols);
  TARFA_CHECK(group == 0 || (group % 8 == 0 && cols % group == 0), "bad group %d", group);
  TARFA_CHECK(aligned16(out), "out not 16-byte aligned");
  if (rows == 0) return TARFA_OK;
  const int64_t n = rows * (cols / 8);
  const int threads = 256;
  const int64_t grid = (n + threads - 1) / threads;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TARFA_BF16)
    dequant_int4_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>(
        reinterpret_cast<const uint32_t*>(packed), static_cast<const __nv_bfloat16*>(scale), rows,
        cols, group, static_cast<__nv_bfloat16*>(out));
  else if (dtype == TARFA_F16)
    dequant_int4_kernel<__half><<<grid, threads, 0, st>>>(
        reinterpret_cast<const uint32_t*>(packed), static_cast<const __half*>(scale), rows, cols,
        group, static_cast<__half*>(out));
  else
    return fail(TARFA_ERR_INVALID, "dtype %d", dtype);
  TARFA_CUDA(cudaGetLastError());
  return TARFA_OK;
}

int tarfa_b200_quantize_int4(const void* w, int64_t rows, int64_t cols, int32_t group,
                             int32_t* packed, void* scale, void* stream) {
  TARFA_CHECK(w && packed && scale, "null argument");
  TARFA_CHECK(rows >= 0 && cols > 0, "bad shape");
  TARFA_CHECK(group % 128 == 0 && group >= 128 && group <= 1024 && cols % group == 0,
              "group %d must be a multiple of 128 in [128, 1024] dividing cols", group);
  TARFA_CHECK(aligned16(w), "w not 16-byte aligned");
  if (rows == 0) return TARFA_OK;
  const int64_t warps = rows * (cols / group);
  const int threads = 256;
  const int64_t grid = (warps * 32 + threads - 1) / threads;
  quantize_int4_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(w), rows, cols, group, reinterpret_cast<uint32_t*>(packed),
      static_cast<__nv_bfloat16*>(scale));
  TARFA_CUDA(cudaGetLastError());
  return TARFA_OK;
}

// ---- expert parallelism over peer memory ------------------------------------
size_t tarfa_b200_ep_box_bytes(const tarfa_moe_shape* shape, int32_t world, int64_t max_tokens) {
  if (!shape || world < 1 || max_tokens < 1) return 0;
  const int S = (int)(max_tokens * shape->top_k);
  return ep::box_layout(world, S, (int)shape->hidden).total;
}

size_t tarfa_b200_ep_workspace_size(const tarfa_moe_shape* shape, int32_t world, int64_t max_tokens) {
  if (!shape || world < 1 || max_tokens < 1) return 0;
  return ep_layout(*shape, world, max_tokens).w.total;
}

int tarfa_b200_ep_box_alloc(size_t bytes, void** box, void* ipc_handle) {
  TARFA_CHECK(box && bytes > 0, "ep_box_alloc: null box or zero bytes");
  void* p = nullptr;
  TARFA_CUDA(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess && ipc_handle) {
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e == cudaSuccess) std::memcpy(ipc_handle, &h, sizeof(h));
  }
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(TARFA_ERR_CUDA, "ep_box_alloc: %s", cudaGetErrorString(e));
  }
  *box = p;
  return TARFA_OK;
}

int tarfa_b200_ep_box_open(const void* ipc_handle, void** box) {
  TARFA_CHECK(ipc_handle && box, "ep_box_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  TARFA_CUDA(cudaIpcOpenMemHandle(box, h, cudaIpcMemLazyEnablePeerAccess));
  return TARFA_OK;
}

int tarfa_b200_ep_box_close(void* box) {
  TARFA_CHECK(box, "ep_box_close: null box");
  TARFA_CUDA(cudaIpcCloseMemHandle(box));
  return TARFA_OK;
}

int tarfa_b200_ep_box_free(void* box) {
  TARFA_CHECK(box, "ep_box_free: null box");
  TARFA_CUDA(cudaFree(box));
  return TARFA_OK;
}

int tarfa_b200_ep_moe_layer(const tarfa_moe_shape* shape, const void* hidden,
                            const void* router_weight, const void* router_bias,
                            const tarfa_moe_weights* weights, const tarfa_shared_expert* shared,
                            const tarfa_ep_group* group, void* out, int64_t* top_idx_out,
                            float* top_w_out, void* workspace, size_t workspace_bytes,
                            void* stream) {
  if (int rc = check_shape(shape)) return rc;
  if (int rc = check_ep(shape, group)) return rc;
  tarfa_moe_shape local = *shape;
  local.experts = shape->experts / (group->world / group->tp);
  local.inter = shape->inter / group->tp;
  if (int rc = check_weights(&local, weights)) return rc;
  if (group->tp == 2 && weights->kind == TARFA_W_INT4)
    TARFA_CHECK(weights->group > 0, "ep tp 2 with int4 experts needs group scales (group > 0)");
  TARFA_CHECK(shape->tokens >= 1 && shape->tokens <= group->max_tokens,
              "ep tokens %lld not in [1, max_tokens = %lld]", (long long)shape->tokens,
              (long long)group->max_tokens);
  TARFA_CHECK(hidden && router_weight && out, "null argument");
  TARFA_CHECK(aligned16(hidden) && aligned16(router_weight) && aligned16(out),
              "operands not 16-byte aligned");
  TARFA_CHECK(shape->top_k <= shape->experts, "top_k > experts");
  const bool has_shared = shared && shape->shared_inter > 0;
  if (has_shared) {
    TARFA_CHECK(shared->gate_proj && shared->up_proj && shared->down_proj && shared->gate_weight,
                "null shared-expert weight");
    TARFA_CHECK(aligned16(shared->gate_proj) && aligned16(shared->up_proj) &&
                    aligned16(shared->down_proj) && aligned16(shared->gate_weight),
                "shared-expert weights not 16-byte aligned");
  }
  tarfa_moe_shape s = *shape;
  if (!has_shared) s.shared_inter = 0;
  const EpWs L = ep_layout(s, group->world, group->max_tokens);
  if (workspace_bytes < L.w.total || !workspace)
    return fail(TARFA_ERR_WORKSPACE, "workspace %zu < %zu bytes", workspace_bytes, L.w.total);
  unsigned* status;
  int sms;
  if (int rc = device_info(&status, &sms)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const tarfa_shared_expert* sh = has_shared ? shared : nullptr;
  return s.dtype == TARFA_BF16
             ? run_ep_layer<__nv_bfloat16>(s, hidden, router_weight, router_bias, *weights, sh,
                                           *group, out, top_idx_out, top_w_out, L, workspace,
                                           status, sms, st)
             : run_ep_layer<__half>(s, hidden, router_weight, router_bias, *weights, sh, *group,
                                    out, top_idx_out, top_w_out, L, workspace, status, sms, st);
}

}  // extern "C"
