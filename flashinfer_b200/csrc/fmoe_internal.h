// fmoe_internal.h -- shared constants, workspace layout and kernel launch declarations.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/fmoe.h"

namespace fmoe {

constexpr int kBlock = 128;          // scale block edge (activations: per token per 128 K;
                                     // weights: 128x128)
constexpr int kTopK = 8;
constexpr int kGroups = 8;
constexpr int kTopKGroups = 4;
constexpr int kExpertsGlobal = 256;
constexpr int kMaxLocalExperts = 256;
constexpr int kTileM = 128;          // slots per GEMM tile (one expert per tile)
constexpr int kTileN = 256;          // weight rows per GEMM tile
constexpr int kMaxSplitUnits = 1024; // split-K partial tiles the workspace holds
constexpr int kMaxSplit = 8;

// Plan header words (int32, written by the plan kernel).
enum PlanWord {
  kPlanPairs = 0,      // P: routed (token, local expert) pairs
  kPlanPadded = 1,     // slots incl. per-expert padding to 128
  kPlanMTiles = 2,     // 128-slot tiles
  kPlanSplit1 = 3,     // GEMM1 K splits
  kPlanUnits1 = 4,     // GEMM1 work units = tiles1 * split1
  kPlanSplit2 = 5,
  kPlanUnits2 = 6,
  kPlanTiles1 = 7,
  kPlanTiles2 = 8,
  kPlanWords = 16,
};

struct Layout {
  size_t total;
  size_t status, plan, topk_ids, topk_w, expert_count, expert_base, slot_token, slot_weight;
  size_t token_slot, token_weight, a_perm, a_scale_t, h_hi, h_lo, h_scale_t, y_rows, y_scale;
  size_t partials, counters, block_hist, block_off;
  int64_t cap;          // padded slot capacity
  int64_t partial_rows; // rows stored per split-K partial tile (<= 128)
  int tpb;              // tokens per routing block
  int nblocks;          // routing blocks = ceil(T / tpb)
};

// Tokens per routing block: the scan kernel keeps one count per (block, local expert) in
// shared memory, at most kMaxBlockCounts of them.
constexpr int kMaxBlockCounts = 8192;
__host__ __device__ inline int routing_tpb(int T, int E) {
  int tpb = 8;
  while (static_cast<long>((T + tpb - 1) / tpb) * E > kMaxBlockCounts && tpb < (1 << 20)) tpb *= 2;
  return tpb;
}

// Host + device: compute the workspace layout.
__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

__host__ __device__ inline Layout make_layout(int T, int E, int H, int I) {
  Layout L{};
  const int64_t picks = (int64_t)(E < kTopK ? E : kTopK);
  const int64_t pmax = (int64_t)T * picks;
  const int64_t pad = 127 * (pmax < E ? pmax : (int64_t)E);
  L.cap = (int64_t)align_up((size_t)(pmax + pad), kTileM);
  L.partial_rows = T < kTileM ? (T > 0 ? T : 1) : kTileM;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  L.status = take(16);
  L.plan = take(kPlanWords * 4);
  L.topk_ids = take((size_t)T * kTopK * 4);
  L.topk_w = take((size_t)T * kTopK * 4);
  L.expert_count = take((size_t)E * 4);
  L.expert_base = take((size_t)(E + 1) * 4);
  L.slot_token = take((size_t)L.cap * 4);
  L.slot_weight = take((size_t)L.cap * 4);
  L.token_slot = take((size_t)T * kTopK * 4);
  L.token_weight = take((size_t)T * kTopK * 4);
  L.a_perm = take((size_t)L.cap * H);
  L.a_scale_t = take((size_t)(H / kBlock) * L.cap * 4);
  L.h_hi = take((size_t)L.cap * I);
  L.h_lo = take((size_t)L.cap * I);
  L.h_scale_t = take((size_t)(I / kBlock) * L.cap * 4);
  L.y_rows = take((size_t)L.cap * H * 2);
  L.y_scale = take((size_t)L.cap * (H / kTileN) * 4);
  L.partials = take((size_t)kMaxSplitUnits * L.partial_rows * kTileN * 4);
  L.counters = take((size_t)2 * kMaxSplitUnits * 4);
  L.tpb = routing_tpb(T, E);
  L.nblocks = T > 0 ? (T + L.tpb - 1) / L.tpb : 0;
  L.block_hist = take((size_t)(L.nblocks > 0 ? L.nblocks : 1) * E * 4);
  L.block_off = take((size_t)(L.nblocks > 0 ? L.nblocks : 1) * E * 4);
  L.total = o;
  return L;
}

// Routing method and top_k of a call, packed for the routing kernels: method | top_k << 8.
__host__ __device__ constexpr int route_mode(int method, int top_k) { return method | (top_k << 8); }
constexpr int kRouteDeepSeek = route_mode(FMOE_ROUTING_DEEPSEEK_V3, kTopK);

struct RunParams {
  // inputs
  const void* logits;
  int logits_dtype;
  const void* bias;
  int bias_dtype;
  const uint8_t* hidden;
  const float* hidden_scale;   // [H/128, T]
  const uint8_t* w1;           // [E, 2I, H] e4m3
  const float* w1_scale;       // [E, 2I/128, H/128]
  const uint8_t* w2;           // [E, H, I] e4m3
  const float* w2_scale;       // [E, H/128, I/128]
  void* output;                // [T, H] bf16, or fp32 (out_mode FMOE_OUT_F32)
  int T, H, I, E, local_start;
  float rsf;
  int route_mode;              // route_mode(method, top_k)
  // pre-routed call (expert parallelism): picks given, optional regions of valid tokens
  const int32_t* in_ids;       // [T, 8] global ids or nullptr
  const float* in_w;           // [T, 8]
  const int32_t* region_counts;
  int region_tokens;
  int out_mode;                // FMOE_OUT_*
  void* region_out[FMOE_EP_MAX_RANKS];
  // failure-path test (fmoe_debug_arm_timeout): GEMM 1 or 2 waits on a barrier nothing arrives
  // on, every GEMM wait limited to wait_ns (0 = the default limit)
  int inject_gemm;
  unsigned long long wait_ns;
  // workspace
  uint8_t* ws;
  Layout L;
  int num_sms;
};

// Launchers (fmoe_kernels.cu / fmoe_gemm.cu). Return cudaGetLastError() of the launch.
cudaError_t launch_route(const void* logits, int logits_dtype, const void* bias, int bias_dtype,
                         int T, float rsf, int32_t* topk_ids, float* topk_w, cudaStream_t s);
// routing + per-block local-expert histogram -> scan -> scatter + activation gather
cudaError_t launch_route_hist(const RunParams& p, cudaStream_t s);
cudaError_t launch_scan(const RunParams& p, cudaStream_t s);
cudaError_t launch_scatter_gather(const RunParams& p, cudaStream_t s);
cudaError_t launch_gather(const RunParams& p, cudaStream_t s);
// Split-K (GEMM units over K ranges) only for T <= kSplitMaxT, where a call can have fewer tiles
// than SMs; the split partial tiles are finished by launch_split_finish(kind) after each GEMM.
// The finish launch itself costs about 4 us even when the plan picks no split: its CTAs wait for
// the whole GEMM1 grid, so GEMM2's CTAs no longer start (and prefetch weights) as GEMM1's CTAs
// leave. At 16 <= T <= 32 the plan had picked no split anyway (8-9 active experts, 128-144 GEMM1
// tiles): T=16 83.1 -> 79.9 us and T=32 86.1 -> 83.1 us without the launch; at T=8 the split is
// worth it (99.9 us with it, 114.8 without).
constexpr int kSplitMaxT = 8;
cudaError_t launch_split_finish(const RunParams& p, int kind, cudaStream_t s);
// T <= kGemvMaxT (fmoe_gemv.cu): after the plan kernel, GEMM1 + SwiGLU and GEMM2 + the combine as
// weight-streaming matrix-vector kernels on the CUDA cores (launch_gemv(p, 1), then 2), for calls
// that gemv_eligible accepts (plain routed calls with a bf16 or fp32 output). Same-box graph
// timings against the grouped GEMMs: T=1 (one active expert) 29.7 -> 21.7 us, T=2 13.8 -> 10.4;
// with three or more active experts the grouped GEMMs stream weights faster (T=3: 59.0 vs 66.3,
// T=4: 46.2 vs 45.9, T=8: 98.8 vs 148.3).
constexpr int kGemvMaxT = 2;
bool gemv_eligible(const RunParams& p);
cudaError_t launch_gemv(const RunParams& p, int which, cudaStream_t s);
// T <= kSmallT: routing + histogram + plan + scatter in one kernel (replaces the three above):
// one CTA (one warp per token) per 8 tokens, up to 8 CTAs in one cluster exchanging counts
// through distributed shared memory
constexpr int kSmallTokensPerCta = 8;
constexpr int kSmallT = 8 * kSmallTokensPerCta;
cudaError_t launch_plan_small(const RunParams& p, cudaStream_t s);
// GEMM2 for T <= kPackedMaxT (every tile then has at most 64 routed slots) packs the hi and lo
// terms of a tile's first 64 slots into one A tile; tm_hi and tm_lo then have 64-row boxes.
constexpr int kPackedMaxT = 64;
cudaError_t launch_gemm1(const RunParams& p, const CUtensorMap& tm_a, const CUtensorMap& tm_w1,
                         const CUtensorMap& tm_sa, cudaStream_t s);
cudaError_t launch_gemm2(const RunParams& p, const CUtensorMap& tm_hi, const CUtensorMap& tm_lo,
                         const CUtensorMap& tm_w2, const CUtensorMap& tm_sa, cudaStream_t s);
cudaError_t launch_combine(const RunParams& p, cudaStream_t s);
// pre-routed: copies the given picks into the workspace (-1 for tokens outside their region's
// count) with the per-block histogram, in place of launch_route_hist
cudaError_t launch_hist_given(const RunParams& p, cudaStream_t s);
// bf16 [T, H] -> e4m3 [T, H] + fp32 scales [H/128, T] (fmoe_quant.cu)
cudaError_t launch_quantize_act(const void* x, int T, int H, void* q, float* scale_t,
                                int num_sms, cudaStream_t s);

// Routing + permutation with every buffer passed explicitly (used by the entry point whose
// scratch lives in a statically allocated device array).
struct PermuteBuffers {
  // scratch
  int32_t* topk_ids;      // [T, 8]
  float* topk_w;          // [T, 8]
  int32_t* block_hist;    // [nblocks, E]
  int32_t* block_off;     // [nblocks, E]
  int32_t* plan;          // [kPlanWords]
  int32_t* counters;      // [2 * kMaxSplitUnits]
  int32_t* status;        // [1]
  // outputs
  int32_t* expert_count;  // [E]
  int32_t* expert_base;   // [E + 1]
  int32_t* slot_token;    // [cap]
  float* slot_weight;     // [cap]
  int32_t* token_slot;    // [T, 8]
  float* token_weight;    // [T, 8]
};
cudaError_t launch_route_permute(const void* logits, int logits_dtype, const void* bias,
                                 int bias_dtype, int T, int E, int local_start, float rsf,
                                 int H, int I, int num_sms, const PermuteBuffers& b,
                                 cudaStream_t s);

// ---------------------------------------------------------------- output stores
// Eight fp32 values of an output row as bf16 (round to nearest even) or fp32; v counts groups of
// eight columns.
__device__ __forceinline__ void store8(__nv_bfloat16* out, size_t v, const float (&acc)[8]) {
  uint4 o;
  __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i) oh[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
  reinterpret_cast<uint4*>(out)[v] = o;
}
__device__ __forceinline__ void store8(float* out, size_t v, const float (&acc)[8]) {
  float4* o = reinterpret_cast<float4*>(out) + 2 * v;
  o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

// ---------------------------------------------------------------- 256-bit global accesses
__device__ __forceinline__ void st_global_v8(void* p, const uint32_t (&w)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(w[0]), "r"(w[1]),
               "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

__device__ __forceinline__ void ld_global_nc_v8(const void* p, uint32_t (&w)[8]) {
  asm volatile("ld.global.nc.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]),
                 "=r"(w[6]), "=r"(w[7])
               : "l"(p));
}

// ---------------------------------------------------------------- programmatic dependent launch
// Every kernel of the path is launched with programmatic stream serialisation. A kernel first
// lets the next kernel in the stream be scheduled (its CTAs are placed as resources free up and
// park in griddepcontrol.wait), then waits for the previous grid to complete and its memory to
// become visible before it reads anything. Results are the same as plain stream order; the
// launch latency between the seven kernels of a call overlaps the previous kernel's tail.
__device__ __forceinline__ void pdl_begin() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// The same with the order reversed, for a kernel that a GEMM follows: the GEMM reads the work
// plan before its own wait, and when it starts, its predecessor has passed this wait, so every
// earlier kernel of the call (the plan kernel included) has completed.
__device__ __forceinline__ void pdl_begin_in_order() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// The same with a thread-block cluster of cluster_x CTAs along x (grid.x a multiple of it).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block,
                                      size_t smem, cudaStream_t s, int cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace fmoe
