// fmoe_api.cu -- the C ABI (include/fmoe.h): argument checks, workspace layout, TMA tensor
// maps and the stream-ordered launch chain route -> plan -> gather -> GEMM1 -> GEMM2 -> combine.
//
// Replaces the host driver of the reference operator, solution/triton/kernel.py:600-825. Where
// the reference synchronises three times per call (.item() at kernel.py:572, :718, :773) to size
// its grids and temporaries, here the plan kernel writes the schedule to device memory and the
// persistent GEMM kernels read it, so a call never waits on the device.
#include <cuda.h>
#include <cuda_runtime.h>
#include <string.h>

#include <mutex>

#include "fmoe_internal.h"

namespace fmoe {
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D fp32 tensor map over a row-major [rows, cols] matrix, box = box_cols x 1 (unswizzled).
bool make_tmap_f32_rows(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows,
                        uint32_t box_cols) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 4};
  const cuuint32_t box[2] = {box_cols, 1};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D uint8 tensor map over a row-major [rows, cols] matrix with a 128-byte-swizzled box.
bool make_tmap_u8(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows,
                  uint64_t row_stride, uint32_t box_cols, uint32_t box_rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_stride};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct DeviceInfo {
  int sms = 0;
  int major = 0;
  int minor = 0;
  int device = -1;
};

int device_info(DeviceInfo* out) {
  static DeviceInfo cache[64];
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FMOE_ERR_CUDA;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev].sms == 0) {
    DeviceInfo d;
    if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return FMOE_ERR_CUDA;
    d.device = dev;
    cache[dev] = d;
  }
  *out = cache[dev];
  return FMOE_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_sizes(int T, int E, int H, int I) {
  if (T < 0 || E < 1 || E > kMaxLocalExperts) return FMOE_ERR_SHAPE;
  if (H <= 0 || I <= 0 || H % kTileN != 0 || I % kBlock != 0) return FMOE_ERR_SHAPE;
  if (H / kBlock > 64 || I / kBlock > 64) return FMOE_ERR_SHAPE;  // GEMM weight-scale tables
  return FMOE_OK;
}

int validate(const FmoeArgs* a) {
  if (!a) return FMOE_ERR_NULL;
  int rc = check_sizes(a->num_tokens, a->num_local_experts, a->hidden_size,
                       a->intermediate_size);
  if (rc) return rc;
  if (a->num_experts != kExpertsGlobal) return FMOE_ERR_SHAPE;
  switch (a->routing_method) {
    case FMOE_ROUTING_DEEPSEEK_V3:
      if (a->top_k != kTopK || a->n_group != kGroups || a->topk_group != kTopKGroups)
        return FMOE_ERR_SHAPE;
      break;
    case FMOE_ROUTING_LLAMA4:
      if (a->top_k != 1) return FMOE_ERR_SHAPE;
      break;
    case FMOE_ROUTING_DEFAULT:
    case FMOE_ROUTING_RENORMALIZE:
    case FMOE_ROUTING_RENORMALIZE_NAIVE:
    case FMOE_ROUTING_TOPK:
      if (a->top_k < 1 || a->top_k > kTopK) return FMOE_ERR_SHAPE;
      break;
    default:
      return FMOE_ERR_SHAPE;
  }
  if (a->local_expert_offset < 0 ||
      a->local_expert_offset + a->num_local_experts > a->num_experts)
    return FMOE_ERR_OFFSET;
  if (a->gemm_path != FMOE_PATH_AUTO && a->gemm_path != FMOE_PATH_GEMM) return FMOE_ERR_SHAPE;
  const bool pre_routed = a->topk_ids != nullptr;
  if ((!pre_routed && ((a->logits_dtype != FMOE_DTYPE_F32 && a->logits_dtype != FMOE_DTYPE_BF16) ||
                       (a->bias_dtype != FMOE_DTYPE_F32 && a->bias_dtype != FMOE_DTYPE_BF16))) ||
      (a->output_dtype != FMOE_OUT_BF16 && a->output_dtype != FMOE_OUT_F32 &&
       a->output_dtype != FMOE_OUT_F16S))
    return FMOE_ERR_DTYPE;
  // partial rows and token regions only for pre-routed calls (the receiving side of expert
  // parallelism); regions must tile the tokens, at most one per rank
  if (a->output_dtype == FMOE_OUT_F16S && !pre_routed) return FMOE_ERR_DTYPE;
  if (a->region_counts != nullptr &&
      (!pre_routed || a->region_tokens <= 0 || a->num_tokens % a->region_tokens != 0 ||
       a->num_tokens / a->region_tokens > FMOE_EP_MAX_RANKS))
    return FMOE_ERR_SHAPE;
  if (a->num_tokens == 0) return FMOE_OK;
  const void* ptrs[] = {pre_routed ? a->topk_ids : a->routing_logits,
                        pre_routed ? static_cast<const void*>(a->topk_weights) : a->routing_bias,
                        a->hidden_states, a->hidden_states_scale, a->gemm1_weights,
                        a->gemm1_weights_scale, a->gemm2_weights, a->gemm2_weights_scale,
                        a->output_dtype == FMOE_OUT_F16S ? a->region_output[0] : a->output,
                        a->workspace};
  for (const void* p : ptrs)
    if (!p) return FMOE_ERR_NULL;
  for (const void* p : ptrs)
    if (!aligned16(p)) return FMOE_ERR_ALIGN;
  if (a->output_dtype == FMOE_OUT_F16S) {
    const int regions = a->region_counts ? a->num_tokens / a->region_tokens : 1;
    for (int r = 0; r < regions; ++r) {
      if (!a->region_output[r]) return FMOE_ERR_NULL;
      // rows are written with 32-byte stores (FMOE_EP_ROW_BYTES is a multiple of 32)
      if ((reinterpret_cast<uintptr_t>(a->region_output[r]) & 31u) != 0) return FMOE_ERR_ALIGN;
    }
  }
  return FMOE_OK;
}

// One-shot failure-path injection armed by fmoe_debug_arm_timeout for this host thread's next
// fmoe_run.
struct ArmedTimeout {
  int gemm = 0;
  unsigned long long wait_ns = 0;
};
thread_local ArmedTimeout g_armed;

}  // namespace
}  // namespace fmoe

using namespace fmoe;

extern "C" {

int fmoe_debug_arm_timeout(int32_t gemm, uint64_t wait_ns) {
  if (gemm != 1 && gemm != 2) return FMOE_ERR_SHAPE;
  if (wait_ns < 100000ull || wait_ns > 2000000000ull) return FMOE_ERR_SHAPE;
  g_armed.gemm = gemm;
  g_armed.wait_ns = wait_ns;
  return FMOE_OK;
}

const char* fmoe_version(void) { return "flashinfer_b200 fmoe 0.1 (sm_100a, tcgen05)"; }

int fmoe_device_sm_count(int32_t* sms) {
  if (!sms) return FMOE_ERR_NULL;
  DeviceInfo d;
  int rc = device_info(&d);
  if (rc) return rc;
  *sms = d.sms;
  return FMOE_OK;
}

int fmoe_workspace_layout(int32_t T, int32_t E, int32_t H, int32_t I, FmoeLayout* out) {
  if (!out) return FMOE_ERR_NULL;
  int rc = check_sizes(T, E, H, I);
  if (rc) return rc;
  const Layout L = make_layout(T, E, H, I);
  memset(out, 0, sizeof(*out));
  out->total_bytes = L.total;
  out->status = L.status;
  out->plan = L.plan;
  out->topk_ids = L.topk_ids;
  out->topk_weights = L.topk_w;
  out->expert_count = L.expert_count;
  out->expert_base = L.expert_base;
  out->slot_token = L.slot_token;
  out->slot_weight = L.slot_weight;
  out->token_slot = L.token_slot;
  out->token_weight = L.token_weight;
  out->a_perm = L.a_perm;
  out->a_scale_t = L.a_scale_t;
  out->h_hi = L.h_hi;
  out->h_lo = L.h_lo;
  out->h_scale_t = L.h_scale_t;
  out->y_rows = L.y_rows;
  out->y_scale = L.y_scale;
  out->partials = L.partials;
  out->counters = L.counters;
  out->block_hist = L.block_hist;
  out->block_off = L.block_off;
  out->cap_slots = L.cap;
  out->max_units = kMaxSplitUnits;
  out->tokens_per_block = L.tpb;
  out->num_blocks = L.nblocks;
  return FMOE_OK;
}

int fmoe_workspace_size(int32_t T, int32_t E, int32_t H, int32_t I, size_t* bytes) {
  if (!bytes) return FMOE_ERR_NULL;
  FmoeLayout l;
  int rc = fmoe_workspace_layout(T, E, H, I, &l);
  if (rc) return rc;
  *bytes = l.total_bytes;
  return FMOE_OK;
}

int fmoe_quantize_activations(const void* x, int32_t T, int32_t H, void* q, float* scale_t,
                              void* stream) {
  if (T < 0 || H <= 0 || H % kBlock != 0) return FMOE_ERR_SHAPE;
  if (static_cast<int64_t>(T) * (H / kBlock) > (int64_t{1} << 30)) return FMOE_ERR_SHAPE;
  if (T == 0) return FMOE_OK;
  if (!x || !q || !scale_t) return FMOE_ERR_NULL;
  if (!aligned16(x) || !aligned16(q) || !aligned16(scale_t)) return FMOE_ERR_ALIGN;
  const auto lo = [](const void* p) { return reinterpret_cast<uintptr_t>(p); };
  const uintptr_t xb = lo(x), xe = xb + static_cast<uintptr_t>(T) * H * 2;
  const uintptr_t qb = lo(q), qe = qb + static_cast<uintptr_t>(T) * H;
  const uintptr_t sb = lo(scale_t), se = sb + static_cast<uintptr_t>(T) * (H / kBlock) * 4;
  if ((qb < xe && xb < qe) || (sb < xe && xb < se) || (sb < qe && qb < se)) return FMOE_ERR_SHAPE;
  DeviceInfo d;
  int rc = device_info(&d);
  if (rc) return rc;
  if (d.major != 10) return FMOE_ERR_DEVICE;
  return launch_quantize_act(x, T, H, q, scale_t, d.sms, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? FMOE_OK
             : FMOE_ERR_CUDA;
}

int fmoe_route(const void* logits, int32_t logits_dtype, const void* bias, int32_t bias_dtype,
               int32_t T, int32_t E_global, int32_t top_k, int32_t n_group, int32_t topk_group,
               float rsf, int32_t* topk_ids, float* topk_weights, void* stream) {
  if (T < 0 || E_global != kExpertsGlobal || top_k != kTopK || n_group != kGroups ||
      topk_group != kTopKGroups)
    return FMOE_ERR_SHAPE;
  if ((logits_dtype != FMOE_DTYPE_F32 && logits_dtype != FMOE_DTYPE_BF16) ||
      (bias_dtype != FMOE_DTYPE_F32 && bias_dtype != FMOE_DTYPE_BF16))
    return FMOE_ERR_DTYPE;
  if (T == 0) return FMOE_OK;
  if (!logits || !bias || !topk_ids || !topk_weights) return FMOE_ERR_NULL;
  if (!aligned16(logits) || !aligned16(bias) || !aligned16(topk_ids) || !aligned16(topk_weights))
    return FMOE_ERR_ALIGN;
  DeviceInfo d;
  int rc = device_info(&d);
  if (rc) return rc;
  if (d.major != 10) return FMOE_ERR_DEVICE;
  return launch_route(logits, logits_dtype, bias, bias_dtype, T, rsf, topk_ids, topk_weights,
                      static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? FMOE_OK
             : FMOE_ERR_CUDA;
}

}  // extern "C"

namespace {

// The GEMMs' seven TMA tensor maps depend only on the workspace and weight pointers and the
// shapes; a call re-encodes them only when those change. Each host thread keeps the maps of its
// last 16 argument sets (one per layer of a model, say), replaced round robin.
struct TensorMaps {
  CUtensorMap a, w1, hi, lo, w2, sa1, sa2;
};

struct TensorMapKey {
  const void* ws;
  const void* w1;
  const void* w2;
  int T, E, H, I, device;
  bool operator==(const TensorMapKey& o) const {
    return ws == o.ws && w1 == o.w1 && w2 == o.w2 && T == o.T && E == o.E && H == o.H &&
           I == o.I && device == o.device;
  }
};

constexpr int kTensorMapCache = 16;

const TensorMaps* tensor_maps(const RunParams& p, const FmoeArgs* a, const Layout& L,
                              int device) {
  struct Entry {
    bool valid;
    TensorMapKey key;
    TensorMaps maps;
  };
  thread_local Entry cache[kTensorMapCache] = {};
  thread_local int next = 0;
  const int T = p.T, E = p.E, H = p.H, I = p.I;
  const TensorMapKey key{p.ws, a->gemm1_weights, a->gemm2_weights, T, E, H, I, device};
  for (Entry& e : cache)
    if (e.valid && e.key == key) return &e.maps;
  Entry& e = cache[next];
  e.valid = false;
  TensorMaps* m = &e.maps;
  if (!make_tmap_u8(&m->a, p.ws + L.a_perm, H, L.cap, H, 128, 128) ||
      !make_tmap_u8(&m->w1, a->gemm1_weights, H, static_cast<uint64_t>(E) * 2 * I, H, 128, 128) ||
      !make_tmap_u8(&m->hi, p.ws + L.h_hi, I, L.cap, I, 128, T <= kPackedMaxT ? 64 : 128) ||
      !make_tmap_u8(&m->lo, p.ws + L.h_lo, I, L.cap, I, 128, T <= kPackedMaxT ? 64 : 128) ||
      !make_tmap_u8(&m->w2, a->gemm2_weights, I, static_cast<uint64_t>(E) * H, I, 128, 256) ||
      // per-K-block activation scales, [K blocks][cap] fp32: one 128-slot row per load
      !make_tmap_f32_rows(&m->sa1, p.ws + L.a_scale_t, L.cap, H / kBlock, 128) ||
      !make_tmap_f32_rows(&m->sa2, p.ws + L.h_scale_t, L.cap, I / kBlock, 128))
    return nullptr;
  e.key = key;
  e.valid = true;
  next = (next + 1) % kTensorMapCache;
  return m;
}

}  // namespace

extern "C" {

int fmoe_run(const FmoeArgs* a, void* stream_ptr) {
  int rc = validate(a);
  if (rc) return rc;
  if (a->num_tokens == 0) return FMOE_OK;
  DeviceInfo d;
  rc = device_info(&d);
  if (rc) return rc;
  if (d.major != 10) return FMOE_ERR_DEVICE;
  const int T = a->num_tokens, E = a->num_local_experts, H = a->hidden_size,
            I = a->intermediate_size;
  const Layout L = make_layout(T, E, H, I);
  if (a->workspace_bytes < L.total) return FMOE_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream_ptr);

  RunParams p{};
  p.logits = a->routing_logits;
  p.logits_dtype = a->logits_dtype;
  p.bias = a->routing_bias;
  p.bias_dtype = a->bias_dtype;
  p.hidden = static_cast<const uint8_t*>(a->hidden_states);
  p.hidden_scale = a->hidden_states_scale;
  p.w1 = static_cast<const uint8_t*>(a->gemm1_weights);
  p.w1_scale = a->gemm1_weights_scale;
  p.w2 = static_cast<const uint8_t*>(a->gemm2_weights);
  p.w2_scale = a->gemm2_weights_scale;
  p.output = a->output;
  p.T = T;
  p.H = H;
  p.I = I;
  p.E = E;
  p.local_start = a->local_expert_offset;
  p.rsf = a->routed_scaling_factor;
  p.route_mode = route_mode(a->routing_method, a->top_k);
  p.in_ids = a->topk_ids;
  p.in_w = a->topk_weights;
  p.region_counts = a->region_counts;
  p.region_tokens = a->region_counts ? a->region_tokens : T;
  p.out_mode = a->output_dtype;
  for (int r = 0; r < FMOE_EP_MAX_RANKS; ++r) p.region_out[r] = a->region_output[r];
  p.inject_gemm = g_armed.gemm;
  p.wait_ns = g_armed.wait_ns;
  g_armed = ArmedTimeout{};
  p.ws = static_cast<uint8_t*>(a->workspace);
  p.L = L;
  p.num_sms = d.sms;

  auto mark = [&](int i) -> bool {
    if (!a->phase_events || i >= a->num_phase_events || !a->phase_events[i]) return true;
    return cudaEventRecord(static_cast<cudaEvent_t>(a->phase_events[i]), s) == cudaSuccess;
  };
  if (!mark(0)) return FMOE_ERR_CUDA;
  // The plan kernel (k_scan or k_plan_small) clears the status word before any GEMM can set it.
  if (p.in_ids != nullptr) {
    // pre-routed: the given picks replace the routing; the permutation is the same
    if (launch_hist_given(p, s) != cudaSuccess || launch_scan(p, s) != cudaSuccess || !mark(1))
      return FMOE_ERR_CUDA;
    if (launch_scatter_gather(p, s) != cudaSuccess || !mark(2)) return FMOE_ERR_CUDA;
  } else if (T <= kSmallT) {
    if (launch_plan_small(p, s) != cudaSuccess || !mark(1)) return FMOE_ERR_CUDA;
    if (a->gemm_path == FMOE_PATH_AUTO && a->stop_after == FMOE_STOP_NONE && gemv_eligible(p)) {
      // small batch: GEMM1 + SwiGLU, then GEMM2 + combine, as matrix-vector kernels
      if (!mark(2) || launch_gemv(p, 1, s) != cudaSuccess || !mark(3)) return FMOE_ERR_CUDA;
      if (launch_gemv(p, 2, s) != cudaSuccess || !mark(4) || !mark(5)) return FMOE_ERR_CUDA;
      return FMOE_OK;
    }
    if (launch_gather(p, s) != cudaSuccess || !mark(2)) return FMOE_ERR_CUDA;
  } else {
    if (launch_route_hist(p, s) != cudaSuccess || launch_scan(p, s) != cudaSuccess || !mark(1))
      return FMOE_ERR_CUDA;
    if (launch_scatter_gather(p, s) != cudaSuccess || !mark(2)) return FMOE_ERR_CUDA;
  }
  if (a->stop_after == FMOE_STOP_ROUTE || a->stop_after == FMOE_STOP_GATHER) return FMOE_OK;

  const TensorMaps* tm = tensor_maps(p, a, L, d.device);
  if (!tm) return FMOE_ERR_CUDA;
  const CUtensorMap &tm_a = tm->a, &tm_w1 = tm->w1, &tm_hi = tm->hi, &tm_lo = tm->lo,
                    &tm_w2 = tm->w2, &tm_sa1 = tm->sa1, &tm_sa2 = tm->sa2;

  if (launch_gemm1(p, tm_a, tm_w1, tm_sa1, s) != cudaSuccess) return FMOE_ERR_CUDA;
  if (T <= kSplitMaxT && launch_split_finish(p, 1, s) != cudaSuccess) return FMOE_ERR_CUDA;
  if (!mark(3)) return FMOE_ERR_CUDA;
  if (a->stop_after == FMOE_STOP_GEMM1) return FMOE_OK;
  if (launch_gemm2(p, tm_hi, tm_lo, tm_w2, tm_sa2, s) != cudaSuccess) return FMOE_ERR_CUDA;
  if (T <= kSplitMaxT && launch_split_finish(p, 2, s) != cudaSuccess) return FMOE_ERR_CUDA;
  if (!mark(4)) return FMOE_ERR_CUDA;
  if (a->stop_after == FMOE_STOP_GEMM2) return FMOE_OK;
  if (launch_combine(p, s) != cudaSuccess || !mark(5)) return FMOE_ERR_CUDA;
  return FMOE_OK;
}

int fmoe_read_status(const void* workspace, void* stream, int32_t* status) {
  if (!workspace || !status) return FMOE_ERR_NULL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(status, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost, s) !=
          cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return FMOE_ERR_CUDA;
  return FMOE_OK;
}

}  // extern "C"
