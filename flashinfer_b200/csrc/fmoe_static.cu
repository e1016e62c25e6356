// fmoe_static.cu -- routing + permutation for callers that cannot allocate device memory.
//
// Some callers of this library have no way to allocate device memory at the point where
// they need the MoE routing tables: an inference engine that plans every buffer ahead of
// time and forbids allocation while it enqueues work, code running inside a CUDA graph
// capture whose memory pool is fixed, or a host program bound to the C ABI from a language
// runtime that has no device allocator of its own. fmoe_route_permute_noalloc() serves them:
// the caller passes the routing inputs and the output tables, and the intermediate scratch
// (top-k picks, per-block histograms and offsets, plan words) lives in the file-scope device
// array below, sized for at most kNoallocMaxTokens tokens. It computes exactly what
// fmoe_run() computes for the same inputs before its GEMMs (same kernels, same results).
//
// The array belongs to the library image: every GPU that loads the library holds it until
// the process exits, and every call on that GPU shares it. A call leaves the previous call's
// contents behind; nothing in it has to start at zero, because each kernel writes every word
// it later reads. Two calls whose executions overlap on the GPU (different streams without
// ordering between them) race on the array and produce undefined tables.
#include <cuda_runtime.h>

#include <mutex>

#include "fmoe_internal.h"

namespace fmoe {
namespace {

constexpr int kNoallocMaxTokens = 4096;

// Byte offsets of the scratch regions inside the array.
constexpr size_t kOffTopkIds = 0;
constexpr size_t kOffTopkW = kOffTopkIds + static_cast<size_t>(kNoallocMaxTokens) * kTopK * 4;
constexpr size_t kOffHist = kOffTopkW + static_cast<size_t>(kNoallocMaxTokens) * kTopK * 4;
constexpr size_t kOffBlockOff = kOffHist + static_cast<size_t>(kMaxBlockCounts) * 4;
constexpr size_t kOffPlan = kOffBlockOff + static_cast<size_t>(kMaxBlockCounts) * 4;
constexpr size_t kOffCounters = kOffPlan + 256;
constexpr size_t kOffStatus = kOffCounters + static_cast<size_t>(2 * kMaxSplitUnits) * 4;
constexpr size_t kNoallocScratchBytes = kOffStatus + 256;  // 336,384 bytes

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

struct DeviceScratch {
  unsigned char* base = nullptr;  // device address of g_noalloc_scratch on this device
  int sms = 0;
};

// Per-device set-up: the host-side name of the array is not a device address, so its address
// on each device is looked up once, with that device current, and cached.
int scratch_for_current_device(DeviceScratch* out) {
  static DeviceScratch cache[64];
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FMOE_ERR_CUDA;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev].base == nullptr) {
    int major = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return FMOE_ERR_CUDA;
    if (major != 10) return FMOE_ERR_DEVICE;
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr)
      return FMOE_ERR_CUDA;
    cache[dev].base = static_cast<unsigned char*>(ptr);
    cache[dev].sms = sms;
  }
  *out = cache[dev];
  return FMOE_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

}  // namespace
}  // namespace fmoe

using namespace fmoe;

extern "C" int fmoe_route_permute_noalloc(const void* logits, int32_t logits_dtype,
                                          const void* bias, int32_t bias_dtype, int32_t T,
                                          int32_t E, int32_t local_expert_offset, float rsf,
                                          int32_t* expert_count, int32_t* expert_base,
                                          int32_t* slot_token, float* slot_weight,
                                          int32_t* token_slot, float* token_weight,
                                          void* stream) {
  if (T < 0 || E < 1 || E > kMaxLocalExperts) return FMOE_ERR_SHAPE;
  if (T > kNoallocMaxTokens) return FMOE_ERR_NOALLOC_LIMIT;
  if (local_expert_offset < 0 || local_expert_offset + E > kExpertsGlobal) return FMOE_ERR_OFFSET;
  if ((logits_dtype != FMOE_DTYPE_F32 && logits_dtype != FMOE_DTYPE_BF16) ||
      (bias_dtype != FMOE_DTYPE_F32 && bias_dtype != FMOE_DTYPE_BF16))
    return FMOE_ERR_DTYPE;
  if (T == 0) return FMOE_OK;
  if (!logits || !bias || !expert_count || !expert_base || !slot_token || !slot_weight ||
      !token_slot || !token_weight)
    return FMOE_ERR_NULL;
  if (!aligned(logits, 16) || !aligned(bias, 16) || !aligned(expert_count, 4) ||
      !aligned(expert_base, 4) || !aligned(slot_token, 4) || !aligned(slot_weight, 4) ||
      !aligned(token_slot, 4) || !aligned(token_weight, 4))
    return FMOE_ERR_ALIGN;
  DeviceScratch d;
  int rc = scratch_for_current_device(&d);
  if (rc) return rc;
  PermuteBuffers b{};
  b.topk_ids = reinterpret_cast<int32_t*>(d.base + kOffTopkIds);
  b.topk_w = reinterpret_cast<float*>(d.base + kOffTopkW);
  b.block_hist = reinterpret_cast<int32_t*>(d.base + kOffHist);
  b.block_off = reinterpret_cast<int32_t*>(d.base + kOffBlockOff);
  b.plan = reinterpret_cast<int32_t*>(d.base + kOffPlan);
  b.counters = reinterpret_cast<int32_t*>(d.base + kOffCounters);
  b.status = reinterpret_cast<int32_t*>(d.base + kOffStatus);
  b.expert_count = expert_count;
  b.expert_base = expert_base;
  b.slot_token = slot_token;
  b.slot_weight = slot_weight;
  b.token_slot = token_slot;
  b.token_weight = token_weight;
  // H and I only size the plan words kept in scratch; the tables do not depend on them.
  return launch_route_permute(logits, logits_dtype, bias, bias_dtype, T, E, local_expert_offset,
                              rsf, 7168, 2048, d.sms, b, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? FMOE_OK
             : FMOE_ERR_CUDA;
}
