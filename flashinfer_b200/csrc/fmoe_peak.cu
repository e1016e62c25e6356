// fmoe_peak.cu -- the FP8 tensor-core peak of this device, measured with the GEMMs' own MMA shape.
//
// Every CTA (one per SM) keeps an e4m3 A tile (128 x 128) and B tile (256 x 128) in shared memory
// and issues chains of tcgen05.mma.kind::f8f6f4 M=128 N=256 K=32 -- the instruction the grouped
// GEMMs issue -- into alternating 256-column TMEM accumulators, 4 per 128-wide K block, with no
// memory traffic and no epilogue. FLOPs / time is the dense FP8 rate the GEMMs' roofline uses as
// its denominator (the benchmark runs it briefly for the burst figure and for about a second for
// the sustained one). No counterpart in the reference.
#include <cuda_runtime.h>

#include "fmoe_internal.h"
#include "fmoe_ptx.cuh"

namespace fmoe {
namespace {

constexpr int kPeakThreads = 128;
constexpr int kPeakSmem = 16384 + 32768 + 1024 + 64;

__global__ void __launch_bounds__(kPeakThreads, 1) k_fp8_peak(int k_blocks, int32_t* status) {
  extern __shared__ uint8_t raw[];
  uint8_t* smem = raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u);
  uint64_t* done = reinterpret_cast<uint64_t*>(smem + 49152);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 49152 + 16);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // small e4m3 values (0.5-ish): the accumulators stay finite
  for (int i = threadIdx.x; i < 49152 / 4; i += blockDim.x)
    reinterpret_cast<uint32_t*>(smem)[i] = 0x30303030u;
  if (threadIdx.x == 0) {
    mbar_init(done, 1);
    fence_mbar_init();
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0 && lane == 0) {
    constexpr uint32_t idesc = idesc_e4m3_f32(128, 256);
    const uint64_t a = smem_desc_k128(smem_u32(smem));
    const uint64_t b = smem_desc_k128(smem_u32(smem) + 16384);
    for (int kb = 0; kb < k_blocks; ++kb) {
      const uint32_t d = tmem + (kb & 1) * 256;
#pragma unroll
      for (int j = 0; j < 4; ++j) mma_f8f6f4(d, a + 2 * j, b + 2 * j, idesc, j > 0 ? 1u : 0u);
    }
    mma_commit(done);
    if (!mbar_wait(done, 0)) atomicOr(status, 1);  // bounded: gives up after FMOE_WAIT_NS
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace
}  // namespace fmoe

using namespace fmoe;

extern "C" int fmoe_fp8_mma_peak(int32_t k_blocks, int32_t* status, double* flops,
                                 void* cuda_stream) {
  // at most 500,000 K blocks per launch (about 0.2 s): well inside the bounded wait
  if (k_blocks <= 0 || k_blocks > 500000) return FMOE_ERR_SHAPE;
  if (!status || !flops) return FMOE_ERR_NULL;
  int dev = 0, sms = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return FMOE_ERR_CUDA;
  if (major != 10) return FMOE_ERR_DEVICE;
  if (cudaFuncSetAttribute(k_fp8_peak, cudaFuncAttributeMaxDynamicSharedMemorySize, kPeakSmem) !=
      cudaSuccess)
    return FMOE_ERR_CUDA;
  k_fp8_peak<<<sms, kPeakThreads, kPeakSmem, static_cast<cudaStream_t>(cuda_stream)>>>(k_blocks,
                                                                                      status);
  if (cudaGetLastError() != cudaSuccess) return FMOE_ERR_CUDA;
  *flops = 2.0 * 128 * 256 * 128 * static_cast<double>(k_blocks) * sms;
  return FMOE_OK;
}
