// fmoe_ep.cu -- expert parallelism over NVLink: token dispatch and partial-output reduction by
// plain stores into the other GPUs' memory (CUDA IPC mappings), plus the buffer and IPC helpers.
//
// The reference has no multi-GPU code; its per-rank contract is run() over the local expert range
// (solution/triton/kernel.py:442-452, the local filter of the routing kernel). One layer call on
// rank r of R:
//   fmoe_route           global top-8 picks of r's tokens
//   fmoe_ep_dispatch     k_ep_plan: per token the ranks owning a pick, its slot at each (tokens
//                        ascending); k_ep_send: one warp per token stores the e4m3 row, scales,
//                        picks and weights into region r of each destination's receive buffer
//   (collective)         orders every destination after every sender
//   fmoe_run             pre-routed, on the receive buffer; its combine stores each token's
//                        partial row (fp16 + power-of-two scales) into region <this rank> of the
//                        sender's return buffer
//   (collective)
//   fmoe_ep_reduce       per token, the partials of the destinations in ascending rank order,
//                        fp32 sums, one rounding to bf16
// No atomics anywhere: every slot is computed by a scan, so results are deterministic. No TMA or
// bulk copy touches another GPU's memory; the peer traffic is st.global from ordinary threads.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <string.h>

#include "fmoe_internal.h"

namespace fmoe {
namespace {

constexpr int kPlanThreads = 1024;

struct PeerBases {
  uint8_t* p[FMOE_EP_MAX_RANKS];
};

struct EpLayout {
  size_t total, recv_hidden, recv_scale, recv_ids, recv_weights, recv_counts, ret_rows;
  int64_t cap;
  size_t row_bytes;
};

EpLayout ep_layout(int R, int T, int H) {
  EpLayout L{};
  L.cap = T;
  L.row_bytes = FMOE_EP_ROW_BYTES(H);
  const size_t n = static_cast<size_t>(R) * static_cast<size_t>(T);
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  L.recv_hidden = take(n * H);
  L.recv_scale = take(static_cast<size_t>(H / kBlock) * n * 4);
  L.recv_ids = take(n * kTopK * 4);
  L.recv_weights = take(n * kTopK * 4);
  L.recv_counts = take(static_cast<size_t>(FMOE_EP_MAX_RANKS) * 4);
  L.ret_rows = take(n * L.row_bytes);
  L.total = o;
  return L;
}

// Destination mask of one token: bit d set when one of its picks lies in rank d's experts.
__device__ __forceinline__ uint32_t dest_mask(const int32_t* ids, int epr, int R) {
  const int4 a = __ldg(reinterpret_cast<const int4*>(ids));
  const int4 b = __ldg(reinterpret_cast<const int4*>(ids) + 1);
  const int v[kTopK] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t m = 0;
#pragma unroll
  for (int k = 0; k < kTopK; ++k) {
    const int d = v[k] / epr;
    if (v[k] >= 0 && d < R) m |= 1u << d;
  }
  return m;
}

// One CTA: thread i takes the i-th contiguous chunk of tokens, so a block-wide exclusive scan of
// the per-thread destination counts gives every token its slot at each destination (tokens
// ascending). The totals go to the destinations' recv_counts[rank].
__global__ void __launch_bounds__(kPlanThreads) k_ep_plan(const int32_t* __restrict__ ids, int T,
                                                          int R, int rank, int epr,
                                                          int32_t* __restrict__ token_dest_slot,
                                                          const PeerBases peers,
                                                          size_t counts_off) {
  __shared__ int warp_tot[32][FMOE_EP_MAX_RANKS];
  pdl_begin();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (T + kPlanThreads - 1) / kPlanThreads;
  const int t0 = min(T, tid * per), t1 = min(T, t0 + per);
  int cnt[FMOE_EP_MAX_RANKS];
#pragma unroll
  for (int d = 0; d < FMOE_EP_MAX_RANKS; ++d) cnt[d] = 0;
  for (int t = t0; t < t1; ++t) {
    const uint32_t m = dest_mask(ids + static_cast<size_t>(t) * kTopK, epr, R);
#pragma unroll
    for (int d = 0; d < FMOE_EP_MAX_RANKS; ++d) cnt[d] += (m >> d) & 1u;
  }
  // inclusive warp scan per destination, then the warps' totals
  int inc[FMOE_EP_MAX_RANKS];
#pragma unroll
  for (int d = 0; d < FMOE_EP_MAX_RANKS; ++d) {
    int v = cnt[d];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    inc[d] = v;
    if (lane == 31) warp_tot[warp][d] = v;
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int d = 0; d < FMOE_EP_MAX_RANKS; ++d) {
      const int w = warp_tot[lane][d];
      int v = w;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      warp_tot[lane][d] = v - w;  // exclusive prefix over warps
      if (lane == 31 && d < R)     // total for destination d
        reinterpret_cast<int32_t*>(peers.p[d] + counts_off)[rank] = v;
    }
  }
  __syncthreads();
  int next[FMOE_EP_MAX_RANKS];
#pragma unroll
  for (int d = 0; d < FMOE_EP_MAX_RANKS; ++d) next[d] = warp_tot[warp][d] + inc[d] - cnt[d];
  for (int t = t0; t < t1; ++t) {
    const uint32_t m = dest_mask(ids + static_cast<size_t>(t) * kTopK, epr, R);
    int32_t* out = token_dest_slot + static_cast<size_t>(t) * R;
#pragma unroll
    for (int d = 0; d < FMOE_EP_MAX_RANKS; ++d)
      if (d < R) out[d] = (m >> d) & 1u ? next[d]++ : -1;
  }
  __threadfence_system();  // the counts reach the destinations before the collective that follows
}

// One warp per token: its row (H bytes), scales and picks, read once, stored into each
// destination's region `rank` at the token's slot there.
__global__ void __launch_bounds__(256) k_ep_send(const int32_t* __restrict__ ids,
                                                 const float* __restrict__ wts,
                                                 const uint8_t* __restrict__ hidden,
                                                 const float* __restrict__ hidden_scale, int T,
                                                 int H, int R, int rank, int64_t cap,
                                                 const int32_t* __restrict__ token_dest_slot,
                                                 const PeerBases peers, EpLayout L) {
  constexpr int kMaxVec = 16;  // H <= 8192: 16 B x 16 per lane
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const int warp0 = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  const int nvec = H / 16, nkb = H / kBlock;
  const size_t n = static_cast<size_t>(R) * cap;
  for (int t = warp0; t < T; t += nwarps) {
    const int my_slot = lane < R ? token_dest_slot[static_cast<size_t>(t) * R + lane] : -1;
    const uint4* src = reinterpret_cast<const uint4*>(hidden + static_cast<size_t>(t) * H);
    uint4 row[kMaxVec];
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i)
      if (lane + 32 * i < nvec) row[i] = __ldg(src + lane + 32 * i);
    const float sc0 = lane < nkb ? __ldg(hidden_scale + static_cast<size_t>(lane) * T + t) : 0.f;
    const float sc1 =
        lane + 32 < nkb ? __ldg(hidden_scale + static_cast<size_t>(lane + 32) * T + t) : 0.f;
    const int pid = lane < kTopK ? __ldg(ids + static_cast<size_t>(t) * kTopK + lane) : 0;
    const float pw = lane < kTopK ? __ldg(wts + static_cast<size_t>(t) * kTopK + lane) : 0.f;
    for (int d = 0; d < R; ++d) {
      const int slot = __shfl_sync(0xffffffffu, my_slot, d);
      if (slot < 0) continue;
      const size_t rix = static_cast<size_t>(rank) * cap + slot;  // row in d's receive buffer
      uint8_t* base = peers.p[d];
      uint4* dst = reinterpret_cast<uint4*>(base + L.recv_hidden + rix * H);
#pragma unroll
      for (int i = 0; i < kMaxVec; ++i)
        if (lane + 32 * i < nvec) dst[lane + 32 * i] = row[i];
      float* sc = reinterpret_cast<float*>(base + L.recv_scale);
      if (lane < nkb) sc[static_cast<size_t>(lane) * n + rix] = sc0;
      if (lane + 32 < nkb) sc[static_cast<size_t>(lane + 32) * n + rix] = sc1;
      if (lane < kTopK) {
        reinterpret_cast<int32_t*>(base + L.recv_ids)[rix * kTopK + lane] = pid;
        reinterpret_cast<float*>(base + L.recv_weights)[rix * kTopK + lane] = pw;
      }
    }
  }
  __threadfence_system();  // the rows reach the destinations before the collective that follows
}

// out[t] = bf16(sum_d partial_d[t]) over the destinations that hold a partial of token t, in
// ascending rank order. Thread: 32 consecutive columns of one token (inside one 256-column scale
// block); the partial rows were stored by other GPUs, so they are read through L2 (ld.global.cg).
constexpr int kReduceThreads = 128;
__global__ void __launch_bounds__(kReduceThreads) k_ep_reduce(const int32_t* __restrict__ tds,
                                                              const uint8_t* __restrict__ ret,
                                                              int64_t cap, size_t row_bytes,
                                                              int T, int H, int R,
                                                              __nv_bfloat16* __restrict__ out) {
  pdl_begin();
  const int ncol = H / 32;  // 32-column pieces per token
  const int chunks = (ncol + kReduceThreads - 1) / kReduceThreads;
  const long work = static_cast<long>(T) * chunks;
  for (long wi = blockIdx.x; wi < work; wi += gridDim.x) {
    const int t = static_cast<int>(wi / chunks);
    const int piece = static_cast<int>(wi - static_cast<long>(t) * chunks) * kReduceThreads +
                      threadIdx.x;
    if (piece >= ncol) continue;
    const int col0 = piece * 32;
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
    for (int d = 0; d < R; ++d) {
      const int slot = __ldg(tds + static_cast<size_t>(t) * R + d);
      if (slot < 0) continue;
      const uint8_t* row = ret + (static_cast<size_t>(d) * cap + slot) * row_bytes;
      const float f = __ldcg(reinterpret_cast<const float*>(row + static_cast<size_t>(H) * 2) +
                             col0 / kTileN);
      const uint4* src = reinterpret_cast<const uint4*>(row + static_cast<size_t>(col0) * 2);
      uint4 v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __ldcg(src + i);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __half2* h = reinterpret_cast<const __half2*>(&v[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 q = __half22float2(h[j]);
          acc[i * 8 + 2 * j] = fmaf(f, q.x, acc[i * 8 + 2 * j]);
          acc[i * 8 + 2 * j + 1] = fmaf(f, q.y, acc[i * 8 + 2 * j + 1]);
        }
      }
    }
    uint4 o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        oh[j] = __floats2bfloat162_rn(acc[i * 8 + 2 * j], acc[i * 8 + 2 * j + 1]);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H + col0);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = o[i];
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int num_sms_current() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 0;
  return sms;
}

}  // namespace
}  // namespace fmoe

using namespace fmoe;

extern "C" {

int fmoe_ep_layout(int32_t R, int32_t T, int32_t H, FmoeEpLayout* out) {
  if (!out) return FMOE_ERR_NULL;
  if (R < 1 || R > FMOE_EP_MAX_RANKS || T < 0 || H <= 0 || H % kTileN != 0 || H / kBlock > 64)
    return FMOE_ERR_SHAPE;
  const EpLayout L = ep_layout(R, T, H);
  out->total_bytes = L.total;
  out->recv_hidden = L.recv_hidden;
  out->recv_scale = L.recv_scale;
  out->recv_ids = L.recv_ids;
  out->recv_weights = L.recv_weights;
  out->recv_counts = L.recv_counts;
  out->ret_rows = L.ret_rows;
  out->cap = L.cap;
  out->row_bytes = L.row_bytes;
  return FMOE_OK;
}

int fmoe_ep_alloc(size_t bytes, void** ptr) {
  if (!ptr) return FMOE_ERR_NULL;
  *ptr = nullptr;
  return cudaMalloc(ptr, bytes > 0 ? bytes : 256) == cudaSuccess ? FMOE_OK : FMOE_ERR_CUDA;
}

int fmoe_ep_free(void* ptr) {
  if (!ptr) return FMOE_OK;
  return cudaFree(ptr) == cudaSuccess ? FMOE_OK : FMOE_ERR_CUDA;
}

int fmoe_ipc_get_handle(const void* ptr, void* handle64) {
  if (!ptr || !handle64) return FMOE_ERR_NULL;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  return cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle64), const_cast<void*>(ptr)) ==
                 cudaSuccess
             ? FMOE_OK
             : FMOE_ERR_CUDA;
}

int fmoe_ipc_open(const void* handle64, void** ptr) {
  if (!handle64 || !ptr) return FMOE_ERR_NULL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess
             ? FMOE_OK
             : FMOE_ERR_CUDA;
}

int fmoe_ipc_close(void* ptr) {
  if (!ptr) return FMOE_ERR_NULL;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? FMOE_OK : FMOE_ERR_CUDA;
}

int fmoe_ep_dispatch(const int32_t* ids, const float* wts, const void* hidden,
                     const float* hidden_scale, int32_t T, int32_t capacity, int32_t H, int32_t R,
                     int32_t rank, void* const* peer_buffers, int32_t* token_dest_slot,
                     void* stream) {
  if (R < 1 || R > FMOE_EP_MAX_RANKS || rank < 0 || rank >= R || T < 0 || T > capacity ||
      H <= 0 || H % kTileN != 0 || H / kBlock > 64 || kExpertsGlobal % R != 0)
    return FMOE_ERR_SHAPE;
  if (!peer_buffers) return FMOE_ERR_NULL;
  PeerBases peers{};
  for (int d = 0; d < R; ++d) {
    if (!peer_buffers[d]) return FMOE_ERR_NULL;
    if ((reinterpret_cast<uintptr_t>(peer_buffers[d]) & 255u) != 0) return FMOE_ERR_ALIGN;
    peers.p[d] = static_cast<uint8_t*>(peer_buffers[d]);
  }
  const EpLayout L = ep_layout(R, capacity, H);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (T == 0) {
    // still tell every destination that nothing comes from this rank
    (void)launch_pdl(k_ep_plan, 1, kPlanThreads, 0, s, ids, 0, static_cast<int>(R),
                     static_cast<int>(rank), kExpertsGlobal / R, token_dest_slot, peers,
                     L.recv_counts);
    return cudaGetLastError() == cudaSuccess ? FMOE_OK : FMOE_ERR_CUDA;
  }
  if (!ids || !wts || !hidden || !hidden_scale || !token_dest_slot) return FMOE_ERR_NULL;
  if (!aligned16(ids) || !aligned16(wts) || !aligned16(hidden) || !aligned16(hidden_scale))
    return FMOE_ERR_ALIGN;
  const int sms = num_sms_current();
  if (sms <= 0) return FMOE_ERR_CUDA;
  (void)launch_pdl(k_ep_plan, 1, kPlanThreads, 0, s, ids, static_cast<int>(T),
                   static_cast<int>(R), static_cast<int>(rank), kExpertsGlobal / R,
                   token_dest_slot, peers, L.recv_counts);
  if (cudaGetLastError() != cudaSuccess) return FMOE_ERR_CUDA;
  int blocks = (T + 7) / 8;
  if (blocks > sms * 8) blocks = sms * 8;
  (void)launch_pdl(k_ep_send, blocks, 256, 0, s, ids, wts, static_cast<const uint8_t*>(hidden),
                   hidden_scale, static_cast<int>(T), static_cast<int>(H), static_cast<int>(R),
                   static_cast<int>(rank), static_cast<int64_t>(L.cap),
                   static_cast<const int32_t*>(token_dest_slot), peers, L);
  return cudaGetLastError() == cudaSuccess ? FMOE_OK : FMOE_ERR_CUDA;
}

int fmoe_ep_reduce(const int32_t* token_dest_slot, const void* buffer, int32_t T,
                   int32_t capacity, int32_t H, int32_t R, void* out, void* stream) {
  if (R < 1 || R > FMOE_EP_MAX_RANKS || T < 0 || T > capacity || H <= 0 || H % kTileN != 0 ||
      H / kBlock > 64)
    return FMOE_ERR_SHAPE;
  if (T == 0) return FMOE_OK;
  if (!token_dest_slot || !buffer || !out) return FMOE_ERR_NULL;
  if (!aligned16(out) || (reinterpret_cast<uintptr_t>(buffer) & 255u) != 0) return FMOE_ERR_ALIGN;
  const EpLayout L = ep_layout(R, capacity, H);
  const int sms = num_sms_current();
  if (sms <= 0) return FMOE_ERR_CUDA;
  const long work = static_cast<long>(T) * ((H / 32 + kReduceThreads - 1) / kReduceThreads);
  const int blocks = static_cast<int>(work < sms * 16L ? work : sms * 16L);
  (void)launch_pdl(k_ep_reduce, blocks, kReduceThreads, 0, static_cast<cudaStream_t>(stream),
                   token_dest_slot, static_cast<const uint8_t*>(buffer) + L.ret_rows,
                   static_cast<int64_t>(L.cap), L.row_bytes, static_cast<int>(T),
                   static_cast<int>(H), static_cast<int>(R), static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError() == cudaSuccess ? FMOE_OK : FMOE_ERR_CUDA;
}

}  // extern "C"
