// fmoe_kernels.cu -- routing, permutation plan, activation gather and weighted combine.
//
// Reference counterparts (solution/triton/kernel.py):
//   k_route    <- _route_select_local_kernel        kernel.py:371-457
//   k_plan     <- _count_local_experts_kernel        kernel.py:460-477
//                 _scatter_local_tokens_kernel       kernel.py:480-505
//                 host cumsum + tile offsets         kernel.py:508-516, :572-581, :717-718
//   k_gather   <- index_select of rows and scales    kernel.py:699-703
//   k_combine  <- _weighted_scatter_add_kernel       kernel.py:337-368 + bf16 cast :820-823
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include <type_traits>

#include "fmoe_internal.h"
#include "fmoe_ptx.cuh"
#include "fmoe_route.cuh"

namespace fmoe {

template <typename TL, typename TB>
__global__ void __launch_bounds__(256) k_route(const TL* __restrict__ logits,
                                               const TB* __restrict__ bias, int T, float rsf,
                                               int mode, int32_t* __restrict__ ids_out,
                                               float* __restrict__ w_out) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const int warp0 = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  float b[8];
  load8<TB>(bias + lane * 8, b);
  for (int t = warp0; t < T; t += nwarps) {
    int ids[kTopK];
    float w[kTopK];
    route_token<TL>(logits + static_cast<size_t>(t) * kExpertsGlobal, b, rsf, mode, lane, ids,
                    w);
    if (lane == 0) store_picks(ids_out, w_out, t, ids, w);
  }
}

// Routing fused with the per-block local-expert histogram. Block b owns tokens
// [b*tpb, min(T, (b+1)*tpb)); the histogram is order-free (shared-memory atomics on counts).
template <typename TL, typename TB>
__global__ void __launch_bounds__(256) k_route_hist(const TL* __restrict__ logits,
                                                    const TB* __restrict__ bias, int T, int tpb,
                                                    float rsf, int mode, int local_start, int E,
                                                    int32_t* __restrict__ ids_out,
                                                    float* __restrict__ w_out,
                                                    int32_t* __restrict__ block_hist) {
  __shared__ int hist[kMaxLocalExperts];
  pdl_begin();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  float b[8];
  load8<TB>(bias + lane * 8, b);
  const int t0 = blockIdx.x * tpb;
  const int t1 = min(T, t0 + tpb);
  for (int t = t0 + warp; t < t1; t += blockDim.x >> 5) {
    int ids[kTopK];
    float w[kTopK];
    route_token<TL>(logits + static_cast<size_t>(t) * kExpertsGlobal, b, rsf, mode, lane, ids,
                    w);
    if (lane == 0) store_picks(ids_out, w_out, t, ids, w);
    if (lane < kTopK) {
      int mine = ids[0];
#pragma unroll
      for (int k = 1; k < kTopK; ++k)
        if (lane == k) mine = ids[k];
      const int le = mine - local_start;
      if (le >= 0 && le < E) atomicAdd(&hist[le], 1);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    block_hist[static_cast<size_t>(blockIdx.x) * E + e] = hist[e];
}

// Pre-routed calls (expert parallelism): the picks come from the sending rank's routing. Block
// b copies its tokens' picks into the workspace tables -- a token outside its region's count
// gets no picks (-1 / 0) -- and counts its local picks per expert, like k_route_hist.
// With copy == 0 the picks are already the workspace tables (routed by k_route just before):
// the block only counts them.
__global__ void __launch_bounds__(256) k_hist_given(const int32_t* in_ids, const float* in_w,
                                                    const int32_t* __restrict__ region_counts,
                                                    int region_tokens, int T, int tpb,
                                                    int local_start, int E, int copy,
                                                    int32_t* ids_out, float* w_out,
                                                    int32_t* __restrict__ block_hist) {
  __shared__ int hist[kMaxLocalExperts];
  pdl_begin();
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int t0 = blockIdx.x * tpb;
  const int t1 = min(T, t0 + tpb);
  for (int t = t0 + static_cast<int>(threadIdx.x); t < t1; t += blockDim.x) {
    bool valid = true;
    if (region_counts != nullptr) {
      const int r = t / region_tokens;
      valid = t - r * region_tokens < __ldg(region_counts + r);
    }
    const int4* ip = reinterpret_cast<const int4*>(in_ids + static_cast<size_t>(t) * kTopK);
    const float4* wp = reinterpret_cast<const float4*>(in_w + static_cast<size_t>(t) * kTopK);
    int4 i0 = make_int4(-1, -1, -1, -1), i1 = i0;
    float4 w0 = make_float4(0.f, 0.f, 0.f, 0.f), w1 = w0;
    if (valid) {  // plain loads: with copy == 0 the previous kernel wrote these tables
      i0 = ip[0];
      i1 = ip[1];
      w0 = wp[0];
      w1 = wp[1];
    }
    if (copy) {
      int4* io = reinterpret_cast<int4*>(ids_out + static_cast<size_t>(t) * kTopK);
      float4* wo = reinterpret_cast<float4*>(w_out + static_cast<size_t>(t) * kTopK);
      io[0] = i0;
      io[1] = i1;
      wo[0] = w0;
      wo[1] = w1;
    }
    const int ids[kTopK] = {i0.x, i0.y, i0.z, i0.w, i1.x, i1.y, i1.z, i1.w};
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
      const int le = ids[k] - local_start;
      if (ids[k] >= 0 && le >= 0 && le < E) atomicAdd(&hist[le], 1);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    block_hist[static_cast<size_t>(blockIdx.x) * E + e] = hist[e];
}

cudaError_t launch_route(const void* logits, int logits_dtype, const void* bias, int bias_dtype,
                         int T, float rsf, int32_t* topk_ids, float* topk_w, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  const int warps_per_block = 8;
  int blocks = (T + warps_per_block - 1) / warps_per_block;
  if (blocks > 148 * 16) blocks = 148 * 16;
  const dim3 grid(blocks), block(warps_per_block * 32);
  if (logits_dtype == FMOE_DTYPE_F32 && bias_dtype == FMOE_DTYPE_BF16)
    (void)launch_pdl(k_route<float, __nv_bfloat16>, grid, block, 0, s,
        static_cast<const float*>(logits), static_cast<const __nv_bfloat16*>(bias), T, rsf,
        kRouteDeepSeek, topk_ids, topk_w);
  else if (logits_dtype == FMOE_DTYPE_F32 && bias_dtype == FMOE_DTYPE_F32)
    (void)launch_pdl(k_route<float, float>, grid, block, 0, s, static_cast<const float*>(logits),
                                                  static_cast<const float*>(bias), T, rsf,
                                                  kRouteDeepSeek, topk_ids, topk_w);
  else if (logits_dtype == FMOE_DTYPE_BF16 && bias_dtype == FMOE_DTYPE_BF16)
    (void)launch_pdl(k_route<__nv_bfloat16, __nv_bfloat16>, grid, block, 0, s,
        static_cast<const __nv_bfloat16*>(logits), static_cast<const __nv_bfloat16*>(bias), T,
        rsf, kRouteDeepSeek, topk_ids, topk_w);
  else
    (void)launch_pdl(k_route<__nv_bfloat16, float>, grid, block, 0, s,
        static_cast<const __nv_bfloat16*>(logits), static_cast<const float*>(bias), T, rsf,
        kRouteDeepSeek, topk_ids, topk_w);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------
// Permutation plan, deterministic and stable (tokens ascending within each expert).
//   k_route_hist  per routing block: how many of its tokens pick each local expert
//   k_scan        one CTA: exclusive scan over blocks per expert, padded expert bases, the
//                 GEMM work plan (tiles, K splits), counter and status reset
//   k_scatter     per routing block: rank of each (token, expert) among the block's earlier
//                 tokens (warp ballots), slot = block offset + rank; then the block copies the
//                 e4m3 rows and 128-column scales of its picks into the permuted buffers and
//                 zero-fills the padding slots it owns.
// ------------------------------------------------------------------------------------------
// The expert bases padded to 128 slots and the GEMM work plan from the per-expert counts, by one
// warp (lane l takes experts [8l, 8l+8), a shuffle scan gives the bases); also clears the status
// word before any GEMM can set it. With plan == nullptr only the bases are written.
// K splits per tile for a persistent grid of G CTAs are allowed for small batches only (a split
// unit stores its partial tile and k_split_finish sums them). Cost, in quarter K blocks on the
// busiest CTA: 4 * waves * ceil(nkb / s) plus per-unit overheads; the least cost wins, ties to
// the smaller split. Lanes 0-7 price s = 1..8 for GEMM1, lanes 8-15 for GEMM2.
__device__ void write_plan_warp(const int* cnt, int E, int H, int I, int G, int allow_split,
                                int* base, int32_t* plan, int32_t* status, int lane) {
  constexpr int kPer = kMaxLocalExperts / 32;
  const int e0 = lane * kPer;
  int c[kPer];
  int padded = 0, pairs = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    c[j] = e0 + j < E ? cnt[e0 + j] : 0;
    padded += (c[j] + kTileM - 1) / kTileM * kTileM;
    pairs += c[j];
  }
  int inc = padded;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, inc, off);
    if (lane >= off) inc += o;
  }
  int acc = inc - padded;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    if (e0 + j < E) base[e0 + j] = acc;
    acc += (c[j] + kTileM - 1) / kTileM * kTileM;
  }
  const int total = __shfl_sync(0xffffffffu, inc, 31);
  if (lane == 0) base[E] = total;
  pairs = __reduce_add_sync(0xffffffffu, pairs);
  if (plan == nullptr) return;
  const int mtiles = total / kTileM;
  const int tiles1 = mtiles * (I / kBlock);
  const int tiles2 = mtiles * (H / kTileN);
  const int which = lane >> 3;  // 0: GEMM1, 1: GEMM2
  const int sp = (lane & 7) + 1;
  const int tiles = which == 0 ? tiles1 : tiles2;
  const int nkb = which == 0 ? H / kBlock : I / kBlock;
  long long cost = 0x7fffffffffffffLL;
  const bool valid = which < 2 && sp <= kMaxSplit &&
                     (sp == 1 || (allow_split && tiles > 0 && sp <= nkb &&
                                  static_cast<long long>(tiles) * sp <= kMaxSplitUnits));
  if (valid) {
    const long long waves = (static_cast<long long>(tiles) * sp + G - 1) / G;
    const long long per = (nkb + sp - 1) / sp;
    cost = 4 * waves * per + waves * (sp > 1 ? 12 : 8);
  }
  long long key = cost * 8 + (sp - 1);
#pragma unroll
  for (int off = 4; off > 0; off >>= 1) {
    const long long o = __shfl_xor_sync(0xffffffffu, key, off);
    key = o < key ? o : key;
  }
  const int s1 = static_cast<int>(__shfl_sync(0xffffffffu, key, 0) & 7) + 1;
  const int s2 = static_cast<int>(__shfl_sync(0xffffffffu, key, 8) & 7) + 1;
  if (lane == 0) {
    plan[kPlanPairs] = pairs;
    plan[kPlanPadded] = total;
    plan[kPlanMTiles] = mtiles;
    plan[kPlanSplit1] = s1;
    plan[kPlanUnits1] = tiles1 * s1;
    plan[kPlanSplit2] = s2;
    plan[kPlanUnits2] = tiles2 * s2;
    plan[kPlanTiles1] = tiles1;
    plan[kPlanTiles2] = tiles2;
    status[0] = 0;
  }
}

__global__ void __launch_bounds__(1024) k_scan(const int32_t* __restrict__ block_hist,
                                               int nblocks, int E, int H, int I, int G,
                                               int allow_split,
                                               int32_t* __restrict__ block_off,
                                               int32_t* __restrict__ plan,
                                               int32_t* __restrict__ expert_count,
                                               int32_t* __restrict__ expert_base,
                                               int32_t* __restrict__ counters,
                                               int32_t* __restrict__ status) {
  __shared__ int sh[kMaxBlockCounts];
  __shared__ int cnt[kMaxLocalExperts];
  __shared__ int base[kMaxLocalExperts + 1];
  pdl_begin();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
  const int n = nblocks * E;
  {
    // all of a thread's loads in flight at once (the scan runs as a single CTA)
    constexpr int kPer = kMaxBlockCounts / 1024;
    int v[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = threadIdx.x + j * 1024;
      v[j] = i < n ? __ldg(block_hist + i) : 0;
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = threadIdx.x + j * 1024;
      if (i < n) sh[i] = v[j];
    }
  }
  __syncthreads();
  // warp w scans experts w, w+32, ...: exclusive prefix over blocks, 32 blocks per step
  for (int e = warp; e < E; e += nwarp) {
    int run = 0;
    for (int b0 = 0; b0 < nblocks; b0 += 32) {
      const int b = b0 + lane;
      const int v = b < nblocks ? sh[b * E + e] : 0;
      int inc = v;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += o;
      }
      if (b < nblocks) sh[b * E + e] = run + inc - v;
      run += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) cnt[e] = run;
  }
  __syncthreads();
  if (warp == 0) write_plan_warp(cnt, E, H, I, G, allow_split, base, plan, status, lane);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    expert_count[e] = cnt[e];
    expert_base[e] = base[e];
  }
  if (threadIdx.x == 0) expert_base[E] = base[E];
  for (int i = threadIdx.x; i < n; i += blockDim.x) block_off[i] = base[i % E] + sh[i];
  for (int i = threadIdx.x; i < 2 * kMaxSplitUnits; i += blockDim.x) counters[i] = 0;
}

struct ScatterSmem {
  int wcnt[8][kMaxLocalExperts];  // per-warp counts, then per-warp exclusive offsets
  int run[kMaxLocalExperts];      // slots already handed out per expert in this block
};

__global__ void __launch_bounds__(256) k_scatter(
    const int32_t* __restrict__ ids, const float* __restrict__ wts, int T, int tpb,
    int local_start, int E, const int32_t* __restrict__ block_off,
    const int32_t* __restrict__ expert_count, const int32_t* __restrict__ expert_base,
    int32_t* __restrict__ slot_token, float* __restrict__ slot_weight,
    int32_t* __restrict__ token_slot, float* __restrict__ token_weight) {
  __shared__ ScatterSmem sm;
  pdl_begin();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.x;
  const int t_begin = b * tpb;
  const int t_end = min(T, t_begin + tpb);
  for (int e = tid; e < E; e += blockDim.x) sm.run[e] = block_off[static_cast<size_t>(b) * E + e];
  const int nwords = (E + 31) >> 5;
  for (int c0 = t_begin; c0 < t_end; c0 += blockDim.x) {
    const int t = c0 + tid;
    int le[kTopK];
    float lw[kTopK];
    int nloc = 0;
    if (t < t_end) {
#pragma unroll
      for (int k = 0; k < kTopK; ++k) {
        const int e = ids[static_cast<size_t>(t) * kTopK + k] - local_start;
        if (e >= 0 && e < E) {
          const float w = wts[static_cast<size_t>(t) * kTopK + k];
          int j = nloc;  // insertion into the ascending list le[0..nloc)
          while (j > 0 && le[j - 1] > e) {
            le[j] = le[j - 1];
            lw[j] = lw[j - 1];
            --j;
          }
          le[j] = e;
          lw[j] = w;
          ++nloc;
        }
      }
    }
    int rank[kTopK];
    {
      int jp = 0;
      for (int wd = 0; wd < nwords; ++wd) {
        uint32_t m = 0;
        for (int j = 0; j < nloc; ++j)
          if ((le[j] >> 5) == wd) m |= 1u << (le[j] & 31);
        const int ebase = wd * 32;
        const int nb = min(32, E - ebase);
        for (int bit = 0; bit < nb; ++bit) {
          const bool has = (m >> bit) & 1u;
          const uint32_t bal = __ballot_sync(0xffffffffu, has);
          if (lane == 0) sm.wcnt[warp][ebase + bit] = __popc(bal);
          if (has) rank[jp++] = __popc(bal & ((1u << lane) - 1u));
        }
      }
    }
    __syncthreads();
    for (int e = tid; e < E; e += blockDim.x) {
      int acc = sm.run[e];
      for (int w = 0; w < 8; ++w) {
        const int c = sm.wcnt[w][e];
        sm.wcnt[w][e] = acc;
        acc += c;
      }
      sm.run[e] = acc;
    }
    __syncthreads();
    if (t < t_end) {
      int* ts = token_slot + static_cast<size_t>(t) * kTopK;
      float* tw = token_weight + static_cast<size_t>(t) * kTopK;
      for (int j = 0; j < kTopK; ++j) {
        if (j < nloc) {
          const int slot = sm.wcnt[warp][le[j]] + rank[j];
          slot_token[slot] = t;
          slot_weight[slot] = lw[j];
          ts[j] = slot;
          tw[j] = lw[j];
        } else {
          ts[j] = -1;
          tw[j] = 0.0f;
        }
      }
    }
    __syncthreads();
  }
  // Padding slots of the experts this block owns (expert e -> block e mod nblocks) are marked
  // empty. Their activation rows are never initialised: a padding row of the A tile only feeds
  // the same row of the accumulator, which the epilogue replaces with zeros.
  const int nblocks = gridDim.x;
  for (int e = b; e < E; e += nblocks) {
    const int first = expert_base[e] + expert_count[e];
    const int end = expert_base[e + 1];
    for (int s = first + tid; s < end; s += blockDim.x) {
      slot_token[s] = -1;
      slot_weight[s] = 0.0f;
    }
  }
}

// Small batches (T <= kSmallT): routing, the histogram, the plan and the scatter in one
// kernel, replacing k_route_hist + k_scan + k_scatter (three dependent launches of a few tokens
// each). One cluster of ceil(T / 8) CTAs of 8 warps; CTA r routes tokens [8r, 8r + 8), one token
// per warp (the routing's double-precision exponentials are spread over up to 8 SMs), and keeps
// per local expert its token count and a mask of its tokens that picked the expert. After one cluster barrier every CTA reads the other CTAs' counts through distributed
// shared memory: the totals give the plan and the expert bases (the same serial scan in every
// CTA), the counts of lower-ranked CTAs give the rank offset of this CTA's tokens. Same results
// as the three-kernel path: a token's slot rank for expert e is the number of earlier tokens that
// picked e (stable, tokens ascending), its picks are listed by ascending expert, and padding
// slots are marked empty.
template <typename TL, typename TB>
__global__ void __launch_bounds__(32 * kSmallTokensPerCta) k_plan_small(
    const TL* __restrict__ logits, const TB* __restrict__ bias, int T, float rsf, int mode,
    int local_start, int E, int H, int I, int G, int allow_split, int32_t* __restrict__ ids_out,
    float* __restrict__ w_out, int32_t* __restrict__ plan, int32_t* __restrict__ expert_count,
    int32_t* __restrict__ expert_base, int32_t* __restrict__ counters,
    int32_t* __restrict__ status, int32_t* __restrict__ slot_token,
    float* __restrict__ slot_weight, int32_t* __restrict__ token_slot,
    float* __restrict__ token_weight) {
  constexpr int kTok = kSmallTokensPerCta;
  __shared__ int cnt[kMaxLocalExperts];       // this CTA's tokens per local expert
  __shared__ int tot[kMaxLocalExperts];       // all tokens per local expert
  __shared__ int off[kMaxLocalExperts];       // tokens of lower-ranked CTAs per local expert
  __shared__ int base[kMaxLocalExperts + 1];
  __shared__ uint32_t tokmask[kMaxLocalExperts];  // bit i: token 8r + i picked the expert
  __shared__ int ids_s[kTok][kTopK];
  __shared__ float w_s[kTok][kTopK];
  pdl_begin();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
  const uint32_t rank = cluster_ctarank(), ncta = cluster_nctarank();
  const int t0 = static_cast<int>(rank) * kTok;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    cnt[e] = 0;
    tokmask[e] = 0u;
  }
  __syncthreads();
  if (warp < kTok && t0 + warp < T) {
    const int t = t0 + warp;
    float b[8];
    load8<TB>(bias + lane * 8, b);
    int ids[kTopK];
    float w[kTopK];
    route_token<TL>(logits + static_cast<size_t>(t) * kExpertsGlobal, b, rsf, mode, lane, ids, w);
    if (lane == 0) {
      store_picks(ids_out, w_out, t, ids, w);
#pragma unroll
      for (int k = 0; k < kTopK; ++k) {
        ids_s[warp][k] = ids[k];
        w_s[warp][k] = w[k];
      }
    }
    if (lane < kTopK) {
      int mine = ids[0];
#pragma unroll
      for (int k = 1; k < kTopK; ++k)
        if (lane == k) mine = ids[k];
      const int le = mine - local_start;
      if (le >= 0 && le < E) {
        atomicAdd(&cnt[le], 1);
        atomicOr(&tokmask[le], 1u << warp);
      }
    }
  }
  __syncthreads();
  cluster_arrive();  // counts of every CTA are complete and visible cluster-wide
  cluster_wait();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int sum = 0, lower = 0;
    for (uint32_t r = 0; r < ncta; ++r) {
      const int c = r == rank ? cnt[e] : ld_dsmem_s32(&cnt[e], r);
      sum += c;
      if (r < rank) lower += c;
    }
    tot[e] = sum;
    off[e] = lower;
  }
  cluster_arrive();  // this CTA's remote reads are done; matched by the wait before exit
  __syncthreads();
  if (warp == 0)
    write_plan_warp(tot, E, H, I, G, allow_split, base, rank == 0 ? plan : nullptr, status,
                    lane);
  // token t0 + i (thread i < 8): its local picks in ascending expert order
  const int i = threadIdx.x;
  const int t = t0 + i;
  int le[kTopK];
  float lw[kTopK];
  int nloc = 0;
  if (i < kTok && t < T) {
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
      const int e = ids_s[i][k] - local_start;
      if (e >= 0 && e < E) {
        int j = nloc;  // insertion into the ascending list le[0..nloc)
        while (j > 0 && le[j - 1] > e) {
          le[j] = le[j - 1];
          lw[j] = lw[j - 1];
          --j;
        }
        le[j] = e;
        lw[j] = w_s[i][k];
        ++nloc;
      }
    }
  }
  __syncthreads();  // base[] is visible
  if (rank == 0) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      expert_count[e] = tot[e];
      expert_base[e] = base[e];
    }
    if (threadIdx.x == 0) expert_base[E] = base[E];
  }
  for (int c = threadIdx.x + static_cast<int>(rank) * blockDim.x; c < 2 * kMaxSplitUnits;
       c += ncta * blockDim.x)
    counters[c] = 0;
  if (i < kTok && t < T) {
    int* ts = token_slot + static_cast<size_t>(t) * kTopK;
    float* tw = token_weight + static_cast<size_t>(t) * kTopK;
    const uint32_t below = (1u << i) - 1u;
    for (int j = 0; j < kTopK; ++j) {
      if (j < nloc) {
        const int e = le[j];
        const int slot = base[e] + off[e] + __popc(tokmask[e] & below);
        slot_token[slot] = t;
        slot_weight[slot] = lw[j];
        ts[j] = slot;
        tw[j] = lw[j];
      } else {
        ts[j] = -1;
        tw[j] = 0.0f;
      }
    }
  }
  // padding slots: expert e by warp (e / ncta) of CTA e mod ncta
  for (int e = warp * static_cast<int>(ncta) + static_cast<int>(rank); e < E;
       e += nwarp * static_cast<int>(ncta))
    for (int sl = base[e] + tot[e] + lane; sl < base[e + 1]; sl += 32) {
      slot_token[sl] = -1;
      slot_weight[sl] = 0.0f;
    }
  cluster_wait();  // no CTA exits while another may still read its counts
}

// Gather: one warp per token reads the token's e4m3 row once (7168 B = 14 x 16 B per lane)
// and writes it, with its 128-column scales, to each of the token's slots.
__global__ void __launch_bounds__(256) k_gather_tokens(const int32_t* __restrict__ token_slot,
                                                       const uint8_t* __restrict__ hidden,
                                                       const float* __restrict__ hidden_scale,
                                                       int T, int H, int64_t cap,
                                                       uint8_t* __restrict__ a_perm,
                                                       float* __restrict__ a_scale_t) {
  constexpr int kMaxVec = 16;  // H <= 8192 (at most 64 scale blocks; 16 B per lane per step)
  pdl_begin_in_order();  // GEMM1, which follows, reads the plan before its own wait
  const int lane = threadIdx.x & 31;
  const int warp0 = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  const int nvec = H / 16;
  const int nkb = H / kBlock;
  for (int t = warp0; t < T; t += nwarps) {
    const int my_slot = lane < kTopK ? __ldg(token_slot + static_cast<size_t>(t) * kTopK + lane) : -1;
    const int nloc = __popc(__ballot_sync(0xffffffffu, my_slot >= 0));
    if (nloc == 0) continue;
    const uint4* src = reinterpret_cast<const uint4*>(hidden + static_cast<size_t>(t) * H);
    uint4 row[kMaxVec];
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i)
      if (lane + 32 * i < nvec) row[i] = __ldg(src + lane + 32 * i);
    const float sc0 = lane < nkb ? __ldg(hidden_scale + static_cast<size_t>(lane) * T + t) : 0.f;
    const float sc1 =
        lane + 32 < nkb ? __ldg(hidden_scale + static_cast<size_t>(lane + 32) * T + t) : 0.f;
    for (int j = 0; j < nloc; ++j) {
      const int slot = __shfl_sync(0xffffffffu, my_slot, j);
      uint4* dst = reinterpret_cast<uint4*>(a_perm + static_cast<size_t>(slot) * H);
#pragma unroll
      for (int i = 0; i < kMaxVec; ++i)
        if (lane + 32 * i < nvec) dst[lane + 32 * i] = row[i];
      if (lane < nkb) a_scale_t[static_cast<size_t>(lane) * cap + slot] = sc0;
      if (lane + 32 < nkb) a_scale_t[static_cast<size_t>(lane + 32) * cap + slot] = sc1;
    }
  }
}


cudaError_t launch_route_hist(const RunParams& p, cudaStream_t s) {
  if (p.T <= 0) return cudaSuccess;
  uint8_t* ws = p.ws;
  const Layout& L = p.L;
  if (L.nblocks < p.num_sms) {
    // Few routing blocks (many local experts: at most 8,192 per-block counts): routing in the
    // fused kernel would run on nblocks CTAs only, so the tokens are routed by a grid over every
    // SM (one warp per token) and the blocks then count the picks from the workspace tables.
    cudaError_t e = dispatch_dtypes(p.logits_dtype, p.bias_dtype, [&](auto tl, auto tb) {
      using TL = decltype(tl);
      using TB = decltype(tb);
      int blocks = (p.T + 7) / 8;
      if (blocks > p.num_sms * 16) blocks = p.num_sms * 16;
      (void)launch_pdl(k_route<TL, TB>, blocks, 256, 0, s, static_cast<const TL*>(p.logits),
                       static_cast<const TB*>(p.bias), p.T, p.rsf, p.route_mode,
                       reinterpret_cast<int32_t*>(ws + L.topk_ids),
                       reinterpret_cast<float*>(ws + L.topk_w));
      return cudaGetLastError();
    });
    if (e != cudaSuccess) return e;
    auto* ids = reinterpret_cast<int32_t*>(ws + L.topk_ids);
    auto* w = reinterpret_cast<float*>(ws + L.topk_w);
    (void)launch_pdl(k_hist_given, L.nblocks, 256, 0, s, static_cast<const int32_t*>(ids),
                     static_cast<const float*>(w), static_cast<const int32_t*>(nullptr), p.T,
                     p.T, L.tpb, p.local_start, p.E, 0, ids, w,
                     reinterpret_cast<int32_t*>(ws + L.block_hist));
    return cudaGetLastError();
  }
  return dispatch_dtypes(p.logits_dtype, p.bias_dtype, [&](auto tl, auto tb) {
    using TL = decltype(tl);
    using TB = decltype(tb);
    (void)launch_pdl(k_route_hist<TL, TB>, L.nblocks, 256, 0, s,
        static_cast<const TL*>(p.logits), static_cast<const TB*>(p.bias), p.T, L.tpb, p.rsf,
        p.route_mode, p.local_start, p.E, reinterpret_cast<int32_t*>(ws + L.topk_ids),
        reinterpret_cast<float*>(ws + L.topk_w), reinterpret_cast<int32_t*>(ws + L.block_hist));
    return cudaGetLastError();
  });
}

cudaError_t launch_hist_given(const RunParams& p, cudaStream_t s) {
  if (p.T <= 0) return cudaSuccess;
  uint8_t* ws = p.ws;
  const Layout& L = p.L;
  (void)launch_pdl(k_hist_given, L.nblocks, 256, 0, s, p.in_ids, p.in_w, p.region_counts,
                   p.region_tokens, p.T, L.tpb, p.local_start, p.E, 1,
                   reinterpret_cast<int32_t*>(ws + L.topk_ids),
                   reinterpret_cast<float*>(ws + L.topk_w),
                   reinterpret_cast<int32_t*>(ws + L.block_hist));
  return cudaGetLastError();
}

cudaError_t launch_scan(const RunParams& p, cudaStream_t s) {
  uint8_t* ws = p.ws;
  const Layout& L = p.L;
  (void)launch_pdl(k_scan, 1, 1024, 0, s, reinterpret_cast<const int32_t*>(ws + L.block_hist), L.nblocks, p.E,
                            p.H, p.I, p.num_sms, p.T <= kSplitMaxT ? 1 : 0,
                            reinterpret_cast<int32_t*>(ws + L.block_off),
                            reinterpret_cast<int32_t*>(ws + L.plan),
                            reinterpret_cast<int32_t*>(ws + L.expert_count),
                            reinterpret_cast<int32_t*>(ws + L.expert_base),
                            reinterpret_cast<int32_t*>(ws + L.counters),
                            reinterpret_cast<int32_t*>(ws + L.status));
  return cudaGetLastError();
}

cudaError_t launch_scatter_gather(const RunParams& p, cudaStream_t s) {
  if (p.T <= 0) return cudaSuccess;
  uint8_t* ws = p.ws;
  const Layout& L = p.L;
  (void)launch_pdl(k_scatter, L.nblocks, 256, 0, s,
      reinterpret_cast<const int32_t*>(ws + L.topk_ids),
      reinterpret_cast<const float*>(ws + L.topk_w), p.T, L.tpb, p.local_start, p.E,
      reinterpret_cast<const int32_t*>(ws + L.block_off),
      reinterpret_cast<const int32_t*>(ws + L.expert_count),
      reinterpret_cast<const int32_t*>(ws + L.expert_base),
      reinterpret_cast<int32_t*>(ws + L.slot_token), reinterpret_cast<float*>(ws + L.slot_weight),
      reinterpret_cast<int32_t*>(ws + L.token_slot),
      reinterpret_cast<float*>(ws + L.token_weight));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_gather(p, s);
}

cudaError_t launch_gather(const RunParams& p, cudaStream_t s) {
  if (p.T <= 0) return cudaSuccess;
  uint8_t* ws = p.ws;
  const Layout& L = p.L;
  int blocks = (p.T + 7) / 8;
  if (blocks > p.num_sms * 8) blocks = p.num_sms * 8;
  (void)launch_pdl(k_gather_tokens, blocks, 256, 0, s, reinterpret_cast<const int32_t*>(ws + L.token_slot),
                                         p.hidden, p.hidden_scale, p.T, p.H, L.cap,
                                         ws + L.a_perm, reinterpret_cast<float*>(ws + L.a_scale_t));
  return cudaGetLastError();
}

cudaError_t launch_plan_small(const RunParams& p, cudaStream_t s) {
  if (p.T <= 0) return cudaSuccess;
  if (p.T > kSmallT) return cudaErrorInvalidValue;
  uint8_t* ws = p.ws;
  const Layout& L = p.L;
  return dispatch_dtypes(p.logits_dtype, p.bias_dtype, [&](auto tl, auto tb) {
    using TL = decltype(tl);
    using TB = decltype(tb);
    // one CTA runs as the implicit single-CTA cluster (no cluster launch attribute)
    const int ncta = (p.T + kSmallTokensPerCta - 1) / kSmallTokensPerCta;
    auto kern = k_plan_small<TL, TB>;
    auto launch = [&](auto... a) {
      return ncta == 1 ? launch_pdl(kern, 1, 32 * kSmallTokensPerCta, 0, s, a...)
                       : launch_pdl_cluster(kern, ncta, 32 * kSmallTokensPerCta, 0, s, ncta, a...);
    };
    (void)launch(static_cast<const TL*>(p.logits),
                     static_cast<const TB*>(p.bias), p.T, p.rsf, p.route_mode, p.local_start,
                     p.E, p.H, p.I,
                     p.num_sms, p.T <= kSplitMaxT ? 1 : 0,
                     reinterpret_cast<int32_t*>(ws + L.topk_ids),
                     reinterpret_cast<float*>(ws + L.topk_w), reinterpret_cast<int32_t*>(ws + L.plan),
                     reinterpret_cast<int32_t*>(ws + L.expert_count),
                     reinterpret_cast<int32_t*>(ws + L.expert_base),
                     reinterpret_cast<int32_t*>(ws + L.counters),
                     reinterpret_cast<int32_t*>(ws + L.status),
                     reinterpret_cast<int32_t*>(ws + L.slot_token),
                     reinterpret_cast<float*>(ws + L.slot_weight),
                     reinterpret_cast<int32_t*>(ws + L.token_slot),
                     reinterpret_cast<float*>(ws + L.token_weight));
    return cudaGetLastError();
  });
}

cudaError_t launch_route_permute(const void* logits, int logits_dtype, const void* bias,
                                 int bias_dtype, int T, int E, int local_start, float rsf,
                                 int H, int I, int num_sms, const PermuteBuffers& bf,
                                 cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  const int tpb = routing_tpb(T, E);
  const int nblocks = (T + tpb - 1) / tpb;
  cudaError_t e = dispatch_dtypes(logits_dtype, bias_dtype, [&](auto tl, auto tb) {
    using TL = decltype(tl);
    using TB = decltype(tb);
    (void)launch_pdl(k_route_hist<TL, TB>, nblocks, 256, 0, s, static_cast<const TL*>(logits),
                                                  static_cast<const TB*>(bias), T, tpb, rsf,
                                                  kRouteDeepSeek, local_start, E, bf.topk_ids,
                                                  bf.topk_w,
                                                  bf.block_hist);
    return cudaGetLastError();
  });
  if (e != cudaSuccess) return e;
  (void)launch_pdl(k_scan, 1, 1024, 0, s, bf.block_hist, nblocks, E, H, I, num_sms,
                   T <= kSplitMaxT ? 1 : 0, bf.block_off, bf.plan,
                            bf.expert_count, bf.expert_base, bf.counters, bf.status);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  (void)launch_pdl(k_scatter, nblocks, 256, 0, s, bf.topk_ids, bf.topk_w, T, tpb, local_start, E,
                                    bf.block_off, bf.expert_count, bf.expert_base, bf.slot_token,
                                    bf.slot_weight, bf.token_slot, bf.token_weight);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------
// Combine: one CTA per (token, 8 * blockDim columns) sums w * Y[slot] over the token's local
// picks in ascending expert order (the definition's loop order, moe.py:79-98), in registers,
// then writes bf16; small T still spreads over every SM.
// Y rows are fp16 with a power-of-two scale per 256 columns (exact to apply). Tokens without
// local picks get zeros (kernel.py:692-695 zero-fills when nothing is local).
// ------------------------------------------------------------------------------------------

// Each thread owns 32 consecutive output columns (inside one 256-column scale tile) of one
// token: per local pick it issues both 32-byte loads of the y row at once (64 bytes in flight);
// the picks are added in ascending expert order.
constexpr int kCombineVec = 4;
constexpr int kCombineThreads = 128;

// Destinations of FMOE_OUT_F16S rows: token t = r * region_tokens + j goes to p[r] + j * rowbytes.
struct RegionOut {
  void* p[FMOE_EP_MAX_RANKS];
};

// Exponent k of the smallest 2^k with amax / 2^k <= 16384: fp16 range kept, scaling exact.
__device__ __forceinline__ int pow2_exp_f16(float amax) {
  int ex = 0;
  const float m = frexpf(amax, &ex);
  return (m > 0.5f ? ex : ex - 1) - 14;
}

// One 32-column piece of a partial row: fp16 values with the 256-column block's power-of-two
// scale (the block's 8 owning threads, consecutive lanes, agree on it by a shuffle reduction).
__device__ __forceinline__ void store_f16s(uint8_t* row, int H, int col0, unsigned mask,
                                           const float (&acc)[kCombineVec][8]) {
  float m = 0.0f;
#pragma unroll
  for (int k = 0; k < kCombineVec; ++k)
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(acc[k][i]));
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) m = fmaxf(m, __shfl_xor_sync(mask, m, o));
  const int e = pow2_exp_f16(m);
  const float inv = ldexpf(1.0f, -e);
  uint32_t w[2][8];
#pragma unroll
  for (int k = 0; k < kCombineVec; ++k)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 h = __floats2half2_rn(acc[k][2 * i] * inv, acc[k][2 * i + 1] * inv);
      w[k >> 1][(k & 1) * 4 + i] = *reinterpret_cast<const uint32_t*>(&h);
    }
  st_global_v8(row + static_cast<size_t>(col0) * 2, w[0]);
  st_global_v8(row + static_cast<size_t>(col0) * 2 + 32, w[1]);
  if ((col0 & (kTileN - 1)) == 0)
    reinterpret_cast<float*>(row + static_cast<size_t>(H) * 2)[col0 / kTileN] = ldexpf(1.0f, e);
}

template <typename TOut>
__global__ void __launch_bounds__(kCombineThreads) k_combine(const int32_t* __restrict__ token_slot,
                                                             const float* __restrict__ token_weight,
                                                             const __half* __restrict__ y,
                                                             const float* __restrict__ y_scale,
                                                             int T, int H, TOut* __restrict__ out,
                                                             const RegionOut regions,
                                                             int region_tokens) {
  pdl_begin();
  const int nvec = H / 8;
  const int ntile = H / kTileN;
  const int per_block = kCombineThreads * kCombineVec;
  const int chunks = (nvec + per_block - 1) / per_block;
  const long work = static_cast<long>(T) * chunks;
  for (long wi = blockIdx.x; wi < work; wi += gridDim.x) {
    const int t = static_cast<int>(wi / chunks);
    const int v0 = static_cast<int>(wi - static_cast<long>(t) * chunks) * per_block +
                   threadIdx.x * kCombineVec;
    const int4* ts = reinterpret_cast<const int4*>(token_slot + static_cast<size_t>(t) * kTopK);
    const float4* tw = reinterpret_cast<const float4*>(token_weight + static_cast<size_t>(t) * kTopK);
    const int4 s0 = __ldg(ts), s1 = __ldg(ts + 1);
    const float4 w0 = __ldg(tw), w1 = __ldg(tw + 1);
    const int slots[kTopK] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const float w[kTopK] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    if (v0 >= nvec) continue;
    // partial rows: a token without a local pick was not received (its row is not written)
    if (std::is_same<TOut, uint8_t>::value && slots[0] < 0) continue;
    const int col0 = v0 * 8;  // 32 columns: two 32-byte loads of the y row
    const int tile = col0 / kTileN;
    float acc[kCombineVec][8];
#pragma unroll
    for (int k = 0; k < kCombineVec; ++k)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[k][i] = 0.0f;
    // local picks occupy slots[0 .. nloc) in ascending expert order
#pragma unroll
    for (int j = 0; j < kTopK; ++j) {
      if (slots[j] < 0) break;
      const size_t row = static_cast<size_t>(slots[j]);
      uint32_t raw[2][8];
      ld_global_nc_v8(y + row * H + col0, raw[0]);
      ld_global_nc_v8(y + row * H + col0 + 16, raw[1]);
      const float f = __ldg(y_scale + row * ntile + tile) * w[j];
#pragma unroll
      for (int k = 0; k < kCombineVec; ++k) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t bits = raw[k >> 1][(k & 1) * 4 + i];
          const float2 q = __half22float2(*reinterpret_cast<const __half2*>(&bits));
          acc[k][2 * i] = fmaf(f, q.x, acc[k][2 * i]);
          acc[k][2 * i + 1] = fmaf(f, q.y, acc[k][2 * i + 1]);
        }
      }
    }
    if constexpr (std::is_same<TOut, uint8_t>::value) {
      // the 8 threads of a 256-column block are consecutive lanes with the same token, and a
      // token's threads are all active or all skipped: the shuffle mask is the lane's octet
      const unsigned mask = 0xffu << (threadIdx.x & 24);
      const int r = t / region_tokens;
      uint8_t* row = static_cast<uint8_t*>(regions.p[r]) +
                     static_cast<size_t>(t - r * region_tokens) * FMOE_EP_ROW_BYTES(H);
      store_f16s(row, H, col0, mask, acc);
    } else {
#pragma unroll
      for (int k = 0; k < kCombineVec; ++k)
        store8(out + static_cast<size_t>(t) * H, v0 + k, acc[k]);
    }
  }
}

cudaError_t launch_combine(const RunParams& p, cudaStream_t s) {
  if (p.T <= 0) return cudaSuccess;
  uint8_t* ws = p.ws;
  const Layout& L = p.L;
  const int per_block = kCombineThreads * kCombineVec;
  const long work = static_cast<long>(p.T) * ((p.H / 8 + per_block - 1) / per_block);
  const int blocks = static_cast<int>(work < p.num_sms * 16L ? work : p.num_sms * 16L);
  RegionOut regions{};
  for (int r = 0; r < FMOE_EP_MAX_RANKS; ++r) regions.p[r] = p.region_out[r];
  const int rt = p.region_tokens > 0 ? p.region_tokens : p.T;
  const auto* ts = reinterpret_cast<const int32_t*>(ws + L.token_slot);
  const auto* tw = reinterpret_cast<const float*>(ws + L.token_weight);
  const auto* yr = reinterpret_cast<const __half*>(ws + L.y_rows);
  const auto* ys = reinterpret_cast<const float*>(ws + L.y_scale);
  if (p.out_mode == FMOE_OUT_F32)
    (void)launch_pdl(k_combine<float>, blocks, kCombineThreads, 0, s, ts, tw, yr, ys, p.T, p.H,
                     static_cast<float*>(p.output), regions, rt);
  else if (p.out_mode == FMOE_OUT_F16S)
    (void)launch_pdl(k_combine<uint8_t>, blocks, kCombineThreads, 0, s, ts, tw, yr, ys, p.T, p.H,
                     static_cast<uint8_t*>(nullptr), regions, rt);
  else
    (void)launch_pdl(k_combine<__nv_bfloat16>, blocks, kCombineThreads, 0, s, ts, tw, yr, ys, p.T,
                     p.H, static_cast<__nv_bfloat16*>(p.output), regions, rt);
  return cudaGetLastError();
}

}  // namespace fmoe
