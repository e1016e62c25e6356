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
#include <math.h>

#include "fmoe_internal.h"

namespace fmoe {

// ------------------------------------------------------------------------------------------
// Routing: one warp per token, lane l owns experts [8l, 8l+8). Group g = lanes 4g..4g+3.
// ------------------------------------------------------------------------------------------
template <typename TL>
__device__ __forceinline__ void load8(const TL* p, float (&x)[8]);

template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&x)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&x)[8]) {
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

// sigmoid with the same three roundings as 1/(1+exp(-x)) in fp32: exp(-x) correctly rounded
// to fp32 (evaluated in double), then an IEEE fp32 add and an IEEE fp32 divide.
__device__ __forceinline__ float sigmoid_rn(float x) {
  const float e = static_cast<float>(exp(-static_cast<double>(x)));
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
}

template <typename TL, typename TB>
__global__ void __launch_bounds__(256) k_route(const TL* __restrict__ logits,
                                               const TB* __restrict__ bias, int T, float rsf,
                                               int32_t* __restrict__ ids_out,
                                               float* __restrict__ w_out) {
  const int lane = threadIdx.x & 31;
  const int warp0 = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  float b[8];
  load8<TB>(bias + lane * 8, b);
  const float NEG_INF = -INFINITY;

  for (int t = warp0; t < T; t += nwarps) {
    float x[8], s[8], sb[8];
    load8<TL>(logits + static_cast<size_t>(t) * kExpertsGlobal + lane * 8, x);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s[i] = sigmoid_rn(x[i]);
      sb[i] = __fadd_rn(s[i], b[i]);
    }
    // Top-2 of the biased scores in each group of 32 (kernel.py:406-416).
    float m1 = NEG_INF, m2 = NEG_INF;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float v = sb[i];
      if (v > m1) {
        m2 = m1;
        m1 = v;
      } else if (v > m2) {
        m2 = v;
      }
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      const float o1 = __shfl_xor_sync(0xffffffffu, m1, off);
      const float o2 = __shfl_xor_sync(0xffffffffu, m2, off);
      const float n1 = fmaxf(m1, o1);
      const float n2 = fmaxf(fminf(m1, o1), fmaxf(m2, o2));
      m1 = n1;
      m2 = n2;
    }
    const float gscore = __fadd_rn(m1, m2);
    float gs[kGroups];
#pragma unroll
    for (int g = 0; g < kGroups; ++g) gs[g] = __shfl_sync(0xffffffffu, gscore, 4 * g);
    // Keep the 4 best groups; ties go to the lower group index (kernel.py:418-426).
    uint32_t gmask = 0;
#pragma unroll
    for (int g = 0; g < kGroups; ++g) {
      int rank = 0;
#pragma unroll
      for (int h = 0; h < kGroups; ++h)
        rank += (gs[h] > gs[g]) || (gs[h] == gs[g] && h < g);
      if (rank < kTopKGroups) gmask |= 1u << g;
    }
    const bool kept = (gmask >> (lane >> 2)) & 1u;
    // Top-8 over the kept groups by biased score; ties to the lowest index (kernel.py:428-438).
    uint32_t taken = kept ? 0u : 0xffu;
    int ids[kTopK];
    float sv[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
      float bv = NEG_INF, bs = 0.0f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        // strict '>' keeps the lowest index among equal scores
        if (!((taken >> i) & 1u) && (bi == 0x7fffffff || sb[i] > bv)) {
          bv = sb[i];
          bs = s[i];
          bi = lane * 8 + i;
        }
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const float os = __shfl_xor_sync(0xffffffffu, bs, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        const bool better = (oi != 0x7fffffff) &&
                            (bi == 0x7fffffff || ov > bv || (ov == bv && oi < bi));
        if (better) {
          bv = ov;
          bs = os;
          bi = oi;
        }
      }
      ids[k] = bi;
      sv[k] = bs;
      if ((bi >> 3) == lane) taken |= 1u << (bi & 7);
    }
    // Weights from the un-biased scores (moe.py:165-168): (s / (sum + 1e-20)) * rsf, with the
    // sum taken in selection order.
    float denom = 0.0f;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) denom = __fadd_rn(denom, sv[k]);
    denom = __fadd_rn(denom, 1e-20f);
    if (lane == 0) {
      int4* io = reinterpret_cast<int4*>(ids_out + static_cast<size_t>(t) * kTopK);
      float4* wo = reinterpret_cast<float4*>(w_out + static_cast<size_t>(t) * kTopK);
      float w[kTopK];
#pragma unroll
      for (int k = 0; k < kTopK; ++k) w[k] = __fmul_rn(__fdiv_rn(sv[k], denom), rsf);
      io[0] = make_int4(ids[0], ids[1], ids[2], ids[3]);
      io[1] = make_int4(ids[4], ids[5], ids[6], ids[7]);
      wo[0] = make_float4(w[0], w[1], w[2], w[3]);
      wo[1] = make_float4(w[4], w[5], w[6], w[7]);
    }
  }
}

cudaError_t launch_route(const void* logits, int logits_dtype, const void* bias, int bias_dtype,
                         int T, float rsf, int32_t* topk_ids, float* topk_w, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  const int warps_per_block = 8;
  int blocks = (T + warps_per_block - 1) / warps_per_block;
  if (blocks > 148 * 16) blocks = 148 * 16;
  const dim3 grid(blocks), block(warps_per_block * 32);
  if (logits_dtype == FMOE_DTYPE_F32 && bias_dtype == FMOE_DTYPE_BF16)
    k_route<float, __nv_bfloat16><<<grid, block, 0, s>>>(
        static_cast<const float*>(logits), static_cast<const __nv_bfloat16*>(bias), T, rsf,
        topk_ids, topk_w);
  else if (logits_dtype == FMOE_DTYPE_F32 && bias_dtype == FMOE_DTYPE_F32)
    k_route<float, float><<<grid, block, 0, s>>>(static_cast<const float*>(logits),
                                                  static_cast<const float*>(bias), T, rsf,
                                                  topk_ids, topk_w);
  else if (logits_dtype == FMOE_DTYPE_BF16 && bias_dtype == FMOE_DTYPE_BF16)
    k_route<__nv_bfloat16, __nv_bfloat16><<<grid, block, 0, s>>>(
        static_cast<const __nv_bfloat16*>(logits), static_cast<const __nv_bfloat16*>(bias), T,
        rsf, topk_ids, topk_w);
  else
    k_route<__nv_bfloat16, float><<<grid, block, 0, s>>>(
        static_cast<const __nv_bfloat16*>(logits), static_cast<const float*>(bias), T, rsf,
        topk_ids, topk_w);
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------
// Plan: one CTA of 1024 threads builds the deterministic, stable permutation.
//   pass 1: per-expert counts (order-free shared-memory atomics) -> padded bases
//   pass 2: chunks of 1024 tokens; per-warp ballots give each (token, expert) its rank among
//           earlier tokens, so slots are ascending in token id within each expert
//   pass 3: padding slots, split-K choice, counter reset
// ------------------------------------------------------------------------------------------
__device__ int choose_split(int tiles, int nkb, int G) {
  if (tiles <= 0 || tiles >= G) return 1;
  int best = 1;
  long best_cost = 0x7fffffffffffL;
  for (int s = 1; s <= kMaxSplit && s <= nkb; ++s) {
    if (static_cast<long>(tiles) * s > kMaxSplitUnits) break;
    const long waves = (static_cast<long>(tiles) * s + G - 1) / G;
    const long per = (nkb + s - 1) / s;
    const long cost = waves * per + (s > 1 ? 1 : 0);
    if (cost < best_cost) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

struct PlanSmem {
  int cnt[kMaxLocalExperts];
  int base[kMaxLocalExperts + 1];
  int run[kMaxLocalExperts];
  int wcnt[32][kMaxLocalExperts];
};

__global__ void __launch_bounds__(1024) k_plan(const int32_t* __restrict__ ids,
                                               const float* __restrict__ wts, int T,
                                               int local_start, int E, int H, int I, int G,
                                               int64_t cap, int32_t* __restrict__ plan,
                                               int32_t* __restrict__ expert_count,
                                               int32_t* __restrict__ expert_base,
                                               int32_t* __restrict__ slot_token,
                                               float* __restrict__ slot_weight,
                                               int32_t* __restrict__ token_slot,
                                               float* __restrict__ token_weight,
                                               int32_t* __restrict__ counters,
                                               int32_t* __restrict__ status) {
  __shared__ PlanSmem sm;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < E; e += blockDim.x) {
    sm.cnt[e] = 0;
    sm.run[e] = 0;
  }
  __syncthreads();
  // pass 1: counts
  for (int t = tid; t < T; t += blockDim.x) {
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
      const int le = ids[static_cast<size_t>(t) * kTopK + k] - local_start;
      if (le >= 0 && le < E) atomicAdd(&sm.cnt[le], 1);
    }
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0, pairs = 0;
    for (int e = 0; e < E; ++e) {
      sm.base[e] = acc;
      acc += (sm.cnt[e] + kTileM - 1) / kTileM * kTileM;
      pairs += sm.cnt[e];
    }
    sm.base[E] = acc;
    const int mtiles = acc / kTileM;
    const int tiles1 = mtiles * (I / kBlock);
    const int tiles2 = mtiles * (H / kTileN);
    const int s1 = choose_split(tiles1, H / kBlock, G);
    const int s2 = choose_split(tiles2, I / kBlock, G);
    plan[kPlanPairs] = pairs;
    plan[kPlanPadded] = acc;
    plan[kPlanMTiles] = mtiles;
    plan[kPlanSplit1] = s1;
    plan[kPlanUnits1] = tiles1 * s1;
    plan[kPlanSplit2] = s2;
    plan[kPlanUnits2] = tiles2 * s2;
    plan[kPlanTiles1] = tiles1;
    plan[kPlanTiles2] = tiles2;
    status[0] = 0;
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    expert_count[e] = sm.cnt[e];
    expert_base[e] = sm.base[e];
  }
  if (tid == 0) expert_base[E] = sm.base[E];
  for (int i = tid; i < 2 * kMaxSplitUnits; i += blockDim.x) counters[i] = 0;

  // pass 2: stable slots
  const int nwords = (E + 31) >> 5;
  for (int c0 = 0; c0 < T; c0 += blockDim.x) {
    const int t = c0 + tid;
    int le[kTopK];
    float lw[kTopK];
    int nloc = 0;
    if (t < T) {
#pragma unroll
      for (int k = 0; k < kTopK; ++k) {
        const int e = ids[static_cast<size_t>(t) * kTopK + k] - local_start;
        if (e >= 0 && e < E) {
          // insertion into the ascending list le[0..nloc)
          int j = nloc;
          const float w = wts[static_cast<size_t>(t) * kTopK + k];
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
          if (has) {
            rank[jp] = __popc(bal & ((1u << lane) - 1u));
            ++jp;
          }
        }
      }
    }
    __syncthreads();
    for (int e = tid; e < E; e += blockDim.x) {
      int acc = sm.run[e];
      for (int w = 0; w < 32; ++w) {
        const int c = sm.wcnt[w][e];
        sm.wcnt[w][e] = acc;
        acc += c;
      }
      sm.run[e] = acc;
    }
    __syncthreads();
    if (t < T) {
      int* ts = token_slot + static_cast<size_t>(t) * kTopK;
      float* tw = token_weight + static_cast<size_t>(t) * kTopK;
      for (int j = 0; j < kTopK; ++j) {
        if (j < nloc) {
          const int e = le[j];
          const int slot = sm.base[e] + sm.wcnt[warp][e] + rank[j];
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
  // pass 3: padding slots
  for (int e = 0; e < E; ++e) {
    const int first = sm.base[e] + sm.cnt[e];
    const int end = sm.base[e + 1];
    for (int s = first + tid; s < end; s += blockDim.x) {
      slot_token[s] = -1;
      slot_weight[s] = 0.0f;
    }
  }
}

cudaError_t launch_plan(const RunParams& p, cudaStream_t s) {
  uint8_t* ws = p.ws;
  const Layout& L = p.L;
  k_plan<<<1, 1024, 0, s>>>(
      reinterpret_cast<const int32_t*>(ws + L.topk_ids),
      reinterpret_cast<const float*>(ws + L.topk_w), p.T, p.local_start, p.E, p.H, p.I,
      p.num_sms, L.cap, reinterpret_cast<int32_t*>(ws + L.plan),
      reinterpret_cast<int32_t*>(ws + L.expert_count),
      reinterpret_cast<int32_t*>(ws + L.expert_base),
      reinterpret_cast<int32_t*>(ws + L.slot_token), reinterpret_cast<float*>(ws + L.slot_weight),
      reinterpret_cast<int32_t*>(ws + L.token_slot),
      reinterpret_cast<float*>(ws + L.token_weight), reinterpret_cast<int32_t*>(ws + L.counters),
      reinterpret_cast<int32_t*>(ws + L.status));
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------
// Gather: one warp per slot copies the token's e4m3 row and transposes its 128-column scales
// into the [H/128, cap] layout the GEMM1 epilogue reads. Padding slots get zeros.
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_gather(const int32_t* __restrict__ plan,
                                                const int32_t* __restrict__ slot_token,
                                                const uint8_t* __restrict__ hidden,
                                                const float* __restrict__ hidden_scale, int T,
                                                int H, int64_t cap, uint8_t* __restrict__ a_perm,
                                                float* __restrict__ a_scale_t) {
  const int lane = threadIdx.x & 31;
  const int warp0 = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  const int padded = plan[kPlanPadded];
  const int nvec = H / 16;
  const int nkb = H / kBlock;
  for (int slot = warp0; slot < padded; slot += nwarps) {
    const int tok = slot_token[slot];
    uint4* dst = reinterpret_cast<uint4*>(a_perm + static_cast<size_t>(slot) * H);
    if (tok >= 0) {
      const uint4* src = reinterpret_cast<const uint4*>(hidden + static_cast<size_t>(tok) * H);
      for (int i = lane; i < nvec; i += 32) dst[i] = __ldg(src + i);
      for (int kb = lane; kb < nkb; kb += 32)
        a_scale_t[static_cast<size_t>(kb) * cap + slot] =
            __ldg(hidden_scale + static_cast<size_t>(kb) * T + tok);
    } else {
      const uint4 z = make_uint4(0, 0, 0, 0);
      for (int i = lane; i < nvec; i += 32) dst[i] = z;
      for (int kb = lane; kb < nkb; kb += 32) a_scale_t[static_cast<size_t>(kb) * cap + slot] = 0.f;
    }
  }
}

cudaError_t launch_gather(const RunParams& p, cudaStream_t s) {
  uint8_t* ws = p.ws;
  const Layout& L = p.L;
  int blocks = static_cast<int>((L.cap + 7) / 8);
  const int max_blocks = p.num_sms * 8;
  if (blocks > max_blocks) blocks = max_blocks;
  if (blocks < 1) blocks = 1;
  k_gather<<<blocks, 256, 0, s>>>(
      reinterpret_cast<const int32_t*>(ws + L.plan),
      reinterpret_cast<const int32_t*>(ws + L.slot_token), p.hidden, p.hidden_scale, p.T, p.H,
      L.cap, ws + L.a_perm, reinterpret_cast<float*>(ws + L.a_scale_t));
  return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------
// Combine: one CTA per token sums w * Y[slot] over the token's local picks in ascending
// expert order (the definition's loop order, moe.py:79-98), in registers, then writes bf16.
// Tokens without local picks get zeros (kernel.py:692-695 zero-fills when nothing is local).
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) k_combine(const int32_t* __restrict__ token_slot,
                                                 const float* __restrict__ token_weight,
                                                 const __nv_bfloat16* __restrict__ y, int T,
                                                 int H, __nv_bfloat16* __restrict__ out) {
  const int nvec = H / 8;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    int slots[kTopK];
    float w[kTopK];
#pragma unroll
    for (int j = 0; j < kTopK; ++j) {
      slots[j] = __ldg(token_slot + static_cast<size_t>(t) * kTopK + j);
      w[j] = __ldg(token_weight + static_cast<size_t>(t) * kTopK + j);
    }
    for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
#pragma unroll
      for (int j = 0; j < kTopK; ++j) {
        if (slots[j] < 0) break;
        const uint4 raw =
            __ldg(reinterpret_cast<const uint4*>(y + static_cast<size_t>(slots[j]) * H) + v);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(h[i]);
          acc[2 * i] = fmaf(w[j], f.x, acc[2 * i]);
          acc[2 * i + 1] = fmaf(w[j], f.y, acc[2 * i + 1]);
        }
      }
      uint4 o;
      __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) oh[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H)[v] = o;
    }
  }
}

cudaError_t launch_combine(const RunParams& p, cudaStream_t s) {
  if (p.T <= 0) return cudaSuccess;
  uint8_t* ws = p.ws;
  const Layout& L = p.L;
  int blocks = p.T < p.num_sms * 16 ? p.T : p.num_sms * 16;
  k_combine<<<blocks, 128, 0, s>>>(reinterpret_cast<const int32_t*>(ws + L.token_slot),
                                   reinterpret_cast<const float*>(ws + L.token_weight),
                                   reinterpret_cast<const __nv_bfloat16*>(ws + L.y_rows), p.T,
                                   p.H, p.output);
  return cudaGetLastError();
}

}  // namespace fmoe
