// fmoe_route.cuh -- the routing of one token by one warp (DeepSeek-V3 grouped routing and the
// other routing methods of the definition family), shared by the routing/plan kernels
// (fmoe_kernels.cu) and the small-batch matrix-vector kernels (fmoe_gemv.cu), plus the
// host-side dispatch over the logits / bias dtypes.
#pragma once

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
// to fp32 (evaluated in double), then an IEEE fp32 add and an IEEE fp32 divide (1/y correctly
// rounded, computed as the correctly rounded reciprocal).
__device__ __forceinline__ float sigmoid_rn(float x) {
  const float e = static_cast<float>(exp(-static_cast<double>(x)));
  return __frcp_rn(__fadd_rn(1.0f, e));
}

// Routes one token with one warp. Returns, in every lane, the 8 picks (selection order:
// descending biased score, lowest index first on ties) and their weights.
template <typename TL>
__device__ __forceinline__ void route_token_ds(const TL* __restrict__ row, const float (&b)[8],
                                               float rsf, int lane, int (&ids)[kTopK],
                                               float (&wts)[kTopK]) {
  const float NEG_INF = -INFINITY;
  float x[8], s[8], sb[8];
  load8<TL>(row + lane * 8, x);
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
  const float gscore = __fadd_rn(m1, m2);  // the same in the 4 lanes of a group
  // Keep the 4 best groups; ties go to the lower group index (kernel.py:418-426). Each lane
  // ranks its own group against the 8 group scores.
  const int myg = lane >> 2;
  int grank = 0;
#pragma unroll
  for (int h = 0; h < kGroups; ++h) {
    const float gh = __shfl_sync(0xffffffffu, gscore, 4 * h);
    grank += (gh > gscore) || (gh == gscore && h < myg);
  }
  const bool kept = grank < kTopKGroups;
  // Top-8 over the kept groups by biased score; ties to the lowest index (kernel.py:428-438).
  // Each candidate becomes an order-preserving 32-bit key, so one warp-wide max reduction
  // (redux.sync) finds the best score and a second one the lowest index holding it.
  uint32_t key[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t u = __float_as_uint(sb[i] + 0.0f);  // -0 -> +0
    key[i] = kept ? ((u & 0x80000000u) ? ~u : (u | 0x80000000u)) : 0u;
  }
  float sv[kTopK];
#pragma unroll
  for (int k = 0; k < kTopK; ++k) {
    uint32_t best = 0;
    int bi = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (key[i] > best) {  // strict '>' keeps the lowest local index among equal keys
        best = key[i];
        bi = i;
      }
    }
    const uint32_t top = __reduce_max_sync(0xffffffffu, best);
    const uint32_t mine = (best == top) ? static_cast<uint32_t>(255 - (lane * 8 + bi)) : 0u;
    const int win = 255 - static_cast<int>(__reduce_max_sync(0xffffffffu, mine));
    const int wl = win >> 3, wi = win & 7;
    float s_win = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i == wi) s_win = s[i];
    sv[k] = __shfl_sync(0xffffffffu, s_win, wl);
    ids[k] = win;
    if (lane == wl) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i == wi) key[i] = 0u;
    }
  }
  // Weights from the un-biased scores (moe.py:165-168): (s / (sum + 1e-20)) * rsf, with the
  // sum taken in selection order; lane k divides pick k, then every lane gathers the eight.
  float denom = 0.0f;
  float my_sv = sv[0];
#pragma unroll
  for (int k = 0; k < kTopK; ++k) {
    denom = __fadd_rn(denom, sv[k]);
    if (lane == k) my_sv = sv[k];
  }
  denom = __fadd_rn(denom, 1e-20f);
  const float my_w = __fmul_rn(__fdiv_rn(my_sv, denom), rsf);
#pragma unroll
  for (int k = 0; k < kTopK; ++k) wts[k] = __shfl_sync(0xffffffffu, my_w, k);
}

// Order-preserving 32-bit key of a float (larger value, larger key; -0 and +0 equal).
__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t u = __float_as_uint(v + 0.0f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// The other routing methods of the definition family (flashinfer/trace/templates/moe.py:
// 187-390), one warp per token, lane l holding experts 8l..8l+7. z = logit + bias (fp32).
// DEFAULT / RENORMALIZE_NAIVE select on softmax(z) (max-subtracted exponentials, expf, one
// warp-wide sum, IEEE divide); RENORMALIZE, LLAMA4 and TOPK select on z. The top-K picks come
// in descending order, ties to the lower expert index (one redux.sync max of the value's key,
// a second for the index, per pick); picks k >= K are -1 with weight 0.
template <typename TL>
__device__ __forceinline__ void route_token_other(const TL* __restrict__ row, const float (&b)[8],
                                                  float rsf, int method, int K, int lane,
                                                  int (&ids)[kTopK], float (&wts)[kTopK]) {
  float x[8], z[8], sel[8];
  load8<TL>(row + lane * 8, x);
#pragma unroll
  for (int i = 0; i < 8; ++i) z[i] = __fadd_rn(x[i], b[i]);
  const bool softmax_first =
      method == FMOE_ROUTING_DEFAULT || method == FMOE_ROUTING_RENORMALIZE_NAIVE;
  if (softmax_first) {
    float m = z[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) m = fmaxf(m, z[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float part = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      sel[i] = expf(__fsub_rn(z[i], m));
      part = __fadd_rn(part, sel[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, o));
#pragma unroll
    for (int i = 0; i < 8; ++i) sel[i] = __fdiv_rn(sel[i], part);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) sel[i] = z[i];
  }
  uint32_t key[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) key[i] = order_key(sel[i]);
  float pv[kTopK], pz[kTopK];  // each pick's selection value and its z
#pragma unroll
  for (int k = 0; k < kTopK; ++k) {
    ids[k] = -1;
    pv[k] = 0.0f;
    pz[k] = 0.0f;
    if (k >= K) continue;  // K is the same in every lane
    uint32_t best = 0;
    int bi = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (key[i] > best) {
        best = key[i];
        bi = i;
      }
    const uint32_t top = __reduce_max_sync(0xffffffffu, best);
    const uint32_t mine = (best == top) ? static_cast<uint32_t>(255 - (lane * 8 + bi)) : 0u;
    const int win = 255 - static_cast<int>(__reduce_max_sync(0xffffffffu, mine));
    const int wl = win >> 3, wi = win & 7;
    float v = 0.0f, zz = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i == wi) {
        v = sel[i];
        zz = z[i];
      }
    pv[k] = __shfl_sync(0xffffffffu, v, wl);
    pz[k] = __shfl_sync(0xffffffffu, zz, wl);
    ids[k] = win;
    if (lane == wl) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i == wi) key[i] = 0u;
    }
  }
  // weights (the same in every lane)
  if (method == FMOE_ROUTING_DEFAULT) {
#pragma unroll
    for (int k = 0; k < kTopK; ++k) wts[k] = k < K ? __fmul_rn(pv[k], rsf) : 0.0f;
  } else if (method == FMOE_ROUTING_RENORMALIZE_NAIVE) {
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < kTopK; ++k)
      if (k < K) sum = __fadd_rn(sum, pv[k]);
    sum = __fadd_rn(sum, 1e-20f);
#pragma unroll
    for (int k = 0; k < kTopK; ++k)
      wts[k] = k < K ? __fmul_rn(__fdiv_rn(pv[k], sum), rsf) : 0.0f;
  } else if (method == FMOE_ROUTING_RENORMALIZE) {
    float e[kTopK], sum = 0.0f;  // softmax over the picks; pz[0] is their maximum
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
      e[k] = k < K ? expf(__fsub_rn(pz[k], pz[0])) : 0.0f;
      if (k < K) sum = __fadd_rn(sum, e[k]);
    }
#pragma unroll
    for (int k = 0; k < kTopK; ++k)
      wts[k] = k < K ? __fmul_rn(__fdiv_rn(e[k], sum), rsf) : 0.0f;
  } else if (method == FMOE_ROUTING_LLAMA4) {
#pragma unroll
    for (int k = 0; k < kTopK; ++k) wts[k] = 0.0f;
    wts[0] = __fmul_rn(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-pz[0]))), rsf);
  } else {  // FMOE_ROUTING_TOPK
    const float u = __fdiv_rn(rsf, static_cast<float>(K));
#pragma unroll
    for (int k = 0; k < kTopK; ++k) wts[k] = k < K ? u : 0.0f;
  }
}

// Routes one token with one warp by the call's routing mode (route_mode(method, top_k)).
template <typename TL>
__device__ __forceinline__ void route_token(const TL* __restrict__ row, const float (&b)[8],
                                            float rsf, int mode, int lane, int (&ids)[kTopK],
                                            float (&wts)[kTopK]) {
  const int method = mode & 0xff;
  if (method == FMOE_ROUTING_DEEPSEEK_V3)
    route_token_ds<TL>(row, b, rsf, lane, ids, wts);
  else
    route_token_other<TL>(row, b, rsf, method, mode >> 8, lane, ids, wts);
}

__device__ __forceinline__ void store_picks(int32_t* ids_out, float* w_out, int t,
                                            const int (&ids)[kTopK], const float (&w)[kTopK]) {
  int4* io = reinterpret_cast<int4*>(ids_out + static_cast<size_t>(t) * kTopK);
  float4* wo = reinterpret_cast<float4*>(w_out + static_cast<size_t>(t) * kTopK);
  io[0] = make_int4(ids[0], ids[1], ids[2], ids[3]);
  io[1] = make_int4(ids[4], ids[5], ids[6], ids[7]);
  wo[0] = make_float4(w[0], w[1], w[2], w[3]);
  wo[1] = make_float4(w[4], w[5], w[6], w[7]);
}


// Calls f(TL(), TB()) for the logits and bias element types of a call.
template <typename F>
inline cudaError_t dispatch_dtypes(int ld, int bd, F&& f) {
  if (ld == FMOE_DTYPE_F32 && bd == FMOE_DTYPE_BF16) return f(float(), __nv_bfloat16());
  if (ld == FMOE_DTYPE_F32 && bd == FMOE_DTYPE_F32) return f(float(), float());
  if (ld == FMOE_DTYPE_BF16 && bd == FMOE_DTYPE_BF16) return f(__nv_bfloat16(), __nv_bfloat16());
  return f(__nv_bfloat16(), float());
}

}  // namespace fmoe
