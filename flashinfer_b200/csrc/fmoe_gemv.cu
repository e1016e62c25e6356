// fmoe_gemv.cu -- the small-batch path (T <= kGemvMaxT): both expert GEMMs as weight-streaming
// matrix-vector products on the CUDA cores, SwiGLU and the weighted combine fused in.
//
// Where it wins: with one or two active experts its fixed costs are far below the grouped
// GEMMs' (T=1: 21.7 against 29.7 us per call); per active expert it streams weights at about
// 2.9 TB/s (a warp waits for each group of its loads before computing on it), slower than the
// grouped GEMMs, so from three active experts on those take over (kGemvMaxT).
//
// At a few tokens every local expert holds one or two routed rows, so a 128-row tensor-core
// tile is almost all padding and the call is bound by streaming the active experts' weights
// (44 MB per expert) plus the fixed costs around the GEMMs: TMEM allocation and barrier set-up,
// split-K partial tiles and their finish kernels, the activation gather and the combine. Here a
// call is three kernels -- the routing/plan kernel (k_plan_small), k_gemv1 and k_gemv2 -- and
// every weight byte is loaded once, straight into registers (16 bytes per lane per load), with
// the arithmetic of the reference's block-scaled GEMMs (solution/triton/kernel.py:158-171,
// :262-271):
//
//   k_gemv1   per CTA a range of intermediate columns j, per warp one (active expert, j) at a
//             time: the gate row j and the up row I + j of W1 against each routed row of that
//             expert. Products of e4m3 values are exact in fp32 (fma.rn.f32.f16 on the values
//             converted to f16, which holds every e4m3 value exactly); a lane's 16 products per
//             128-column block are summed in fp32 and promoted by a_scale[token, kb] *
//             w_scale[row block, kb]; lanes are summed by shuffles, then h = silu(up) * gate,
//             kept in fp32 ([P, I] rows in pair order, P = routed pairs).
//   k_gemv2   per CTA a range of about 24 output columns (rows of W2), per warp item 4 of them
//             for one active expert: each W2 row against the fp32 h of every pair of the expert,
//             promoted per 128-wide K block by w_scale; the per-pair results go to shared
//             memory, and each (token, column) then sums its picks in ascending expert order
//             (routing weight times the pair's value) and is rounded once to bf16 (or left in
//             fp32). The first item's W2 rows are requested before the grid-dependency wait.
//
// Differences from the tensor-core path: the intermediate stays fp32 (no two-term e4m3
// re-encoding) and the per-pair output rows are not rounded to fp16 before the combine, so the
// result is at least as close to the reference; sums are taken in another order, so the bits
// differ from the grouped GEMMs' in the last places. No atomics; deterministic.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "fmoe_gemm_common.cuh"

namespace fmoe {

namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kChunk = 512;          // K bytes of one warp-wide load round (32 lanes x 16 B)
constexpr int kMaxChunks1 = 14;      // GEMV1 K = H <= 7168
constexpr int kMaxChunks2 = 4;       // GEMV2 K = I <= 2048
constexpr int kGroup1 = 4;           // k_gemv1: loads per weight row in flight (K group)
constexpr int kRows1 = 4;            // k_gemv1: routed rows of one expert per pass
constexpr int kColsPerItem2 = 4;     // k_gemv2: output columns (W2 rows) per warp item
constexpr int kColsPerCta2 = 32;     // k_gemv2: output columns per CTA at most
constexpr int kGemvMaxPairs = kGemvMaxT * kTopK;

struct GemvArgs {
  const int32_t* expert_count;   // [E]
  const int32_t* expert_base;    // [E + 1] first slot of each expert
  const int32_t* slot_token;     // [cap]
  const int32_t* token_slot;     // [T, 8] slots of a token's local picks, expert ascending
  const float* token_weight;     // [T, 8]
  const uint8_t* hidden;         // [T, H] e4m3
  const float* hidden_scale;     // [H/128, T]
  const uint8_t* w1;             // [E, 2I, H] e4m3
  const float* w1_scale;         // [E, 2I/128, H/128]
  const uint8_t* w2;             // [E, H, I] e4m3
  const float* w2_scale;         // [E, H/128, I/128]
  float* h;                      // [P, I] fp32 (workspace)
  void* out;                     // [T, H] bf16 or fp32
  int out_f32;
  int T, H, I, E;
};

// The local experts that hold routed rows, in ascending order, with their first pair index
// (pairs numbered expert by expert), row count and first slot. One warp: lane l takes experts
// [8l, 8l + 8) and two shuffle scans give the positions.
struct ActiveExperts {
  int n;
  int e[kMaxLocalExperts];
  int q0[kMaxLocalExperts];
  int cnt[kMaxLocalExperts];
  int s0[kMaxLocalExperts];
};

__device__ void build_active(const GemvArgs& a, ActiveExperts& ax) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int c[8];
    int na = 0, nq = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane * 8 + i;
      c[i] = e < a.E ? __ldcg(a.expert_count + e) : 0;
      na += c[i] > 0 ? 1 : 0;
      nq += c[i];
    }
    int sa = na, sq = nq;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int ua = __shfl_up_sync(0xffffffffu, sa, off);
      const int uq = __shfl_up_sync(0xffffffffu, sq, off);
      if (lane >= off) {
        sa += ua;
        sq += uq;
      }
    }
    int ia = sa - na, iq = sq - nq;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (c[i] > 0) {
        const int e = lane * 8 + i;
        ax.e[ia] = e;
        ax.q0[ia] = iq;
        ax.cnt[ia] = c[i];
        ax.s0[ia] = __ldcg(a.expert_base + e);
        ++ia;
        iq += c[i];
      }
    }
    if (lane == 31) ax.n = sa;
  }
  __syncthreads();
}

// 16 bytes of weights, read once: not kept in L1.
__device__ __forceinline__ uint4 ld_weights16(const uint8_t* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

// Two e4m3 values (the low 16 bits of w) -> f16x2, exactly (the first byte in the low half).
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t w) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(static_cast<unsigned short>(w & 0xffffu)));
  return r;
}

// 16 e4m3 values -> 8 f16x2 (value 2i in the low half of f[i], 2i + 1 in the high half).
__device__ __forceinline__ void e4m3x16_to_f16(const uint4 v, uint32_t (&f)[8]) {
  f[0] = e4m3x2_to_f16x2(v.x);
  f[1] = e4m3x2_to_f16x2(v.x >> 16);
  f[2] = e4m3x2_to_f16x2(v.y);
  f[3] = e4m3x2_to_f16x2(v.y >> 16);
  f[4] = e4m3x2_to_f16x2(v.z);
  f[5] = e4m3x2_to_f16x2(v.z >> 16);
  f[6] = e4m3x2_to_f16x2(v.w);
  f[7] = e4m3x2_to_f16x2(v.w >> 16);
}

// c + a.lo * b.lo + a.hi * b.hi for f16x2 a and b: each product is formed exactly in fp32 and
// added with one rounding (fma.rn.f32.f16).
__device__ __forceinline__ float fma_f16x2_f32(uint32_t a, uint32_t b, float c) {
  asm("{\n\t.reg .b16 al, ah, bl, bh;\n\t"
      "mov.b32 {al, ah}, %1;\n\t"
      "mov.b32 {bl, bh}, %2;\n\t"
      "fma.rn.f32.f16 %0, al, bl, %0;\n\t"
      "fma.rn.f32.f16 %0, ah, bh, %0;\n\t}"
      : "+f"(c)
      : "r"(a), "r"(b));
  return c;
}

// Dot product of one 16-value chunk of f16x2 activations and weights, four independent chains.
__device__ __forceinline__ float dot16_f16(const uint32_t (&x)[8], const uint32_t (&w)[8]) {
  float p0 = 0.0f, p1 = 0.0f, p2 = 0.0f, p3 = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; i += 4) {
    p0 = fma_f16x2_f32(x[i], w[i], p0);
    p1 = fma_f16x2_f32(x[i + 1], w[i + 1], p1);
    p2 = fma_f16x2_f32(x[i + 2], w[i + 2], p2);
    p3 = fma_f16x2_f32(x[i + 3], w[i + 3], p3);
  }
  return (p0 + p1) + (p2 + p3);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

}  // namespace

// GEMM1 + SwiGLU for the small-batch path. Two CTAs of 8 warps per SM (at most 128 registers
// a thread): a warp's item is one (active expert, intermediate column j), its K range in groups
// of 4 loads per row (gate and up), so 16 warps per SM keep 4 KB each of weights in flight.
__global__ void __launch_bounds__(kGemvThreads, 2) k_gemv1(const GemvArgs a) {
  __shared__ ActiveExperts ax;
  pdl_begin_in_order();  // the plan is complete after the wait; k_gemv2 reads it before its own
  build_active(a, ax);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = a.H, I = a.I, T = a.T;
  const int nch = H / kChunk, nkb = H / kBlock;
  const int G = gridDim.x;
  // this CTA's columns: [j0, j1) of the intermediate, the same range for every active expert
  const int j0 = static_cast<int>(static_cast<int64_t>(blockIdx.x) * I / G);
  const int j1 = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * I / G);
  const int ncol = j1 - j0;
  const int items = ax.n * ncol;
  for (int it = warp; it < items; it += kGemvWarps) {
    const int ai = it / ncol;
    const int j = j0 + (it - ai * ncol);
    const int e = ax.e[ai], cnt = ax.cnt[ai], q0 = ax.q0[ai], s0 = ax.s0[ai];
    const uint8_t* wg = a.w1 + (static_cast<size_t>(e) * 2 * I + j) * H + lane * 16;
    const uint8_t* wu = wg + static_cast<size_t>(I) * H;
    const float* sg = a.w1_scale + (static_cast<size_t>(e) * (2 * I / kBlock) + j / kBlock) * nkb;
    const float* su = a.w1_scale + (static_cast<size_t>(e) * (2 * I / kBlock) + (I + j) / kBlock) * nkb;
    for (int r0 = 0; r0 < cnt; r0 += kRows1) {
      const int nr = min(kRows1, cnt - r0);
      float accg[kRows1], accu[kRows1];
#pragma unroll
      for (int r = 0; r < kRows1; ++r) accg[r] = accu[r] = 0.0f;
      for (int c0 = 0; c0 < nch; c0 += kGroup1) {
        uint4 vg[kGroup1], vu[kGroup1];
#pragma unroll
        for (int c = 0; c < kGroup1; ++c) {
          if (c0 + c < nch) {
            vg[c] = ld_weights16(wg + (c0 + c) * kChunk);
            vu[c] = ld_weights16(wu + (c0 + c) * kChunk);
          }
        }
        for (int r = 0; r < nr; ++r) {
          const int t = __ldcg(a.slot_token + s0 + r0 + r);
          const uint8_t* ar = a.hidden + static_cast<size_t>(t) * H + lane * 16;
          uint4 av[kGroup1];
#pragma unroll
          for (int c = 0; c < kGroup1; ++c)
            if (c0 + c < nch) av[c] = __ldg(reinterpret_cast<const uint4*>(ar + (c0 + c) * kChunk));
          float g = 0.0f, u = 0.0f;
#pragma unroll
          for (int c = 0; c < kGroup1; ++c) {
            if (c0 + c < nch) {
              const int kb = (c0 + c) * (kChunk / kBlock) + (lane >> 3);
              const float as = __ldg(a.hidden_scale + static_cast<size_t>(kb) * T + t);
              uint32_t ha[8], hw[8];
              e4m3x16_to_f16(av[c], ha);
              e4m3x16_to_f16(vg[c], hw);
              g = fmaf(dot16_f16(ha, hw), as * __ldg(sg + kb), g);
              e4m3x16_to_f16(vu[c], hw);
              u = fmaf(dot16_f16(ha, hw), as * __ldg(su + kb), u);
            }
          }
          // row r's sums (registers indexed by a loop variable: select by compare)
#pragma unroll
          for (int rr = 0; rr < kRows1; ++rr) {
            if (rr == r) {
              accg[rr] += g;
              accu[rr] += u;
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < kRows1; ++r) {
        if (r < nr) {
          const float g = warp_sum(accg[r]);
          const float u = warp_sum(accu[r]);
          if (lane == 0) a.h[static_cast<size_t>(q0 + r0 + r) * I + j] = swiglu(u, g);
        }
      }
    }
  }
}

// GEMM2 + the weighted combine for the small-batch path. Two CTAs of 8 warps per SM; a CTA owns
// about 24 output columns (rows of W2). A warp's item is one (active expert, group of 4 of those
// columns): the 4 W2 rows stay in registers while every pair of the expert passes (its fp32 h
// row read through L1, one 512-wide K chunk at a time); the per-pair results go to shared memory,
// and after all items each (token, column) sums its picks in ascending expert order.
__global__ void __launch_bounds__(kGemvThreads, 2) k_gemv2(const GemvArgs a) {
  __shared__ ActiveExperts ax;
  __shared__ float ybuf[kGemvMaxPairs * kColsPerCta2];
  // Before the wait: k_gemv1 starts this grid only after its own wait, so the plan is complete.
  build_active(a, ax);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = a.H, I = a.I, T = a.T;
  const int kch = I / kChunk, nkb = I / kBlock;
  const int G = gridDim.x;
  const int c0 = static_cast<int>(static_cast<int64_t>(blockIdx.x) * H / G);
  const int c1 = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * H / G);
  const int ncols = c1 - c0;  // <= kColsPerCta2 (checked on the host)
  const int ngroups = (ncols + kColsPerItem2 - 1) / kColsPerItem2;
  const int items = ax.n * ngroups;
  bool waited = false;
  for (int it = warp; it < items; it += kGemvWarps) {
    const int ai = it / ngroups;
    const int cg = (it - ai * ngroups) * kColsPerItem2;  // first column of the group, CTA-local
    const int e = ax.e[ai], cnt = ax.cnt[ai], q0 = ax.q0[ai];
    uint4 vw[kColsPerItem2][kMaxChunks2];
#pragma unroll
    for (int m = 0; m < kColsPerItem2; ++m) {
      const uint8_t* wr = a.w2 + (static_cast<size_t>(e) * H + c0 + cg + m) * I + lane * 16;
#pragma unroll
      for (int c = 0; c < kMaxChunks2; ++c)
        if (cg + m < ncols && c < kch) vw[m][c] = ld_weights16(wr + c * kChunk);
    }
    if (!waited) {
      // h comes from k_gemv1: the first item's weights are already in flight
      asm volatile("griddepcontrol.wait;" ::: "memory");
      waited = true;
    }
    const float* wsb = a.w2_scale + static_cast<size_t>(e) * (H / kBlock) * nkb + (lane >> 3);
    for (int p = 0; p < cnt; ++p) {
      const float* hp = a.h + static_cast<size_t>(q0 + p) * I + lane * 16;
      float y[kColsPerItem2];
#pragma unroll
      for (int m = 0; m < kColsPerItem2; ++m) y[m] = 0.0f;
#pragma unroll
      for (int c = 0; c < kMaxChunks2; ++c) {
        if (c < kch) {
          float hv[16];
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const float4 x = reinterpret_cast<const float4*>(hp + c * kChunk)[v];
            hv[4 * v] = x.x;
            hv[4 * v + 1] = x.y;
            hv[4 * v + 2] = x.z;
            hv[4 * v + 3] = x.w;
          }
#pragma unroll
          for (int m = 0; m < kColsPerItem2; ++m) {
            if (cg + m < ncols) {
              uint32_t f[8];
              e4m3x16_to_f16(vw[m][c], f);
              float2 s0 = make_float2(0.0f, 0.0f), s1 = make_float2(0.0f, 0.0f);
#pragma unroll
              for (int i = 0; i < 8; i += 2) {
                const float2 w0 = __half22float2(*reinterpret_cast<const __half2*>(&f[i]));
                const float2 w1 = __half22float2(*reinterpret_cast<const __half2*>(&f[i + 1]));
                s0 = __ffma2_rn(make_float2(hv[2 * i], hv[2 * i + 1]), w0, s0);
                s1 = __ffma2_rn(make_float2(hv[2 * i + 2], hv[2 * i + 3]), w1, s1);
              }
              const float wsc = __ldg(wsb + ((c0 + cg + m) / kBlock) * nkb + c * (kChunk / kBlock));
              y[m] = fmaf((s0.x + s0.y) + (s1.x + s1.y), wsc, y[m]);
            }
          }
        }
      }
#pragma unroll
      for (int m = 0; m < kColsPerItem2; ++m) {
        if (cg + m < ncols) {
          const float v = warp_sum(y[m]);
          if (lane == 0) ybuf[(q0 + p) * kColsPerCta2 + cg + m] = v;
        }
      }
    }
  }
  if (!waited) asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __syncthreads();
  // Combine: token t's picks are its slots in ascending expert order (token_slot); a slot's pair
  // index follows from the active expert that holds it.
  for (int i = threadIdx.x; i < T * ncols; i += blockDim.x) {
    const int t = i / ncols, col = i - t * ncols;
    float acc = 0.0f;
#pragma unroll 1
    for (int k = 0; k < kTopK; ++k) {
      const int slot = __ldcg(a.token_slot + static_cast<size_t>(t) * kTopK + k);
      if (slot < 0) break;
      int lo = 0, hi = ax.n - 1;  // the active expert whose slots hold `slot`
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (ax.s0[mid] <= slot)
          lo = mid;
        else
          hi = mid - 1;
      }
      const int q = ax.q0[lo] + (slot - ax.s0[lo]);
      acc = fmaf(__ldcg(a.token_weight + static_cast<size_t>(t) * kTopK + k),
                 ybuf[q * kColsPerCta2 + col], acc);
    }
    const size_t o = static_cast<size_t>(t) * H + c0 + col;
    if (a.out_f32)
      static_cast<float*>(a.out)[o] = acc;
    else
      static_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(acc);
  }
}

static GemvArgs gemv_args(const RunParams& p) {
  const Layout& L = p.L;
  GemvArgs a{};
  a.expert_count = reinterpret_cast<const int32_t*>(p.ws + L.expert_count);
  a.expert_base = reinterpret_cast<const int32_t*>(p.ws + L.expert_base);
  a.slot_token = reinterpret_cast<const int32_t*>(p.ws + L.slot_token);
  a.token_slot = reinterpret_cast<const int32_t*>(p.ws + L.token_slot);
  a.token_weight = reinterpret_cast<const float*>(p.ws + L.token_weight);
  a.hidden = p.hidden;
  a.hidden_scale = p.hidden_scale;
  a.w1 = p.w1;
  a.w1_scale = p.w1_scale;
  a.w2 = p.w2;
  a.w2_scale = p.w2_scale;
  a.h = reinterpret_cast<float*>(p.ws + L.partials);
  a.out = p.output;
  a.out_f32 = p.out_mode == FMOE_OUT_F32 ? 1 : 0;
  a.T = p.T;
  a.H = p.H;
  a.I = p.I;
  a.E = p.E;
  return a;
}

bool gemv_eligible(const RunParams& p) {
  if (p.T < 1 || p.T > kGemvMaxT || p.in_ids != nullptr || p.inject_gemm != 0) return false;
  if (p.out_mode != FMOE_OUT_BF16 && p.out_mode != FMOE_OUT_F32) return false;
  if (p.H % kChunk != 0 || p.H > kMaxChunks1 * kChunk) return false;
  if (p.I % kChunk != 0 || p.I > kMaxChunks2 * kChunk) return false;
  const int g2 = 2 * p.num_sms;  // k_gemv2 grid
  if (p.num_sms < 1 || (p.H + g2 - 1) / g2 > kColsPerCta2) return false;
  // h: [P, I] fp32 in the partial-tile region, P <= T * 8
  const size_t h_bytes = static_cast<size_t>(p.T) * kTopK * p.I * 4;
  return h_bytes <= static_cast<size_t>(kMaxSplitUnits) * p.L.partial_rows * kTileN * 4;
}

cudaError_t launch_gemv(const RunParams& p, int which, cudaStream_t s) {
  const GemvArgs a = gemv_args(p);
  if (which == 1)
    (void)launch_pdl(k_gemv1, 2 * p.num_sms, kGemvThreads, 0, s, a);
  else
    (void)launch_pdl(k_gemv2, 2 * p.num_sms, kGemvThreads, 0, s, a);
  return cudaGetLastError();
}

}  // namespace fmoe
