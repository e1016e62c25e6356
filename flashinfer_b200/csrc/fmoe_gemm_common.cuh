// fmoe_gemm_common.cuh -- the grouped GEMM kernels' (fmoe_gemm.cu) kernel arguments, shared-memory
// layout of a CTA, work-unit decomposition, bounded waits and epilogue arithmetic.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "fmoe_internal.h"
#include "fmoe_ptx.cuh"

namespace fmoe {

struct GemmArgs {
  const int32_t* plan;
  const int32_t* expert_base;
  const int32_t* expert_count;
  const float* a_scale_t;  // [nkb][cap]
  const float* w_scale;    // KIND1 [E][2I/128][H/128], KIND2 [E][H/128][I/128]
  float* partials;
  int32_t* counters;
  int32_t* status;
  uint8_t* h_hi;
  uint8_t* h_lo;
  float* h_scale_t;        // [I/128][cap]
  __half* y;               // [cap][H] fp16, scaled by y_scale
  float* y_scale;          // [cap][H/256] power-of-two scale per slot per n-tile
  int E, H, I;
  int64_t cap;
  int partial_rows;
  // every bounded wait of the pipeline gives up after wait_ns of global time; inject != 0 makes
  // the MMA warp wait on a barrier nothing arrives on (tests of the failure path only)
  unsigned long long wait_ns;
  int inject;
};

template <int KIND>
struct Cfg;
template <>
struct Cfg<1> {
  static constexpr int NS = 4;
  static constexpr int A_TILES = 1;
  static constexpr int STAGE = 128 * 128 * A_TILES + 256 * 128;  // 48 KB
};
template <>
struct Cfg<2> {
  static constexpr int NS = 3;
  static constexpr int A_TILES = 2;
  static constexpr int STAGE = 128 * 128 * A_TILES + 256 * 128;  // 64 KB
};
// GEMM2 for tiles of at most 64 routed slots (T <= kPackedMaxT): one A tile holds the hi term of
// the tile's first 64 slots in rows 0-63 and their lo term in rows 64-127, so a K block takes
// four MMAs instead of eight; at the tile end the lo rows' fp32 sums are added to the hi rows'
// through shared memory (xbuf), 16 rows per round.
template <>
struct Cfg<3> {
  static constexpr int NS = 4;
  static constexpr int A_TILES = 1;
  static constexpr int STAGE = 128 * 128 * A_TILES + 256 * 128;  // 48 KB
};

constexpr int kThreads = 384;
constexpr int kEpiWarps = 8;
constexpr int kEpiWarp0 = 4;       // first epilogue warp (warpgroups 1 and 2)
constexpr int kProducer2Warp = 2;
constexpr int kRegsControl = 56;   // setmaxnreg of warpgroup 0 (producers, MMA)
constexpr int kRegsEpilogue = 224; // setmaxnreg of the epilogue warpgroups
static_assert(kRegsControl * 128 + kRegsEpilogue * 256 <= 168 * kThreads,
              "register split exceeds the launch allocation (168 per thread at 384 threads)");
constexpr int kTmemCols = 512;
constexpr int kATileBytes = 128 * 128;
// Activation scales of K iteration it land (by TMA, counted on full[s]) in ring entry it % 8.
// The producer runs at most NS stages ahead of the MMA warp, which runs at most two K blocks
// ahead of the epilogue, so an entry is never refilled before the epilogue has read it.
constexpr int kSaRing = 8;
constexpr int kSaBytes = 128 * 4;
constexpr int kMaxKb = 64;  // K blocks per GEMM (H/128 and I/128); checked on the host
// Row buffer of the tile end (xbuf): per tile row the 256 fp32 sums in accumulator order (column
// group g at g * 128: its 64 first-half columns, then its 64 second-half columns), rows padded
// by 4 floats (a warp's 16-byte accesses to consecutive rows then cover all 32 banks). It holds
// the rows of a tile with at most kXSmall routed rows, which all epilogue threads then finish,
// and for KIND 3 the lo rows of 16 slots per exchange round.
constexpr int kXRow = 2 * 128 + 4;
constexpr int kXSmall = 16;
template <int KIND>
constexpr int xbuf_bytes() {
  return kXSmall * kXRow * 4;
}

struct alignas(16) GemmTail {
  uint64_t full[4];
  uint64_t empty[4];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint64_t never;  // armed, never arrived on: the injected wait of a failure-path test
  uint32_t tmem_base;
  int last_flag;
  int abort_flag;
  int pad_;
  int last_issue[2][4];  // per producer, per stage: last round issued (-1 = none)
  float amax_x[2][128];
  float w_sc[2][2][kMaxKb];  // [unit parity][tile half][K block] weight scales of a unit
  int ebase[kMaxLocalExperts + 1];
  int ecnt[kMaxLocalExperts];
};

template <int KIND>
constexpr size_t gemm_smem_bytes() {
  static_assert(Cfg<KIND>::NS + 3 <= kSaRing, "activation-scale ring too short");
  static_assert(sizeof(GemmTail) % 16 == 0, "xbuf follows the tail 16-byte aligned");
  return static_cast<size_t>(Cfg<KIND>::NS) * Cfg<KIND>::STAGE + kSaRing * kSaBytes +
         sizeof(GemmTail) + xbuf_bytes<KIND>() + 1024;
}
static_assert(gemm_smem_bytes<1>() <= 227 * 1024 && gemm_smem_bytes<2>() <= 227 * 1024 &&
                  gemm_smem_bytes<3>() <= 227 * 1024,
              "shared memory per CTA");

struct Unit {
  int e, n, row0, nrows, kb0, kb1;
};

__device__ __forceinline__ Unit decode_unit(int unit, int S, int NT, int nkb, const int* ebase,
                                            const int* ecnt, int E) {
  const int tile = unit / S;
  const int split = unit - tile * S;
  int lo = 0, hi = E;
  while (lo < hi) {  // first expert e with tile < tile_base(e + 1)
    const int mid = (lo + hi) >> 1;
    if (tile < (ebase[mid + 1] >> 7) * NT)
      hi = mid;
    else
      lo = mid + 1;
  }
  const int e = lo < E ? lo : E - 1;
  const int mt = max(1, (ebase[e + 1] - ebase[e]) >> 7);
  const int local = tile - (ebase[e] >> 7) * NT;
  const int n = local / mt;
  const int m = local - n * mt;
  Unit u;
  u.e = e;
  u.n = n;
  u.row0 = ebase[e] + m * 128;
  u.nrows = min(128, ecnt[e] - m * 128);
  u.kb0 = split * nkb / S;
  u.kb1 = (split + 1) * nkb / S;
  return u;
}

// Bounded wait that also gives up when another role of this CTA has already aborted. Spins on
// the non-suspending test_wait: this wait sits on the MMA <-> epilogue hand-off, the pipeline's
// critical path.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity,
                                              volatile int* abort_flag, uint64_t limit_ns) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((++spins & 255u) == 0) {
      if (*abort_flag) return false;
      if (global_timer_ns() - t0 > limit_ns) return false;
    }
  }
}

// The same for a thread that is not on the critical path (the TMA producers): each poll may
// park the thread for up to 2 us, leaving its issue slots to the epilogue warps.
__device__ __forceinline__ bool wait_or_abort_parked(uint64_t* bar, uint32_t parity,
                                                     volatile int* abort_flag, uint64_t limit_ns) {
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 2000u)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
}

__device__ __forceinline__ void raise_abort(GemmTail* tail, int32_t* status, int code) {
  *reinterpret_cast<volatile int*>(&tail->abort_flag) = 1;
  atomicOr(status, code);
}

// Row maximum over the two column groups of epilogue warps that share a row (through shared
// memory; every epilogue thread takes part).
__device__ __forceinline__ float exchange_amax(GemmTail* tail, int g, int r, float amax) {
  tail->amax_x[g][r] = amax;
  named_bar_sync(1, kEpiWarps * 32);
  return fmaxf(tail->amax_x[0][r], tail->amax_x[1][r]);
}

// Every lane polls the barrier; the warp agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          uint64_t limit_ns) {
  const bool got = wait_or_abort(bar, parity, abort_flag, limit_ns);
  return __all_sync(0xffffffffu, got);
}

// acc[0..16) += v[0..16) * f with packed fp32 FMA (same rounding as 16 fmaf).
__device__ __forceinline__ void fma16(float* acc, const float* v, float f) {
  const float2 ff = make_float2(f, f);
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    const float2 r = __ffma2_rn(make_float2(v[i], v[i + 1]), ff, make_float2(acc[i], acc[i + 1]));
    acc[i] = r.x;
    acc[i + 1] = r.y;
  }
}

// silu(up) * gate (moe.py:90-92) with the fast exponential and divide: relative error about
// 1e-6, far below the e4m3 encoding that follows; for up < -87 the denominator is +inf and the
// result is -0.
__device__ __forceinline__ float swiglu(float up, float gate) {
  return __fdividef(up, 1.0f + __expf(-up)) * gate;
}

// Two-term e4m3 encoding of 32 values: x * inv = hi + lo with hi = e4m3(x * inv) and
// lo = e4m3(x * inv - hi); one 32-byte store (a full DRAM sector) per term.
__device__ __forceinline__ void encode_e4m3_2term32(const float* x, float inv, uint8_t* hi_dst,
                                                    uint8_t* lo_dst) {
  uint32_t hw[8], lw[8];
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    uint32_t hbits = 0, lbits = 0;
#pragma unroll
    for (int pr = 0; pr < 2; ++pr) {
      const float x0 = x[w * 4 + pr * 2] * inv;
      const float x1 = x[w * 4 + pr * 2 + 1] * inv;
      const uint16_t hp = pack_e4m3x2(x0, x1);
      const float2 back = unpack_e4m3x2(hp);
      const uint16_t lp = pack_e4m3x2(x0 - back.x, x1 - back.y);
      hbits |= static_cast<uint32_t>(hp) << (16 * pr);
      lbits |= static_cast<uint32_t>(lp) << (16 * pr);
    }
    hw[w] = hbits;
    lw[w] = lbits;
  }
  st_global_v8(hi_dst, hw);
  st_global_v8(lo_dst, lw);
}

// 16 values times a power-of-two inv, rounded to fp16, stored with one 32-byte store to
// y[slot][col, col + 16) (a full DRAM sector per store).
__device__ __forceinline__ void store_f16x16(const float* x, float inv, __half* y, size_t slot,
                                             int col, int H) {
  uint32_t wv[8];
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const __half2 pr = __floats2half2_rn(x[2 * w] * inv, x[2 * w + 1] * inv);
    wv[w] = *reinterpret_cast<const uint32_t*>(&pr);
  }
  st_global_v8(y + slot * static_cast<size_t>(H) + col, wv);
}

// Exponent k of the smallest 2^k with amax / 2^k <= 16384 (ceil(log2(amax)) - 14): the fp16
// range is never exceeded, the scaling is exact and the relative precision stays 2^-11.
__device__ __forceinline__ int pow2_exponent_for_f16(float amax) {
  int ex = 0;
  const float m = frexpf(amax, &ex);  // amax = m * 2^ex, m in [0.5, 1)
  return (m > 0.5f ? ex : ex - 1) - 14;
}

}  // namespace fmoe
