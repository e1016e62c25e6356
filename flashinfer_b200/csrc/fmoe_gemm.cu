// fmoe_gemm.cu -- grouped FP8 e4m3 GEMMs with 128x128 block-scale promotion on tcgen05.
//
// Reference counterparts (solution/triton/kernel.py):
//   KIND 1  <- _persistent_gemm1_kernel kernel.py:69-186 (+ _swiglu_kernel :301-330 fused in
//              the epilogue; output re-encoded as two e4m3 terms with one scale per 128 cols)
//   KIND 2  <- _persistent_gemm2_kernel kernel.py:193-293 (the reference runs this GEMM in
//              TF32 on an fp32 intermediate; here A = hi + lo e4m3 terms, two MMAs per K block)
//
// Per CTA (persistent, one per SM, 384 threads = three warpgroups):
//   warps 0,2   TMA producers, alternating K iterations: A tile [128 slots x 128 K] (+ the lo
//               term for KIND 2) and the weight tile [256 rows x 128 K] into an NS-stage
//               shared-memory ring. One issuing warp sustains about 42 B/cycle per SM of
//               128-row boxes; two sustain about 79 B/cycle, above the 48 KB per 520-cycle
//               K block that the MMA consumes.
//   warp 1      MMA issuer: per 128-wide K block, tcgen05.mma kind::f8f6f4 M=128 N=256 K=32
//               x4 (x8 for KIND 2) into one of two TMEM partial buffers (2 x 256 columns).
//   warp 3      idle (completes warpgroup 0, whose register budget is handed to the epilogue).
//   warps 4-11  promotion + epilogue: read each K block's partial from TMEM, scale it by
//               a_scale[slot, kb] * w_scale[n-block, kb] and accumulate in fp32 registers
//               with packed FMA (the reference's "partial * sa * sb" promotion,
//               kernel.py:167-171).
// After the prologue warpgroup 0 gives up registers (setmaxnreg.dec to 56) and the two
// epilogue warpgroups take them (setmaxnreg.inc to 224): 168 x 384 = 56 x 128 + 224 x 256, so
// each epilogue thread holds its 128 accumulators, two 16-column TMEM load buffers and the tile
// end's working set without spilling in the K loop.
// The hand-offs between the MMA warp and the epilogue are the pipeline's critical path (only two
// 256-column TMEM buffers fit in TMEM): waits spin on mbarrier.test_wait (a suspended try_wait
// wakes up late) and every epilogue lane arrives on the buffer-empty barrier itself (no warp
// synchronisation before the arrive). Splitting each tile's MMA into two N=128 halves with a
// TMEM double buffer per epilogue warpgroup (so the warpgroups run half a K block apart) was
// built and measured 10-12% slower on both GEMMs (same box, same inputs).
// Work unit = (tile, K split). Tiles are ordered expert -> n-tile -> m-tile so concurrently
// running CTAs share weight tiles in L2. For small batches with fewer tiles than SMs the K range
// is split; every split writes its fp32 partial tile and k_split_finish (a separate kernel,
// one CTA per tile) sums them in split order and runs the epilogue -- deterministic, and no CTA
// ever waits on another.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>

#include "fmoe_gemm_common.cuh"

namespace fmoe {

template <int KIND>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm(const __grid_constant__ CUtensorMap tm_a0, const __grid_constant__ CUtensorMap tm_a1,
           const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_sa,
           const GemmArgs args) {
  using C = Cfg<KIND>;
  constexpr int NS = C::NS;
  static_assert(NS >= 2 && NS <= 4, "barrier arrays hold 4 stages; alternating producers need 2");
  constexpr int STAGE = C::STAGE;
  constexpr int kErr = KIND == 1 ? FMOE_STATUS_TIMEOUT_GEMM1 : FMOE_STATUS_TIMEOUT_GEMM2;
  // Until griddepcontrol.wait below, the previous kernel may still run. The plan and the expert
  // tables are complete: the gather releases GEMM1 only after its own wait (pdl_begin_in_order),
  // and GEMM2 starts after GEMM1 has.
  // The prologue and the weight loads of the first NS K iterations, which need nothing else,
  // run before the wait; the activations are loaded after it.

  // Read through L2 (ld.global.cg): the plan kernel wrote these while lines of the previous
  // call's tables may still sit in this SM's (non-coherent) L1.
  const int S = __ldcg(args.plan + (KIND == 1 ? kPlanSplit1 : kPlanSplit2));
  const int units = __ldcg(args.plan + (KIND == 1 ? kPlanUnits1 : kPlanUnits2));
  if (static_cast<int>(blockIdx.x) >= units) return;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  float* sa_ring = reinterpret_cast<float*>(smem + NS * STAGE);  // [kSaRing][128]
  GemmTail* tail = reinterpret_cast<GemmTail*>(smem + NS * STAGE + kSaRing * kSaBytes);
  float* xbuf = reinterpret_cast<float*>(tail + 1);  // [kXSmall][kXRow]
  volatile int* abort_flag = &tail->abort_flag;
  const uint64_t wait_ns = args.wait_ns;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int E = args.E;
  const int nkb = KIND == 1 ? args.H / kBlock : args.I / kBlock;
  const int NT = KIND == 1 ? args.I / kBlock : args.H / kTileN;

  for (int i = threadIdx.x; i <= E; i += blockDim.x) {
    tail->ebase[i] = __ldcg(args.expert_base + i);
    if (i < E) tail->ecnt[i] = __ldcg(args.expert_count + i);
  }
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&tail->full[s], 1);
      mbar_init(&tail->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tail->tfull[b], 1);
      mbar_init(&tail->tempty[b], kEpiWarps * 32);  // every epilogue lane arrives
    }
    mbar_init(&tail->drain, 1);
    mbar_init(&tail->never, 1);
    tail->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_a0);
    if (KIND != 1) tma_prefetch_desc(&tm_a1);
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_sa);
  }
  if (warp == 1) {
    tmem_alloc(&tail->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tail->tmem_base;

  // The weight boxes of iteration it (K block kb of unit u) into stage s, with the stage's
  // transaction count for the whole stage (weights, activations and activation scales).
  // L2 policy of a weight box: an expert with more than 128 routed rows has several m-tiles,
  // whose units (consecutive, so on CTAs running side by side) all stream the same weight tile,
  // so its boxes are kept (evict_last); otherwise a box is read once and goes first
  // (evict_first), leaving L2 to the activations. With evict_first everywhere the headline
  // batch (T=16384 over 256 experts, ~4 m-tiles per expert) read its weights from DRAM 2.7
  // times per GEMM; the per-expert choice took GEMM1 from 5.36 to 4.75 ms there and left the
  // one-m-tile batches unchanged.
  auto issue_weights = [&](int s, const Unit& u, int kb, uint64_t pol_first, uint64_t pol_last) {
    const uint64_t pol_w = tail->ecnt[u.e] > kTileM ? pol_last : pol_first;
    uint8_t* st = smem + s * STAGE;
    mbar_arrive_expect_tx(&tail->full[s], STAGE + kSaBytes);
    const int kx = kb * kBlock;
    if (KIND == 1) {
      const int wrow = u.e * 2 * args.I + u.n * kBlock;
      tma_load_2d(st + kATileBytes, &tm_w, &tail->full[s], kx, wrow, pol_w);
      tma_load_2d(st + 2 * kATileBytes, &tm_w, &tail->full[s], kx, wrow + args.I, pol_w);
    } else {
      tma_load_2d(st + C::A_TILES * kATileBytes, &tm_w, &tail->full[s], kx,
                  u.e * args.H + u.n * kTileN, pol_w);
    }
  };
  // Each role branch starts with its warpgroup's register change (ptxas allocates each branch
  // under the limit its setmaxnreg sets), then waits for the previous grid.
  if (warp < kEpiWarp0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
    if ((warp == 0 || warp == kProducer2Warp) && lane == 0) {
      const int pw = warp == 0 ? 0 : 1;
      const uint64_t pol_first = policy_evict_first();
      const uint64_t pol_last = policy_evict_last();
      int it = 0;
      for (int unit = blockIdx.x; unit < units && it < NS; unit += gridDim.x) {
        const Unit u = decode_unit(unit, S, NT, nkb, tail->ebase, tail->ecnt, E);
        for (int kb = u.kb0; kb < u.kb1 && it < NS; ++kb, ++it)
          if ((it & 1) == pw) issue_weights(it, u, kb, pol_first, pol_last);
      }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0 || warp == kProducer2Warp) {
    // ------------------------------------------------------------------ TMA producers
    const int pw = warp == 0 ? 0 : 1;  // issues the K iterations it with (it & 1) == pw
    if (lane == 0) {
      const uint64_t pol_first = policy_evict_first();
      const uint64_t pol_a = policy_evict_last();
      int last_round[NS];
#pragma unroll
      for (int s = 0; s < NS; ++s) last_round[s] = -1;
      int it = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < units && ok; unit += gridDim.x) {
        const Unit u = decode_unit(unit, S, NT, nkb, tail->ebase, tail->ecnt, E);
        for (int kb = u.kb0; kb < u.kb1; ++kb, ++it) {
          if ((it & 1) != pw) continue;
          const int s = it % NS;
          const int r = it / NS;
          // This producer issued iteration it - 2 after the release of it - 2 - NS, and the MMA
          // warp releases in order, so round r - 2 of this stage is already released: the empty
          // barrier is at most one phase behind and the parity wait is unambiguous.
          if (r > 0 && !wait_or_abort_parked(&tail->empty[s], (r & 1) ^ 1, abort_flag, wait_ns)) {
            raise_abort(tail, args.status, kErr);
            ok = false;
            break;
          }
          uint8_t* st = smem + s * STAGE;
          if (it >= NS) issue_weights(s, u, kb, pol_first, pol_a);  // else issued before the wait
          const int kx = kb * kBlock;
          tma_load_2d(sa_ring + (it % kSaRing) * 128, &tm_sa, &tail->full[s], u.row0, kb, pol_a);
          if (KIND == 1) {
            tma_load_2d(st, &tm_a0, &tail->full[s], kx, u.row0, pol_a);
          } else if (KIND == 2) {
            tma_load_2d(st, &tm_a0, &tail->full[s], kx, u.row0, pol_a);
            tma_load_2d(st + kATileBytes, &tm_a1, &tail->full[s], kx, u.row0, pol_a);
          } else {  // 64-row boxes: hi rows 0-63, lo rows 64-127 of the one A tile
            tma_load_2d(st, &tm_a0, &tail->full[s], kx, u.row0, pol_a);
            tma_load_2d(st + kATileBytes / 2, &tm_a1, &tail->full[s], kx, u.row0, pol_a);
          }
          last_round[s] = r;
        }
      }
#pragma unroll
      for (int s = 0; s < NS; ++s) tail->last_issue[pw][s] = last_round[s];
    }
    named_bar_sync(2, 64);
    // Never leave a bulk copy in flight into shared memory that is about to be released. Each
    // stage's latest round (over both producers) was issued after every earlier round of that
    // stage had landed, so one wait per stage on the latest round suffices.
    if (pw == 0 && lane == 0) {
#pragma unroll
      for (int s = 0; s < NS; ++s) {
        const int r = max(tail->last_issue[0][s], tail->last_issue[1][s]);
        if (r >= 0) (void)mbar_wait(&tail->full[s], r & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(128, 256);
      int it = 0, kt = 0;
      // failure-path test: a wait on a barrier nothing arrives on runs out, and the CTA takes
      // the abort path below (status bit, producers stop and drain, TMEM freed)
      bool ok = args.inject == 0 || wait_or_abort(&tail->never, 0, abort_flag, wait_ns);
      for (int unit = blockIdx.x; unit < units && ok; unit += gridDim.x) {
        const Unit u = decode_unit(unit, S, NT, nkb, tail->ebase, tail->ecnt, E);
        for (int kb = u.kb0; kb < u.kb1; ++kb, ++it, ++kt) {
          const int s = it % NS;
          const int r = it / NS;
          const int b = kt & 1;
          const int rb = kt >> 1;
          if (!wait_or_abort(&tail->full[s], r & 1, abort_flag, wait_ns) ||
              (rb > 0 && !wait_or_abort(&tail->tempty[b], (rb & 1) ^ 1, abort_flag, wait_ns))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + b * kTileN;
          const uint32_t st = smem_u32(smem + s * STAGE);
          const uint64_t a_desc = smem_desc_k128(st);
          const uint64_t b_desc = smem_desc_k128(st + C::A_TILES * kATileBytes);
#pragma unroll
          for (int j = 0; j < 4; ++j)  // 4 x K=32 covers the 128-byte row
            mma_f8f6f4(d, a_desc + 2 * j, b_desc + 2 * j, idesc, j > 0 ? 1u : 0u);
          if (KIND == 2) {
            const uint64_t lo_desc = smem_desc_k128(st + kATileBytes);
#pragma unroll
            for (int j = 0; j < 4; ++j) mma_f8f6f4(d, lo_desc + 2 * j, b_desc + 2 * j, idesc, 1u);
          }
          mma_commit(&tail->empty[s]);
          mma_commit(&tail->tfull[b]);
        }
      }
      if (!ok) raise_abort(tail, args.status, kErr);
      mma_commit(&tail->drain);
      (void)mbar_wait(&tail->drain, 0);
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsEpilogue));
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // ------------------------------------------------------------------ promotion + epilogue
    const int ew = warp - kEpiWarp0;
    const int g = ew >> 2;        // column group: 0 -> cols [0,64)+[128,192), 1 -> [64,128)+...
    const int q = warp & 3;       // TMEM lane quarter this warp may access
    const int r = q * 32 + lane;  // accumulator row owned by this thread
    // Slot offset of that row within the tile, and (KIND 3) whether it holds the lo term.
    const int prow = KIND == 3 ? (r & 63) : r;
    const bool lo_row = KIND == 3 && r >= 64;
    const int etid = ew * 32 + lane;
    const int64_t cap = args.cap;
    int kt = 0;
    bool ok = true;
    float acc[128];
    // Weight scales of a unit's two 128-row halves (gate/up, or two n-blocks) for all its K
    // blocks (2 * nkb <= 128 values, one per epilogue thread), kept in w_sc[par]; a unit's
    // table is fetched during the previous unit's epilogue and published by the unit-start
    // barrier.
    auto fetch_w_scale = [&](const Unit& uu) -> float {
      if (etid >= 2 * nkb) return 0.0f;
      const int h = etid >= nkb ? 1 : 0;
      const int kb = etid - h * nkb;
      size_t row;
      if (KIND == 1) {
        const int nb1 = args.I / kBlock;
        row = static_cast<size_t>(uu.e) * 2 * nb1 + h * nb1 + uu.n;
      } else {
        row = static_cast<size_t>(uu.e) * (args.H / kBlock) + 2 * uu.n + h;
      }
      return __ldg(args.w_scale + row * nkb + kb);
    };
    auto store_w_scale = [&](int to_par, float v) {
      if (etid < 2 * nkb) tail->w_sc[to_par][etid >= nkb ? 1 : 0][etid % nkb] = v;
    };
    int par = 0;
    store_w_scale(0, fetch_w_scale(decode_unit(blockIdx.x, S, NT, nkb, tail->ebase, tail->ecnt, E)));
    for (int unit = blockIdx.x; unit < units; unit += gridDim.x, par ^= 1) {
      const Unit u = decode_unit(unit, S, NT, nkb, tail->ebase, tail->ecnt, E);
      // every epilogue thread has finished the previous unit and written this unit's w_sc
      named_bar_sync(1, kEpiWarps * 32);
      // Warps whose 32 rows are all padding skip the TMEM reads (their rows are discarded);
      // they still wait for each half before releasing it, which keeps the phases aligned.
      const bool warp_rows = (KIND == 3 ? (q & 1) : q) * 32 < u.nrows;
#pragma unroll
      for (int i = 0; i < 128; ++i) acc[i] = 0.0f;
      const bool has_next = unit + static_cast<int>(gridDim.x) < units;
      float w_next = 0.0f;  // the next unit's weight scale, fetched during the last K block
      for (int kb = u.kb0; kb < u.kb1; ++kb, ++kt) {
        if (has_next && kb == u.kb1 - 1)
          w_next = fetch_w_scale(decode_unit(unit + gridDim.x, S, NT, nkb, tail->ebase,
                                             tail->ecnt, E));
        if (!ok) continue;
        const int b = kt & 1;
        const int rb = kt >> 1;
        if (!warp_wait(&tail->tfull[b], rb & 1, abort_flag, wait_ns)) {
          if (lane == 0) raise_abort(tail, args.status, kErr);
          ok = false;
          continue;
        }
        if (warp_rows) {
          tc_fence_after();
          const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + b * kTileN;
          // 8 chunks of 16 columns: gate (or n-block 0) cols g*64 + [0,64), then up (n-block 1)
          // cols 128 + g*64 + [0,64). Chunk c+1 is in flight while chunk c is accumulated.
          float va[16], vb[16];
          tmem_ld_32x32b_x16(taddr + g * 64, va);
          // the activation scale reached shared memory before the MMA that this wait follows;
          // the shared-memory reads overlap the first TMEM load
          const float sa = sa_ring[(kt % kSaRing) * 128 + prow];
          const float f0 = sa * tail->w_sc[par][0][kb];
          const float f1 = sa * tail->w_sc[par][1][kb];
          tmem_ld_wait16(va);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const int cn = c + 1;
            const int coln = (cn < 4 ? 0 : 128) + g * 64 + (cn & 3) * 16;
            const float f = c < 4 ? f0 : f1;
            if ((c & 1) == 0) {
              if (cn < 8) tmem_ld_32x32b_x16(taddr + coln, vb);
              fma16(acc + c * 16, va, f);
              if (cn < 8) tmem_ld_wait16(vb);
            } else {
              if (cn < 8) tmem_ld_32x32b_x16(taddr + coln, va);
              fma16(acc + c * 16, vb, f);
              if (cn < 8) tmem_ld_wait16(va);
            }
          }
          tc_fence_before();
        }
        mbar_arrive(&tail->tempty[b]);
      }
      // w_sc[par ^ 1] was last read in the previous unit, which every epilogue thread has left
      if (has_next) store_w_scale(par ^ 1, w_next);

      if (S == 1 && u.nrows <= kXSmall) {
        // A tile with few routed rows (the decode case): their owners -- the warps of one or
        // (KIND 3) two lane quarters -- park the rows' fp32 sums in xbuf (KIND 3: lo rows
        // first, then the hi rows add theirs), and every epilogue thread finishes one row's 8
        // intermediate columns (KIND 1) or 16 output columns (KIND 2/3): thread etid takes row
        // etid / 16, column chunk etid % 16, and the row maximum is a 16-lane shuffle
        // reduction. Each value sees the same operations as on the per-row path below.
        const bool own = prow < u.nrows;
        float4* x = reinterpret_cast<float4*>(xbuf + prow * kXRow + g * 128);
        if (KIND == 3) {
          if (lo_row && own) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              x[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
          }
          named_bar_sync(1, kEpiWarps * 32);
          if (!lo_row && own) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float4 v = x[i];
              x[i] = make_float4(acc[4 * i] + v.x, acc[4 * i + 1] + v.y, acc[4 * i + 2] + v.z,
                                 acc[4 * i + 3] + v.w);
            }
          }
        } else if (own) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            x[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
        }
        named_bar_sync(1, kEpiWarps * 32);
        const int rr = etid >> 4, c = etid & 15;
        const bool live = rr < u.nrows;
        const float* xr = xbuf + rr * kXRow;
        const size_t orow = static_cast<size_t>(u.row0) + rr;
        if (KIND == 1) {
          // intermediate columns hc + [0, 8): gate (first half) and up (second half) sums
          const int hc = c * 8;
          const float* gp = xr + (hc >> 6) * 128 + (hc & 63);
          float gv[8], uv[8];
          *reinterpret_cast<float4*>(gv) = *reinterpret_cast<const float4*>(gp);
          *reinterpret_cast<float4*>(gv + 4) = *reinterpret_cast<const float4*>(gp + 4);
          *reinterpret_cast<float4*>(uv) = *reinterpret_cast<const float4*>(gp + 64);
          *reinterpret_cast<float4*>(uv + 4) = *reinterpret_cast<const float4*>(gp + 68);
          float h[8];
          float m = 0.0f;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            h[j] = swiglu(uv[j], gv[j]);
            m = fmaxf(m, fabsf(h[j]));
          }
#pragma unroll
          for (int off = 8; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
          if (live) {
            const float inv = m > 0.0f ? 448.0f / m : 0.0f;
            uint32_t hw[2] = {0u, 0u}, lw[2] = {0u, 0u};
#pragma unroll
            for (int pr = 0; pr < 4; ++pr) {
              const float x0 = h[2 * pr] * inv, x1 = h[2 * pr + 1] * inv;
              const uint16_t hp = pack_e4m3x2(x0, x1);
              const float2 back = unpack_e4m3x2(hp);
              const uint16_t lp = pack_e4m3x2(x0 - back.x, x1 - back.y);
              hw[pr >> 1] |= static_cast<uint32_t>(hp) << (16 * (pr & 1));
              lw[pr >> 1] |= static_cast<uint32_t>(lp) << (16 * (pr & 1));
            }
            const size_t off = orow * args.I + static_cast<size_t>(u.n) * kBlock + hc;
            *reinterpret_cast<uint2*>(args.h_hi + off) = make_uint2(hw[0], hw[1]);
            *reinterpret_cast<uint2*>(args.h_lo + off) = make_uint2(lw[0], lw[1]);
            if (c == 0) args.h_scale_t[static_cast<size_t>(u.n) * cap + orow] = m / 448.0f;
          }
        } else {
          // output columns oc + [0, 16) of the tile's 256
          const int oc = c * 16;
          const float* vp = xr + ((oc & 127) >> 6) * 128 + (oc >= 128 ? 64 : 0) + (oc & 63);
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; j += 4)
            *reinterpret_cast<float4*>(v + j) = *reinterpret_cast<const float4*>(vp + j);
          float m = 0.0f;
#pragma unroll
          for (int j = 0; j < 16; ++j) m = fmaxf(m, fabsf(v[j]));
#pragma unroll
          for (int off = 8; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
          const int k = pow2_exponent_for_f16(m);
          if (live) {
            store_f16x16(v, ldexpf(1.0f, -k), args.y, orow, u.n * kTileN + oc, args.H);
            if (c == 0) args.y_scale[orow * (args.H / kTileN) + u.n] = ldexpf(1.0f, k);
          }
        }
        continue;
      }
      if (KIND == 3) {
        // add the lo rows' sums to the hi rows' (same slot, same columns, same scales), 16
        // slots per round through xbuf
        const int rounds = (u.nrows + kXSmall - 1) / kXSmall;
        for (int rd = 0; rd < rounds; ++rd) {
          const bool mine = prow >= rd * kXSmall && prow < (rd + 1) * kXSmall && prow < u.nrows;
          float4* x = reinterpret_cast<float4*>(xbuf + (mine ? prow - rd * kXSmall : 0) * kXRow +
                                                g * 128);
          if (lo_row && mine) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              x[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
          }
          named_bar_sync(1, kEpiWarps * 32);
          if (!lo_row && mine) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float4 v = x[i];
              acc[4 * i] += v.x;
              acc[4 * i + 1] += v.y;
              acc[4 * i + 2] += v.z;
              acc[4 * i + 3] += v.w;
            }
          }
          named_bar_sync(1, kEpiWarps * 32);  // xbuf is rewritten by the next round
        }
      }
      const bool valid = prow < u.nrows && !lo_row;
      const size_t row = static_cast<size_t>(u.row0) + prow;
      if (S > 1) {
        // split-K: publish this split's partial tile (valid rows); k_split_finish sums the
        // splits of each tile in split order and runs the epilogue
        if (valid) {
          float* pr = args.partials + (static_cast<size_t>(unit) * args.partial_rows + prow) * kTileN;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float4* dst = reinterpret_cast<float4*>(pr + h * 128 + g * 64);
#pragma unroll
            for (int i = 0; i < 16; ++i)
              dst[i] = make_float4(acc[h * 64 + 4 * i], acc[h * 64 + 4 * i + 1],
                                   acc[h * 64 + 4 * i + 2], acc[h * 64 + 4 * i + 3]);
          }
        }
        continue;
      }

      if (KIND == 1) {
        // SwiGLU (moe.py:90-92: silu(second half) * first half), then the two-term e4m3
        // encoding with one scale per slot per 128 intermediate columns. Padding slots are
        // skipped: GEMM2 only writes the output rows of valid slots, so their intermediate
        // rows and scales are never read into a result.
        float amax = 0.0f;
        if (valid) {
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            const float h = swiglu(acc[64 + c], acc[c]);
            acc[c] = h;
            amax = fmaxf(amax, fabsf(h));
          }
        }
        amax = exchange_amax(tail, g, r, amax);
        if (valid) {
          const float inv = amax > 0.0f ? 448.0f / amax : 0.0f;
          uint8_t* hi_dst = args.h_hi + row * args.I + u.n * kBlock + g * 64;
          uint8_t* lo_dst = args.h_lo + row * args.I + u.n * kBlock + g * 64;
#pragma unroll
          for (int cc = 0; cc < 2; ++cc)
            encode_e4m3_2term32(acc + cc * 32, inv, hi_dst + cc * 32, lo_dst + cc * 32);
          if (g == 0) args.h_scale_t[static_cast<size_t>(u.n) * cap + row] = amax / 448.0f;
        }
      } else {
        float amax = 0.0f;
        if (valid) {
#pragma unroll
          for (int c = 0; c < 128; ++c) amax = fmaxf(amax, fabsf(acc[c]));
        }
        amax = exchange_amax(tail, g, r, amax);
        const int k = pow2_exponent_for_f16(amax);
        const float inv = ldexpf(1.0f, -k);
        if (valid) {
#pragma unroll
          for (int cc = 0; cc < 8; ++cc)
            store_f16x16(acc + cc * 16, inv, args.y, row,
                         u.n * kTileN + (cc >> 2) * 128 + g * 64 + (cc & 3) * 16, args.H);
          if (g == 0) args.y_scale[row * (args.H / kTileN) + u.n] = ldexpf(1.0f, k);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Split-K finish (small batches): one CTA per tile sums the tile's S partial tiles in split
// order into shared memory -- every thread takes (row, 4-column) items and keeps four splits'
// loads in flight -- then runs the tile's epilogue with one warp per valid row: SwiGLU and the
// two-term e4m3 encoding (KIND 1) or fp16 with a power-of-two scale (KIND 2), the same
// arithmetic as k_gemm's register epilogue.
// Dependents are released before the wait: GEMM2 reads the plan before its own wait, and the
// plan was complete before GEMM1 launched (the gather releases GEMM1 only after its own wait),
// so GEMM2 may start and prefetch weights while this kernel waits for GEMM1; GEMM2's wait then
// covers this kernel, which ends after GEMM1. T=8: 99.1 -> 98.4 us per call.
template <int KIND>
__global__ void __launch_bounds__(256) k_split_finish(const GemmArgs args) {
  pdl_begin();
  const int S = args.plan[KIND == 1 ? kPlanSplit1 : kPlanSplit2];
  if (S <= 1) return;
  const int tiles = args.plan[KIND == 1 ? kPlanTiles1 : kPlanTiles2];
  __shared__ int ebase[kMaxLocalExperts + 1];
  __shared__ int ecnt[kMaxLocalExperts];
  extern __shared__ float red[];  // [partial_rows][kTileN]
  const int E = args.E;
  for (int i = threadIdx.x; i <= E; i += blockDim.x) {
    ebase[i] = args.expert_base[i];
    if (i < E) ecnt[i] = args.expert_count[i];
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = blockDim.x >> 5;
  const int nkb = KIND == 1 ? args.H / kBlock : args.I / kBlock;
  const int NT = KIND == 1 ? args.I / kBlock : args.H / kTileN;
  const size_t split_stride = static_cast<size_t>(args.partial_rows) * kTileN;
  for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const Unit u = decode_unit(tile * S, S, NT, nkb, ebase, ecnt, E);
    const float* tile0 = args.partials + static_cast<size_t>(tile * S) * split_stride;
    for (int item = threadIdx.x; item < u.nrows * (kTileN / 4); item += blockDim.x) {
      const int rr = item / (kTileN / 4);
      const int c4 = (item - rr * (kTileN / 4)) * 4;
      const float* src = tile0 + static_cast<size_t>(rr) * kTileN + c4;
      float4 sum = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      for (int sp0 = 0; sp0 < S; sp0 += 4) {
        float4 x[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (sp0 + j < S) x[j] = __ldcg(reinterpret_cast<const float4*>(src + (sp0 + j) * split_stride));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (sp0 + j < S) {
            sum.x += x[j].x;
            sum.y += x[j].y;
            sum.z += x[j].z;
            sum.w += x[j].w;
          }
        }
      }
      *reinterpret_cast<float4*>(red + rr * kTileN + c4) = sum;
    }
    __syncthreads();
    for (int rr = warp; rr < u.nrows; rr += nwarp) {
      const size_t row = static_cast<size_t>(u.row0) + rr;
      const float* v = red + rr * kTileN;
      if (KIND == 1) {
        // lane: intermediate columns lane*4 + [0,4) of the tile's 128 (gate | up halves)
        float h[4];
        float m = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          h[j] = swiglu(v[128 + lane * 4 + j], v[lane * 4 + j]);
          m = fmaxf(m, fabsf(h[j]));
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        const float inv = m > 0.0f ? 448.0f / m : 0.0f;
        uint32_t hw = 0, lw = 0;
#pragma unroll
        for (int pr = 0; pr < 2; ++pr) {
          const float x0 = h[2 * pr] * inv, x1 = h[2 * pr + 1] * inv;
          const uint16_t hp = pack_e4m3x2(x0, x1);
          const float2 back = unpack_e4m3x2(hp);
          const uint16_t lp = pack_e4m3x2(x0 - back.x, x1 - back.y);
          hw |= static_cast<uint32_t>(hp) << (16 * pr);
          lw |= static_cast<uint32_t>(lp) << (16 * pr);
        }
        const size_t off = row * args.I + static_cast<size_t>(u.n) * kBlock + lane * 4;
        *reinterpret_cast<uint32_t*>(args.h_hi + off) = hw;
        *reinterpret_cast<uint32_t*>(args.h_lo + off) = lw;
        if (lane == 0) args.h_scale_t[static_cast<size_t>(u.n) * args.cap + row] = m / 448.0f;
      } else {
        // lane: output columns lane*8 + [0,8) of the tile's 256
        float x[8];
        float m = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          x[j] = v[lane * 8 + j];
          m = fmaxf(m, fabsf(x[j]));
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        const int k = pow2_exponent_for_f16(m);
        const float inv = ldexpf(1.0f, -k);
        uint32_t wv[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const __half2 pr = __floats2half2_rn(x[2 * w] * inv, x[2 * w + 1] * inv);
          wv[w] = *reinterpret_cast<const uint32_t*>(&pr);
        }
        *reinterpret_cast<uint4*>(args.y + row * args.H + static_cast<size_t>(u.n) * kTileN +
                                  lane * 8) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        if (lane == 0) args.y_scale[row * (args.H / kTileN) + u.n] = ldexpf(1.0f, k);
      }
    }
    __syncthreads();  // red is rewritten by the next tile
  }
}

template <int KIND>
static GemmArgs gemm_args(const RunParams& p) {
  uint8_t* ws = p.ws;
  const Layout& L = p.L;
  GemmArgs a{};
  a.plan = reinterpret_cast<const int32_t*>(ws + L.plan);
  a.expert_base = reinterpret_cast<const int32_t*>(ws + L.expert_base);
  a.expert_count = reinterpret_cast<const int32_t*>(ws + L.expert_count);
  a.a_scale_t = reinterpret_cast<const float*>(ws + (KIND == 1 ? L.a_scale_t : L.h_scale_t));
  a.w_scale = KIND == 1 ? p.w1_scale : p.w2_scale;
  a.partials = reinterpret_cast<float*>(ws + L.partials);
  a.counters = reinterpret_cast<int32_t*>(ws + L.counters);
  a.status = reinterpret_cast<int32_t*>(ws + L.status);
  a.h_hi = ws + L.h_hi;
  a.h_lo = ws + L.h_lo;
  a.h_scale_t = reinterpret_cast<float*>(ws + L.h_scale_t);
  a.y = reinterpret_cast<__half*>(ws + L.y_rows);
  a.y_scale = reinterpret_cast<float*>(ws + L.y_scale);
  a.E = p.E;
  a.H = p.H;
  a.I = p.I;
  a.cap = L.cap;
  a.partial_rows = static_cast<int>(L.partial_rows);
  a.wait_ns = p.wait_ns != 0 ? p.wait_ns : FMOE_WAIT_NS;
  a.inject = p.inject_gemm == (KIND == 1 ? 1 : 2) ? 1 : 0;
  return a;
}

template <int KIND>
static cudaError_t launch_gemm_kind(const RunParams& p, const CUtensorMap& a0,
                                    const CUtensorMap& a1, const CUtensorMap& w,
                                    const CUtensorMap& sa, cudaStream_t s) {
  const size_t smem = gemm_smem_bytes<KIND>();
  // The shared-memory opt-in is a per-device function attribute: set once per device (an
  // idempotent call, so two host threads that both see it unset only repeat it).
  static std::atomic<bool> configured[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured[dev].store(true, std::memory_order_release);
  }
  const GemmArgs a = gemm_args<KIND>(p);
  (void)launch_pdl(k_gemm<KIND>, p.num_sms, kThreads, smem, s, a0, a1, w, sa, a);
  return cudaGetLastError();
}

cudaError_t launch_split_finish(const RunParams& p, int kind, cudaStream_t s) {
  // at most partial_rows (<= kSplitMaxT) rows of 256 fp32 per tile in shared memory; two CTAs
  // per SM, so up to 2 * num_sms split tiles (T=8: 160 GEMM1 tiles) finish in one round
  const size_t smem = static_cast<size_t>(p.L.partial_rows) * kTileN * 4;
  if (kind == 1)
    (void)launch_pdl(k_split_finish<1>, 2 * p.num_sms, 256, smem, s, gemm_args<1>(p));
  else
    (void)launch_pdl(k_split_finish<2>, 2 * p.num_sms, 256, smem, s, gemm_args<2>(p));
  return cudaGetLastError();
}

cudaError_t launch_gemm1(const RunParams& p, const CUtensorMap& tm_a, const CUtensorMap& tm_w1,
                         const CUtensorMap& tm_sa, cudaStream_t s) {
  return launch_gemm_kind<1>(p, tm_a, tm_a, tm_w1, tm_sa, s);
}

cudaError_t launch_gemm2(const RunParams& p, const CUtensorMap& tm_hi, const CUtensorMap& tm_lo,
                         const CUtensorMap& tm_w2, const CUtensorMap& tm_sa, cudaStream_t s) {
  if (p.T <= kPackedMaxT) return launch_gemm_kind<3>(p, tm_hi, tm_lo, tm_w2, tm_sa, s);
  return launch_gemm_kind<2>(p, tm_hi, tm_lo, tm_w2, tm_sa, s);
}

}  // namespace fmoe
