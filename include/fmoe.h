/*
 * fmoe.h -- C ABI of the B200 (sm_100a) fused FP8 block-scale MoE with DeepSeek-V3 routing.
 *
 * Operator: moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048. The entry
 * points replace the reference's Python/Triton operator
 *   solution/triton/kernel.py:600-825   run(routing_logits, routing_bias, hidden_states,
 *                                           hidden_states_scale, gemm1_weights,
 *                                           gemm1_weights_scale, gemm2_weights,
 *                                           gemm2_weights_scale, local_expert_offset,
 *                                           routed_scaling_factor, output)
 * and the empty CUDA slot the reference leaves for a compiled solution
 *   solution/cuda/binding.py:11-25      (TVM-FFI "flashinfer.kernel" stub)
 *   solution/cuda/kernel.cu:13-20
 *
 * Conventions: plain device pointers and sizes only; every launch goes on the given
 * cudaStream_t (pass the caller's current stream); no call allocates device memory or
 * synchronises the host -- the caller supplies a workspace of fmoe_workspace_size()
 * bytes. All functions return 0 on success or a negative FMOE_ERR_* code.
 */
#ifndef FMOE_H_
#define FMOE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FMOE_API __attribute__((visibility("default")))
#else
#define FMOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Error codes (argument checks happen on the host before any launch). */
#define FMOE_OK                 0
#define FMOE_ERR_NULL         (-1)  /* a required pointer is NULL                          */
#define FMOE_ERR_SHAPE        (-2)  /* unsupported hidden/intermediate/expert/top-k sizes   */
#define FMOE_ERR_ALIGN        (-3)  /* a pointer is not 16-byte aligned                     */
#define FMOE_ERR_OFFSET       (-4)  /* local_expert_offset + num_local_experts > E_global   */
#define FMOE_ERR_WORKSPACE    (-5)  /* workspace missing or smaller than fmoe_workspace_size */
#define FMOE_ERR_DTYPE        (-6)  /* unsupported routing logits / bias dtype              */
#define FMOE_ERR_CUDA         (-7)  /* a CUDA runtime or driver call failed                 */
#define FMOE_ERR_DEVICE       (-8)  /* the current device is not sm_100                     */
#define FMOE_ERR_NOALLOC_LIMIT (-9) /* more tokens than fmoe_route_permute_noalloc supports  */

/* Device status word bits (fmoe_read_status): set by a kernel whose bounded wait ran out. */
#define FMOE_STATUS_TIMEOUT_GEMM1  0x1
#define FMOE_STATUS_TIMEOUT_GEMM2  0x2

/* output dtypes */
#define FMOE_OUT_BF16    0
#define FMOE_OUT_F32     1
/* Partial rows for expert parallelism: each token's row is H fp16 values followed by H/256
 * fp32 power-of-two scales (value = fp16 * scale of its 256-column block), padded to a multiple
 * of 32 bytes (the rows are written with 32-byte stores): FMOE_EP_ROW_BYTES(H) bytes at the row
 * address that FmoeArgs.region_output gives for the token (32-byte aligned). */
#define FMOE_OUT_F16S    2
#define FMOE_EP_ROW_BYTES(H) (((size_t)(H) * 2 + (size_t)(H) / 256 * 4 + 31) / 32 * 32)
#define FMOE_EP_MAX_RANKS 8

/* dtype tags for the routing inputs */
#define FMOE_DTYPE_F32   0
#define FMOE_DTYPE_BF16  1

/* Routing methods (FmoeArgs.routing_method). DeepSeek-V3 is the hot path of kernel.py:371-457
 * and the zero value; the others are the same definition family's routing references
 * (flashinfer/trace/templates/moe.py:187-390; their RoutingMethodType number in brackets), all
 * with routing_bias added to the logits first:
 *   DEFAULT [0]            softmax -> top_k; weight = softmax value * rsf
 *   RENORMALIZE [1]        top_k of the logits -> softmax over the picks * rsf
 *   LLAMA4 [3]             top-1 of the logits; weight = sigmoid(logit) * rsf (top_k = 1)
 *   RENORMALIZE_NAIVE [4]  softmax -> top_k -> divided by their sum (+1e-20) * rsf
 *   TOPK [5]               top_k of the logits; every weight rsf / top_k
 * Ties go to the lower expert index. top_k may be 1..8 except for DeepSeek-V3 (8) and
 * Llama4 (1); n_group and topk_group are used by DeepSeek-V3 only. */
#define FMOE_ROUTING_DEEPSEEK_V3       0
#define FMOE_ROUTING_DEFAULT           1
#define FMOE_ROUTING_RENORMALIZE       2
#define FMOE_ROUTING_LLAMA4            3
#define FMOE_ROUTING_RENORMALIZE_NAIVE 4
#define FMOE_ROUTING_TOPK              5

/* Stop points for staged execution (tests inspect the workspace in between). */
#define FMOE_PATH_AUTO     0
#define FMOE_PATH_GEMM     1

#define FMOE_STOP_NONE     0
#define FMOE_STOP_ROUTE    1   /* after routing, permutation and the activation gather */
#define FMOE_STOP_GATHER   2   /* same point (the gather is fused into the permutation) */
#define FMOE_STOP_GEMM1    3   /* after GEMM1 + SwiGLU (intermediate)  */
#define FMOE_STOP_GEMM2    4   /* after GEMM2 (per-slot output rows)   */

typedef struct FmoeArgs {
  /* reference kernel.py:602  routing_logits  [T, E_global]  fp32 (or bf16, see logits_dtype) */
  const void* routing_logits;
  int32_t logits_dtype;
  /* kernel.py:603  routing_bias  [E_global]  bf16 (or fp32, see bias_dtype)                  */
  const void* routing_bias;
  int32_t bias_dtype;
  /* kernel.py:604  hidden_states  [T, H]  float8_e4m3fn                                      */
  const void* hidden_states;
  /* kernel.py:605  hidden_states_scale  [H/128, T]  fp32                                     */
  const float* hidden_states_scale;
  /* kernel.py:606  gemm1_weights  [E_local, 2*I, H]  float8_e4m3fn (rows 0..I-1 gate, I.. up)*/
  const void* gemm1_weights;
  /* kernel.py:607  gemm1_weights_scale  [E_local, 2*I/128, H/128]  fp32                      */
  const float* gemm1_weights_scale;
  /* kernel.py:608  gemm2_weights  [E_local, H, I]  float8_e4m3fn                             */
  const void* gemm2_weights;
  /* kernel.py:609  gemm2_weights_scale  [E_local, H/128, I/128]  fp32                        */
  const float* gemm2_weights_scale;
  /* kernel.py:612  output  [T, H]  bf16, written in place (destination-passing)              */
  void* output;
  int32_t num_tokens;            /* T >= 0                                                  */
  int32_t hidden_size;           /* H: multiple of 256 (7168)                               */
  int32_t intermediate_size;     /* I: multiple of 128 (2048)                               */
  int32_t num_experts;           /* E_global: 256                                           */
  int32_t num_local_experts;     /* E_local: 1..256                                         */
  int32_t top_k;                 /* 8                                                       */
  int32_t n_group;               /* 8                                                       */
  int32_t topk_group;            /* 4                                                       */
  int32_t local_expert_offset;   /* kernel.py:610                                           */
  float routed_scaling_factor;   /* kernel.py:611                                           */
  void* workspace;               /* device buffer, >= fmoe_workspace_size() bytes           */
  size_t workspace_bytes;
  int32_t stop_after;            /* FMOE_STOP_*; 0 runs the whole operator                   */
  /* Optional phase timing (the reference's FIB_PROFILE_PHASES, kernel.py:631-672): when
   * non-NULL, an array of num_phase_events cudaEvent_t recorded on the stream at phase
   * boundaries: [0] start, [1] routed + planned, [2] gathered, [3] GEMM1 done,
   * [4] GEMM2 done, [5] combined. Extra entries are ignored; NULL entries are skipped. */
  void* const* phase_events;
  int32_t num_phase_events;
  /* FMOE_OUT_BF16 (the reference's output, kernel.py:822) or FMOE_OUT_F32: the same sum left
   * in fp32, for callers that add several partial outputs (expert parallelism) before the
   * single final rounding to bf16. */
  int32_t output_dtype;
  /* FMOE_ROUTING_*; 0 (DeepSeek-V3) for callers that zero the struct. */
  int32_t routing_method;
  /* Pre-routed calls (the receiving side of expert parallelism; NULL for a normal call). When
   * topk_ids is set, the routing step is skipped: token t's picks are the GLOBAL expert ids
   * topk_ids[t*8 .. t*8+8) (-1 = no pick) with weights topk_weights[t*8 ..] (device arrays),
   * exactly as the routing of the sending rank produced them; routing_logits and routing_bias
   * are not read. With region_counts set as well, the T tokens form T / region_tokens regions
   * of region_tokens tokens (one per sending rank) and token j of region r takes part only if
   * j < region_counts[r] (a device array; the other tokens are ignored). */
  const int32_t* topk_ids;
  const float* topk_weights;
  const int32_t* region_counts;
  int32_t region_tokens;
  /* FMOE_OUT_F16S only: token j of region r is written to region_output[r] + j *
   * FMOE_EP_ROW_BYTES(H) (32-byte aligned device addresses; may be another GPU's memory mapped
   * into this process). Tokens without a local pick are not written. */
  void* region_output[FMOE_EP_MAX_RANKS];
  /* FMOE_PATH_AUTO (0): calls of at most 2 tokens with a bf16 or fp32 output run the
   * matrix-vector path (GEMM1 and GEMM2 streamed on the CUDA cores, SwiGLU and the combine fused
   * in; 3 kernels); FMOE_PATH_GEMM: always the grouped tensor-core GEMMs. Staged calls
   * (stop_after != 0) always take the grouped GEMMs. */
  int32_t gemm_path;
} FmoeArgs;

/* Offsets (bytes from the workspace base) of the regions tests and tools read back. */
typedef struct FmoeLayout {
  size_t total_bytes;
  size_t status;          /* int32  [4]      device status word (bits FMOE_STATUS_*)          */
  size_t plan;            /* int32  [16]     P, padded slots, m-tiles, split/units per GEMM    */
  size_t topk_ids;        /* int32  [T, 8]   global expert ids, selection order               */
  size_t topk_weights;    /* fp32   [T, 8]   routing weights, same order                     */
  size_t expert_count;    /* int32  [E_local]                                                 */
  size_t expert_base;     /* int32  [E_local+1] first slot of each expert (multiples of 128)   */
  size_t slot_token;      /* int32  [cap]    token of each slot (-1 = padding)                 */
  size_t slot_weight;     /* fp32   [cap]                                                     */
  size_t token_slot;      /* int32  [T, 8]   slots of a token's local picks, expert ascending  */
  size_t token_weight;    /* fp32   [T, 8]                                                    */
  size_t a_perm;          /* e4m3   [cap, H] gathered activation rows                          */
  size_t a_scale_t;       /* fp32   [H/128, cap]                                               */
  size_t h_hi;            /* e4m3   [cap, I] SwiGLU output, leading term                       */
  size_t h_lo;            /* e4m3   [cap, I] SwiGLU output, residual term                      */
  size_t h_scale_t;       /* fp32   [I/128, cap]                                               */
  size_t y_rows;          /* fp16   [cap, H] per-slot GEMM2 output rows, scaled by y_scale     */
  size_t y_scale;         /* fp32   [cap, H/256] power-of-two scale per slot per 256 columns   */
  size_t partials;        /* fp32   split-K partial tiles                                      */
  size_t counters;        /* int32  split-K arrival counters                                   */
  size_t block_hist;      /* int32  [nblocks, E_local] local picks per routing block           */
  size_t block_off;       /* int32  [nblocks, E_local] first slot of each block per expert     */
  int64_t cap_slots;      /* padded slot capacity                                             */
  int64_t max_units;      /* split-K partial tile capacity                                    */
  int64_t tokens_per_block; /* tokens per routing block                                       */
  int64_t num_blocks;     /* routing blocks                                                   */
} FmoeLayout;

/* Workspace bytes for T tokens and E_local local experts (H, I as in FmoeArgs).
 * No counterpart in the reference: its run() allocates temporaries per call
 * (kernel.py:535-581, :710, :747, :769, :801). */
FMOE_API int fmoe_workspace_size(int32_t num_tokens, int32_t num_local_experts, int32_t hidden_size,
                        int32_t intermediate_size, size_t* bytes);

/* Region offsets of the workspace (same arguments as fmoe_workspace_size). */
FMOE_API int fmoe_workspace_layout(int32_t num_tokens, int32_t num_local_experts, int32_t hidden_size,
                          int32_t intermediate_size, FmoeLayout* layout);

/* The fused operator: routing -> permutation -> GEMM1+SwiGLU -> GEMM2 -> weighted combine.
 * Replaces kernel.py:600-825 run(...). Stream-ordered, no host synchronisation, no
 * allocation; graph-capturable. */
FMOE_API int fmoe_run(const FmoeArgs* args, void* cuda_stream);

/* Routing only: global top-k ids [T, top_k] (int32) and weights [T, top_k] (fp32).
 * Replaces the routing half of kernel.py:519-557 (_route_select_local_kernel), but keeps
 * the global ids (callers derive locality themselves, as kernel.py:448-452 does). */
FMOE_API int fmoe_route(const void* routing_logits, int32_t logits_dtype, const void* routing_bias,
               int32_t bias_dtype, int32_t num_tokens, int32_t num_experts, int32_t top_k,
               int32_t n_group, int32_t topk_group, float routed_scaling_factor,
               int32_t* topk_ids, float* topk_weights, void* cuda_stream);

/* Routing + permutation without any device allocation, for callers that cannot allocate
 * device memory where they enqueue work (engines that plan every buffer ahead and forbid
 * allocation at enqueue time, code inside a CUDA graph capture with a fixed memory pool, host
 * programs bound to the C ABI from runtimes without a device allocator). No counterpart in
 * the reference, whose run() allocates its temporaries on every call.
 *
 * Writes the same tables fmoe_run() builds before its GEMMs: expert_count [E_local],
 * expert_base [E_local+1] (first slot of each expert, multiples of 128), slot_token and
 * slot_weight (the caller sizes them [cap], cap = cap_slots of fmoe_workspace_layout; only
 * slots [0, expert_base[E_local]) are written -- the padding slots inside that range hold
 * -1 / 0 -- and entries from expert_base[E_local] up to cap are left as the caller had them),
 * token_slot and token_weight [T, 8] (a token's local picks in ascending expert order, -1 /
 * 0 after them). Its scratch is one statically allocated device array of 336,384 bytes,
 * which every GPU that loads this library keeps until the process exits:
 *   - num_tokens may be at most 4096; larger requests return FMOE_ERR_NOALLOC_LIMIT;
 *   - the first call on a device looks up the array's device address (cudaGetSymbolAddress)
 *     with that device current and keeps it for the life of the process; make that first
 *     call before any stream capture, and do not use this entry point after a device reset
 *     (cudaDeviceReset, or the primary context destroyed and re-created), which may move the
 *     array;
 *   - all calls on a device share the array, so calls whose executions overlap on the GPU
 *     race and produce undefined tables: order them on one stream. */
FMOE_API int fmoe_route_permute_noalloc(const void* routing_logits, int32_t logits_dtype,
                                        const void* routing_bias, int32_t bias_dtype,
                                        int32_t num_tokens, int32_t num_local_experts,
                                        int32_t local_expert_offset,
                                        float routed_scaling_factor, int32_t* expert_count,
                                        int32_t* expert_base, int32_t* slot_token,
                                        float* slot_weight, int32_t* token_slot,
                                        float* token_weight, void* cuda_stream);

/* Input quantisation, the step that produces the operator's activation inputs: bf16
 * x [T, H] (row-major, 16-byte aligned) -> e4m3 q [T, H] and fp32 scale_t [H/128, T], per token
 * and 128-column block scale = max(amax, 1e-30) / 448, q = e4m3(x / scale) rounded to nearest
 * even. No counterpart in the reference, which receives hidden_states already quantised in
 * this layout (kernel.py:601-602; hidden_states_scale indexed [kb, token] at kernel.py:169).
 * H must be a multiple of 128; q and scale_t must not overlap x. */
FMOE_API int fmoe_quantize_activations(const void* x_bf16, int32_t num_tokens, int32_t hidden_size,
                                       void* q_e4m3, float* scale_t, void* cuda_stream);

/* ---------------------------------------------------------------- expert parallelism
 * One rank of R (R <= FMOE_EP_MAX_RANKS) owns experts [rank*256/R, (rank+1)*256/R) and
 * T_rank tokens. The reference's per-rank contract is run() over the local expert range
 * (kernel.py:442-452); these entry points move tokens to the ranks that own their picks and the
 * partial outputs back, with plain stores into the other GPUs' memory (CUDA IPC mappings, no
 * multicast) -- no counterpart in the reference, which has no multi-GPU code.
 *
 * Every rank holds one device buffer of the layout below (allocate it with fmoe_ep_alloc so it
 * can be exported, then map every other rank's buffer with fmoe_ipc_open):
 *   recv_hidden  e4m3 [R * cap, H]     rows sent to this rank, region r = sender r
 *   recv_scale   fp32 [H/128, R * cap] their 128-column scales (scale-major, as run() reads)
 *   recv_ids     int32 [R * cap, 8]    the sender's routing picks (global ids) ...
 *   recv_weights fp32 [R * cap, 8]     ... and weights
 *   recv_counts  int32 [R]             tokens received from each sender
 *   ret_rows     [R * cap] rows of FMOE_EP_ROW_BYTES(H): partial outputs returned to this
 *                rank, region d = from rank d, row = the token's slot at d
 * with cap = the most tokens any rank processes per call (a sender may send all its tokens to
 * one rank); every rank uses the same cap, so the regions sit at the same offsets everywhere. */
typedef struct FmoeEpLayout {
  size_t total_bytes;
  size_t recv_hidden, recv_scale, recv_ids, recv_weights, recv_counts, ret_rows;
  int64_t cap;
  size_t row_bytes;
} FmoeEpLayout;

FMOE_API int fmoe_ep_layout(int32_t world, int32_t capacity, int32_t hidden_size,
                            FmoeEpLayout* layout);

/* Device memory that other processes can map (cudaMalloc; fmoe_run itself never allocates). */
FMOE_API int fmoe_ep_alloc(size_t bytes, void** ptr);
FMOE_API int fmoe_ep_free(void* ptr);
/* CUDA IPC: a 64-byte handle of an fmoe_ep_alloc buffer, and its mapping in another process
 * (peer access enabled on first use). fmoe_ipc_close unmaps. */
FMOE_API int fmoe_ipc_get_handle(const void* ptr, void* handle64);
FMOE_API int fmoe_ipc_open(const void* handle64, void** ptr);
FMOE_API int fmoe_ipc_close(void* ptr);

/* Dispatch on the sending rank: for each of its T_rank tokens (picks topk_ids/topk_weights
 * [T_rank, 8] from fmoe_route), the ranks that own at least one pick; the token's slot at such
 * a rank is its position among this rank's tokens sent there (tokens ascending). Writes the
 * token's e4m3 row, scales, picks and weights into region `rank` of every destination's buffer
 * (peer_buffers[d]: rank d's buffer as mapped here, this rank's own buffer at d == rank), the
 * per-destination count into their recv_counts[rank], and token_dest_slot [T_rank, R] (-1 = not
 * sent) for the reduction. tokens <= capacity (the cap of fmoe_ep_layout). A system-scope fence
 * ends the kernels; the caller then orders the destinations after them (a collective on every
 * rank's stream). peer_buffers is a host array of `world` device addresses. */
FMOE_API int fmoe_ep_dispatch(const int32_t* topk_ids, const float* topk_weights,
                              const void* hidden_states, const float* hidden_states_scale,
                              int32_t tokens, int32_t capacity, int32_t hidden_size,
                              int32_t world, int32_t rank, void* const* peer_buffers,
                              int32_t* token_dest_slot, void* cuda_stream);

/* Reduction on the sending rank, after every destination's fmoe_run (FMOE_OUT_F16S into region
 * `rank` of this rank's ret_rows): out[t] = bf16(sum over d = 0..R-1 of the partial row from d),
 * in ascending rank order (= ascending expert order, the single-GPU sum order), fp32 sums. */
FMOE_API int fmoe_ep_reduce(const int32_t* token_dest_slot, const void* buffer, int32_t tokens,
                            int32_t capacity, int32_t hidden_size, int32_t world,
                            void* output_bf16, void* cuda_stream);

/* Failure-path test (no counterpart in the reference): arms the next fmoe_run of the calling
 * host thread so that GEMM `gemm` (1 or 2) waits on a barrier nothing arrives on, with every wait
 * of that call's GEMMs limited to wait_ns (100 us .. 2 s) instead of 2 s. The wait runs out, the
 * kernel sets FMOE_STATUS_TIMEOUT_GEMM<gemm> in the status word, stops its producers, waits for
 * its copies in flight, frees its tensor memory and returns; the call's output is not valid, and
 * the next call runs normally (its plan kernel clears the status word). One-shot. */
FMOE_API int fmoe_debug_arm_timeout(int32_t gemm, uint64_t wait_ns);

/* Copies the device status word into *status (synchronises the stream). Non-zero means a
 * kernel gave up on a bounded wait and its outputs are not valid. */
FMOE_API int fmoe_read_status(const void* workspace, void* cuda_stream, int32_t* status);

/* The device's dense FP8 tensor rate with the GEMMs' MMA shape (no counterpart in the
 * reference): one CTA per SM issues k_blocks x 4 tcgen05.mma kind::f8f6f4 M=128 N=256 K=32 from
 * shared memory, nothing else. Enqueued on the stream (time it with events around the call);
 * *flops receives the FLOPs it performs; a bounded wait that ran out sets bit 0 of the device
 * word *status. k_blocks: 1..500000. */
FMOE_API int fmoe_fp8_mma_peak(int32_t k_blocks, int32_t* status, double* flops,
                               void* cuda_stream);

/* Number of SMs the persistent GEMM kernels size their grid for on the current device. */
FMOE_API int fmoe_device_sm_count(int32_t* sms);

/* Build identification string (static storage). */
FMOE_API const char* fmoe_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FMOE_H_ */
