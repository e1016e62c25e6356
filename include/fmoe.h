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

/* Copies the device status word into *status (synchronises the stream). Non-zero means a
 * kernel gave up on a bounded wait and its outputs are not valid. */
FMOE_API int fmoe_read_status(const void* workspace, void* cuda_stream, int32_t* status);

/* Number of SMs the persistent GEMM kernels size their grid for on the current device. */
FMOE_API int fmoe_device_sm_count(int32_t* sms);

/* Build identification string (static storage). */
FMOE_API const char* fmoe_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FMOE_H_ */
