/*
 * moe_b200.h - C ABI of the B200 (sm_100a) fused FP8 block-scale MoE forward.
 *
 * Drop-in for the hot path of nikhilnd/mlsys26-flashinfer-moe, whose whole
 * product is the Python entry point
 *
 *   run(routing_logits, routing_bias, hidden_states, hidden_states_scale,
 *       gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
 *       local_expert_offset, routed_scaling_factor, output)      (kernel.py:562-575)
 *
 * The reference has no native library; these entry points are what its
 * Triton launches (kernel.py:624-729) become when they are bound through a
 * plain C interface (ctypes / cffi / any FFI).  Signatures hold only plain
 * pointers, sizes and a cudaStream_t passed as void*: no framework types.
 *
 * Layouts (all row-major, e4m3 = OCP float8 e4m3fn stored as bytes):
 *   routing_logits      [T, E_global]              fp32
 *   routing_bias        [E_global]                 fp32 / bf16 / fp16 (bias_dtype)
 *   hidden_states       [T, H]                     e4m3
 *   hidden_states_scale [H/128, T]                 fp32 (token-minor, kernel.py:603)
 *   gemm1_weights       [E_local, 2*I, H]          e4m3 (rows [0,I) multiply, [I,2I) gate the SiLU)
 *   gemm1_weights_scale [E_local, 2*I/128, H/128]  fp32
 *   gemm2_weights       [E_local, H, I]            e4m3
 *   gemm2_weights_scale [E_local, H/128, I/128]    fp32
 *   output              [T, H]                     bf16
 *
 * Every call is asynchronous on `stream`, performs no host<->device
 * synchronisation and allocates nothing: scratch lives in the caller's
 * workspace (see moe_fp8_workspace_size).
 */
#ifndef MOE_B200_H_
#define MOE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (0 = success).  The Python layer maps shape/dtype errors to
 * AssertionError (reference kernel.py:591-607) and the rest to RuntimeError. */
#define MOE_OK 0
#define MOE_ERR_INVALID_ARG (-1)     /* null pointer or bad enum value */
#define MOE_ERR_SHAPE (-2)           /* unsupported or inconsistent shape */
#define MOE_ERR_ALIGNMENT (-3)       /* a pointer is not 16-byte aligned */
#define MOE_ERR_WORKSPACE (-4)       /* workspace missing or too small */
#define MOE_ERR_CUDA (-5)            /* a CUDA runtime / driver call failed */
#define MOE_ERR_TIMEOUT (-6)         /* a device-side bounded wait expired */
#define MOE_ERR_DEVICE (-7)          /* device is not sm_100 */
#define MOE_ERR_TOO_LARGE (-8)       /* beyond the fixed scratch of moe_fp8_route_noalloc */
#define MOE_ERR_BOUNDS (-9)          /* MOE_FLAG_DEBUG: a dispatch table or a workspace guard
                                        failed its check; info = MOE_CHECK_* << 24 | index */

/* routing_bias element type */
#define MOE_BIAS_F32 0
#define MOE_BIAS_BF16 1
#define MOE_BIAS_F16 2

/* MoeFwdArgs.flags */
/* Fixed-order combine: GEMM2 stores every (token, expert) row's weighted fp32
 * result and a gather adds a token's rows in routing-selection order, so the
 * output is bit-identical from run to run.  The default adds rows with fp32
 * atomics in whatever order they finish, as the reference does
 * (kernel.py:246-250).  Costs one extra fp32 write and read per assignment row
 * (rows_out in the workspace). */
#define MOE_FLAG_DETERMINISTIC 0x1u
/* Debug bounds checks.  The forward writes a 16-byte guard pattern after every
 * workspace buffer, checks the routing and dispatch tables on the device before
 * any kernel uses them as indices (moe_fp8_check_workspace's checks), lets the
 * GEMMs do no work when a check failed, and checks the guards after the last
 * kernel.  A failure records MOE_ERR_BOUNDS with info = (MOE_CHECK_* << 24) |
 * the failing element's index (clamped to 24 bits) in the control block; read it
 * with moe_fp8_device_error.  The output is not meaningful after a failure.  The
 * reference has no counterpart (its kernels index without checks). */
#define MOE_FLAG_DEBUG 0x2u
/* Failure-detection tests only: the first MMA issuer of each GEMM1 CTA waits
 * on a barrier that nothing completes, so its bounded wait runs out after
 * wait_limit_ns; the layer then drains, records MOE_ERR_TIMEOUT (info = the
 * wait site) and returns without faulting.  The output is not computed. */
#define MOE_FLAG_TEST_STALL 0x100u

typedef struct MoeFwdArgs {
  const float* routing_logits;
  const void* routing_bias;
  const void* hidden_states;
  const float* hidden_states_scale;
  const void* gemm1_weights;
  const float* gemm1_weights_scale;
  const void* gemm2_weights;
  const float* gemm2_weights_scale;
  void* output;
  int64_t T;                   /* tokens (may be 0), at most 2^24 */
  int64_t H;                   /* hidden size, multiple of 256 */
  int64_t I;                   /* intermediate size, multiple of 128 */
  int64_t E_global;            /* routed experts, <= 256 */
  int64_t E_local;             /* experts with weights here, <= E_global */
  int64_t local_expert_offset; /* first local expert (reference kernel.py:572) */
  int64_t n_group;             /* expert groups (8 for DeepSeek-V3) */
  int64_t topk_group;          /* groups kept per token (4) */
  int64_t top_k;               /* experts per token (8), <= 8 */
  float routed_scaling_factor;
  int32_t bias_dtype;          /* MOE_BIAS_* */
  void* workspace;             /* device scratch, 256-byte aligned */
  size_t workspace_bytes;
  uint32_t flags;              /* MOE_FLAG_*; 0 = reference behaviour */
  uint32_t reserved;           /* must be 0 */
  uint64_t wait_limit_ns;      /* bound of every device-side wait; 0 = 2 s */
  /* Optional: the down-projection weights prepared once by
   * moe_fp8_prepare_gemm2_bf16, [E_local, H, I] bf16.  When set, batches on the
   * prefill path run GEMM2 on bf16 operands without block-scale promotion
   * (GEMM1 then writes the dequantised intermediate); NULL = FP8 path. */
  const void* gemm2_weights_bf16;
  /* Shared experts (0 or 1; DeepSeek-V3 has one, intermediate size I).  When 1,
   * the weight tensors hold E_local + 1 experts: the routed experts
   * [local_expert_offset, local_expert_offset + E_local) followed by the shared
   * expert, i.e. gemm1_weights [E_local + 1, 2I, H], gemm2_weights
   * [E_local + 1, H, I] and their scales likewise.  Every token also goes
   * through the shared expert with weight 1, summed into the same output as
   * its routed experts (y = sum_k w_k E_k(x) + S(x)).  The reference has no
   * shared expert (kernel.py:562 computes the routed sum only); callers that
   * run it separately add it afterwards.  Not combined with
   * gemm2_weights_bf16. */
  int64_t n_shared_experts;
} MoeFwdArgs;

/* Offsets (bytes from the workspace base) of the per-stage buffers a forward
 * leaves behind; tests read them to check each stage on its own.  npad is the
 * row capacity of the expert-contiguous (permuted) buffers. */
typedef struct MoeWorkspaceLayout {
  size_t total_bytes;
  int64_t npad;            /* rows of the permuted buffers (multiple of 128) */
  int64_t route_blocks;    /* blocks of the routing kernel */
  int64_t tokens_per_block;
  size_t ctrl;             /* control block: done counter, device error code */
  size_t topk_idx;         /* [T, top_k] int32   routed global expert ids, selection order */
  size_t topk_weights;     /* [T, top_k] fp32    routing weights */
  size_t block_base;       /* [route_blocks, E_local] int32 per-block bucket offsets */
  size_t counts;           /* [E_local + n_shared_experts] int32  rows per bucket (local
                              experts, then the shared expert's T) */
  size_t tile_start;       /* [E_local + n_shared_experts + 1] int32 prefix sum of 128-row tiles */
  size_t row_token;        /* [npad] int32       token of each permuted row */
  size_t row_weight;       /* [npad] fp32        routing weight of each permuted row */
  size_t a_perm;           /* [npad, H] e4m3     permuted hidden states */
  size_t a_scale_perm;     /* [H/128, npad] fp32 their scales */
  size_t inter;            /* [npad, I] e4m3     SwiGLU output, requantised */
  size_t inter_scale;      /* [I/64, npad] fp32  its per-64-column scales */
  size_t out_f32;          /* [T, H] fp32        scatter-add accumulator */
  size_t assign_row;       /* [T, top_k] int32   permuted row of each assignment (-1: not local) */
  size_t rows_out;         /* [npad, H] fp32     weighted GEMM2 rows (MOE_FLAG_DETERMINISTIC only) */
  size_t inter_bf16;       /* [npad, I] bf16     dequantised intermediate (gemm2_weights_bf16 only) */
} MoeWorkspaceLayout;

/* Workspace bytes needed for the shape in `a` (pointers are not read).
 * Replaces the torch allocations of kernel.py:629-630, 348, 358, 364-368,
 * 664-670 and 704. */
int moe_fp8_workspace_size(const MoeFwdArgs* a, size_t* bytes);

/* Byte offsets of the stage buffers inside the workspace. */
int moe_fp8_workspace_layout(const MoeFwdArgs* a, MoeWorkspaceLayout* out);

/* The whole layer: routing -> dispatch -> GEMM1+SwiGLU+requant -> GEMM2 with
 * weighted scatter-add -> bf16 output.  Replaces run() (kernel.py:562-729).
 * Only experts [local_expert_offset, local_expert_offset + E_local) contribute;
 * tokens routed elsewhere get zeros, as in the reference. */
int moe_fp8_forward(const MoeFwdArgs* a, void* stream);

/* moe_fp8_forward that also records CUDA events (cudaEvent_t handles, already
 * created) on `stream` at the stage boundaries, for per-kernel timing:
 *   events[0] start, [1] after routing (+ accumulator zeroing), [2] after the
 *   permute/pack, [3] after GEMM1, [4] after GEMM2, [5] after the bf16 cast.
 * For T <= 4 routing and packing are one kernel ([1] and [2] are recorded
 * together after it); for T <= 2 GEMM2 also writes the bf16 output ([4] and [5]
 * together).  Events between kernels can reduce the overlap that programmatic
 * dependent launch gives an unprofiled forward.
 * n_events must be 6.  No counterpart in the reference (profiling aid). */
#define MOE_PROFILE_EVENTS 6
int moe_fp8_forward_profiled(const MoeFwdArgs* a, void* stream, void* const* events,
                             int n_events);

/* Routing only: writes topk_idx / topk_weights (and the dispatch counters) in
 * the workspace.  Replaces moe_routing_kernel (kernel.py:428-542) plus the
 * counting pass of build_expert_dispatch (kernel.py:252-285, 327-361). */
int moe_fp8_route(const MoeFwdArgs* a, void* stream);

/* Device-side error word of the last forward on this workspace (0 = none).
 * Reads the control block with a blocking copy on `stream`. */
int moe_fp8_device_error(const MoeFwdArgs* a, void* stream, int32_t* code, int32_t* info);

/* What failed, in bits 24-31 of the info word of MOE_ERR_BOUNDS; bits 0-23
 * hold the index of the failing element (expert, assignment t*top_k+k, row or
 * guard number). */
#define MOE_CHECK_COUNTS 1       /* counts[e] outside [0, T] (the shared bucket's: not T) */
#define MOE_CHECK_TILE_START 2   /* tile_start not the 128-row prefix of counts, or past npad */
#define MOE_CHECK_TOPK_IDX 3     /* routed expert id outside [0, E_global) or repeated in a token */
#define MOE_CHECK_TOPK_WEIGHT 4  /* routing weight not finite */
#define MOE_CHECK_ROW_TOKEN 5    /* a live permuted row's token outside [0, T) */
#define MOE_CHECK_ROW_WEIGHT 6   /* a live row's weight differs from its assignment's */
#define MOE_CHECK_ROW_EXPERT 7   /* a live row's token was not routed to the row's expert
                                    (shared bucket: row i of the bucket is not token i) */
#define MOE_CHECK_ASSIGN_ROW 8   /* an assignment's row is not the live row holding it */
#define MOE_CHECK_GUARD 9        /* the guard after workspace buffer `index` was overwritten */

/* Checks the routing and dispatch tables that the last forward left in the
 * workspace, and, when a->flags has MOE_FLAG_DEBUG (the last forward wrote the
 * guards), the workspace guards.  Clears the control block's error word first;
 * the result is read with moe_fp8_device_error.  Reads the tables only with
 * indices it has checked, so it is safe on any workspace contents.  Asynchronous
 * on `stream`.  No counterpart in the reference (debugging aid). */
int moe_fp8_check_workspace(const MoeFwdArgs* a, void* stream);

/* Routing for callers that cannot allocate device memory.  No counterpart in
 * the reference.
 *
 * Some hosts must not allocate while this layer runs: an inference engine's
 * plugin callback where allocation is forbidden, a serving loop whose device
 * memory is owned by another pool, or a foreign-language caller with no device
 * allocator.  This entry point needs no workspace.  The caller passes the
 * router inputs (logits [T, E_global] fp32, bias [E_global]) and the outputs:
 * topk_idx [T, top_k] int32 and topk_weights [T, top_k] fp32 (as moe_fp8_route
 * writes them) and expert_counts [E_local] int32 (assignments per local
 * expert, the reference's token_counts, kernel.py:357).
 *
 * Scratch lives in a fixed device array inside the library (263,428 bytes) that
 * every GPU which loads the library keeps until the process exits.  Limits:
 * T <= 65536 (more tokens return MOE_ERR_TOO_LARGE); the router's shape rules
 * (E_global <= 256 among them) are those of moe_fp8_forward and a violation
 * returns MOE_ERR_SHAPE.  The first call on each device looks up that array's
 * device address (with the device current) and keeps it for the life of the
 * process; make this first call before any stream capture, and do not use the
 * library across cudaDeviceReset (the kept address, like the kernels' shared
 * memory settings, belongs to the context that reset destroys).  All calls
 * share the one array, so calls that overlap on the GPU (different streams,
 * or different host threads on the same device) race: order them on a
 * single stream. */
int moe_fp8_route_noalloc(const float* routing_logits, const void* routing_bias,
                          int32_t bias_dtype, int64_t T, int64_t E_global, int64_t n_group,
                          int64_t topk_group, int64_t top_k, int64_t E_local,
                          int64_t local_expert_offset, float routed_scaling_factor,
                          int32_t* topk_idx, float* topk_weights, int32_t* expert_counts,
                          void* stream);

/* One-time relayout of the down-projection weights for the bf16 GEMM2:
 * out[e, h, i] = bf16(float(W2[e, h, i]) * W2_scale[e, h/128, i/128]), the
 * reference's dequantised weight (kernel.py:224-234) rounded once to bf16.
 * w2 [E_local, H, I] e4m3, w2_scale [E_local, H/128, I/128] fp32, out
 * [E_local, H, I] bf16 (twice the bytes of w2).  Pass `out` as
 * MoeFwdArgs.gemm2_weights_bf16 to later forwards with the same weights.  No
 * counterpart in the reference (a one-time weight relayout).  Asynchronous
 * on `stream`, no allocation; H, I multiples of 128, pointers 16-byte aligned. */
int moe_fp8_prepare_gemm2_bf16(const void* w2, const float* w2_scale, int64_t E_local, int64_t H,
                               int64_t I, void* out, void* stream);

/* Router logits, the producer of routing_logits (DeepSeek-V3's gate):
 * logits[T, E] = x[T, H] . w_gate[E, H]^T with bf16 x and w_gate (row-major),
 * products exact in fp32 and fp32 accumulation, fp32 logits [T, E].  The
 * reference receives the logits as an input (kernel.py:562); this op is the
 * step before it (the router GEMM), with no counterpart there.
 * Batches of at most 128 tokens, and shapes with E not a multiple of 256 or H
 * not a multiple of 64, run on CUDA cores in a fixed summation order with every
 * addition rounded to nearest (no workspace needed: pass NULL, 0); larger
 * batches run on the tensor cores (tcgen05 kind::f16, whose fp32 accumulator
 * does not round each addition to nearest: about 1e-5 of the largest logit at
 * H=7168) and need moe_router_workspace_size bytes of workspace (256-byte
 * aligned).  Both paths give the same bits on every run.  H must be a multiple of 8; x, w_gate and logits 16-byte
 * aligned; T < 2^24, E <= 65536.  Asynchronous on `stream`, no allocation. */
int moe_router_workspace_size(int64_t T, int64_t H, int64_t E, size_t* bytes);
int moe_router_logits_bf16(const void* x, const void* w_gate, int64_t T, int64_t H, int64_t E,
                           float* logits, void* workspace, size_t workspace_bytes, void* stream);

/* bf16 -> FP8 e4m3 quantisation of activations with one fp32 scale per token
 * and 128 columns: x [T, H] bf16 (row-major) -> q [T, H] e4m3 and
 * scale [H/128, T] fp32, scale = max(amax * fp32(1/448), 1e-12),
 * q = e4m3_rne(x / scale) (saturating) -- the values torch produces for
 * max(amax / 448, 1e-12) and (x / scale).to(float8_e4m3fn).  Produces the forward's hidden_states / hidden_states_scale in the
 * layout run() asserts (reference kernel.py:603); the reference itself receives
 * them already quantised, so this replaces the quantisation step of its callers
 * (the FlashInfer-Bench workloads; the expert-parallel layer's bf16 inputs).
 * H must be a multiple of 128, x and q 16-byte aligned.  Asynchronous on
 * `stream`, no allocation. */
int moe_bf16_to_fp8_1x128(const void* x, int64_t T, int64_t H, void* q, float* scale,
                          void* stream);

/* ---------------------------------------------------------------------------
 * Expert-parallel layer with the token exchange done over NVLink peer memory.
 *
 * No counterpart function exists in the reference: its API expresses one shard
 * (local_expert_offset + a contiguous weight slice, kernel.py:572) and leaves
 * the exchange of tokens between shards to the caller.  One process per GPU;
 * rank r of `world` owns experts [r*E/world, (r+1)*E/world) and up to T_max
 * tokens.  Each rank's receive buffers are mapped into every peer with CUDA
 * IPC; the caller moves the 64-byte handles (moe_ep_ipc_handle, e.g. with an
 * all-gather of bytes) and passes all of them to moe_ep_connect.  Per forward,
 * in this order on one stream per rank, with the caller's collectives between:
 *   moe_ep_send_plan   route own tokens; send_cnt[world] = rows for each rank
 *   (all-gather send_cnt of every rank into cnt_all[world][world], source-major)
 *   moe_ep_dispatch    store FP8 rows, scales and logits into the owners' buffers
 *   (barrier across ranks)
 *   moe_ep_experts     local experts on the received rows; bf16 partials stored
 *                      back into the sources' buffers
 *   (barrier across ranks)
 *   moe_ep_finalize    sum of a token's partials in rank order -> bf16 output
 * The routing bias must be the same on every rank. */
typedef struct MoeEpConfig {
  int32_t world, rank;
  int64_t T_max;             /* most tokens any rank passes in one forward, < 2^24 */
  int64_t H, I, E_global, n_group, topk_group, top_k;
} MoeEpConfig;

typedef struct MoeEp MoeEp;

/* Allocates this rank's receive region (world*T_max rows) and workspaces on the
 * current device. */
int moe_ep_create(const MoeEpConfig* cfg, MoeEp** out);
/* 64-byte CUDA IPC handle of this rank's receive region. */
int moe_ep_ipc_handle(MoeEp* ep, void* handle_out);
/* all_handles: world consecutive 64-byte handles, rank order. */
int moe_ep_connect(MoeEp* ep, const void* all_handles);
int moe_ep_send_plan(MoeEp* ep, const float* routing_logits, const void* routing_bias,
                     int32_t bias_dtype, int64_t T, float routed_scaling_factor,
                     int32_t* send_cnt, void* stream);
/* hidden_states [T, H] e4m3, hidden_states_scale [H/128, T], routing_logits [T, E]. */
int moe_ep_dispatch(MoeEp* ep, const void* hidden_states, const float* hidden_states_scale,
                    const float* routing_logits, int64_t T, const int32_t* cnt_all,
                    void* stream);
/* Weights: this rank's contiguous expert slice, reference layouts. */
int moe_ep_experts(MoeEp* ep, const void* routing_bias, int32_t bias_dtype,
                   float routed_scaling_factor, const void* gemm1_weights,
                   const float* gemm1_weights_scale, const void* gemm2_weights,
                   const float* gemm2_weights_scale, const int32_t* cnt_all, void* stream);
/* output [T, H] bf16. */
int moe_ep_finalize(MoeEp* ep, int64_t T, void* output, void* stream);
/* First non-zero error word of the handle's kernels (blocks on `stream`). */
int moe_ep_device_error(MoeEp* ep, void* stream, int32_t* code, int32_t* info);
/* Unmaps peers and frees this rank's buffers (synchronises the device). */
int moe_ep_destroy(MoeEp* ep);

/* Human-readable name of a status code. */
const char* moe_fp8_status_string(int code);

/* Number of streaming multiprocessors the persistent kernels size their grid
 * to (queried once per device). */
int moe_fp8_num_sms(int device, int32_t* out);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H_ */
