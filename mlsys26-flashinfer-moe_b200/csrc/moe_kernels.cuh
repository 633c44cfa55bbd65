// Kernel parameter blocks and launch constants shared by the host glue
// (moe_api.cu) and the kernels (moe_route.cu, moe_gemm.cu).
#pragma once

#include "moe_common.cuh"

namespace moe {

constexpr int kMaxExperts = 256;       // E_global (and hence E_local) limit
// Dispatch buckets: the local routed experts plus at most one shared expert
// (MoeFwdArgs.n_shared_experts), which is bucket E_local.
constexpr int kMaxBuckets = kMaxExperts + 1;
constexpr int kMaxTopK = 8;
constexpr int kRouteThreads = 256;     // 8 warps, one token per warp at a time
constexpr int kMaxTokensPerBlock = 256;
// Batches routed and permuted by one block (moe_route_permute_tiny_kernel).  At
// 8 tokens that block's serial row copies took 31 us against 20 + 12 us for the
// routing kernel and the split permute.
constexpr int kTinyMaxTokens = 4;
constexpr int kFuseFinalMaxTokens = 2;   // decode GEMM2 also writes the bf16 output
constexpr int kTileM = 128;            // rows (assignments) per GEMM tile
constexpr int kTileN = 256;            // output columns per GEMM tile
constexpr int kBlockK = 128;           // K per pipeline stage = scale block
constexpr int kInterScaleBlock = 64;   // requant granularity of the intermediate (kernel.py:643)
constexpr int kStages = 4;             // smem pipeline depth
constexpr int kGemmThreads = 384;      // warpgroups 0-1: epilogue; 2: TMA warp, MMA warp, 2 idle
constexpr int kEpilogueRegs = 232;     // setmaxnreg split: 8*32*232 + 4*32*40 = 384*168
constexpr int kControlRegs = 40;
constexpr int kMmaIssuers = 2;        // warps 9 and 10, one per TMEM buffer
constexpr int kStageABytes = kTileM * kBlockK;     // 16 KB
constexpr int kStageBBytes = kTileN * kBlockK;     // 32 KB
constexpr int kStageBytes = kStageABytes + kStageBBytes;
// Per promotion warp, a 32-row x 64-byte staging tile that transposes the
// epilogue's row-per-lane results so that global writes go out row-contiguous.
constexpr int kXposeBytesPerWarp = 32 * 64;
constexpr int kXposeBytes = 8 * kXposeBytesPerWarp;
constexpr int kTmemCols = 512;         // two 256-column fp32 partial accumulators

struct RouteParams {
  const float* logits;
  const void* bias;
  int bias_dtype;
  int T, E, n_group, topk_group, top_k;
  int lanes_per_group, experts_per_lane;
  int E_local, local_expert_offset;
  float routed_scaling_factor;
  int tokens_per_block;
  int* topk_idx;
  float* topk_weights;
  int* block_base;   // [blocks, E_local]
  int* counts;       // [E_local]
  int* tile_start;   // [E_local + n_shared + 1]
  CtrlBlock* ctrl;
  const int* T_dev;  // when set, the number of rows is min(*T_dev, T) (expert-parallel receive side)
  int n_shared;      // 1: bucket E_local holds every token (counts[E_local] = T)
};

struct PermuteParams {
  int T, H, top_k, E_local, local_expert_offset, tokens_per_block;
  int64_t npad;
  const int* topk_idx;
  const float* topk_weights;
  const int* block_base;
  const int* tile_start;
  const uint8_t* hidden;
  const float* hs_scale;
  int64_t scale_ld;    // row stride of hs_scale [H/128, scale_ld] (T on the single-GPU path)
  int* row_token;
  float* row_weight;
  uint8_t* a_perm;
  float* a_scale_perm;
  const int* T_dev;    // as RouteParams::T_dev
  float* zero_rows;    // when set, rows t of this [T, H] fp32 buffer are zeroed for every token
  int* assign_row;     // when set, [T, top_k]: permuted row of every assignment, -1 if not local
  int n_shared;        // 1: token t also fills row 128 * tile_start[E_local] + t, weight 1
};

// One persistent grouped GEMM launch.  Work units are (expert tile, N tile)
// pairs, enumerated expert by expert with the N tile outer and the expert's
// 128-row tiles inner, so consecutive units share a weight tile in L2.
struct GemmParams {
  const int* tile_start;   // [E_local + 1] prefix sum of 128-row tiles
  const int* counts;       // [E_local] rows per expert
  int E_local;             // dispatch buckets: local experts (+ the shared expert), <= kMaxBuckets
  int num_k_blocks;        // K / 128
  int n_tiles;             // N tiles of 256 output columns
  int b_rows_per_expert;   // rows of one expert's weight matrix (2I or H)
  int inter;               // I
  int hidden;              // H
  int64_t npad;            // row capacity of the permuted buffers
  const float* a_scale;    // GEMM1: [H/128, npad]   GEMM2: [I/64, npad]
  const float* b_scale;    // GEMM1: [E, 2I/128, H/128]   GEMM2: [E, H/128, I/128]
  uint8_t* inter_out;      // GEMM1 output [npad, I] e4m3
  float* inter_scale;      // GEMM1 output [I/64, npad]
  const int* row_token;    // GEMM2: token of each permuted row
  const float* row_weight; // GEMM2: routing weight of each permuted row
  float* out_f32;          // GEMM2: [T, H] accumulator
  __nv_bfloat16* final_out;  // decode GEMM2 with few tokens: bf16 output written by the last CTA
  int64_t final_n8;        // T * H / 8
  float* rows_out;         // GEMM2, deterministic combine: [npad, H] weighted rows, stored
                           // instead of added into out_f32
  __nv_bfloat16* inter_bf16;  // GEMM1 with prepared bf16 W2: [npad, I] dequantised
                              // intermediate (bf16(code * scale)) instead of codes + scales
  unsigned int wait_limit_us;         // bound of the bounded waits (wait_limit_us())
  int stall;               // GEMM1, failure-detection tests: first MMA issuer waits forever
  int skip_on_error;       // MOE_FLAG_DEBUG: no units when the control block holds an error
  CtrlBlock* ctrl;
};

// Router logits (moe_router.cu).  Batches up to kRouterGemvMaxTokens tokens,
// and shapes outside the tensor-core path (E a multiple of 256, H of 64), take
// the CUDA-core kernel: a block per kRouterRows experts x kRouterGemvTokens
// tokens, each token row loaded once for the block's experts.  Above
// kRouterGemvMaxTokens the tensor-core path is faster (it streams the gate
// weight once per 128 tokens).  Measured alternatives (1 or 2 experts a block,
// 16 or 32 warps, unrolled loads) were no faster at T <= 8, where the launch
// dominates, and up to 3x slower at T = 64-256.
constexpr int kRouterRows = 4;
constexpr int kRouterGemvTokens = 8;
constexpr int64_t kRouterGemvMaxTokens = 128;
int launch_router_gemv(const __nv_bfloat16* x, const __nv_bfloat16* w, int64_t T, int64_t H,
                       int64_t E, float* out, cudaStream_t s);
__global__ void moe_router_setup_kernel(int T, int npad, int* tile_start, int* counts,
                                        int* row_token, float* row_weight, CtrlBlock* ctrl);

// Debug checks (moe_check.cu).  Guards are 16-byte patterns written after the
// workspace buffers; `guard` holds their byte offsets from `base`.
constexpr int kMaxGuards = 24;
constexpr int kGuardBytes = 16;
struct GuardList {
  uint8_t* base;
  int n;
  size_t off[kMaxGuards];
};

struct CheckParams {
  int T, top_k, E_global, E_local, local_expert_offset, n_shared;
  int64_t npad;
  const int* counts;
  const int* tile_start;
  const int* topk_idx;
  const float* topk_weights;
  const int* row_token;
  const float* row_weight;
  const int* assign_row;
  CtrlBlock* ctrl;
};

// MOE_CHECK_* checks of the routing and dispatch tables; reports the first
// failure as MOE_ERR_BOUNDS.
__global__ void moe_check_dispatch_kernel(CheckParams p);
// write != 0: stores the pattern into every guard; else reports the first
// guard that differs from it (MOE_CHECK_GUARD, index = guard number).
__global__ void moe_guard_kernel(GuardList g, int write, CtrlBlock* ctrl);

__global__ void moe_route_kernel(RouteParams p);
__global__ void moe_permute_kernel(PermuteParams p);
__global__ void moe_route_permute_tiny_kernel(RouteParams rp, PermuteParams pp, float* acc,
                                              int64_t acc_n4);
__global__ void moe_finalize_kernel(const float* __restrict__ in, __nv_bfloat16* __restrict__ out,
                                    int64_t n8);
// Deterministic combine: out[t] = bf16(sum over k of rows_out[assign_row[t, k]]),
// k in routing-selection order, then the shared expert's row 128 * *shared_tile
// + t when shared_tile is set.
__global__ void moe_combine_rows_kernel(const float* __restrict__ rows_out,
                                        const int* __restrict__ assign_row,
                                        __nv_bfloat16* __restrict__ out, int T, int H, int top_k,
                                        const int* __restrict__ shared_tile);

constexpr int kGemm1 = 0;   // gate/up GEMM, SwiGLU + 1x64 FP8 requant epilogue
constexpr int kGemm2 = 1;   // down GEMM, routing-weighted scatter-add epilogue
// down GEMM on bf16 operands (the dequantised intermediate and a prepared
// bf16(W2 * block scale)): no block scales left, so the tensor core accumulates
// all of K in TMEM and there is no promotion; same epilogue as kGemm2.
constexpr int kGemm2Bf16 = 2;

// Host-side launchers defined next to the kernel templates (moe_gemm.cu).
int gemm_set_smem_attrs();
int launch_gemm(int mode, const CUtensorMap& tm_a, const CUtensorMap& tm_b, const GemmParams& p,
                int grid, cudaStream_t stream);

// The forward takes the decode-shaped GEMMs when T * top_k <= this many rows
// per routed expert on average.
constexpr int64_t kSmallPathMaxAvgRows = 4;
// ... and when a unit's scale blocks (H/128, I/64) fit its shared-memory stage.
constexpr int64_t kSmallMaxScaleBlocks = 64;

// Decode-shaped variant with swapped operands (moe_gemm_small.cu): weight rows
// are the M=128 operand, 16 permuted token rows the N operand.  n_tiles counts
// 128-feature tiles for both GEMMs.
int gemm_small_set_smem_attrs();
int launch_gemm_small(int mode, const CUtensorMap& tm_w, const CUtensorMap& tm_tok,
                      const GemmParams& p, int grid, cudaStream_t stream);

// The layer forward of moe_api.cu with a device-resident row count (a->T is
// the capacity): route, permute (zeroing the fp32 accumulator rows), GEMM1,
// GEMM2 into the workspace's out_f32; no memset of the whole accumulator and no
// bf16 finalize.  Used by the expert-parallel receive side (moe_ep.cu).
int forward_device_rows(const MoeFwdArgs* a, const int* T_dev, cudaStream_t s);
int validate_shape_public(const MoeFwdArgs* a);
// Router + expert histogram only, into a->workspace (layout of a full forward).
int route_only(const MoeFwdArgs* a, cudaStream_t s);
// SM count of the current device (checks that it is an sm_100 part).
int num_sms(int* out);
MoeWorkspaceLayout workspace_layout_for(const MoeFwdArgs* a);

// bf16(W2 * block scale) for the bf16 GEMM2 (moe_quant.cu).
int launch_prepare_w2_bf16(const void* w2, const float* w2s, int64_t E, int64_t H, int64_t I,
                           void* out, int sms, cudaStream_t stream);

// bf16 -> e4m3 1x128 activation quantisation (moe_quant.cu).
int launch_quant_1x128(const void* x, int64_t T, int64_t H, void* q, float* scale, int sms,
                       cudaStream_t stream);

// Dynamic shared memory a CTA may opt into on sm_100 (227 KB).
constexpr int kMaxDynSmemBytes = 232448;

constexpr int gemm_smem_bytes() {
  return 1024 /*alignment slack*/ + kStages * kStageBytes + kXposeBytes +
         4096 /*barriers + tables*/;
}
static_assert(gemm_smem_bytes() <= kMaxDynSmemBytes, "GEMM stages exceed shared memory");
// Barriers (full and empty per stage, two tfull, two tempty, drain, never:
// 8 B each), TMEM slot and abort words (12 B) and the unit tables (tile_start,
// counts, skip flag) fit the 4096-byte area.
static_assert((2 * kStages + 6) * 8 + 12 + (2 * kMaxBuckets + 2) * 4 <= 4096,
              "GEMM tables exceed their area");

}  // namespace moe
