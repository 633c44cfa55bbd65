// Router logits, the producer of the forward's routing_logits:
//   logits[T, E] = x[T, H] . w_gate[E, H]^T   (bf16 inputs, fp32 accumulate and output)
//
// DeepSeek-V3's gate multiplies the bf16 hidden state by a bf16 [E, H] weight
// and keeps the logits in fp32; the reference receives them as an input
// (run()'s routing_logits, kernel.py:562), so this op sits just before it.
//
//   moe_router_gemv_kernel   decode-sized batches and shapes the tensor-core
//                            path does not take: one block per (4 experts, 8
//                            tokens), its 8 warps over 8 slices of H, summed
//                            in a fixed order.
//   moe_router_setup_kernel  row tables of the tensor-core path, which runs the
//                            grouped bf16 GEMM (moe_gemm_kernel<kGemm2Bf16>) as
//                            one "expert" whose rows are the tokens in order,
//                            with weight 1 and a store epilogue into logits.
#include "moe_kernels.cuh"

namespace moe {

__global__ void __launch_bounds__(256)
    moe_router_gemv_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                           int T, int H, int E, float* __restrict__ out) {
  // Block = kRouterRows experts x kRouterGemvTokens tokens; warp q sums the
  // q-th of 8 slices of H, each lane 16-byte pieces of it, every x piece
  // loaded once for the block's experts.  Partial sums meet in a fixed order:
  // lane pieces in K order, a butterfly over the lanes, then the 8 slices.
  constexpr int kR = kRouterRows, kTok = kRouterGemvTokens, kWarps = 8;
  __shared__ float red[kWarps][kR * kTok];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row_groups = (E + kR - 1) / kR;
  const int e0 = (blockIdx.x % row_groups) * kR;
  const int t0 = (blockIdx.x / row_groups) * kTok;
  const int nt = min(kTok, T - t0), nr = min(kR, E - e0);
  const int pieces = H / 8;
  const int per_warp = (pieces + kWarps - 1) / kWarps;
  const int p_lo = warp * per_warp, p_hi = min(pieces, p_lo + per_warp);
  float acc[kR][kTok];
#pragma unroll
  for (int r = 0; r < kR; ++r)
#pragma unroll
    for (int i = 0; i < kTok; ++i) acc[r][i] = 0.f;
  for (int p = p_lo + lane; p < p_hi; p += 32) {
    uint4 wv[kR], xv[kTok];
#pragma unroll
    for (int r = 0; r < kR; ++r)
      wv[r] = r < nr ? __ldg(reinterpret_cast<const uint4*>(w + static_cast<int64_t>(e0 + r) * H) + p)
                     : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int i = 0; i < kTok; ++i)
      xv[i] = i < nt ? __ldg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t0 + i) * H) + p)
                     : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 wf[kR];
#pragma unroll
      for (int r = 0; r < kR; ++r)
        wf[r] = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(&wv[r])[j]);
#pragma unroll
      for (int i = 0; i < kTok; ++i) {
        const float2 xf = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(&xv[i])[j]);
#pragma unroll
        for (int r = 0; r < kR; ++r) {
          acc[r][i] = fmaf(xf.x, wf[r].x, acc[r][i]);
          acc[r][i] = fmaf(xf.y, wf[r].y, acc[r][i]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kR; ++r)
#pragma unroll
    for (int i = 0; i < kTok; ++i) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc[r][i] += __shfl_xor_sync(0xffffffffu, acc[r][i], off);
    }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < kR; ++r)
#pragma unroll
      for (int i = 0; i < kTok; ++i) red[warp][r * kTok + i] = acc[r][i];
  }
  __syncthreads();
  if (threadIdx.x < kR * kTok) {
    const int r = threadIdx.x / kTok, i = threadIdx.x % kTok;
    float v = red[0][threadIdx.x];
#pragma unroll
    for (int q = 1; q < kWarps; ++q) v += red[q][threadIdx.x];
    if (r < nr && i < nt) out[static_cast<int64_t>(t0 + i) * E + e0 + r] = v;
  }
}

int launch_router_gemv(const __nv_bfloat16* x, const __nv_bfloat16* w, int64_t T, int64_t H,
                       int64_t E, float* out, cudaStream_t s) {
  const int64_t blocks = (E + kRouterRows - 1) / kRouterRows *
                         ((T + kRouterGemvTokens - 1) / kRouterGemvTokens);
  if (blocks > 0x7fffffff) return MOE_ERR_SHAPE;
  moe_router_gemv_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(
      x, w, static_cast<int>(T), static_cast<int>(H), static_cast<int>(E), out);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

__global__ void moe_router_setup_kernel(int T, int npad, int* tile_start, int* counts,
                                        int* row_token, float* row_weight, CtrlBlock* ctrl) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < npad;
       r += stride) {
    row_token[r] = static_cast<int>(r);
    row_weight[r] = 1.f;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    tile_start[0] = 0;
    tile_start[1] = (T + kTileM - 1) / kTileM;
    counts[0] = T;
    ctrl->done = 0u;
    ctrl->error = 0;
    ctrl->error_info = 0;
    ctrl->gemm_done = 0u;
  }
}

}  // namespace moe
