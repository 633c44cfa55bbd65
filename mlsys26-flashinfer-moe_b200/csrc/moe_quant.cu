// bf16 -> FP8 e4m3 activation quantisation with one fp32 scale per token and
// 128 columns: the producer of the forward's hidden_states / hidden_states_scale
// when a layer starts from bf16 activations (the expert-parallel layer does,
// before its FP8 dispatch).  The reference receives these two tensors already
// quantised; its workloads quantise with scale = max(amax / 448, 1e-12) and
// q = e4m3_rne(x / scale), which this kernel reproduces bit for bit: torch
// evaluates amax / 448 (a tensor by a host scalar) as amax * fp32(1/448), and
// x / scale (tensor by tensor) as an IEEE division, followed by a
// round-to-nearest-even conversion that never leaves the finite range here.
//
// One warp per (token, 128-column block): each lane loads 4 bf16 (8 bytes), the
// block amax is a 5-step shuffle reduction, each lane stores its 4 codes as one
// 32-bit word (128 contiguous bytes per warp) and lane 0 writes the scale into
// the transposed [H/128, T] scale matrix.  Memory-bound: 3 bytes per element
// plus 4 bytes per block.
#include "moe_kernels.cuh"

namespace moe {

namespace {

constexpr int kQuantThreads = 256;

__global__ void __launch_bounds__(kQuantThreads)
    moe_quant_1x128_kernel(const __nv_bfloat16* __restrict__ x, int64_t T, int64_t H,
                           uint8_t* __restrict__ q, float* __restrict__ scale) {
  const int lane = threadIdx.x & 31;
  const int64_t nblk = H / 128;
  const int64_t total = T * nblk;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kQuantThreads / 32);
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * (kQuantThreads / 32) + (threadIdx.x >> 5);
       w < total; w += warps) {
    const int64_t t = w / nblk;
    const int64_t b = w - t * nblk;
    const int64_t off = t * H + b * 128 + lane * 4;
    const uint2 raw = __ldcs(reinterpret_cast<const uint2*>(x + off));
    const __nv_bfloat162 p0 = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
    const __nv_bfloat162 p1 = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
    const float v[4] = {__low2float(p0), __high2float(p0), __low2float(p1), __high2float(p1)};
    float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s = fmaxf(m * (1.0f / 448.0f), 1e-12f);
    const uint32_t lo = pack_e4m3x2(__fdiv_rn(v[0], s), __fdiv_rn(v[1], s));
    const uint32_t hi = pack_e4m3x2(__fdiv_rn(v[2], s), __fdiv_rn(v[3], s));
    *reinterpret_cast<uint32_t*>(q + off) = lo | (hi << 16);
    if (lane == 0) scale[b * T + t] = s;
  }
}

}  // namespace

int launch_quant_1x128(const void* x, int64_t T, int64_t H, void* q, float* scale, int sms,
                       cudaStream_t stream) {
  const int64_t warps_needed = T * (H / 128);
  int64_t blocks = (warps_needed + kQuantThreads / 32 - 1) / (kQuantThreads / 32);
  if (blocks > static_cast<int64_t>(sms) * 16) blocks = static_cast<int64_t>(sms) * 16;
  if (blocks < 1) blocks = 1;
  moe_quant_1x128_kernel<<<static_cast<int>(blocks), kQuantThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), T, H, static_cast<uint8_t*>(q), scale);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

}  // namespace moe
