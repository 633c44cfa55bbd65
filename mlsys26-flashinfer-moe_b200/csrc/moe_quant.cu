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

// ---------------------------------------------------------------------------
// One-time relayout of the down-projection weights for the bf16 GEMM2:
// out[e, h, i] = bf16(float(W2[e, h, i]) * W2_scale[e, h/128, i/128]), i.e. the
// reference's dequantised weight (kernel.py:224-234 multiplies the FP8 dot by
// this block scale) rounded once to bf16.  Each thread converts 16 codes (one
// 16-byte load, two 16-byte stores); the 16 share one scale block because
// 16 divides 128.  Memory-bound: 3 bytes per element.
// ---------------------------------------------------------------------------

namespace {

__global__ void __launch_bounds__(256)
    moe_prepare_w2_bf16_kernel(const uint8_t* __restrict__ w, const float* __restrict__ s,
                               __nv_bfloat16* __restrict__ out, int64_t n16, int64_t H,
                               int64_t I) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t hi_blocks = H / 128, ii_blocks = I / 128;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < n16;
       c += stride) {
    const int64_t off = c * 16;
    const int64_t e = off / (H * I);
    const int64_t rem = off - e * H * I;
    const int64_t h = rem / I;
    const int64_t i = rem - h * I;
    const float sc = __ldg(s + (e * hi_blocks + h / 128) * ii_blocks + i / 128);
    const uint4 codes = __ldcs(reinterpret_cast<const uint4*>(w) + c);
    const uint32_t wd[4] = {codes.x, codes.y, codes.z, codes.w};
    uint32_t o[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const __nv_fp8x2_storage_t two =
            static_cast<__nv_fp8x2_storage_t>((wd[k] >> (16 * half)) & 0xffffu);
        const float2 f = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(two, __NV_E4M3)));
        const __nv_bfloat162 b = __floats2bfloat162_rn(f.x * sc, f.y * sc);
        o[2 * k + half] = *reinterpret_cast<const uint32_t*>(&b);
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(out + off);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

}  // namespace

int launch_prepare_w2_bf16(const void* w2, const float* w2s, int64_t E, int64_t H, int64_t I,
                           void* out, int sms, cudaStream_t stream) {
  const int64_t n16 = E * H * I / 16;
  int64_t blocks = (n16 + 255) / 256;
  if (blocks > static_cast<int64_t>(sms) * 8) blocks = static_cast<int64_t>(sms) * 8;
  if (blocks < 1) blocks = 1;
  moe_prepare_w2_bf16_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(
      static_cast<const uint8_t*>(w2), w2s, static_cast<__nv_bfloat16*>(out), n16, H, I);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

}  // namespace moe
