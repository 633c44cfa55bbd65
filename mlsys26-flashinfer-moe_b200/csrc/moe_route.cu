// Routing and dispatch for the fused FP8 MoE forward (sm_100a).
//
//   moe_route_kernel    DeepSeek-V3 no-aux group-limited top-k router, one warp
//                       per token, fused with the per-block expert histogram;
//                       the last block to finish turns the histograms into
//                       bucket offsets and the 128-row tile schedule.
//                       Replaces moe_routing_kernel (reference kernel.py:428-542),
//                       _count_kernel (252-285), the host sum/cumsum of
//                       build_expert_dispatch (356-361) and build_tile_schedule
//                       (384-407) -- without any device->host synchronisation.
//   moe_permute_kernel  Places every (token, local expert) assignment at its
//                       row of the expert-contiguous buffers, in token order
//                       inside each expert, and packs the token's FP8 row and
//                       scales there.  Replaces _scatter_kernel (288-324) and the
//                       index_select packing (663-665).
//   moe_route_permute_tiny_kernel  both of the above in one launch for decode-sized
//                       batches.
//   moe_finalize_kernel fp32 accumulator -> bf16 output (reference kernel.py:729).
#include "moe_kernels.cuh"

namespace moe {

namespace {

__device__ __forceinline__ float load_bias(const void* bias, int dtype, int i) {
  if (dtype == MOE_BIAS_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[i]);
  if (dtype == MOE_BIAS_F16) return __half2float(static_cast<const __half*>(bias)[i]);
  return static_cast<const float*>(bias)[i];
}

// Sigmoid evaluated in double and rounded once to float, so that the result is
// the correctly rounded float in all but astronomically rare cases and the
// routing decisions are reproducible on any host.
__device__ __forceinline__ float sigmoid_f32(float x) {
  return static_cast<float>(1.0 / (1.0 + exp(-static_cast<double>(x))));
}

// Unsigned key with the order of the float: flip all bits of negatives, the
// sign bit of the rest (-inf is the smallest key).
__device__ __forceinline__ unsigned ordered_key(float v) {
  const unsigned b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// One token on one warp.  Lane l holds experts [l*EPL, (l+1)*EPL); a group of
// G experts spans LPG = G/EPL consecutive lanes.
// Lane's logits of token t (zeros past E).
template <int EPL>
__device__ __forceinline__ void load_logits(const RouteParams& p, int t, int lane, float (&x)[EPL]) {
  const int e0 = lane * EPL;
  const float* row = p.logits + static_cast<int64_t>(t) * p.E;
#pragma unroll
  for (int j = 0; j < EPL; ++j) x[j] = e0 < p.E ? __ldg(row + e0 + j) : 0.f;
}

template <int EPL>
__device__ __forceinline__ void route_one_token(const RouteParams& p, int t, int lane,
                                                const float (&x)[EPL], const float (&bias)[EPL],
                                                int* hist_s, int* idx_s) {
  const unsigned full = 0xffffffffu;
  const int e0 = lane * EPL;
  const bool active = e0 < p.E;
  float s[EPL], sb[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    s[j] = sigmoid_f32(x[j]);
    const float v = s[j] + bias[j];
    // A NaN score (NaN logit or bias) ranks below every number, so the
    // comparisons below stay a total order.
    sb[j] = active && !isnan(v) ? v : -INFINITY;
  }
  // --- group score: sum of the two largest sb in the group (kernel.py:479-488)
  float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    if (sb[j] > m1) {
      m2 = m1;
      m1 = sb[j];
    } else if (sb[j] > m2) {
      m2 = sb[j];
    }
  }
  for (int off = 1; off < p.lanes_per_group; off <<= 1) {
    const float o1 = __shfl_xor_sync(full, m1, off);
    const float o2 = __shfl_xor_sync(full, m2, off);
    const float hi = fmaxf(m1, o1);
    m2 = fmaxf(fminf(m1, o1), fmaxf(m2, o2));
    m1 = hi;
  }
  const float gscore = m1 + m2;
  // --- keep the topk_group best groups, ties to the lowest group (495-501)
  const int my_group = lane / p.lanes_per_group;
  int better = 0;
  for (int g = 0; g < p.n_group; ++g) {
    const float o = __shfl_sync(full, gscore, g * p.lanes_per_group);
    better += (o > gscore) || (o == gscore && g < my_group);
  }
  const bool keep = active && better < p.topk_group;
  // --- top_k experts by sb, ties to the lowest expert id (522-534).  Each
  // round: the lane's best candidate not yet taken (first of equal values, so
  // its lowest expert), the warp maximum of an order-preserving integer key in
  // one redux, and the lowest lane holding it -- lane l owns experts
  // [l*EPL, (l+1)*EPL), so that lane's candidate is the lowest expert id
  // among the equal maxima, as in the reference's max-and-mask.  Taken
  // experts are tracked apart from their scores, so even -inf scores (from
  // -inf biases or NaN inputs) can never be picked twice: the kept groups hold
  // at least top_k experts, so every round finds an untaken one, and a token's
  // experts are always distinct (the permute relies on it).
  unsigned taken = keep ? 0u : (1u << EPL) - 1u;   // lanes of dropped groups offer none
  int my_idx = 0;
  float my_s = 0.f;
  for (int k = 0; k < p.top_k; ++k) {
    float bv = -INFINITY;
    int bj = -1;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      if (!((taken >> j) & 1u) && (bj < 0 || sb[j] > bv)) {
        bv = sb[j];
        bj = j;
      }
    }
    // ordered_key(-inf) = 0x007fffff, above the 0 of a lane with nothing left
    const unsigned key = bj < 0 ? 0u : ordered_key(bv);
    const unsigned kmax = __reduce_max_sync(full, key);
    const int src = __ffs(__ballot_sync(full, key == kmax)) - 1;
    bj = max(bj, 0);
    float sv = 0.f;
    if (lane == src) {
      taken |= 1u << bj;
#pragma unroll
      for (int j = 0; j < EPL; ++j)
        if (j == bj) sv = s[j];
    }
    const int bi = __shfl_sync(full, e0 + bj, src);
    sv = __shfl_sync(full, sv, src);
    if (lane == k) {
      my_idx = bi;
      my_s = sv;
    }
  }
  // --- renormalise by the unbiased scores (537-538)
  float acc = (lane < p.top_k) ? my_s : 0.f;
  float total;
  if ((p.top_k & (p.top_k - 1)) == 0) {
    for (int off = 1; off < p.top_k; off <<= 1) acc = acc + __shfl_down_sync(full, acc, off);
    total = __shfl_sync(full, acc, 0);
  } else {
    total = __shfl_sync(full, my_s, 0);
    for (int k = 1; k < p.top_k; ++k) total = total + __shfl_sync(full, my_s, k);
  }
  total = total + 1e-20f;
  if (lane < p.top_k) {
    const float w = __fdiv_rn(my_s, total) * p.routed_scaling_factor;
    p.topk_idx[static_cast<int64_t>(t) * p.top_k + lane] = my_idx;
    if (idx_s) idx_s[t * p.top_k + lane] = my_idx;
    p.topk_weights[static_cast<int64_t>(t) * p.top_k + lane] = w;
    const int le = my_idx - p.local_expert_offset;
    if (le >= 0 && le < p.E_local) atomicAdd(&hist_s[le], 1);
  }
}

template <int EPL>
// idx_s: optional copy of the routed expert ids in shared memory (one-block launches).
__device__ __forceinline__ void route_block_tokens(const RouteParams& p, int* hist_s,
                                                   int* idx_s = nullptr) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float bias[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = lane * EPL + j;
    bias[j] = e < p.E ? load_bias(p.bias, p.bias_dtype, e) : 0.f;
  }
  const int T = p.T_dev ? min(p.T, *p.T_dev) : p.T;
  const int t0 = blockIdx.x * p.tokens_per_block;
  const int t1 = min(T, t0 + p.tokens_per_block);
  // A warp's tokens are t0 + warp + 8i.  The next token's logits are
  // prefetched into L1 while the current one is routed, so only the first
  // token of a warp waits for DRAM.  (Loading several tokens into registers
  // and routing them from an unrolled loop was 1.6x slower: four copies of the
  // routing code, with its double-precision exp, per template instance.)
  constexpr int kWarps = kRouteThreads / 32;
  for (int t = t0 + warp; t < t1; t += kWarps) {
    float x[EPL];
    load_logits<EPL>(p, t, lane, x);
    if (t + kWarps < t1 && lane * EPL < p.E)
      asm volatile("prefetch.global.L1 [%0];" ::"l"(p.logits + static_cast<int64_t>(t + kWarps) * p.E + lane * EPL));
    route_one_token<EPL>(p, t, lane, x, bias, hist_s, idx_s);
  }
}

}  // namespace

__global__ void __launch_bounds__(kRouteThreads) moe_route_kernel(RouteParams p) {
  __shared__ int hist_s[kMaxExperts];
  __shared__ int warp_sum[kRouteThreads / 32];
  __shared__ int is_last;
  const int tid = threadIdx.x;
  griddep_launch_dependents();   // the permute kernel waits for this grid inside
  for (int i = tid; i < p.E_local; i += kRouteThreads) hist_s[i] = 0;
  __syncthreads();
  switch (p.experts_per_lane) {
    case 1: route_block_tokens<1>(p, hist_s); break;
    case 2: route_block_tokens<2>(p, hist_s); break;
    case 4: route_block_tokens<4>(p, hist_s); break;
    default: route_block_tokens<8>(p, hist_s); break;
  }
  __syncthreads();
  for (int i = tid; i < p.E_local; i += kRouteThreads)
    p.block_base[static_cast<int64_t>(blockIdx.x) * p.E_local + i] = hist_s[i];
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = (atomicAdd(&p.ctrl->done, 1u) == static_cast<unsigned>(gridDim.x - 1));
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // Last block: bucket base of every (block, expert) = that expert's count in
  // all earlier blocks (token order is block order), the per-expert counts,
  // then the prefix sum of 128-row tiles that places every expert's segment in
  // the permuted buffers.  Warp w takes the w-th chunk of blocks and lane l the
  // experts l, l+32, ...: a warp's loads of one block row are coalesced and a
  // thread's loads do not depend on each other, so the scan costs a few
  // round trips to L2 instead of one per block.
  __shared__ int chunk_sum[kRouteThreads / 32][kMaxExperts];
  constexpr int kWarps = kRouteThreads / 32;
  const int lane = tid & 31, warp = tid >> 5;
  const int nb = static_cast<int>(gridDim.x);
  const int per_chunk = (nb + kWarps - 1) / kWarps;
  const int b_lo = min(nb, warp * per_chunk), b_hi = min(nb, b_lo + per_chunk);
  for (int e = lane; e < p.E_local; e += 32) {
    int sum = 0;
#pragma unroll 8
    for (int b = b_lo; b < b_hi; ++b)
      sum += __ldcg(p.block_base + static_cast<int64_t>(b) * p.E_local + e);
    chunk_sum[warp][e] = sum;
  }
  __syncthreads();
  for (int e = lane; e < p.E_local; e += 32) {
    int base = 0;
    for (int w = 0; w < warp; ++w) base += chunk_sum[w][e];
    for (int b0 = b_lo; b0 < b_hi; b0 += 8) {
      int v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        v[i] = b0 + i < b_hi ? __ldcg(p.block_base + static_cast<int64_t>(b0 + i) * p.E_local + e) : 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (b0 + i < b_hi) {
          p.block_base[static_cast<int64_t>(b0 + i) * p.E_local + e] = base;
          base += v[i];
        }
      }
    }
  }
  int count = 0;
  if (tid < p.E_local) {
#pragma unroll
    for (int w = 0; w < kWarps; ++w) count += chunk_sum[w][tid];
    p.counts[tid] = count;
  }
  const int tiles = tid < p.E_local ? (count + kTileM - 1) / kTileM : 0;
  // block-wide exclusive scan of `tiles`
  int incl = tiles;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  if (lane == 31) warp_sum[warp] = incl;
  __syncthreads();
  int before = 0;
  for (int w = 0; w < warp; ++w) before += warp_sum[w];
  incl += before;
  if (tid < p.E_local) p.tile_start[tid] = incl - tiles;
  if (tid == kRouteThreads - 1) {
    p.tile_start[p.E_local] = incl;
    if (p.n_shared) {   // the shared expert's bucket: every token, in order
      const int T = p.T_dev ? min(p.T, *p.T_dev) : p.T;
      p.counts[p.E_local] = T;
      p.tile_start[p.E_local + 1] = incl + (T + kTileM - 1) / kTileM;
    }
  }
  if (tid == 0) p.ctrl->done = 0u;
}

namespace {

// Row of every assignment of tokens [t0, t1), tokens in order inside each
// expert (a token's experts are distinct, so the lanes of one token never touch
// the same cursor).  Warp 0 only; cursor[e] starts at the expert's first row;
// idx holds the routed expert ids [T, top_k] (global memory or a block's copy).
__device__ __forceinline__ void assign_rows(const PermuteParams& p, const int* idx, int* cursor,
                                            int* rows_s, int t0, int t1, int lane) {
  for (int t = t0; t < t1; ++t) {
    if (lane < p.top_k) {
      const int le = idx[static_cast<int64_t>(t) * p.top_k + lane] - p.local_expert_offset;
      int row = -1;
      if (le >= 0 && le < p.E_local) row = cursor[le]++;
      rows_s[(t - t0) * p.top_k + lane] = row;
    }
    __syncwarp();
  }
}

// Packs the rows of tokens [t0, t1) into the permuted buffers: token, weight
// and scales per assignment, then the FP8 rows.  All threads of the block;
// the assignments (and accumulator rows) are shared out over `nsub` blocks
// with the same tokens, this one being number `sub`.
__device__ __forceinline__ void pack_rows(const PermuteParams& p, const int* rows_s, int t0, int t1,
                                          int sub, int nsub) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_assign = (t1 - t0) * p.top_k;
  const int hb = p.H / kBlockK;
  // Scales: one thread per assignment, loads issued in batches of 8 before
  // their stores (restrict-qualified: the compiler may not otherwise overlap a
  // load with the previous store).
  const float* __restrict__ hs = p.hs_scale;
  float* __restrict__ asp = p.a_scale_perm;
  const int nwarps = blockDim.x >> 5;
  // Few assignments (decode batches): a warp per assignment instead, its lanes
  // over the (at most 64) scale blocks, so that a copy is one round trip.
  const bool few = n_assign <= 4 * nwarps * nsub && hb <= 64;
  for (int j = sub * nwarps + warp; few && j < n_assign; j += nwarps * nsub) {
    const int row = rows_s[j];
    if (row < 0) continue;
    const int t = t0 + j / p.top_k;
    if (lane == 0) {
      p.row_token[row] = t;
      p.row_weight[row] = p.topk_weights[static_cast<int64_t>(t) * p.top_k + j % p.top_k];
    }
    float v0 = 0.f, v1 = 0.f;
    if (lane < hb) v0 = __ldg(hs + static_cast<int64_t>(lane) * p.scale_ld + t);
    if (lane + 32 < hb) v1 = __ldg(hs + static_cast<int64_t>(lane + 32) * p.scale_ld + t);
    if (lane < hb) asp[static_cast<int64_t>(lane) * p.npad + row] = v0;
    if (lane + 32 < hb) asp[static_cast<int64_t>(lane + 32) * p.npad + row] = v1;
  }
  for (int j = sub * blockDim.x + tid; !few && j < n_assign; j += blockDim.x * nsub) {
    const int row = rows_s[j];
    if (row < 0) continue;
    const int t = t0 + j / p.top_k;
    p.row_token[row] = t;
    p.row_weight[row] = p.topk_weights[static_cast<int64_t>(t) * p.top_k + j % p.top_k];
    for (int kb0 = 0; kb0 < hb; kb0 += 8) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (kb0 + i < hb) v[i] = __ldg(hs + static_cast<int64_t>(kb0 + i) * p.scale_ld + t);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (kb0 + i < hb) asp[static_cast<int64_t>(kb0 + i) * p.npad + row] = v[i];
    }
  }
  if (p.assign_row) {
    for (int j = sub * blockDim.x + tid; j < n_assign; j += blockDim.x * nsub)
      p.assign_row[static_cast<int64_t>(t0) * p.top_k + j] = rows_s[j];
  }
  if (p.zero_rows) {
    const int64_t n4 = static_cast<int64_t>(t1 - t0) * p.H / 4;
    float4* z = reinterpret_cast<float4*>(p.zero_rows + static_cast<int64_t>(t0) * p.H);
    for (int64_t i = static_cast<int64_t>(sub) * blockDim.x + tid; i < n4;
         i += static_cast<int64_t>(blockDim.x) * nsub)
      z[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  // FP8 rows: one warp per assignment, 16-byte vectors, each lane's loads of a
  // row issued before its stores.
  const int vec = p.H / 16;
  const uint8_t* __restrict__ hid = p.hidden;
  uint8_t* __restrict__ ap = p.a_perm;
  for (int j = sub * nwarps + warp; j < n_assign; j += nwarps * nsub) {
    const int row = rows_s[j];
    if (row < 0) continue;
    const int t = t0 + j / p.top_k;
    const uint4* src = reinterpret_cast<const uint4*>(hid + static_cast<int64_t>(t) * p.H);
    uint4* dst = reinterpret_cast<uint4*>(ap + static_cast<int64_t>(row) * p.H);
    for (int c0 = 0; c0 < vec; c0 += 32 * 8) {
      uint4 v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = c0 + 32 * i + lane;
        if (c < vec) v[i] = __ldg(src + c);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = c0 + 32 * i + lane;
        if (c < vec) dst[c] = v[i];
      }
    }
  }
}

// Exclusive scan of the experts' 128-row tile counts (one thread per local
// expert, E_local <= kRouteThreads): writes tile_start[0..E_local] and returns
// this thread's start.
__device__ __forceinline__ int scan_tiles(int tiles, int* tile_start, int E_local, int* warp_sum,
                                          int shared_rows) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int incl = tiles;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  if (lane == 31) warp_sum[warp] = incl;
  __syncthreads();
  int before = 0;
  for (int w = 0; w < warp; ++w) before += warp_sum[w];
  incl += before;
  if (tid < E_local) tile_start[tid] = incl - tiles;
  if (tid == kRouteThreads - 1) {
    tile_start[E_local] = incl;
    if (shared_rows >= 0) tile_start[E_local + 1] = incl + (shared_rows + kTileM - 1) / kTileM;
  }
  return incl - tiles;
}

// Shared expert: token t of [t0, t1) fills row base + t with weight 1 (its
// token id, scales and FP8 row), shared out over `nsub` blocks as pack_rows.
__device__ __forceinline__ void pack_shared_rows(const PermuteParams& p, int64_t base, int t0, int t1,
                                                 int sub, int nsub) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = t1 - t0;
  const int nthreads = blockDim.x * nsub, first = sub * blockDim.x + tid;
  for (int j = first; j < n; j += nthreads) {
    p.row_token[base + t0 + j] = t0 + j;
    p.row_weight[base + t0 + j] = 1.f;
  }
  // scales [H/128, *]: consecutive threads take consecutive tokens of one block
  const int hb = p.H / kBlockK;
  const int64_t n_sc = static_cast<int64_t>(n) * hb;
  for (int64_t i = first; i < n_sc; i += nthreads) {
    const int kb = static_cast<int>(i / n), j = static_cast<int>(i - static_cast<int64_t>(kb) * n);
    p.a_scale_perm[static_cast<int64_t>(kb) * p.npad + base + t0 + j] =
        __ldg(p.hs_scale + static_cast<int64_t>(kb) * p.scale_ld + t0 + j);
  }
  const int vec = p.H / 16;
  const int nwarps = blockDim.x >> 5;
  for (int j = sub * nwarps + warp; j < n; j += nwarps * nsub) {
    const uint4* src = reinterpret_cast<const uint4*>(p.hidden + static_cast<int64_t>(t0 + j) * p.H);
    uint4* dst = reinterpret_cast<uint4*>(p.a_perm + (base + t0 + j) * p.H);
    for (int c0 = 0; c0 < vec; c0 += 32 * 8) {
      uint4 v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = c0 + 32 * i + lane;
        if (c < vec) v[i] = __ldg(src + c);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = c0 + 32 * i + lane;
        if (c < vec) dst[c] = v[i];
      }
    }
  }
}

}  // namespace

// Grid (route blocks, split): the blocks of one column share the tokens of
// route block x; each of them assigns all their rows (cheap, warp 0) and packs
// its share, so that small batches still have enough copies in flight.
__global__ void __launch_bounds__(kRouteThreads) moe_permute_kernel(PermuteParams p) {
  __shared__ int cursor[kMaxExperts];
  __shared__ int rows_s[kMaxTokensPerBlock * kMaxTopK];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.x;
  griddep_launch_dependents();
  griddep_wait();   // routing results of moe_route_kernel
  const int T = p.T_dev ? min(p.T, *p.T_dev) : p.T;
  const int t0 = b * p.tokens_per_block;
  const int t1 = min(T, t0 + p.tokens_per_block);
  for (int i = tid; i < p.E_local; i += kRouteThreads)
    cursor[i] = kTileM * p.tile_start[i] + p.block_base[static_cast<int64_t>(b) * p.E_local + i];
  __syncthreads();
  if (warp == 0) assign_rows(p, p.topk_idx, cursor, rows_s, t0, t1, lane);
  __syncthreads();
  pack_rows(p, rows_s, t0, t1, blockIdx.y, gridDim.y);
  if (p.n_shared)
    pack_shared_rows(p, static_cast<int64_t>(kTileM) * p.tile_start[p.E_local], t0, t1, blockIdx.y,
                     gridDim.y);
}

// Decode-sized batches (T <= kTinyMaxTokens, host row count): routing, the
// expert histogram, the tile schedule and the permute in block 0 of ONE launch
// (no per-block histograms, no second kernel, no memsets); blocks 1.. zero the
// fp32 accumulator meanwhile.  Results are those of moe_route_kernel followed
// by moe_permute_kernel.
__global__ void __launch_bounds__(kRouteThreads)
    moe_route_permute_tiny_kernel(RouteParams rp, PermuteParams pp, float* acc, int64_t acc_n4) {
  griddep_launch_dependents();   // GEMM1 waits for this grid inside
  if (blockIdx.x > 0) {
    float4* z = reinterpret_cast<float4*>(acc);
    const int64_t stride = static_cast<int64_t>(gridDim.x - 1) * kRouteThreads;
    for (int64_t i = static_cast<int64_t>(blockIdx.x - 1) * kRouteThreads + threadIdx.x; i < acc_n4;
         i += stride)
      z[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  __shared__ int hist_s[kMaxExperts];
  __shared__ int cursor[kMaxExperts];
  __shared__ int warp_sum[kRouteThreads / 32];
  __shared__ int rows_s[kTinyMaxTokens * kMaxTopK];
  __shared__ int idx_s[kTinyMaxTokens * kMaxTopK];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < rp.E_local; i += kRouteThreads) hist_s[i] = 0;
  if (tid == 0) {
    rp.ctrl->done = 0u;
    rp.ctrl->error = 0;
    rp.ctrl->error_info = 0;
    rp.ctrl->gemm_done = 0u;
  }
  __syncthreads();
  switch (rp.experts_per_lane) {
    case 1: route_block_tokens<1>(rp, hist_s, idx_s); break;
    case 2: route_block_tokens<2>(rp, hist_s, idx_s); break;
    case 4: route_block_tokens<4>(rp, hist_s, idx_s); break;
    default: route_block_tokens<8>(rp, hist_s, idx_s); break;
  }
  __syncthreads();
  const int count = tid < rp.E_local ? hist_s[tid] : 0;
  if (tid < rp.E_local) rp.counts[tid] = count;
  if (tid == 0 && rp.n_shared) rp.counts[rp.E_local] = rp.T;
  const int first = scan_tiles(tid < rp.E_local ? (count + kTileM - 1) / kTileM : 0, rp.tile_start,
                               rp.E_local, warp_sum, rp.n_shared ? rp.T : -1);
  if (tid < rp.E_local) cursor[tid] = kTileM * first;
  __syncthreads();   // also publishes tile_start[E_local] (written above) to the block
  if (warp == 0) assign_rows(pp, idx_s, cursor, rows_s, 0, rp.T, lane);
  __syncthreads();
  pack_rows(pp, rows_s, 0, rp.T, 0, 1);
  if (pp.n_shared)
    pack_shared_rows(pp, static_cast<int64_t>(kTileM) * rp.tile_start[rp.E_local], 0, rp.T, 0, 1);
}

__global__ void __launch_bounds__(256) moe_finalize_kernel(const float* __restrict__ in,
                                                           __nv_bfloat16* __restrict__ out,
                                                           int64_t n8) {
  griddep_wait();   // the accumulator is complete once GEMM2 has finished
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += stride) {
    const float4 a = __ldcs(reinterpret_cast<const float4*>(in) + 2 * i);
    const float4 b = __ldcs(reinterpret_cast<const float4*>(in) + 2 * i + 1);
    __nv_bfloat162 r[4];
    r[0] = __floats2bfloat162_rn(a.x, a.y);
    r[1] = __floats2bfloat162_rn(a.z, a.w);
    r[2] = __floats2bfloat162_rn(b.x, b.y);
    r[3] = __floats2bfloat162_rn(b.z, b.w);
    reinterpret_cast<uint4*>(out)[i] = *reinterpret_cast<uint4*>(r);
  }
}

__global__ void __launch_bounds__(256)
    moe_combine_rows_kernel(const float* __restrict__ rows_out, const int* __restrict__ assign_row,
                            __nv_bfloat16* __restrict__ out, int T, int H, int top_k,
                            const int* __restrict__ shared_tile) {
  griddep_wait();   // GEMM2's rows are complete
  const int64_t shared_base = shared_tile ? static_cast<int64_t>(kTileM) * *shared_tile : -1;
  const int n8 = H / 8;
  const int64_t total = static_cast<int64_t>(T) * n8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const int t = static_cast<int>(i / n8);
    const int c8 = static_cast<int>(i - static_cast<int64_t>(t) * n8);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < top_k; ++k) {   // routing-selection order, fixed
      const int r = __ldg(assign_row + static_cast<int64_t>(t) * top_k + k);
      if (r < 0) continue;
      const float4* src = reinterpret_cast<const float4*>(rows_out + static_cast<int64_t>(r) * H) + 2 * c8;
      const float4 a = __ldcs(src), b = __ldcs(src + 1);
      acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
      acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
    }
    if (shared_base >= 0) {   // the shared expert's row, last
      const float4* src = reinterpret_cast<const float4*>(rows_out + (shared_base + t) * H) + 2 * c8;
      const float4 a = __ldcs(src), b = __ldcs(src + 1);
      acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
      acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
    }
    __nv_bfloat162 r2[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) r2[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
    reinterpret_cast<uint4*>(out)[i] = *reinterpret_cast<uint4*>(r2);
  }
}

}  // namespace moe
