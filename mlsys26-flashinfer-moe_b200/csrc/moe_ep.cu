// Expert-parallel MoE layer whose token exchange is done by this library's own
// kernels over NVLink peer memory (one process per GPU, CUDA IPC mappings).
//
// Rank r of W owns experts [r*E/W, (r+1)*E/W) and T_r <= T_max tokens.  Every
// rank holds one "shared" region, mapped into every peer:
//   recv_x      [R_max, H]       e4m3   rows other ranks dispatched to this rank
//   recv_logits [R_max, E]       fp32   their router logits
//   recv_scale  [H/128, R_max]   fp32   their 1x128 scales (the layout run() takes)
//   recv_src    [R_max]          int32  (source rank << 24) | source token
//   comb        [W, T_max, H]    bf16   partial outputs of this rank's tokens, one
//                                        slab per destination rank
// with R_max = W * T_max (a token is sent at most once to each rank).
//
// One forward (the host issues the NCCL steps between the stages):
//   1. moe_ep_send_plan (source): route own tokens (all E experts), destination
//      mask per token, per-destination row counts -> send_cnt[W].
//      NCCL all-gather of send_cnt into cnt_all[W][W] (W*W ints, device side).
//   2. moe_ep_dispatch (source): each token goes once to every rank owning one of
//      its experts, at slot (sum of earlier ranks' counts to that destination) +
//      (its order among this rank's tokens for it).  The kernel stores the FP8 row,
//      scales, logits and token id straight into the destination's shared region
//      (NVLink stores; this replaces the reference's gather + the all-to-all).
//      NCCL barrier.
//   3. moe_ep_experts (destination): the received rows, compact in source order,
//      run through the single-GPU layer (route again -- routing is a pure function
//      of logits and bias, so it reproduces the source's choice -- permute,
//      GEMM1, GEMM2) with the row count read on the device; then each received
//      row's fp32 result is converted to bf16 and stored straight into its source
//      rank's comb slab (NVLink stores; this replaces the combine all-to-all).
//      NCCL barrier.
//   4. moe_ep_finalize (source): out[t] = sum over the destinations of t, in rank
//      order, of comb[d][t] (fp32), rounded to bf16 once.
// Every peer store is bounds-checked against the region sizes; a violation sets
// the handle's error word instead of writing.
#include "moe_kernels.cuh"

#include <cstring>
#include <new>

namespace moe {

constexpr int kEpMaxRanks = 8;
constexpr int kEpThreads = 256;

struct EpPeerPtrs {
  uint8_t* recv_x[kEpMaxRanks];
  float* recv_logits[kEpMaxRanks];
  float* recv_scale[kEpMaxRanks];
  int* recv_src[kEpMaxRanks];
  __nv_bfloat16* comb[kEpMaxRanks];
};

namespace {

struct SendPlanParams {
  int T, top_k, E_local, world, tokens_per_block;
  const int* topk_idx;        // [T, top_k]
  int* block_cnt;             // [blocks, world] -> per-block bases after the scan
  int* send_cnt;              // [world]
  CtrlBlock* ctrl;            // .done is the last-block counter
};

__device__ __forceinline__ uint32_t dest_mask(const int* idx, int top_k, int E_local) {
  uint32_t m = 0;
  for (int k = 0; k < top_k; ++k) m |= 1u << (idx[k] / E_local);
  return m;
}

__global__ void __launch_bounds__(kEpThreads) ep_send_plan_kernel(SendPlanParams p) {
  __shared__ int cnt_s[kEpMaxRanks];
  __shared__ int is_last;
  const int tid = threadIdx.x;
  if (tid < kEpMaxRanks) cnt_s[tid] = 0;
  __syncthreads();
  const int t0 = blockIdx.x * p.tokens_per_block;
  const int t1 = min(p.T, t0 + p.tokens_per_block);
  for (int t = t0 + tid; t < t1; t += kEpThreads) {
    const uint32_t m = dest_mask(p.topk_idx + static_cast<int64_t>(t) * p.top_k, p.top_k, p.E_local);
    for (int d = 0; d < p.world; ++d)
      if (m >> d & 1u) atomicAdd(&cnt_s[d], 1);
  }
  __syncthreads();
  if (tid < p.world) p.block_cnt[blockIdx.x * p.world + tid] = cnt_s[tid];
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(&p.ctrl->done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // Last block: warp d scans destination d over the blocks; lane l owns the
  // l-th chunk of blocks, so a lane's loads are independent of each other.
  const int warp = tid >> 5, lane = tid & 31;
  const int nb = static_cast<int>(gridDim.x);
  const int per_lane = (nb + 31) / 32;
  const int b_lo = min(nb, lane * per_lane), b_hi = min(nb, b_lo + per_lane);
  if (warp < p.world) {
    int sum = 0;
    for (int b = b_lo; b < b_hi; ++b) sum += __ldcg(p.block_cnt + b * p.world + warp);
    int incl = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    int run = incl - sum;
    for (int b0 = b_lo; b0 < b_hi; b0 += 8) {
      int v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = b0 + i < b_hi ? __ldcg(p.block_cnt + (b0 + i) * p.world + warp) : 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (b0 + i < b_hi) {
          p.block_cnt[(b0 + i) * p.world + warp] = run;
          run += v[i];
        }
      }
    }
    if (lane == 31) p.send_cnt[warp] = incl;
  }
  if (tid == 0) p.ctrl->done = 0u;
}

struct DispatchParams {
  int T, H, E, top_k, E_local, world, rank, tokens_per_block;
  int64_t R_max;
  const int* topk_idx;        // [T, top_k]
  const float* logits;        // [T, E]
  const uint8_t* hidden;      // [T, H]
  const float* hs_scale;      // [H/128, T]
  const int* block_cnt;       // per-block bases [blocks, world]
  const int* cnt_all;         // [world (source), world (destination)]
  EpPeerPtrs peers;
  CtrlBlock* ctrl;            // error word
};

__global__ void __launch_bounds__(kEpThreads) ep_dispatch_kernel(DispatchParams p) {
  __shared__ int cursor[kEpMaxRanks];
  __shared__ int pair_t[kMaxTokensPerBlock * kEpMaxRanks];
  __shared__ int pair_slot[kMaxTokensPerBlock * kEpMaxRanks];
  __shared__ unsigned char pair_d[kMaxTokensPerBlock * kEpMaxRanks];
  __shared__ int n_pairs;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = blockIdx.x * p.tokens_per_block;
  const int t1 = min(p.T, t0 + p.tokens_per_block);
  if (tid < p.world) {
    int off = 0;
    for (int s = 0; s < p.rank; ++s) off += p.cnt_all[s * p.world + tid];
    cursor[tid] = off + p.block_cnt[blockIdx.x * p.world + tid];
  }
  __syncthreads();
  if (tid == 0) {
    // Slots in token order: the destination's rows stay in (source, token) order.
    int n = 0;
    for (int t = t0; t < t1; ++t) {
      const uint32_t m = dest_mask(p.topk_idx + static_cast<int64_t>(t) * p.top_k, p.top_k, p.E_local);
      for (int d = 0; d < p.world; ++d) {
        if (m >> d & 1u) {
          pair_t[n] = t;
          pair_d[n] = static_cast<unsigned char>(d);
          pair_slot[n] = cursor[d]++;
          ++n;
        }
      }
    }
    n_pairs = n;
  }
  __syncthreads();
  const int hb = p.H / kBlockK;
  const int vec = p.H / 16;
  const int lvec = p.E / 4;
  for (int j = warp; j < n_pairs; j += kEpThreads / 32) {
    const int t = pair_t[j], d = pair_d[j];
    const int64_t slot = pair_slot[j];
    if (slot < 0 || slot >= p.R_max) {
      if (lane == 0) report_error(p.ctrl, MOE_ERR_INVALID_ARG, 1000 + d);
      continue;
    }
    const uint4* __restrict__ src =
        reinterpret_cast<const uint4*>(p.hidden + static_cast<int64_t>(t) * p.H);
    uint4* __restrict__ dst = reinterpret_cast<uint4*>(p.peers.recv_x[d] + slot * p.H);
    // loads of a row batched ahead of their stores
    for (int c0 = 0; c0 < vec; c0 += 32 * 8) {
      uint4 v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (c0 + 32 * i + lane < vec) v[i] = __ldg(src + c0 + 32 * i + lane);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (c0 + 32 * i + lane < vec) dst[c0 + 32 * i + lane] = v[i];
    }
    const float4* ls = reinterpret_cast<const float4*>(p.logits + static_cast<int64_t>(t) * p.E);
    float4* ld = reinterpret_cast<float4*>(p.peers.recv_logits[d] + slot * p.E);
    for (int c = lane; c < lvec; c += 32) ld[c] = __ldg(ls + c);
    for (int kb = lane; kb < hb; kb += 32)
      p.peers.recv_scale[d][static_cast<int64_t>(kb) * p.R_max + slot] =
          __ldg(p.hs_scale + static_cast<int64_t>(kb) * p.T + t);
    if (lane == 0) p.peers.recv_src[d][slot] = (p.rank << 24) | t;
  }
  __threadfence_system();
}

__global__ void ep_recv_count_kernel(const int* cnt_all, int world, int rank, int* n_recv) {
  if (threadIdx.x == 0) {
    int n = 0;
    for (int s = 0; s < world; ++s) n += cnt_all[s * world + rank];
    *n_recv = n;
  }
}

struct CombineParams {
  int H, world, rank, T_max;
  int64_t R_max;
  const int* n_recv;
  const int* recv_src;        // local
  const float* out_f32;       // [R_max, H] local
  EpPeerPtrs peers;
  CtrlBlock* ctrl;
};

// Received row r -> bf16 -> the source rank's comb[rank][token] (NVLink stores).
__global__ void __launch_bounds__(kEpThreads) ep_combine_kernel(CombineParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = min(static_cast<int64_t>(*p.n_recv), p.R_max);
  const int v8 = p.H / 8;
  for (int r = blockIdx.x * (kEpThreads / 32) + warp; r < n; r += gridDim.x * (kEpThreads / 32)) {
    const int code = p.recv_src[r];
    const int s = code >> 24, t = code & 0xffffff;
    if (s < 0 || s >= p.world || t >= p.T_max) {
      if (lane == 0) report_error(p.ctrl, MOE_ERR_INVALID_ARG, 2000 + s);
      continue;
    }
    const float4* __restrict__ src =
        reinterpret_cast<const float4*>(p.out_f32 + static_cast<int64_t>(r) * p.H);
    uint4* __restrict__ dst = reinterpret_cast<uint4*>(
        p.peers.comb[s] + (static_cast<int64_t>(p.rank) * p.T_max + t) * p.H);
    for (int c0 = 0; c0 < v8; c0 += 32 * 4) {
      float4 a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = c0 + 32 * i + lane;
        if (c < v8) {
          a[i] = __ldcs(src + 2 * c);
          b[i] = __ldcs(src + 2 * c + 1);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = c0 + 32 * i + lane;
        if (c < v8) {
          __nv_bfloat162 h[4] = {__floats2bfloat162_rn(a[i].x, a[i].y),
                                 __floats2bfloat162_rn(a[i].z, a[i].w),
                                 __floats2bfloat162_rn(b[i].x, b[i].y),
                                 __floats2bfloat162_rn(b[i].z, b[i].w)};
          dst[c] = *reinterpret_cast<uint4*>(h);
        }
      }
    }
  }
  __threadfence_system();
}

// out[t] = bf16( sum over destinations d of t, in rank order, of comb[d][t] ).
__global__ void __launch_bounds__(kEpThreads)
    ep_finalize_kernel(int T, int H, int top_k, int E_local, int world, int T_max,
                       const int* topk_idx, const __nv_bfloat16* comb, __nv_bfloat16* out) {
  const int v8 = H / 8;
  const int64_t total = static_cast<int64_t>(T) * v8;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kEpThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kEpThreads) {
    const int t = static_cast<int>(i / v8), c = static_cast<int>(i - static_cast<int64_t>(t) * v8);
    const uint32_t m = dest_mask(topk_idx + static_cast<int64_t>(t) * top_k, top_k, E_local);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int d = 0; d < world; ++d) {
      if (!(m >> d & 1u)) continue;
      const uint4 raw = __ldcs(reinterpret_cast<const uint4*>(
                                   comb + (static_cast<int64_t>(d) * T_max + t) * H) + c);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] += __low2float(h[j]);
        acc[2 * j + 1] += __high2float(h[j]);
      }
    }
    __nv_bfloat162 r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) r[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
    reinterpret_cast<uint4*>(out)[i] = *reinterpret_cast<uint4*>(r);
  }
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

}  // namespace
}  // namespace moe

using namespace moe;

struct MoeEp {
  MoeEpConfig cfg;
  int device;
  int64_t E_local, R_max;
  // shared region (exported over CUDA IPC) and its layout
  void* shared = nullptr;
  size_t shared_bytes = 0;
  size_t off_x, off_logits, off_scale, off_src, off_comb;
  void* peer_base[kEpMaxRanks] = {};
  bool peer_opened[kEpMaxRanks] = {};
  bool connected = false;
  // local memory: send-side routing workspace and receive-side layer workspace
  void* local = nullptr;
  size_t local_bytes = 0;
  MoeWorkspaceLayout send_w;   // layout of the send-side routing workspace (T = T_max, all experts)
  size_t off_send_ws, off_block_cnt, off_n_recv, off_recv_ws, off_ctrl;
  int send_blocks, send_tpb;
  MoeWorkspaceLayout recv_w;
};

namespace {

MoeFwdArgs recv_args(const MoeEp* ep) {
  MoeFwdArgs a{};
  a.T = ep->R_max;
  a.H = ep->cfg.H;
  a.I = ep->cfg.I;
  a.E_global = ep->cfg.E_global;
  a.E_local = ep->E_local;
  a.local_expert_offset = ep->cfg.rank * ep->E_local;
  a.n_group = ep->cfg.n_group;
  a.topk_group = ep->cfg.topk_group;
  a.top_k = ep->cfg.top_k;
  return a;
}

MoeFwdArgs send_args(const MoeEp* ep, int64_t T) {
  MoeFwdArgs a{};
  a.T = T;
  a.H = ep->cfg.H;
  a.I = ep->cfg.I;
  a.E_global = ep->cfg.E_global;
  a.E_local = ep->cfg.E_global;      // route over all experts, histogram unused
  a.local_expert_offset = 0;
  a.n_group = ep->cfg.n_group;
  a.topk_group = ep->cfg.topk_group;
  a.top_k = ep->cfg.top_k;
  return a;
}

EpPeerPtrs peer_ptrs(const MoeEp* ep) {
  EpPeerPtrs pp{};
  for (int r = 0; r < ep->cfg.world; ++r) {
    uint8_t* b = static_cast<uint8_t*>(ep->peer_base[r]);
    pp.recv_x[r] = b + ep->off_x;
    pp.recv_logits[r] = reinterpret_cast<float*>(b + ep->off_logits);
    pp.recv_scale[r] = reinterpret_cast<float*>(b + ep->off_scale);
    pp.recv_src[r] = reinterpret_cast<int*>(b + ep->off_src);
    pp.comb[r] = reinterpret_cast<__nv_bfloat16*>(b + ep->off_comb);
  }
  return pp;
}

template <typename T>
T* at(void* base, size_t off) {
  return reinterpret_cast<T*>(static_cast<uint8_t*>(base) + off);
}

int set_device(const MoeEp* ep) {
  return cudaSetDevice(ep->device) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

}  // namespace

extern "C" {

int moe_ep_create(const MoeEpConfig* cfg, MoeEp** out) {
  if (!cfg || !out) return MOE_ERR_INVALID_ARG;
  *out = nullptr;
  const MoeEpConfig& c = *cfg;
  if (c.world < 1 || c.world > kEpMaxRanks || c.rank < 0 || c.rank >= c.world) return MOE_ERR_SHAPE;
  if (c.T_max < 1 || c.T_max >= (1 << 24) || c.E_global % c.world != 0) return MOE_ERR_SHAPE;
  MoeEp* ep = new (std::nothrow) MoeEp();
  if (!ep) return MOE_ERR_CUDA;
  ep->cfg = c;
  ep->E_local = c.E_global / c.world;
  ep->R_max = static_cast<int64_t>(c.world) * c.T_max;
  if (cudaGetDevice(&ep->device) != cudaSuccess) {
    delete ep;
    return MOE_ERR_CUDA;
  }
  // shapes are checked by the single-GPU validator on the receive-side args
  const MoeFwdArgs ra = recv_args(ep);
  if (int st = validate_shape_public(&ra)) {
    delete ep;
    return st;
  }
  const int64_t H = c.H, E = c.E_global, R = ep->R_max;
  size_t off = 0;
  ep->off_x = off; off = align256(off + static_cast<size_t>(R) * H);
  ep->off_logits = off; off = align256(off + sizeof(float) * R * E);
  ep->off_scale = off; off = align256(off + sizeof(float) * (H / kBlockK) * R);
  ep->off_src = off; off = align256(off + sizeof(int) * R);
  ep->off_comb = off; off = align256(off + sizeof(__nv_bfloat16) * c.world * c.T_max * H);
  ep->shared_bytes = off;
  // local: send-side routing workspace, per-block destination counts, n_recv,
  // control block, receive-side layer workspace
  const MoeFwdArgs sa = send_args(ep, c.T_max);
  ep->send_w = workspace_layout_for(&sa);
  ep->send_tpb = static_cast<int>(ep->send_w.tokens_per_block);
  ep->send_blocks = static_cast<int>(ep->send_w.route_blocks);
  ep->recv_w = workspace_layout_for(&ra);
  size_t lo = 0;
  ep->off_send_ws = lo; lo = align256(lo + ep->send_w.total_bytes);
  ep->off_block_cnt = lo; lo = align256(lo + sizeof(int) * (ep->send_blocks + 1) * kEpMaxRanks);
  ep->off_n_recv = lo; lo = align256(lo + sizeof(int));
  ep->off_ctrl = lo; lo = align256(lo + sizeof(CtrlBlock));
  ep->off_recv_ws = lo; lo = align256(lo + ep->recv_w.total_bytes);
  ep->local_bytes = lo;
  if (cudaMalloc(&ep->shared, ep->shared_bytes) != cudaSuccess) {
    delete ep;
    return MOE_ERR_CUDA;
  }
  if (cudaMalloc(&ep->local, ep->local_bytes) != cudaSuccess) {
    cudaFree(ep->shared);
    delete ep;
    return MOE_ERR_CUDA;
  }
  if (cudaMemset(ep->shared, 0, ep->shared_bytes) != cudaSuccess ||
      cudaMemset(ep->local, 0, ep->local_bytes) != cudaSuccess) {
    cudaFree(ep->shared);
    cudaFree(ep->local);
    delete ep;
    return MOE_ERR_CUDA;
  }
  ep->peer_base[c.rank] = ep->shared;
  *out = ep;
  return MOE_OK;
}

int moe_ep_ipc_handle(MoeEp* ep, void* handle_out) {
  if (!ep || !handle_out) return MOE_ERR_INVALID_ARG;
  if (set_device(ep)) return MOE_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ep->shared) != cudaSuccess) return MOE_ERR_CUDA;
  std::memcpy(handle_out, &h, sizeof(h));
  return MOE_OK;
}

int moe_ep_connect(MoeEp* ep, const void* all_handles) {
  if (!ep || !all_handles) return MOE_ERR_INVALID_ARG;
  if (set_device(ep)) return MOE_ERR_CUDA;
  const int world = ep->cfg.world;
  for (int r = 0; r < world; ++r) {
    if (r == ep->cfg.rank || ep->peer_opened[r]) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const uint8_t*>(all_handles) + r * sizeof(h), sizeof(h));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
      return MOE_ERR_CUDA;
    ep->peer_base[r] = p;
    ep->peer_opened[r] = true;
  }
  ep->connected = true;
  return MOE_OK;
}

int moe_ep_send_plan(MoeEp* ep, const float* logits, const void* bias, int32_t bias_dtype,
                     int64_t T, float routed_scaling_factor, int32_t* send_cnt, void* stream) {
  if (!ep || !send_cnt) return MOE_ERR_INVALID_ARG;
  if (T < 0 || T > ep->cfg.T_max) return MOE_ERR_SHAPE;
  if (T > 0 && (!logits || !bias)) return MOE_ERR_INVALID_ARG;
  if (set_device(ep)) return MOE_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(send_cnt, 0, sizeof(int) * ep->cfg.world, s) != cudaSuccess) return MOE_ERR_CUDA;
  if (T == 0) return MOE_OK;
  MoeFwdArgs sa = send_args(ep, T);
  sa.routing_logits = logits;
  sa.routing_bias = bias;
  sa.bias_dtype = bias_dtype;
  sa.routed_scaling_factor = routed_scaling_factor;
  sa.workspace = at<uint8_t>(ep->local, ep->off_send_ws);
  sa.workspace_bytes = ep->send_w.total_bytes;
  int st = route_only(&sa, s);
  if (st) return st;
  const MoeWorkspaceLayout w = workspace_layout_for(&sa);
  SendPlanParams p{};
  p.T = static_cast<int>(T);
  p.top_k = static_cast<int>(ep->cfg.top_k);
  p.E_local = static_cast<int>(ep->E_local);
  p.world = ep->cfg.world;
  p.tokens_per_block = static_cast<int>(w.tokens_per_block);
  p.topk_idx = at<int>(sa.workspace, w.topk_idx);
  p.block_cnt = at<int>(ep->local, ep->off_block_cnt);
  p.send_cnt = send_cnt;
  p.ctrl = at<CtrlBlock>(ep->local, ep->off_ctrl);
  ep_send_plan_kernel<<<static_cast<int>(w.route_blocks), kEpThreads, 0, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

int moe_ep_dispatch(MoeEp* ep, const void* hidden_states, const float* hidden_states_scale,
                    const float* logits, int64_t T, const int32_t* cnt_all, void* stream) {
  if (!ep || !cnt_all || !ep->connected) return MOE_ERR_INVALID_ARG;
  if (T < 0 || T > ep->cfg.T_max) return MOE_ERR_SHAPE;
  if (T == 0) return MOE_OK;
  if (!hidden_states || !hidden_states_scale || !logits) return MOE_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(hidden_states) & 15u) != 0 ||
      (reinterpret_cast<uintptr_t>(logits) & 15u) != 0)
    return MOE_ERR_ALIGNMENT;
  if (set_device(ep)) return MOE_ERR_CUDA;
  MoeFwdArgs sa = send_args(ep, T);
  sa.workspace = at<uint8_t>(ep->local, ep->off_send_ws);
  const MoeWorkspaceLayout w = workspace_layout_for(&sa);
  DispatchParams p{};
  p.T = static_cast<int>(T);
  p.H = static_cast<int>(ep->cfg.H);
  p.E = static_cast<int>(ep->cfg.E_global);
  p.top_k = static_cast<int>(ep->cfg.top_k);
  p.E_local = static_cast<int>(ep->E_local);
  p.world = ep->cfg.world;
  p.rank = ep->cfg.rank;
  p.tokens_per_block = static_cast<int>(w.tokens_per_block);
  p.R_max = ep->R_max;
  p.topk_idx = at<int>(sa.workspace, w.topk_idx);
  p.logits = logits;
  p.hidden = static_cast<const uint8_t*>(hidden_states);
  p.hs_scale = hidden_states_scale;
  p.block_cnt = at<int>(ep->local, ep->off_block_cnt);
  p.cnt_all = cnt_all;
  p.peers = peer_ptrs(ep);
  p.ctrl = at<CtrlBlock>(ep->local, ep->off_ctrl);
  ep_dispatch_kernel<<<static_cast<int>(w.route_blocks), kEpThreads, 0,
                       static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

int moe_ep_experts(MoeEp* ep, const void* routing_bias, int32_t bias_dtype,
                   float routed_scaling_factor, const void* gemm1_weights,
                   const float* gemm1_weights_scale, const void* gemm2_weights,
                   const float* gemm2_weights_scale, const int32_t* cnt_all, void* stream) {
  if (!ep || !cnt_all || !ep->connected || !routing_bias || !gemm1_weights || !gemm2_weights ||
      !gemm1_weights_scale || !gemm2_weights_scale)
    return MOE_ERR_INVALID_ARG;
  if (set_device(ep)) return MOE_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* n_recv = at<int>(ep->local, ep->off_n_recv);
  ep_recv_count_kernel<<<1, 32, 0, s>>>(cnt_all, ep->cfg.world, ep->cfg.rank, n_recv);
  if (cudaGetLastError() != cudaSuccess) return MOE_ERR_CUDA;
  MoeFwdArgs ra = recv_args(ep);
  ra.routing_logits = at<float>(ep->shared, ep->off_logits);
  ra.routing_bias = routing_bias;
  ra.bias_dtype = bias_dtype;
  ra.hidden_states = at<uint8_t>(ep->shared, ep->off_x);
  ra.hidden_states_scale = at<float>(ep->shared, ep->off_scale);
  ra.gemm1_weights = gemm1_weights;
  ra.gemm1_weights_scale = gemm1_weights_scale;
  ra.gemm2_weights = gemm2_weights;
  ra.gemm2_weights_scale = gemm2_weights_scale;
  ra.routed_scaling_factor = routed_scaling_factor;
  ra.workspace = at<uint8_t>(ep->local, ep->off_recv_ws);
  ra.workspace_bytes = ep->recv_w.total_bytes;
  int st = forward_device_rows(&ra, n_recv, s);
  if (st) return st;
  CombineParams cp{};
  cp.H = static_cast<int>(ep->cfg.H);
  cp.world = ep->cfg.world;
  cp.rank = ep->cfg.rank;
  cp.T_max = static_cast<int>(ep->cfg.T_max);
  cp.R_max = ep->R_max;
  cp.n_recv = n_recv;
  cp.recv_src = at<int>(ep->shared, ep->off_src);
  cp.out_f32 = at<float>(ra.workspace, ep->recv_w.out_f32);
  cp.peers = peer_ptrs(ep);
  cp.ctrl = at<CtrlBlock>(ep->local, ep->off_ctrl);
  int sms = 148;
  if ((st = num_sms(&sms))) return st;
  ep_combine_kernel<<<sms * 4, kEpThreads, 0, s>>>(cp);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

int moe_ep_finalize(MoeEp* ep, int64_t T, void* output, void* stream) {
  if (!ep) return MOE_ERR_INVALID_ARG;
  if (T < 0 || T > ep->cfg.T_max) return MOE_ERR_SHAPE;
  if (T == 0) return MOE_OK;
  if (!output || (reinterpret_cast<uintptr_t>(output) & 15u) != 0) return MOE_ERR_ALIGNMENT;
  if (set_device(ep)) return MOE_ERR_CUDA;
  MoeFwdArgs sa = send_args(ep, T);
  const MoeWorkspaceLayout w = workspace_layout_for(&sa);
  int sms = 148;
  if (int st = num_sms(&sms)) return st;
  ep_finalize_kernel<<<sms * 4, kEpThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<int>(T), static_cast<int>(ep->cfg.H), static_cast<int>(ep->cfg.top_k),
      static_cast<int>(ep->E_local), ep->cfg.world, static_cast<int>(ep->cfg.T_max),
      at<int>(at<uint8_t>(ep->local, ep->off_send_ws), w.topk_idx),
      at<__nv_bfloat16>(ep->shared, ep->off_comb), static_cast<__nv_bfloat16*>(output));
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

int moe_ep_device_error(MoeEp* ep, void* stream, int32_t* code, int32_t* info) {
  if (!ep || !code || !info) return MOE_ERR_INVALID_ARG;
  if (set_device(ep)) return MOE_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CtrlBlock c[2];
  if (cudaMemcpyAsync(&c[0], at<CtrlBlock>(ep->local, ep->off_ctrl), sizeof(CtrlBlock),
                      cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaMemcpyAsync(&c[1],
                      at<CtrlBlock>(at<uint8_t>(ep->local, ep->off_recv_ws), ep->recv_w.ctrl),
                      sizeof(CtrlBlock), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return MOE_ERR_CUDA;
  *code = c[0].error ? c[0].error : c[1].error;
  *info = c[0].error ? c[0].error_info : c[1].error_info;
  return MOE_OK;
}

int moe_ep_destroy(MoeEp* ep) {
  if (!ep) return MOE_OK;
  cudaSetDevice(ep->device);
  cudaDeviceSynchronize();
  for (int r = 0; r < kEpMaxRanks; ++r)
    if (ep->peer_opened[r]) cudaIpcCloseMemHandle(ep->peer_base[r]);
  cudaFree(ep->shared);
  cudaFree(ep->local);
  delete ep;
  return MOE_OK;
}

}  // extern "C"
