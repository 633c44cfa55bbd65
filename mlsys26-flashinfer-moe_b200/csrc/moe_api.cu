// C ABI of the fused FP8 MoE forward: argument validation, workspace layout,
// TMA descriptor construction and the launch sequence.  No allocation and no
// host<->device synchronisation happen on the forward path.
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "moe_kernels.cuh"

namespace moe {
namespace {

// The routing grid aims at this many blocks (8 warps each, a multiple of
// 8 tokens per block): enough warps per SM to overlap the per-token shuffle
// chains, few enough for the last block's scan over all block histograms, and
// the bound the fixed scratch of moe_fp8_route_noalloc is sized for.
constexpr int kRouteTargetBlocks = 256;
constexpr int kLayoutSms = 148;   // B200 SM count: sizes the permute grid
constexpr size_t kAlign = 1024;

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

bool is_pow2(int64_t x) { return x > 0 && (x & (x - 1)) == 0; }

// Shape rules, mirroring the reference's asserts (kernel.py:591-607) but
// generalised to any layer this kernel family supports.
int validate_shape(const MoeFwdArgs* a) {
  // Row numbers of the expert-padded buffers (up to T * top_k + E * 127) are
  // 32-bit: T <= 2^24 keeps them far from overflow.
  if (a->T < 0 || a->T > (int64_t(1) << 24)) return MOE_ERR_SHAPE;
  if (a->H < 256 || a->H % 256 != 0 || a->H > 65536) return MOE_ERR_SHAPE;
  if (a->I < 128 || a->I % 128 != 0 || a->I > 65536) return MOE_ERR_SHAPE;
  const int64_t e = a->E_global;
  if (e < 1 || e > kMaxExperts) return MOE_ERR_SHAPE;
  if (a->n_group < 1 || e % a->n_group != 0) return MOE_ERR_SHAPE;
  const int64_t g = e / a->n_group;
  const int64_t epl = e <= 32 ? 1 : e / 32;
  if (e > 32 && e % 32 != 0) return MOE_ERR_SHAPE;
  if (!is_pow2(epl) || epl > 8 || g % epl != 0 || !is_pow2(g / epl)) return MOE_ERR_SHAPE;
  if (a->topk_group < 1 || a->topk_group > a->n_group) return MOE_ERR_SHAPE;
  if (a->top_k < 1 || a->top_k > kMaxTopK || a->top_k > a->topk_group * g) return MOE_ERR_SHAPE;
  if (a->E_local < 1 || a->E_local > e) return MOE_ERR_SHAPE;
  if (a->local_expert_offset < 0 || a->local_expert_offset + a->E_local > e) return MOE_ERR_SHAPE;
  if (a->bias_dtype != MOE_BIAS_F32 && a->bias_dtype != MOE_BIAS_BF16 &&
      a->bias_dtype != MOE_BIAS_F16)
    return MOE_ERR_INVALID_ARG;
  if ((a->flags & ~(MOE_FLAG_DETERMINISTIC | MOE_FLAG_DEBUG | MOE_FLAG_TEST_STALL)) != 0 ||
      a->reserved != 0)
    return MOE_ERR_INVALID_ARG;
  if (a->n_shared_experts < 0 || a->n_shared_experts > 1) return MOE_ERR_SHAPE;
  if (a->n_shared_experts && a->gemm2_weights_bf16) return MOE_ERR_INVALID_ARG;
  return MOE_OK;
}

// Dispatch buckets: the local routed experts, then the shared expert if any.
int64_t buckets(const MoeFwdArgs* a) { return a->E_local + a->n_shared_experts; }

bool deterministic(const MoeFwdArgs* a) { return (a->flags & MOE_FLAG_DETERMINISTIC) != 0; }
bool debug_checks(const MoeFwdArgs* a) { return (a->flags & MOE_FLAG_DEBUG) != 0; }

struct Layout {
  MoeWorkspaceLayout w;
  int tokens_per_block;
  int blocks;
  int permute_split;   // permute blocks per routing block (grid.y)
  GuardList guards;    // offsets of the buffers' guards (base set at launch)
};

// Decode-shaped batches (few rows per expert on average) take the
// swapped-operand kernels; the choice only depends on the shape, never on the
// routing, and both paths are exact for any routing.
bool use_small_path(const MoeFwdArgs* a) {
  return a->T * a->top_k <= kSmallPathMaxAvgRows * a->E_global &&
         a->H / kBlockK <= kSmallMaxScaleBlocks && a->I / 64 <= kSmallMaxScaleBlocks;
}

Layout make_layout(const MoeFwdArgs* a, int target_blocks = kRouteTargetBlocks) {
  Layout L{};
  const int64_t T = a->T, H = a->H, I = a->I, El = a->E_local, K = a->top_k;
  int64_t tpw = (T + target_blocks * 8 - 1) / (target_blocks * 8);
  if (tpw < 1) tpw = 1;
  int64_t tpb = 8 * tpw;
  if (tpb > kMaxTokensPerBlock) tpb = kMaxTokensPerBlock;
  L.tokens_per_block = static_cast<int>(tpb);
  L.blocks = static_cast<int>((T + tpb - 1) / tpb);
  // Permute blocks per routing block: about two blocks per SM in all, at
  // least one assignment per warp.
  int64_t split = (2 * kLayoutSms + L.blocks - 1) / (L.blocks > 0 ? L.blocks : 1);
  const int64_t most = tpb * K / (kRouteThreads / 32);
  if (split > most) split = most;
  if (split < 1) split = 1;
  L.permute_split = static_cast<int>(split);
  // Rows: every local assignment plus, with a shared expert, every token once
  // more; each non-empty bucket pads its last tile.
  const int64_t ns = a->n_shared_experts, nb = El + ns;
  const int64_t nmax = T * (K < El ? K : El) + ns * T;
  const int64_t active = nb < nmax ? nb : nmax;
  int64_t tiles = (nmax + active * (kTileM - 1)) / kTileM;
  if (tiles < 1) tiles = 1;
  const int64_t npad = tiles * kTileM;
  MoeWorkspaceLayout& w = L.w;
  w.npad = npad;
  w.route_blocks = L.blocks;
  w.tokens_per_block = tpb;
  // Every buffer is followed by a 16-byte guard (written and checked only by
  // MOE_FLAG_DEBUG forwards) before the next 1024-byte boundary.
  size_t off = 0;
  L.guards.n = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    const size_t guard = align_up(at + bytes, kGuardBytes);
    L.guards.off[L.guards.n++] = guard;
    off = align_up(guard + kGuardBytes, kAlign);
    return at;
  };
  w.ctrl = take(sizeof(CtrlBlock));
  w.topk_idx = take(sizeof(int) * T * K);
  w.topk_weights = take(sizeof(float) * T * K);
  w.block_base = take(sizeof(int) * (L.blocks > 0 ? L.blocks : 1) * El);
  w.counts = take(sizeof(int) * nb);
  w.tile_start = take(sizeof(int) * (nb + 1));
  w.row_token = take(sizeof(int) * npad);
  w.row_weight = take(sizeof(float) * npad);
  w.a_perm = take(static_cast<size_t>(npad) * H);
  w.a_scale_perm = take(sizeof(float) * (H / kBlockK) * npad);
  w.inter = take(static_cast<size_t>(npad) * I);
  w.inter_scale = take(sizeof(float) * (I / kInterScaleBlock) * npad);
  w.out_f32 = take(sizeof(float) * T * H);
  w.assign_row = take(sizeof(int) * T * K);
  w.rows_out = take(deterministic(a) ? sizeof(float) * static_cast<size_t>(npad) * H : 0);
  w.inter_bf16 = take(a->gemm2_weights_bf16 ? 2 * static_cast<size_t>(npad) * I : 0);
  w.total_bytes = off;
  return L;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// device properties and TMA descriptors
// ---------------------------------------------------------------------------

struct DeviceInfo {
  int sms = 0;
  int major = 0;
  bool attrs_set = false;
};
std::mutex g_mu;
DeviceInfo g_dev[64];

int device_info(DeviceInfo** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MOE_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (d.sms == 0) {
    if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return MOE_ERR_CUDA;
    if (cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return MOE_ERR_CUDA;
  }
  if (d.major != 10) return MOE_ERR_DEVICE;
  if (!d.attrs_set) {
    if (gemm_set_smem_attrs() != MOE_OK) return MOE_ERR_CUDA;
    if (gemm_small_set_smem_attrs() != MOE_OK) return MOE_ERR_CUDA;
    d.attrs_set = true;
  }
  *out = &d;
  return MOE_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Byte matrix [rows, cols] (row stride = cols) read in 128x128 boxes with the
// 128-byte swizzle the UMMA descriptors expect.
struct MapKey {
  const void* base;
  uint64_t cols, rows;
  uint32_t box_rows;
  bool operator==(const MapKey& o) const {
    return base == o.base && cols == o.cols && rows == o.rows && box_rows == o.box_rows;
  }
};
struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool used;
};
constexpr int kMapCache = 64;
MapEntry g_maps[kMapCache];
int g_map_next = 0;

// Tensor map of a row-major byte matrix [rows, cols] read in boxes of 128
// columns (one K block) x box_rows rows, 128-byte swizzled.
int byte_tile_map(const void* base, uint64_t cols, uint64_t rows, CUtensorMap* out,
                  uint32_t box_rows = kTileM) {
  const MapKey key{base, cols, rows, box_rows};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    for (int i = 0; i < kMapCache; ++i)
      if (g_maps[i].used && g_maps[i].key == key) {
        *out = g_maps[i].map;
        return MOE_OK;
      }
  }
  auto fn = encode_fn();
  if (!fn) return MOE_ERR_CUDA;
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBlockK), box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return MOE_ERR_CUDA;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    g_maps[g_map_next] = MapEntry{key, m, true};
    g_map_next = (g_map_next + 1) % kMapCache;
  }
  *out = m;
  return MOE_OK;
}

int check_args(const MoeFwdArgs* a, Layout* L) {
  if (!a) return MOE_ERR_INVALID_ARG;
  int st = validate_shape(a);
  if (st) return st;
  *L = make_layout(a);
  if (a->T == 0) return MOE_OK;
  if (!a->routing_logits || !a->routing_bias || !a->hidden_states || !a->hidden_states_scale ||
      !a->gemm1_weights || !a->gemm1_weights_scale || !a->gemm2_weights ||
      !a->gemm2_weights_scale || !a->output)
    return MOE_ERR_INVALID_ARG;
  if (!a->workspace || a->workspace_bytes < L->w.total_bytes) return MOE_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(a->workspace) & 255u) != 0) return MOE_ERR_ALIGNMENT;
  if (!aligned16(a->hidden_states) || !aligned16(a->gemm1_weights) ||
      !aligned16(a->gemm2_weights) || !aligned16(a->output) || !aligned16(a->routing_logits) ||
      !aligned16(a->gemm2_weights_bf16))
    return MOE_ERR_ALIGNMENT;
  return MOE_OK;
}

template <class T>
T* ws_ptr(const MoeFwdArgs* a, size_t off) {
  return reinterpret_cast<T*>(static_cast<uint8_t*>(a->workspace) + off);
}

RouteParams route_params(const MoeFwdArgs* a, const Layout& L, const int* T_dev) {
  const MoeWorkspaceLayout& w = L.w;
  RouteParams rp{};
  rp.logits = a->routing_logits;
  rp.bias = a->routing_bias;
  rp.bias_dtype = a->bias_dtype;
  rp.T = static_cast<int>(a->T);
  rp.E = static_cast<int>(a->E_global);
  rp.n_group = static_cast<int>(a->n_group);
  rp.topk_group = static_cast<int>(a->topk_group);
  rp.top_k = static_cast<int>(a->top_k);
  const int epl = rp.E <= 32 ? 1 : rp.E / 32;
  rp.experts_per_lane = epl;
  rp.lanes_per_group = (rp.E / rp.n_group) / epl;
  rp.E_local = static_cast<int>(a->E_local);
  rp.local_expert_offset = static_cast<int>(a->local_expert_offset);
  rp.routed_scaling_factor = a->routed_scaling_factor;
  rp.tokens_per_block = L.tokens_per_block;
  rp.topk_idx = ws_ptr<int>(a, w.topk_idx);
  rp.topk_weights = ws_ptr<float>(a, w.topk_weights);
  rp.block_base = ws_ptr<int>(a, w.block_base);
  rp.counts = ws_ptr<int>(a, w.counts);
  rp.tile_start = ws_ptr<int>(a, w.tile_start);
  rp.ctrl = ws_ptr<CtrlBlock>(a, w.ctrl);
  rp.T_dev = T_dev;
  rp.n_shared = static_cast<int>(a->n_shared_experts);
  return rp;
}

int launch_route(const MoeFwdArgs* a, const Layout& L, cudaStream_t s,
                 const int* T_dev = nullptr) {
  const RouteParams rp = route_params(a, L, T_dev);
  if (cudaMemsetAsync(rp.ctrl, 0, sizeof(CtrlBlock), s) != cudaSuccess) return MOE_ERR_CUDA;
  moe_route_kernel<<<L.blocks, kRouteThreads, 0, s>>>(rp);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

CheckParams check_params(const MoeFwdArgs* a, const Layout& L) {
  const MoeWorkspaceLayout& w = L.w;
  CheckParams c{};
  c.T = static_cast<int>(a->T);
  c.top_k = static_cast<int>(a->top_k);
  c.E_global = static_cast<int>(a->E_global);
  c.E_local = static_cast<int>(a->E_local);
  c.local_expert_offset = static_cast<int>(a->local_expert_offset);
  c.n_shared = static_cast<int>(a->n_shared_experts);
  c.npad = w.npad;
  c.counts = ws_ptr<int>(a, w.counts);
  c.tile_start = ws_ptr<int>(a, w.tile_start);
  c.topk_idx = ws_ptr<int>(a, w.topk_idx);
  c.topk_weights = ws_ptr<float>(a, w.topk_weights);
  c.row_token = ws_ptr<int>(a, w.row_token);
  c.row_weight = ws_ptr<float>(a, w.row_weight);
  c.assign_row = ws_ptr<int>(a, w.assign_row);
  c.ctrl = ws_ptr<CtrlBlock>(a, w.ctrl);
  return c;
}

int launch_check_dispatch(const MoeFwdArgs* a, const Layout& L, int sms, cudaStream_t s) {
  const CheckParams c = check_params(a, L);
  const int64_t items = c.E_local + c.n_shared + static_cast<int64_t>(c.T) * c.top_k + c.npad;
  int64_t blocks = (items + 255) / 256;
  if (blocks > 4 * sms) blocks = 4 * sms;
  moe_check_dispatch_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(c);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

int launch_guards(const MoeFwdArgs* a, const Layout& L, bool write, cudaStream_t s) {
  GuardList g = L.guards;
  g.base = static_cast<uint8_t*>(a->workspace);
  moe_guard_kernel<<<1, 32, 0, s>>>(g, write ? 1 : 0, ws_ptr<CtrlBlock>(a, L.w.ctrl));
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

int record(void* const* ev, int i, cudaStream_t s) {
  if (!ev) return MOE_OK;
  return cudaEventRecord(static_cast<cudaEvent_t>(ev[i]), s) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

// T_dev (expert-parallel receive side): the row count lives on the device and
// a->T is only its capacity; the fp32 accumulator rows are zeroed by the
// permute kernel for exactly the rows that exist, and the layer stops after
// GEMM2 (the caller combines the fp32 rows).
int launch_forward(const MoeFwdArgs* a, const Layout& L, cudaStream_t s,
                   void* const* ev = nullptr, const int* T_dev = nullptr) {
  DeviceInfo* dev = nullptr;
  int st = device_info(&dev);
  if (st) return st;
  if ((st = record(ev, 0, s))) return st;
  const MoeWorkspaceLayout& w = L.w;
  const int64_t T = a->T, H = a->H, I = a->I, El = a->E_local;
  // Debug checks (single-GPU forward only; the expert-parallel receive side
  // passes flags 0).
  const bool dbg = debug_checks(a) && !T_dev;
  if (dbg && (st = launch_guards(a, L, true, s))) return st;
  float* out_f32 = ws_ptr<float>(a, w.out_f32);
  PermuteParams pp{};
  pp.T = static_cast<int>(T);
  pp.H = static_cast<int>(H);
  pp.top_k = static_cast<int>(a->top_k);
  pp.E_local = static_cast<int>(El);
  pp.local_expert_offset = static_cast<int>(a->local_expert_offset);
  pp.tokens_per_block = L.tokens_per_block;
  pp.npad = w.npad;
  pp.topk_idx = ws_ptr<int>(a, w.topk_idx);
  pp.topk_weights = ws_ptr<float>(a, w.topk_weights);
  pp.block_base = ws_ptr<int>(a, w.block_base);
  pp.tile_start = ws_ptr<int>(a, w.tile_start);
  pp.hidden = static_cast<const uint8_t*>(a->hidden_states);
  pp.hs_scale = a->hidden_states_scale;
  pp.scale_ld = T;
  pp.T_dev = T_dev;
  const bool det = deterministic(a);
  // the accumulator rows of the permute block's tokens (the deterministic
  // combine stores rows instead of adding into the accumulator)
  pp.zero_rows = det ? nullptr : out_f32;
  pp.assign_row = ws_ptr<int>(a, w.assign_row);
  pp.n_shared = static_cast<int>(a->n_shared_experts);
  pp.row_token = ws_ptr<int>(a, w.row_token);
  pp.row_weight = ws_ptr<float>(a, w.row_weight);
  pp.a_perm = ws_ptr<uint8_t>(a, w.a_perm);
  pp.a_scale_perm = ws_ptr<float>(a, w.a_scale_perm);

  if (!T_dev && T <= kTinyMaxTokens) {
    // Decode-sized batch: one launch routes, schedules and packs (block 0)
    // and zeroes the accumulator (the other blocks); events[1] and [2] mark
    // its end.
    RouteParams rp = route_params(a, L, nullptr);
    rp.tokens_per_block = static_cast<int>(T);
    const int64_t n4 = det ? 0 : T * H / 4;
    int64_t zblocks = (n4 + 4 * kRouteThreads - 1) / (4 * kRouteThreads);
    if (zblocks < 1) zblocks = 1;
    if (zblocks > 32) zblocks = 32;
    moe_route_permute_tiny_kernel<<<static_cast<int>(1 + zblocks), kRouteThreads, 0, s>>>(
        rp, pp, out_f32, n4);
    if (cudaGetLastError() != cudaSuccess) return MOE_ERR_CUDA;
    if ((st = record(ev, 1, s))) return st;
    if ((st = record(ev, 2, s))) return st;
  } else {
    st = launch_route(a, L, s, T_dev);
    if (st) return st;
    if ((st = record(ev, 1, s))) return st;
    if (launch_programmatic(moe_permute_kernel, dim3(L.blocks, L.permute_split),
                            dim3(kRouteThreads), 0, s, pp) != cudaSuccess)
      return MOE_ERR_CUDA;
    if ((st = record(ev, 2, s))) return st;
  }
  // Tables checked before the GEMMs read them; on a failure the GEMMs see the
  // error word and schedule no units.
  if (dbg && (st = launch_check_dispatch(a, L, dev->sms, s))) return st;

  const bool small = use_small_path(a);
  // Prepared bf16 W2 (prefill path only; decode streams the FP8 weights).
  const bool bf16_w2 = a->gemm2_weights_bf16 != nullptr && !small;

  const uint32_t tok_box = small ? 16u : static_cast<uint32_t>(kTileM);
  CUtensorMap tm_a1, tm_b1, tm_a2, tm_b2;
  if ((st = byte_tile_map(pp.a_perm, H, w.npad, &tm_a1, tok_box))) return st;
  const int64_t nb = buckets(a);   // the shared expert's weights follow the routed experts'
  if ((st = byte_tile_map(a->gemm1_weights, H, nb * 2 * I, &tm_b1))) return st;
  if (bf16_w2) {
    // bf16 matrices read as byte matrices: 128-byte boxes hold 64 elements of K.
    if ((st = byte_tile_map(ws_ptr<uint8_t>(a, w.inter_bf16), 2 * I, w.npad, &tm_a2))) return st;
    if ((st = byte_tile_map(a->gemm2_weights_bf16, 2 * I, nb * H, &tm_b2))) return st;
  } else {
    if ((st = byte_tile_map(ws_ptr<uint8_t>(a, w.inter), I, w.npad, &tm_a2, tok_box))) return st;
    if ((st = byte_tile_map(a->gemm2_weights, I, nb * H, &tm_b2))) return st;
  }

  GemmParams g1{};
  g1.tile_start = pp.tile_start;
  g1.counts = ws_ptr<int>(a, w.counts);
  g1.E_local = static_cast<int>(nb);
  g1.num_k_blocks = static_cast<int>(H / kBlockK);
  g1.n_tiles = static_cast<int>(I / (kTileN / 2));
  g1.b_rows_per_expert = static_cast<int>(2 * I);
  g1.inter = static_cast<int>(I);
  g1.hidden = static_cast<int>(H);
  g1.npad = w.npad;
  g1.a_scale = pp.a_scale_perm;
  g1.b_scale = a->gemm1_weights_scale;
  g1.inter_out = ws_ptr<uint8_t>(a, w.inter);
  g1.inter_scale = ws_ptr<float>(a, w.inter_scale);
  g1.ctrl = ws_ptr<CtrlBlock>(a, w.ctrl);
  g1.wait_limit_us = wait_limit_us(a->wait_limit_ns);
  g1.inter_bf16 = bf16_w2 ? ws_ptr<__nv_bfloat16>(a, w.inter_bf16) : nullptr;
  g1.stall = (a->flags & MOE_FLAG_TEST_STALL) != 0 ? 1 : 0;
  g1.skip_on_error = dbg ? 1 : 0;
  if (small) {
    if ((st = launch_gemm_small(kGemm1, tm_b1, tm_a1, g1, dev->sms, s))) return st;
  } else if ((st = launch_gemm(kGemm1, tm_a1, tm_b1, g1, dev->sms, s))) {
    return st;
  }
  if ((st = record(ev, 3, s))) return st;

  GemmParams g2 = g1;
  g2.num_k_blocks = static_cast<int>(I / kBlockK);
  g2.n_tiles = static_cast<int>(H / kTileN);
  g2.b_rows_per_expert = static_cast<int>(H);
  g2.a_scale = g1.inter_scale;
  g2.b_scale = a->gemm2_weights_scale;
  g2.inter_out = nullptr;
  g2.inter_scale = nullptr;
  g2.row_token = pp.row_token;
  g2.row_weight = pp.row_weight;
  g2.out_f32 = out_f32;
  g2.stall = 0;
  g2.inter_bf16 = nullptr;
  g2.rows_out = det ? ws_ptr<float>(a, w.rows_out) : nullptr;
  if (bf16_w2) g2.num_k_blocks = static_cast<int>(2 * I / kBlockK);   // 64 bf16 per block
  const bool fuse_final = small && !T_dev && !det && T <= kFuseFinalMaxTokens;
  if (fuse_final) {
    g2.final_out = static_cast<__nv_bfloat16*>(a->output);
    g2.final_n8 = T * H / 8;
  }
  if (small) {
    g2.n_tiles = static_cast<int>(H / kTileM);
    if ((st = launch_gemm_small(kGemm2, tm_b2, tm_a2, g2, dev->sms, s))) return st;
  } else if ((st = launch_gemm(bf16_w2 ? kGemm2Bf16 : kGemm2, tm_a2, tm_b2, g2, dev->sms, s))) {
    return st;
  }
  if ((st = record(ev, 4, s))) return st;
  if (T_dev) return MOE_OK;
  if (fuse_final) {
    if ((st = record(ev, 5, s))) return st;
    return dbg ? launch_guards(a, L, false, s) : MOE_OK;
  }

  const int64_t n8 = T * H / 8;
  int blocks = static_cast<int>((n8 + 255) / 256);
  if (blocks > dev->sms * 8) blocks = dev->sms * 8;
  cudaError_t e;
  if (det)
    e = launch_programmatic(moe_combine_rows_kernel, dim3(blocks), dim3(256), 0, s,
                            static_cast<const float*>(g2.rows_out),
                            static_cast<const int*>(pp.assign_row),
                            static_cast<__nv_bfloat16*>(a->output), static_cast<int>(T),
                            static_cast<int>(H), static_cast<int>(a->top_k),
                            a->n_shared_experts ? static_cast<const int*>(pp.tile_start) + El
                                                : static_cast<const int*>(nullptr));
  else
    e = launch_programmatic(moe_finalize_kernel, dim3(blocks), dim3(256), 0, s,
                            static_cast<const float*>(out_f32),
                            static_cast<__nv_bfloat16*>(a->output), n8);
  if (e != cudaSuccess) return MOE_ERR_CUDA;
  if ((st = record(ev, 5, s))) return st;
  return dbg ? launch_guards(a, L, false, s) : MOE_OK;
}

}  // namespace

int forward_device_rows(const MoeFwdArgs* a, const int* T_dev, cudaStream_t s) {
  int st = validate_shape(a);
  if (st) return st;
  const Layout L = make_layout(a);
  if (a->T == 0) return MOE_OK;
  if (!a->workspace || a->workspace_bytes < L.w.total_bytes) return MOE_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(a->workspace) & 255u) != 0) return MOE_ERR_ALIGNMENT;
  return launch_forward(a, L, s, nullptr, T_dev);
}

int validate_shape_public(const MoeFwdArgs* a) { return validate_shape(a); }

int route_only(const MoeFwdArgs* a, cudaStream_t s) {
  int st = validate_shape(a);
  if (st) return st;
  const Layout L = make_layout(a);
  if (a->T == 0) return MOE_OK;
  if (!a->routing_logits || !a->routing_bias) return MOE_ERR_INVALID_ARG;
  if (!a->workspace || a->workspace_bytes < L.w.total_bytes) return MOE_ERR_WORKSPACE;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev))) return st;
  return launch_route(a, L, s);
}

int num_sms(int* out) {
  DeviceInfo* dev = nullptr;
  const int st = device_info(&dev);
  if (st) return st;
  *out = dev->sms;
  return MOE_OK;
}

MoeWorkspaceLayout workspace_layout_for(const MoeFwdArgs* a) { return make_layout(a).w; }

// ---------------------------------------------------------------------------
// router logits
// ---------------------------------------------------------------------------
namespace {

bool router_shape_ok(int64_t T, int64_t H, int64_t E) {
  return T >= 0 && T < (int64_t(1) << 24) && H >= 8 && H % 8 == 0 && H <= 65536 && E >= 1 &&
         E <= 65536;
}

// The tensor-core path: a batch big enough to fill row tiles, E in whole
// 256-column tiles, H in whole 128-byte (64-element) K blocks.
bool router_uses_tc(int64_t T, int64_t H, int64_t E) {
  return T > kRouterGemvMaxTokens && E % kTileN == 0 && H % 64 == 0;
}

struct RouterLayout {
  int64_t npad;
  size_t ctrl, tile_start, counts, row_token, row_weight, total;
};

RouterLayout router_layout(int64_t T) {
  RouterLayout r{};
  r.npad = (T + kTileM - 1) / kTileM * kTileM;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes, 256);
    return at;
  };
  r.ctrl = take(sizeof(CtrlBlock));
  r.tile_start = take(2 * sizeof(int));
  r.counts = take(sizeof(int));
  r.row_token = take(sizeof(int) * r.npad);
  r.row_weight = take(sizeof(float) * r.npad);
  r.total = off;
  return r;
}

}  // namespace

}  // namespace moe

using namespace moe;

extern "C" {

int moe_fp8_workspace_size(const MoeFwdArgs* a, size_t* bytes) {
  if (!a || !bytes) return MOE_ERR_INVALID_ARG;
  const int st = validate_shape(a);
  if (st) return st;
  *bytes = make_layout(a).w.total_bytes;
  return MOE_OK;
}

int moe_fp8_workspace_layout(const MoeFwdArgs* a, MoeWorkspaceLayout* out) {
  if (!a || !out) return MOE_ERR_INVALID_ARG;
  const int st = validate_shape(a);
  if (st) return st;
  *out = make_layout(a).w;
  return MOE_OK;
}

int moe_fp8_forward(const MoeFwdArgs* a, void* stream) {
  Layout L;
  int st = check_args(a, &L);
  if (st) return st;
  if (a->T == 0) return MOE_OK;
  return launch_forward(a, L, static_cast<cudaStream_t>(stream));
}

int moe_fp8_forward_profiled(const MoeFwdArgs* a, void* stream, void* const* events,
                             int n_events) {
  if (!events || n_events != MOE_PROFILE_EVENTS) return MOE_ERR_INVALID_ARG;
  Layout L;
  int st = check_args(a, &L);
  if (st) return st;
  if (a->T == 0) return MOE_OK;
  return launch_forward(a, L, static_cast<cudaStream_t>(stream), events);
}

int moe_fp8_route(const MoeFwdArgs* a, void* stream) {
  Layout L;
  int st = check_args(a, &L);
  if (st) return st;
  if (a->T == 0) return MOE_OK;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev))) return st;
  return launch_route(a, L, static_cast<cudaStream_t>(stream));
}

int moe_fp8_device_error(const MoeFwdArgs* a, void* stream, int32_t* code, int32_t* info) {
  Layout L;
  if (!a || !code || !info) return MOE_ERR_INVALID_ARG;
  int st = validate_shape(a);
  if (st) return st;
  L = make_layout(a);
  if (!a->workspace || a->workspace_bytes < L.w.total_bytes) return MOE_ERR_WORKSPACE;
  CtrlBlock host;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(&host, ws_ptr<CtrlBlock>(a, L.w.ctrl), sizeof(host), cudaMemcpyDeviceToHost,
                      s) != cudaSuccess)
    return MOE_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return MOE_ERR_CUDA;
  *code = host.error;
  *info = host.error_info;
  return MOE_OK;
}

int moe_fp8_check_workspace(const MoeFwdArgs* a, void* stream) {
  if (!a) return MOE_ERR_INVALID_ARG;
  int st = validate_shape(a);
  if (st) return st;
  const Layout L = make_layout(a);
  if (a->T == 0) return MOE_OK;
  if (!a->workspace || a->workspace_bytes < L.w.total_bytes) return MOE_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(a->workspace) & 255u) != 0) return MOE_ERR_ALIGNMENT;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev))) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CtrlBlock* ctrl = ws_ptr<CtrlBlock>(a, L.w.ctrl);
  // error and error_info are adjacent words
  if (cudaMemsetAsync(&ctrl->error, 0, 2 * sizeof(int), s) != cudaSuccess) return MOE_ERR_CUDA;
  if ((st = launch_check_dispatch(a, L, dev->sms, s))) return st;
  return debug_checks(a) ? launch_guards(a, L, false, s) : MOE_OK;
}

const char* moe_fp8_status_string(int code) {
  switch (code) {
    case MOE_OK: return "ok";
    case MOE_ERR_INVALID_ARG: return "invalid argument";
    case MOE_ERR_SHAPE: return "unsupported or inconsistent shape";
    case MOE_ERR_ALIGNMENT: return "pointer not 16-byte aligned";
    case MOE_ERR_WORKSPACE: return "workspace missing or too small";
    case MOE_ERR_CUDA: return "CUDA call failed";
    case MOE_ERR_TIMEOUT: return "device-side wait timed out";
    case MOE_ERR_DEVICE: return "device is not sm_100 (B200)";
    case MOE_ERR_TOO_LARGE: return "size exceeds the fixed scratch of moe_fp8_route_noalloc";
    case MOE_ERR_BOUNDS: return "a debug check of the dispatch tables or workspace guards failed";
    default: return "unknown status";
  }
}

int moe_fp8_prepare_gemm2_bf16(const void* w2, const float* w2_scale, int64_t E_local, int64_t H,
                               int64_t I, void* out, void* stream) {
  if (E_local < 1 || H < 128 || H % 128 != 0 || I < 128 || I % 128 != 0) return MOE_ERR_SHAPE;
  if (!w2 || !w2_scale || !out) return MOE_ERR_INVALID_ARG;
  if (!aligned16(w2) || !aligned16(out) || (reinterpret_cast<uintptr_t>(w2_scale) & 3u) != 0)
    return MOE_ERR_ALIGNMENT;
  DeviceInfo* dev = nullptr;
  const int st = device_info(&dev);
  if (st) return st;
  return launch_prepare_w2_bf16(w2, w2_scale, E_local, H, I, out, dev->sms,
                                static_cast<cudaStream_t>(stream));
}

int moe_router_workspace_size(int64_t T, int64_t H, int64_t E, size_t* bytes) {
  if (!bytes) return MOE_ERR_INVALID_ARG;
  if (!router_shape_ok(T, H, E)) return MOE_ERR_SHAPE;
  *bytes = router_uses_tc(T, H, E) ? router_layout(T).total : 0;
  return MOE_OK;
}

int moe_router_logits_bf16(const void* x, const void* w_gate, int64_t T, int64_t H, int64_t E,
                           float* logits, void* workspace, size_t workspace_bytes, void* stream) {
  if (!router_shape_ok(T, H, E)) return MOE_ERR_SHAPE;
  if (T == 0) return MOE_OK;
  if (!x || !w_gate || !logits) return MOE_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(w_gate) || !aligned16(logits)) return MOE_ERR_ALIGNMENT;
  DeviceInfo* dev = nullptr;
  int st = device_info(&dev);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const auto* wb = static_cast<const __nv_bfloat16*>(w_gate);
  if (!router_uses_tc(T, H, E)) {
    return launch_router_gemv(xb, wb, T, H, E, logits, s);
  }
  const RouterLayout L = router_layout(T);
  if (!workspace || workspace_bytes < L.total) return MOE_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return MOE_ERR_ALIGNMENT;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* tile_start = reinterpret_cast<int*>(ws + L.tile_start);
  int* counts = reinterpret_cast<int*>(ws + L.counts);
  int* row_token = reinterpret_cast<int*>(ws + L.row_token);
  float* row_weight = reinterpret_cast<float*>(ws + L.row_weight);
  CtrlBlock* ctrl = reinterpret_cast<CtrlBlock*>(ws + L.ctrl);
  int64_t sblocks = (L.npad + 255) / 256;
  if (sblocks > dev->sms) sblocks = dev->sms;
  moe_router_setup_kernel<<<static_cast<int>(sblocks), 256, 0, s>>>(
      static_cast<int>(T), static_cast<int>(L.npad), tile_start, counts, row_token, row_weight,
      ctrl);
  if (cudaGetLastError() != cudaSuccess) return MOE_ERR_CUDA;
  GemmParams g{};
  g.tile_start = tile_start;
  g.counts = counts;
  g.row_token = row_token;
  g.row_weight = row_weight;
  g.ctrl = ctrl;
  // One "expert" whose 128-row tiles are the tokens in order and whose weight
  // rows are the E router rows; bf16 matrices read as byte matrices, so a
  // 128-byte K block holds 64 elements.
  CUtensorMap tm_a, tm_b;
  if ((st = byte_tile_map(x, 2 * H, T, &tm_a))) return st;
  if ((st = byte_tile_map(w_gate, 2 * H, E, &tm_b))) return st;
  g.E_local = 1;
  g.num_k_blocks = static_cast<int>(2 * H / kBlockK);
  g.n_tiles = static_cast<int>(E / kTileN);
  g.b_rows_per_expert = static_cast<int>(E);
  g.hidden = static_cast<int>(E);   // width of the stored rows
  g.npad = L.npad;
  g.rows_out = logits;              // row r of the single "expert" = token r
  g.wait_limit_us = wait_limit_us(0);
  return launch_gemm(kGemm2Bf16, tm_a, tm_b, g, dev->sms, s);
}

int moe_bf16_to_fp8_1x128(const void* x, int64_t T, int64_t H, void* q, float* scale,
                          void* stream) {
  if (T < 0 || H <= 0 || H % 128 != 0) return MOE_ERR_SHAPE;
  if (T == 0) return MOE_OK;
  if (!x || !q || !scale) return MOE_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(q) || (reinterpret_cast<uintptr_t>(scale) & 3u) != 0)
    return MOE_ERR_ALIGNMENT;
  DeviceInfo* dev = nullptr;
  const int st = device_info(&dev);
  if (st) return st;
  return launch_quant_1x128(x, T, H, q, scale, dev->sms, static_cast<cudaStream_t>(stream));
}

int moe_fp8_num_sms(int device, int32_t* out) {
  if (!out) return MOE_ERR_INVALID_ARG;
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return MOE_ERR_CUDA;
  *out = v;
  return MOE_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Routing without a workspace.
//
// Some callers cannot allocate device memory at the point where they route
// tokens: an inference engine that runs this layer from a plugin callback in
// which allocation is forbidden, a serving loop whose device memory is owned in
// full by another pool, or a host in another language that has no device
// allocator to hand.  moe_fp8_route_noalloc serves them: it takes only the
// router inputs and the caller's output arrays and keeps its scratch (the
// per-block expert histograms, the tile prefix sum and the arrival counter of
// the last-block scan) in the fixed device array below.  That array is part of
// the library image, so every GPU that loads the library holds it
// (kNoAllocScratchBytes = 263,428 bytes) until the process exits.
// ---------------------------------------------------------------------------

namespace moe {
namespace {

constexpr int kNoAllocMaxBlocks = 256;                 // route blocks for T <= 65536
constexpr int64_t kNoAllocMaxTokens = 65536;
constexpr size_t kNoAllocHistOffset = sizeof(CtrlBlock);
constexpr size_t kNoAllocTileOffset =
    kNoAllocHistOffset + sizeof(int) * kNoAllocMaxBlocks * kMaxExperts;
constexpr size_t kNoAllocScratchBytes = kNoAllocTileOffset + sizeof(int) * (kMaxExperts + 1);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device, looked up once with the
// device current and kept for the life of the process (so a first call before
// any stream capture makes later calls capturable).  The address belongs to
// the device's primary context: the library is not meant to be used across
// cudaDeviceReset.  Host code must not pass the symbol itself to a kernel: on
// the host it names a host-side stand-in.
unsigned char* g_noalloc_ptr[64];
std::mutex g_noalloc_mu;

int noalloc_scratch(unsigned char** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return MOE_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
      return MOE_ERR_CUDA;
    g_noalloc_ptr[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return MOE_OK;
}

}  // namespace
}  // namespace moe

extern "C" int moe_fp8_route_noalloc(const float* routing_logits, const void* routing_bias,
                                     int32_t bias_dtype, int64_t T, int64_t E_global,
                                     int64_t n_group, int64_t topk_group, int64_t top_k,
                                     int64_t E_local, int64_t local_expert_offset,
                                     float routed_scaling_factor, int32_t* topk_idx,
                                     float* topk_weights, int32_t* expert_counts,
                                     void* stream) {
  using namespace moe;
  MoeFwdArgs a{};
  a.T = T;
  a.H = 256;                      // the router does not read H or I; any valid value
  a.I = 128;
  a.E_global = E_global;
  a.E_local = E_local;
  a.local_expert_offset = local_expert_offset;
  a.n_group = n_group;
  a.topk_group = topk_group;
  a.top_k = top_k;
  a.routed_scaling_factor = routed_scaling_factor;
  a.bias_dtype = bias_dtype;
  int st = validate_shape(&a);
  if (st) return st;
  if (T > kNoAllocMaxTokens) return MOE_ERR_TOO_LARGE;
  if (T == 0) return MOE_OK;
  if (!routing_logits || !routing_bias || !topk_idx || !topk_weights || !expert_counts)
    return MOE_ERR_INVALID_ARG;
  const Layout L = make_layout(&a, kNoAllocMaxBlocks);
  if (L.blocks > kNoAllocMaxBlocks) return MOE_ERR_TOO_LARGE;
  DeviceInfo* dev = nullptr;
  if ((st = device_info(&dev))) return st;
  unsigned char* scratch = nullptr;
  if ((st = noalloc_scratch(&scratch))) return st;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  RouteParams rp{};
  rp.logits = routing_logits;
  rp.bias = routing_bias;
  rp.bias_dtype = bias_dtype;
  rp.T = static_cast<int>(T);
  rp.E = static_cast<int>(E_global);
  rp.n_group = static_cast<int>(n_group);
  rp.topk_group = static_cast<int>(topk_group);
  rp.top_k = static_cast<int>(top_k);
  const int epl = rp.E <= 32 ? 1 : rp.E / 32;
  rp.experts_per_lane = epl;
  rp.lanes_per_group = (rp.E / rp.n_group) / epl;
  rp.E_local = static_cast<int>(E_local);
  rp.local_expert_offset = static_cast<int>(local_expert_offset);
  rp.routed_scaling_factor = routed_scaling_factor;
  rp.tokens_per_block = L.tokens_per_block;
  rp.topk_idx = topk_idx;
  rp.topk_weights = topk_weights;
  rp.counts = expert_counts;
  rp.ctrl = reinterpret_cast<CtrlBlock*>(scratch);
  rp.block_base = reinterpret_cast<int*>(scratch + kNoAllocHistOffset);
  rp.tile_start = reinterpret_cast<int*>(scratch + kNoAllocTileOffset);
  // The array keeps the previous call's contents: the arrival counter of the
  // last-block scan must start at zero.  Histograms and the tile prefix are
  // fully rewritten by every call.
  if (cudaMemsetAsync(scratch, 0, sizeof(CtrlBlock), s) != cudaSuccess) return MOE_ERR_CUDA;
  moe_route_kernel<<<L.blocks, kRouteThreads, 0, s>>>(rp);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}
