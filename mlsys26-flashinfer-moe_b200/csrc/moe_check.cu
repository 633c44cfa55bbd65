// Debug checks of the forward's routing and dispatch tables and of the
// workspace guards (MOE_FLAG_DEBUG, moe_fp8_check_workspace).
//
//   moe_check_dispatch_kernel  one thread per dispatch bucket (local expert or
//                              the shared expert), per (token, k) assignment
//                              and per permuted row, grid-stride:
//                              every index is range-checked before it is used
//                              to read another table, so the kernel is safe on
//                              any contents of the workspace.
//   moe_guard_kernel           writes or compares the 16-byte patterns placed
//                              after the workspace buffers.
//
// The reference indexes its buffers without checks (its GEMM2 even reads up to
// 63 floats past the end of the intermediate scales on the last tile,
// kernel.py:218-220); these checks have no counterpart there.
#include "moe_kernels.cuh"

namespace moe {

namespace {

__device__ __forceinline__ void fail(CtrlBlock* ctrl, int site, int64_t index) {
  const int64_t i = index < 0 ? 0 : (index > 0xFFFFFF ? 0xFFFFFF : index);
  report_error(ctrl, MOE_ERR_BOUNDS, (site << 24) | static_cast<int>(i));
}

__device__ __forceinline__ bool finite(float v) { return isfinite(v); }

// Bucket e of the E buckets whose tile range [128*ts[e], 128*ts[e+1])
// holds row r, or -1.  The table is read at checked indices only, so a
// corrupted (non-monotone) table yields a wrong expert or -1, never a read
// outside it.
__device__ __forceinline__ int expert_of_row(const int* ts, int E, int64_t r) {
  int lo = 0, hi = E - 1;
  while (lo < hi) {   // largest e with 128*ts[e] <= r
    const int mid = (lo + hi + 1) >> 1;
    if (static_cast<int64_t>(ts[mid]) * kTileM <= r) lo = mid;
    else hi = mid - 1;
  }
  const int64_t b0 = static_cast<int64_t>(ts[lo]) * kTileM;
  const int64_t b1 = static_cast<int64_t>(ts[lo + 1]) * kTileM;
  return (r >= b0 && r < b1) ? lo : -1;
}

}  // namespace

__global__ void __launch_bounds__(256) moe_check_dispatch_kernel(CheckParams p) {
  const int64_t n_assign = static_cast<int64_t>(p.T) * p.top_k;
  const int nb = p.E_local + p.n_shared;   // buckets: routed experts, then the shared expert
  const int64_t total = nb + n_assign + p.npad;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    if (i < nb) {
      // ---- per bucket: counts and the 128-row tile prefix (the shared
      // expert's bucket holds every token)
      const int e = static_cast<int>(i);
      const int c = p.counts[e];
      if (c < 0 || c > p.T || (e == p.E_local && c != p.T)) {
        fail(p.ctrl, MOE_CHECK_COUNTS, e);
        continue;
      }
      const int ts0 = p.tile_start[e], ts1 = p.tile_start[e + 1];
      if (e == 0 && ts0 != 0) fail(p.ctrl, MOE_CHECK_TILE_START, 0);
      if (ts1 - ts0 != (c + kTileM - 1) / kTileM) fail(p.ctrl, MOE_CHECK_TILE_START, e + 1);
      if (e == nb - 1 && (ts1 < 0 || static_cast<int64_t>(ts1) * kTileM > p.npad))
        fail(p.ctrl, MOE_CHECK_TILE_START, e + 1);
    } else if (i < nb + n_assign) {
      // ---- per assignment (token t, selection k)
      const int64_t j = i - nb;
      const int t = static_cast<int>(j / p.top_k), k = static_cast<int>(j % p.top_k);
      const int idx = p.topk_idx[j];
      if (!finite(p.topk_weights[j])) fail(p.ctrl, MOE_CHECK_TOPK_WEIGHT, j);
      if (idx < 0 || idx >= p.E_global) {
        fail(p.ctrl, MOE_CHECK_TOPK_IDX, j);
        continue;
      }
      bool repeated = false;
      for (int k2 = 0; k2 < k; ++k2)
        repeated |= p.topk_idx[static_cast<int64_t>(t) * p.top_k + k2] == idx;
      if (repeated) fail(p.ctrl, MOE_CHECK_TOPK_IDX, j);
      if (!p.assign_row) continue;
      const int r = p.assign_row[j];
      const int le = idx - p.local_expert_offset;
      if (le < 0 || le >= p.E_local) {
        if (r != -1) fail(p.ctrl, MOE_CHECK_ASSIGN_ROW, j);
        continue;
      }
      const int64_t lo = static_cast<int64_t>(p.tile_start[le]) * kTileM;
      const int64_t hi = lo + p.counts[le];
      if (r < lo || r >= hi || r < 0 || r >= p.npad || p.row_token[r] != t)
        fail(p.ctrl, MOE_CHECK_ASSIGN_ROW, j);
    } else {
      // ---- per permuted row: live rows hold an assignment of their expert
      const int64_t r = i - nb - n_assign;
      const int e = expert_of_row(p.tile_start, nb, r);
      if (e < 0) continue;   // past the last bucket's tiles
      const int64_t row0 = static_cast<int64_t>(p.tile_start[e]) * kTileM;
      const int64_t live_end = row0 + p.counts[e];
      if (r >= live_end) continue;   // padding row of the bucket's last tile
      const int tok = p.row_token[r];
      if (tok < 0 || tok >= p.T) {
        fail(p.ctrl, MOE_CHECK_ROW_TOKEN, r);
        continue;
      }
      if (e == p.E_local) {   // shared expert: token r - row0, weight 1
        if (tok != r - row0) fail(p.ctrl, MOE_CHECK_ROW_EXPERT, r);
        if (p.row_weight[r] != 1.f) fail(p.ctrl, MOE_CHECK_ROW_WEIGHT, r);
        continue;
      }
      const int g = e + p.local_expert_offset;
      int k = -1;
      for (int k2 = 0; k2 < p.top_k; ++k2)
        if (k < 0 && p.topk_idx[static_cast<int64_t>(tok) * p.top_k + k2] == g) k = k2;
      if (k < 0) {
        fail(p.ctrl, MOE_CHECK_ROW_EXPERT, r);
        continue;
      }
      if (__float_as_uint(p.row_weight[r]) !=
          __float_as_uint(p.topk_weights[static_cast<int64_t>(tok) * p.top_k + k]))
        fail(p.ctrl, MOE_CHECK_ROW_WEIGHT, r);
    }
  }
}

// Guard pattern: four words spelling "MOE" and the guard's number, so a guard
// copied onto another still differs.
__device__ __forceinline__ uint4 guard_pattern(int i) {
  return make_uint4(0x4D4F4547u, 0x55415244u, 0xA5C3E1F0u, 0x00B20000u + static_cast<unsigned>(i));
}

__global__ void moe_guard_kernel(GuardList g, int write, CtrlBlock* ctrl) {
  for (int i = threadIdx.x; i < g.n; i += blockDim.x) {
    uint4* at = reinterpret_cast<uint4*>(g.base + g.off[i]);
    const uint4 want = guard_pattern(i);
    if (write) {
      *at = want;
    } else {
      const uint4 v = *at;
      if (v.x != want.x || v.y != want.y || v.z != want.z || v.w != want.w)
        fail(ctrl, MOE_CHECK_GUARD, i);
    }
  }
}

}  // namespace moe
