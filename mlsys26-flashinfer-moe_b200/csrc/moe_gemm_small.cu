// Grouped GEMMs for decode-shaped batches (a few rows per expert), with the
// operands swapped: the expert's weight rows are the MMA's M=128 operand and
// up to 16 of its permuted token rows the N=16 operand.
//
// With 128-row token tiles a decode step would spend a full promotion pass
// (two 256-column TMEM round trips per thread) on every 128-deep K block for
// one to eight real rows.  Here a TMEM accumulator group is 128 lanes x 32
// columns per 128-deep K block, sixteen of them fit in the 512 allocated
// columns (one CTA per SM), so the tensor core runs up to sixteen K blocks ahead
// of the promotion.  The promotion's cost per group, not its latency, is what
// bounds these kernels: a group covering less than a whole K block (16-column
// groups per 64-deep half in GEMM2) made GEMM2 1.27x slower.
//
// One CTA per SM walks work units (expert, 128 output features, 16 token rows):
//   warps 0-3  promotion + epilogue; thread (warp q, lane l) owns output feature
//              32q + l of the unit for all 16 token columns.
//   warp 4     TMA producer: per 128-deep K block the weight box(es) 128 x 128
//              and the 16 x 128 token box, into a ring of Cfg::kStages stages.
//   warp 5     MMA issuer: tcgen05.mma kind::f8f6f4, M=128 N=16 K=32.
// Every kernel of a forward after the first is launched with programmatic
// stream serialisation: barrier set-up, TMEM allocation and tensor-map prefetch
// run before griddepcontrol.wait, overlapping the previous kernel's tail.
//
// kGemm1 (reference moe_gemm1_kernel, kernel.py:7-151): per K block two MMA
//   chains into the two 16-column halves of the group, X1 = rows n*128.. of
//   W1[e] (multiplied) and X2 = rows I + n*128.. (SiLU input); epilogue
//   C = silu(X2) * X1, amax over 64 features (two warps), scale =
//   max(amax/448, 1e-12), C * (1/scale) -> e4m3, written to the intermediate.
// kGemm2 (reference moe_gemm2_kernel, kernel.py:153-250): W2[e] rows n*128..;
//   the two 64-deep halves of a K block (one 1x64 intermediate scale block
//   each) go to the two 16-column halves of the group; epilogue out[token] +=
//   weight * D with fp32 reductions, 128 contiguous floats per token and warp.
#include "moe_kernels.cuh"

namespace moe {

namespace {

constexpr int kSmallN = 16;                // token rows per unit (MMA N)
constexpr int kSmallThreads = 192;
constexpr int kSmallTmemCols = 512;        // all of TMEM: one CTA per SM
constexpr int kSmallBufsMax = 32;          // barrier slots for TMEM accumulator groups
constexpr int kTokBytes = kSmallN * kBlockK;   // 2 KB token box per K block
// Scale blocks per unit staged in shared memory: activation / intermediate
// scale blocks (H/128 for GEMM1, I/64 for GEMM2) x 16 token rows, and the
// weight scales (2 x H/128 for GEMM1, I/128 for GEMM2).  Two copies, by unit
// parity.
constexpr int kSmallMaxBlk = static_cast<int>(kSmallMaxScaleBlocks);
constexpr int kSmallSwOff = kSmallMaxBlk * kSmallN;
constexpr int kSmallRowOff = kSmallSwOff + 2 * kSmallMaxBlk;   // GEMM2: token, weight of the 16 rows
constexpr int kSmallScaleFloats = kSmallRowOff + 2 * kSmallN;

template <int kMode>
struct SmallCfg {
  static constexpr int kWBytes = kMode == kGemm1 ? 2 * kTileM * kBlockK : kTileM * kBlockK;
  static constexpr int kStageBytes = kWBytes + kTokBytes;
  static constexpr int kStages = kMode == kGemm1 ? 6 : 11;
  // One TMEM group per K block, 2 x 16 columns: the X1 and X2 chains in GEMM1,
  // the two 64-deep halves in GEMM2; 16 groups in the 512 allocated columns.
  static constexpr int kBufCols = 2 * kSmallN;
  static constexpr int kBufs = kSmallTmemCols / kBufCols;
  static_assert(kBufs <= kSmallBufsMax, "TMEM groups exceed the barrier slots");
};

template <int kMode>
constexpr int small_smem_bytes() {
  return 1024 + SmallCfg<kMode>::kStages * SmallCfg<kMode>::kStageBytes +
         2 * kSmallScaleFloats * 4 + 4096 + (2 * kMaxBuckets + 2) * 4;
}
static_assert(small_smem_bytes<kGemm1>() <= kMaxDynSmemBytes, "decode GEMM1 exceeds shared memory");
static_assert(small_smem_bytes<kGemm2>() <= kMaxDynSmemBytes, "decode GEMM2 exceeds shared memory");

struct SmallUnit {
  int e, n, row0, nrows;
};

__device__ __forceinline__ SmallUnit decode_small(int u, const int* ustart, const int* counts,
                                                  const int* tstart, int E, int NT) {
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (ustart[mid] <= u) lo = mid;
    else hi = mid - 1;
  }
  SmallUnit c;
  c.e = lo;
  const int mt = (counts[lo] + kSmallN - 1) / kSmallN;
  const int l = u - ustart[lo];
  c.n = l / mt;
  const int t = l - c.n * mt;
  c.row0 = tstart[lo] * kTileM + t * kSmallN;
  c.nrows = min(kSmallN, counts[lo] - t * kSmallN);
  return c;
}

// A CTA's work as segments (unit, K blocks [kb0, kb1)).  Units are whole and
// dealt round-robin, except in GEMM2 when there are few of them (`split`:
// fewer than kSplitUnitsPerCta per CTA, where a partial last wave would leave
// SMs idle): then the flattened (unit, K block) space is cut into one
// contiguous range per CTA, so every CTA streams the same number of weight
// tiles, and the pieces of a unit cut between CTAs each add their partial
// product to the output (exact with the epilogue's fp32 reductions).  GEMM1
// is never split: its SwiGLU needs whole sums, and measured at one token the
// fix-up of split units cost more than the idle SMs.
constexpr int kSplitUnitsPerCta = 8;

struct Seg {
  int u, kb0, kb1;   // u < 0: no more work
};

struct SegSpace {
  bool split;
  int total_units, KB;
  int64_t n_items;   // total_units * KB
  int ctas;          // CTAs with work in split mode: min(grid, n_items), each range non-empty
  __device__ __forceinline__ int64_t lo(int b) const { return static_cast<int64_t>(b) * n_items / ctas; }
  __device__ __forceinline__ Seg first() const {
    const int b = blockIdx.x;
    if (!split) return b < total_units ? Seg{b, 0, KB} : Seg{-1, 0, 0};
    if (b >= ctas) return Seg{-1, 0, 0};
    const int64_t a = lo(b), e = lo(b + 1);
    const int u = static_cast<int>(a / KB);
    const int kb0 = static_cast<int>(a - static_cast<int64_t>(u) * KB);
    return Seg{u, kb0, static_cast<int>(min(static_cast<int64_t>(KB), kb0 + e - a))};
  }
  __device__ __forceinline__ Seg next(const Seg& sg) const {
    if (!split) {
      const int u = sg.u + static_cast<int>(gridDim.x);
      return u < total_units ? Seg{u, 0, KB} : Seg{-1, 0, 0};
    }
    const int64_t it = static_cast<int64_t>(sg.u) * KB + sg.kb1;
    const int64_t e = lo(static_cast<int>(blockIdx.x) + 1);
    if (it >= e) return Seg{-1, 0, 0};
    return Seg{sg.u + 1, 0, static_cast<int>(min(static_cast<int64_t>(KB), e - it))};
  }
};

__device__ __forceinline__ SegSpace make_seg_space(int total_units, int KB, bool may_split) {
  SegSpace sp;
  sp.total_units = total_units;
  sp.KB = KB;
  sp.n_items = static_cast<int64_t>(total_units) * KB;
  sp.split = may_split && total_units > 0 &&
             total_units < kSplitUnitsPerCta * static_cast<int>(gridDim.x);
  sp.ctas = static_cast<int>(min(static_cast<int64_t>(gridDim.x), sp.n_items));
  return sp;
}

__device__ __forceinline__ void drain_wait_s(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitLimitNs) return;
  }
}

// Barrier among the four promotion warps on an mbarrier (count 4, one arrival
// per warp), so that a warp leaving after an abort cannot strand the others.
__device__ __forceinline__ bool epi_sync(uint64_t* bar, uint32_t& phase, int lane,
                                         volatile int* abort, CtrlBlock* ctrl) {
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
  const bool ok = mbar_wait(bar, phase & 1u, abort, ctrl, 16);
  ++phase;
  return ok;
}

}  // namespace

template <int kMode>
__global__ void __launch_bounds__(kSmallThreads, 1)
    moe_gemm_small_kernel(const __grid_constant__ CUtensorMap tm_w,
                          const __grid_constant__ CUtensorMap tm_tok, GemmParams p) {
  using Cfg = SmallCfg<kMode>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sW = smem;                                   // S x kWBytes (1024-aligned)
  uint8_t* sT = smem + S * Cfg::kWBytes;                // S x 2 KB
  float* scale_s = reinterpret_cast<float*>(sT + S * kTokBytes);   // [2][kSmallScaleFloats]
  uint64_t* full = reinterpret_cast<uint64_t*>(scale_s + 2 * kSmallScaleFloats);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + kSmallBufsMax;
  uint64_t* drain = tempty + kSmallBufsMax;
  uint64_t* ebar = drain + 1;
  uint64_t* never = ebar + 1;      // failure-detection tests: completed by nothing
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(never + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);   // [1]: wait limit
  float* red_s = reinterpret_cast<float*>(tmem_slot + 4);     // [4][16] amax exchange
  int* ustart_s = reinterpret_cast<int*>(red_s + 4 * kSmallN);
  int* counts_s = ustart_s + kMaxBuckets + 1;
  int* tstart_s = counts_s + kMaxBuckets;
  int* skip_s = tstart_s + kMaxBuckets;   // debug checks failed: no units

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = p.E_local, NT = p.n_tiles, KB = p.num_k_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < Cfg::kBufs; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(drain, 1);
    mbar_init(ebar, 4);
    mbar_init(never, 1);
    abort_flag[0] = 0;
    abort_flag[1] = static_cast<int>(p.wait_limit_us);
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, kSmallTmemCols);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_tok);
  }
  // Everything above only touches this CTA's own resources.  GEMM1 waits for
  // the routing kernels (programmatic dependent launch) before it lets GEMM2
  // launch, so when GEMM2 starts the routing tables are complete: GEMM2 reads
  // them, and streams its first weight tiles, before it waits for GEMM1 (see
  // the producer); everything GEMM1 writes is read after that wait.
  if constexpr (kMode == kGemm1) {
    griddep_wait();
    griddep_launch_dependents();
  }
  for (int i = threadIdx.x; i < E; i += kSmallThreads) {
    counts_s[i] = p.counts[i];
    tstart_s[i] = p.tile_start[i];
  }
  if (threadIdx.x == 0)
    *skip_s = p.skip_on_error && *reinterpret_cast<volatile const int*>(&p.ctrl->error) != 0;
  __syncthreads();
  if (warp == 0) {
    // Unit prefix over the buckets: NT x ceil(count / 16) units each, warp
    // scan of kPerLane buckets per lane (32 * kPerLane > kMaxBuckets, so the
    // lanes also cover index E, the total).
    constexpr int kPerLane = (kMaxBuckets + 31) / 32;
    static_assert(32 * kPerLane > kMaxBuckets, "the scan must reach index E");
    int local[kPerLane];
    int sum = 0;
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) {
      const int e = lane * kPerLane + j;
      const int v = e < E ? NT * ((counts_s[e] + kSmallN - 1) / kSmallN) : 0;
      local[j] = sum;
      sum += v;
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const int base = incl - sum;
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) {
      const int e = lane * kPerLane + j;
      if (e <= E) ustart_s[e] = base + local[j];
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total_units = *skip_s ? 0 : ustart_s[E];
  // Split units add partial products, which the deterministic combine's
  // stored rows cannot take.
  const SegSpace segs = make_seg_space(total_units, KB, kMode == kGemm2 && p.rows_out == nullptr);
  if constexpr (kMode == kGemm2) {
    griddep_launch_dependents();
    if (!(warp == 4 && lane == 0)) griddep_wait();   // the producer waits after its early loads
  }

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, issued_phase = 0;
      // GEMM2: the weight boxes of the first S stages (items 0..S-1 of this
      // CTA, stages 0..S-1 of the first ring pass) go out before the wait for
      // GEMM1; the items' token boxes, which GEMM1 writes, after it.  Each
      // stage's barrier expects both boxes either way.
      int early = 0;
      if constexpr (kMode == kGemm2) {
        for (Seg sg = segs.first(); sg.u >= 0 && early < S; sg = segs.next(sg)) {
          const SmallUnit c = decode_small(sg.u, ustart_s, counts_s, tstart_s, E, NT);
          const int w_row0 = c.e * p.b_rows_per_expert + c.n * kTileM;
          for (int kb = sg.kb0; kb < sg.kb1 && early < S; ++kb, ++early) {
            mbar_arrive_expect_tx(&full[early], Cfg::kStageBytes);
            tma_load_2d(sW + early * Cfg::kWBytes, &tm_w, &full[early], kb * kBlockK, w_row0);
            issued |= 1u << early;
          }
        }
        griddep_wait();
      }
      int item = 0;
      for (Seg sg = segs.first(); sg.u >= 0; sg = segs.next(sg)) {
        const SmallUnit c = decode_small(sg.u, ustart_s, counts_s, tstart_s, E, NT);
        const int w_row0 = c.e * p.b_rows_per_expert + c.n * kTileM;
        for (int kb = sg.kb0; kb < sg.kb1; ++kb, ++item) {
          if (item >= early) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.ctrl, 11)) goto producer_done;
            mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
            uint8_t* w_dst = sW + stage * Cfg::kWBytes;
            tma_load_2d(w_dst, &tm_w, &full[stage], kb * kBlockK, w_row0);
            if constexpr (kMode == kGemm1)
              tma_load_2d(w_dst + kTileM * kBlockK, &tm_w, &full[stage], kb * kBlockK,
                          w_row0 + p.inter);
          }
          tma_load_2d(sT + stage * kTokBytes, &tm_tok, &full[stage], kb * kBlockK, c.row0);
          issued |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:
      // Every load this thread issued lands before the CTA can exit, also
      // when a consumer gave up on its stage (abort raised at any time).
      for (int s = 0; s < S; ++s)
        if (issued & (1u << s)) drain_wait_s(&full[s], (issued_phase >> s) & 1u);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_e4m3_f32(kTileM, kSmallN);
      const uint64_t w_desc0 = umma_desc_sw128(smem_u32(sW));
      const uint64_t t_desc0 = umma_desc_sw128(smem_u32(sT));
      int stage = 0;
      uint32_t phase = 0;
      uint32_t g = 0;
      if (kMode == kGemm1 && p.stall && !mbar_wait(never, 0, abort_flag, p.ctrl, 19))
        goto mma_done;
      for (Seg sg = segs.first(); sg.u >= 0; sg = segs.next(sg)) {
        for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.ctrl, 12)) goto mma_done;
          tc_fence_after();
          const uint64_t wd = w_desc0 + ((static_cast<uint32_t>(stage) * Cfg::kWBytes) >> 4);
          const uint64_t td = t_desc0 + ((static_cast<uint32_t>(stage) * kTokBytes) >> 4);
          {
            const uint32_t buf = g % Cfg::kBufs;
            const uint32_t free_parity = ((g / Cfg::kBufs) & 1u) ^ 1u;
            ++g;
            if (!mbar_wait(&tempty[buf], free_parity, abort_flag, p.ctrl, 13))
              goto mma_done;
            tc_fence_after();
            const uint32_t d = tmem_base + buf * Cfg::kBufCols;
            if constexpr (kMode == kGemm1) {
              uint64_t a[4], b[4], a2[4];
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                a[kk] = wd + ((kk * 32) >> 4);
                a2[kk] = wd + ((kTileM * kBlockK + kk * 32) >> 4);
                b[kk] = td + ((kk * 32) >> 4);
              }
              umma_f8_group<4>(d, a, b, idesc);
              umma_f8_group<4>(d + kSmallN, a2, b, idesc);
            } else {
              // the two 64-deep halves (one intermediate scale block each)
              // into the two 16-column halves of the group
              uint64_t a[2], b[2], a2[2], b2[2];
#pragma unroll
              for (int kk = 0; kk < 2; ++kk) {
                a[kk] = wd + ((kk * 32) >> 4);
                b[kk] = td + ((kk * 32) >> 4);
                a2[kk] = wd + ((64 + kk * 32) >> 4);
                b2[kk] = td + ((64 + kk * 32) >> 4);
              }
              umma_f8_group<2>(d, a, b, idesc);
              umma_f8_group<2>(d + kSmallN, a2, b2, idesc);
            }
            umma_commit(&tfull[buf]);
          }
          umma_commit(&empty[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    mma_done:
      umma_commit(drain);
      drain_wait_s(drain, 0);
    }
  } else {
    // ------------------------------------------------------------ promotion + epilogue
    const int q = warp;                       // TMEM lane quarter = feature rows 32q..
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    uint32_t g = 0;
    uint32_t ephase = 0;
    uint32_t unit_parity = 0;
    // Copies the scales of unit cu into dst: activation / intermediate scale
    // blocks x 16 rows, then the weight scales.
    auto stage_scales = [&](const SmallUnit& cu, float* dst) {
      float* dst_w = dst + kSmallSwOff;
      const int nblk = kMode == kGemm1 ? KB : 2 * KB;
      for (int i = threadIdx.x; i < nblk * kSmallN; i += 128)
        cp_async4(smem_u32(dst + i),
                  p.a_scale + static_cast<int64_t>(i >> 4) * p.npad + cu.row0 + (i & 15));
      if constexpr (kMode == kGemm1) {
        // W1 scale [E, 2I/128, H/128]: X1 block n, X2 block I/128 + n.
        const int ib = p.inter / kBlockK;
        const float* ws_x1 = p.b_scale + (static_cast<int64_t>(cu.e) * 2 * ib + cu.n) * KB;
        for (int i = threadIdx.x; i < 2 * KB; i += 128)
          cp_async4(smem_u32(dst_w + i), ws_x1 + (i < KB ? i : static_cast<int64_t>(ib) * KB + i - KB));
      } else {
        // W2 scale [E, H/128, I/128].
        const float* ws = p.b_scale + (static_cast<int64_t>(cu.e) * (p.hidden / kBlockK) + cu.n) * KB;
        for (int i = threadIdx.x; i < KB; i += 128) cp_async4(smem_u32(dst_w + i), ws + i);
        // token and routing weight of the 16 rows, read by the unit's output
        // step (rows past the expert's count are padding and never used)
        if (threadIdx.x < 2 * kSmallN) {
          const int j = threadIdx.x & (kSmallN - 1);
          const void* src = threadIdx.x < kSmallN ? static_cast<const void*>(p.row_token + cu.row0 + j)
                                                  : static_cast<const void*>(p.row_weight + cu.row0 + j);
          cp_async4(smem_u32(dst + kSmallRowOff + threadIdx.x), src);
        }
      }
      cp_async_commit();
    };
    const Seg first = segs.first();
    if (first.u >= 0) stage_scales(decode_small(first.u, ustart_s, counts_s, tstart_s, E, NT), scale_s);
    for (Seg sg = first; sg.u >= 0; sg = segs.next(sg)) {
      const SmallUnit c = decode_small(sg.u, ustart_s, counts_s, tstart_s, E, NT);
      constexpr int kAcc = kMode == kGemm1 ? 2 * kSmallN : kSmallN;
      float acc[kAcc];
#pragma unroll
      for (int i = 0; i < kAcc; ++i) acc[i] = 0.f;
      // The unit's scales were staged in shared memory by 4-byte cp.async
      // copies issued during the previous unit (one DRAM round trip per unit,
      // hidden behind that unit's work); wait for this thread's copies, then for
      // every warp's.
      float* sc = scale_s + (unit_parity & 1u) * kSmallScaleFloats;
      float* sc_w = sc + kSmallSwOff;
      ++unit_parity;
      cp_async_wait_all();
      if (!epi_sync(ebar, ephase, lane, abort_flag, p.ctrl)) goto epi_done;
      // All warps are past the previous unit: its copy can take the next unit's.
      const Seg nx = segs.next(sg);
      if (nx.u >= 0)
        stage_scales(decode_small(nx.u, ustart_s, counts_s, tstart_s, E, NT),
                     scale_s + (unit_parity & 1u) * kSmallScaleFloats);
      if constexpr (kMode == kGemm1) {
        // Groups are consumed kBatch1 at a time: all their TMEM loads go out
        // before one tcgen05.wait::ld, so a batch costs one TMEM round trip.
        constexpr int kBatch1 = 2;
        const int kb_end = sg.kb1;
        for (int kb0 = sg.kb0; kb0 < kb_end; kb0 += kBatch1) {
          uint32_t bufs[kBatch1];
#pragma unroll
          for (int bi = 0; bi < kBatch1; ++bi) {
            const uint32_t gg = g + bi;
            bufs[bi] = gg % Cfg::kBufs;
            if (kb0 + bi < kb_end &&
                !mbar_wait(&tfull[bufs[bi]], (gg / Cfg::kBufs) & 1u, abort_flag, p.ctrl, 14))
              goto epi_done;
          }
          tc_fence_after();
          float v[kBatch1][32];
#pragma unroll
          for (int bi = 0; bi < kBatch1; ++bi)
            if (kb0 + bi < kb_end) tmem_ld32(t_lane + bufs[bi] * Cfg::kBufCols, v[bi]);
          tmem_ld_wait();
          tc_fence_before();
          __syncwarp();
#pragma unroll
          for (int bi = 0; bi < kBatch1; ++bi)
            if (kb0 + bi < kb_end && lane == 0) mbar_arrive(&tempty[bufs[bi]]);
#pragma unroll
          for (int bi = 0; bi < kBatch1; ++bi) {
            const int kb = kb0 + bi;
            if (kb < kb_end) {
              const float w1 = sc_w[kb], w2 = sc_w[KB + kb];
              const float4* s4 = reinterpret_cast<const float4*>(sc + kb * kSmallN);
#pragma unroll
              for (int j4 = 0; j4 < 4; ++j4) {
                const float4 f = s4[j4];
                const float sa[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                  const int j = 4 * j4 + jj;
                  acc[j] = fmaf(v[bi][j], sa[jj] * w1, acc[j]);
                  acc[kSmallN + j] = fmaf(v[bi][kSmallN + j], sa[jj] * w2, acc[kSmallN + j]);
                }
              }
              ++g;
            }
          }
        }
        // SwiGLU + 1x64 requant (kernel.py:128-151): amax over the 64 features
        // of this thread's half (warps 0-1 or 2-3) for every token column.
        float cv[kSmallN];
#pragma unroll
        for (int j = 0; j < kSmallN; ++j) {
          const float x1 = acc[j], x2 = acc[kSmallN + j];
          cv[j] = __fdividef(x2, 1.0f + __expf(-x2)) * x1;   // as the prefill GEMM1
          float m = fabsf(cv[j]);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          if (lane == 0) red_s[q * kSmallN + j] = m;
        }
        if (!epi_sync(ebar, ephase, lane, abort_flag, p.ctrl)) goto epi_done;
        const int qp = q ^ 1;
        const int col = c.n * kTileM + q * 32 + lane;
#pragma unroll
        for (int j = 0; j < kSmallN; ++j) {
          if (j < c.nrows) {
            const float amax = fmaxf(red_s[q * kSmallN + j], red_s[qp * kSmallN + j]);
            const float sc = fmaxf(amax / 448.0f, 1e-12f);
            const float inv = 1.0f / sc;
            const int64_t row = static_cast<int64_t>(c.row0) + j;
            p.inter_out[row * p.inter + col] = static_cast<uint8_t>(pack_e4m3x2(cv[j] * inv, 0.f) & 0xffu);
            if (lane == 0 && (q & 1) == 0)
              p.inter_scale[static_cast<int64_t>(2 * c.n + (q >> 1)) * p.npad + row] = sc;
          }
        }
        // red_s is rewritten by the next unit
        if (!epi_sync(ebar, ephase, lane, abort_flag, p.ctrl)) goto epi_done;
      } else {
        // One TMEM group per K block, its two 16-column halves holding the two
        // 64-deep partial products (one intermediate scale block each);
        // consumed kBatch2 groups at a time, as in GEMM1.
        constexpr int kBatch2 = 4;
        const int kb_end = sg.kb1;
        for (int kb0 = sg.kb0; kb0 < kb_end; kb0 += kBatch2) {
          uint32_t bufs[kBatch2];
#pragma unroll
          for (int bi = 0; bi < kBatch2; ++bi) {
            const uint32_t gg = g + bi;
            bufs[bi] = gg % Cfg::kBufs;
            if (kb0 + bi < kb_end &&
                !mbar_wait(&tfull[bufs[bi]], (gg / Cfg::kBufs) & 1u, abort_flag, p.ctrl, 15))
              goto epi_done;
          }
          tc_fence_after();
          float v[kBatch2][2 * kSmallN];
#pragma unroll
          for (int bi = 0; bi < kBatch2; ++bi)
            if (kb0 + bi < kb_end) tmem_ld32(t_lane + bufs[bi] * Cfg::kBufCols, v[bi]);
          tmem_ld_wait();
          tc_fence_before();
          __syncwarp();
#pragma unroll
          for (int bi = 0; bi < kBatch2; ++bi)
            if (kb0 + bi < kb_end && lane == 0) mbar_arrive(&tempty[bufs[bi]]);
#pragma unroll
          for (int bi = 0; bi < kBatch2; ++bi) {
            const int kb = kb0 + bi;
            if (kb < kb_end) {
              const float sw = sc_w[kb];
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const float4* s4 = reinterpret_cast<const float4*>(sc + (2 * kb + h) * kSmallN);
#pragma unroll
                for (int j4 = 0; j4 < 4; ++j4) {
                  const float4 f = s4[j4];
                  const float* vv = v[bi] + h * kSmallN + 4 * j4;
                  acc[4 * j4] = fmaf(vv[0], f.x * sw, acc[4 * j4]);
                  acc[4 * j4 + 1] = fmaf(vv[1], f.y * sw, acc[4 * j4 + 1]);
                  acc[4 * j4 + 2] = fmaf(vv[2], f.z * sw, acc[4 * j4 + 2]);
                  acc[4 * j4 + 3] = fmaf(vv[3], f.w * sw, acc[4 * j4 + 3]);
                }
              }
              ++g;
            }
          }
        }
        // out[token] += weight * D (kernel.py:236-250): per token, the warp's 32
        // lanes add 32 consecutive floats.  The choice between adding and the
        // deterministic combine's stores is made once per unit, outside the
        // unrolled loop (a per-element branch made the adds 16% slower at T=64).
        const int col = c.n * kTileM + q * 32 + lane;
        if (p.rows_out == nullptr) {
#pragma unroll
          for (int j = 0; j < kSmallN; ++j) {
            if (j < c.nrows) {
              const int tok = reinterpret_cast<const int*>(sc + kSmallRowOff)[j];
              const float w = sc[kSmallRowOff + kSmallN + j];
              atomicAdd(p.out_f32 + static_cast<int64_t>(tok) * p.hidden + col, acc[j] * w);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < kSmallN; ++j) {
            if (j < c.nrows) {   // deterministic combine: the row's own line
              const int64_t row = static_cast<int64_t>(c.row0) + j;
              p.rows_out[row * p.hidden + col] = acc[j] * sc[kSmallRowOff + kSmallN + j];
            }
          }
        }
      }
    }
  epi_done:
    cp_async_wait_all();   // scale copies still in flight after an abort
    if constexpr (kMode == kGemm2) {
      if (p.final_out != nullptr) {
        // Small batches: the last CTA to get here turns the fp32 accumulator
        // into the bf16 output (moe_finalize_kernel's work) without another
        // launch.  Every path out of the loop above reaches these barriers.
        volatile int* last = reinterpret_cast<volatile int*>(red_s);
        __threadfence();   // this thread's reductions into out_f32
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (threadIdx.x == 0)
          *last = atomicAdd(&p.ctrl->gemm_done, 1u) == gridDim.x - 1 ? 1 : 0;
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (*last) {
          __threadfence();
          const float4* in = reinterpret_cast<const float4*>(p.out_f32);
          uint4* out = reinterpret_cast<uint4*>(p.final_out);
          // eight 8-float chunks per thread in flight before their stores
          for (int64_t i0 = threadIdx.x; i0 < p.final_n8; i0 += 8 * 128) {
            float4 a[8], b[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int64_t i = i0 + k * 128;
              if (i < p.final_n8) {
                a[k] = __ldcg(in + 2 * i);
                b[k] = __ldcg(in + 2 * i + 1);
              }
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int64_t i = i0 + k * 128;
              if (i < p.final_n8) {
                __nv_bfloat162 r[4];
                r[0] = __floats2bfloat162_rn(a[k].x, a[k].y);
                r[1] = __floats2bfloat162_rn(a[k].z, a[k].w);
                r[2] = __floats2bfloat162_rn(b[k].x, b[k].y);
                r[3] = __floats2bfloat162_rn(b[k].z, b[k].w);
                out[i] = *reinterpret_cast<uint4*>(r);
              }
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kSmallTmemCols);
  }
}

int gemm_small_set_smem_attrs() {
  if (cudaFuncSetAttribute(moe_gemm_small_kernel<kGemm1>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           small_smem_bytes<kGemm1>()) != cudaSuccess)
    return MOE_ERR_CUDA;
  if (cudaFuncSetAttribute(moe_gemm_small_kernel<kGemm2>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           small_smem_bytes<kGemm2>()) != cudaSuccess)
    return MOE_ERR_CUDA;
  return MOE_OK;
}

int launch_gemm_small(int mode, const CUtensorMap& tm_w, const CUtensorMap& tm_tok,
                      const GemmParams& p, int grid, cudaStream_t stream) {
  // Both kernels wait for their predecessor inside (griddep_wait) after a
  // prologue that only touches their own shared memory and TMEM.
  const cudaError_t e =
      mode == kGemm1
          ? launch_programmatic(moe_gemm_small_kernel<kGemm1>, dim3(grid), dim3(kSmallThreads),
                                small_smem_bytes<kGemm1>(), stream, tm_w, tm_tok, p)
          : launch_programmatic(moe_gemm_small_kernel<kGemm2>, dim3(grid), dim3(kSmallThreads),
                                small_smem_bytes<kGemm2>(), stream, tm_w, tm_tok, p);
  return e == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

}  // namespace moe
