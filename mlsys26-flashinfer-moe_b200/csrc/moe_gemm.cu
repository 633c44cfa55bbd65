// Persistent warp-specialised grouped GEMMs of the MoE forward on tcgen05.
//
// One CTA per SM walks a static list of work units (expert tile of 128
// permuted rows x 256 output columns).  Roles:
//   Warpgroup 2 (warps 8-11) gives registers to warpgroups 0-1 with setmaxnreg.
//   warp 8  (one thread)  TMA producer: A tile 128x128 and B tile 256x128 (two
//                         128-row boxes) per 128-deep K block, 4-stage ring.
//   warps 9, 10 (one thread each) MMA issuers, one per TMEM partial buffer:
//                         tcgen05.mma kind::f8f6f4 (e4m3 x e4m3 -> fp32),
//                         M=128 N=256 K=32, into one of two 256-column TMEM
//                         partial accumulators.
//   warps 0-7             Block-scale promotion and epilogue.  FP8 operands
//                         carry one fp32 scale per 128 (A, W) or 64 (the
//                         intermediate) K elements, which the tensor core
//                         cannot apply, so every partial accumulator covers
//                         exactly one scale block and is folded into fp32
//                         registers as acc += partial * (sa[row] * sw[block]),
//                         reading 64 TMEM columns per wait.  Only two partials
//                         fit in TMEM, so the time a buffer is held bounds the
//                         tensor core: a warp releases it right after its last
//                         tcgen05.ld and does the remaining FMAs afterwards.
//                         Warp w reads TMEM lanes 32*(w%4).. and column half
//                         w/4, so each thread owns one row and 128 columns.
//
// kGemm1 (reference moe_gemm1_kernel, kernel.py:7-151): B rows are the gate
//   half W1[e, n*128 : n*128+128] (multiplied, X1) followed by the SiLU half
//   W1[e, I + n*128 : ...] (X2); epilogue C = silu(X2) * X1, per-row amax over
//   64 columns, scale = max(amax/448, 1e-12), C/scale -> e4m3.
// kGemm2 (reference moe_gemm2_kernel, kernel.py:153-250): B rows are
//   W2[e, n*256 : n*256+256]; epilogue multiplies by the routing weight and
//   does an fp32 vector reduction into out[token] (kernel.py:236-250).
#include "moe_kernels.cuh"

namespace moe {

namespace {

struct Unit {
  int e, m, n, row0, nrows;
};

// Unit u -> (expert, tile of the expert, N tile).  Experts own the contiguous
// unit range [tile_start[e]*NT, tile_start[e+1]*NT); inside it the N tile is
// the outer index so the expert's row tiles reuse each weight tile from L2.
__device__ __forceinline__ Unit decode_unit(int u, const int* tstart, const int* counts, int E,
                                            int NT) {
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tstart[mid] * NT <= u) lo = mid;
    else hi = mid - 1;
  }
  Unit c;
  c.e = lo;
  const int mt = tstart[lo + 1] - tstart[lo];
  const int l = u - tstart[lo] * NT;
  c.n = l / mt;
  c.m = l - c.n * mt;
  c.row0 = (tstart[lo] + c.m) * kTileM;
  c.nrows = min(kTileM, counts[lo] - c.m * kTileM);
  return c;
}

// Bounded wait that ignores the abort flag: used only to let copies and MMAs
// already in flight land before the CTA releases its shared memory and TMEM.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitLimitNs) return;
  }
}

// Byte offset of 16-byte chunk c (0..3) of row r (0..31) in a warp's 32 x 64 B
// staging tile.  The XOR swizzle keeps both access patterns free of bank
// conflicts: row-wise writes (a quarter-warp writes one chunk of 8 rows) and
// column-wise reads (a quarter-warp reads the 4 chunks of 2 rows) each touch 8
// distinct 16-byte bank groups.
__device__ __forceinline__ int xpose_off(int r, int c) { return r * 64 + ((c ^ ((r >> 1) & 3)) << 4); }

// acc[i] += v[i] * s for 64 values, two per paired fp32 FMA instruction (each
// lane of a pair rounds once, as fmaf does): half the issue slots of the
// promotion's FMAs (0.3-2% faster GEMM1 at T=8192, measured).
__device__ __forceinline__ void fma_pairs(float* acc, const float* v, float s) {
  const float2 s2 = make_float2(s, s);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float2 r = __ffma2_rn(make_float2(v[2 * i], v[2 * i + 1]), s2,
                                make_float2(acc[2 * i], acc[2 * i + 1]));
    acc[2 * i] = r.x;
    acc[2 * i + 1] = r.y;
  }
}

// Release a TMEM partial buffer once this warp's tcgen05.ld of it completed.
__device__ __forceinline__ void release_buffer(uint64_t* tempty, int lane) {
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(tempty);
}

}  // namespace

template <int kMode>
__global__ void __launch_bounds__(kGemmThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tm_a,
                    const __grid_constant__ CUtensorMap tm_b, GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kStageABytes;
  uint8_t* xpose = sB + kStages * kStageBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(xpose + kXposeBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* never = drain + 1;     // failure-detection tests: completed by nothing
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(never + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);   // [1]: wait limit
  int* tstart_s = reinterpret_cast<int*>(tmem_slot + 3);
  int* counts_s = tstart_s + kMaxBuckets + 1;
  int* skip_s = counts_s + kMaxBuckets;   // debug checks failed: no units

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = p.E_local, NT = p.n_tiles, KB = p.num_k_blocks;

  for (int i = threadIdx.x; i <= E; i += kGemmThreads) tstart_s[i] = p.tile_start[i];
  for (int i = threadIdx.x; i < E; i += kGemmThreads) counts_s[i] = p.counts[i];
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kMode == kGemm2 ? 2 : 1);   // one commit per scale group
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    mbar_init(drain, kMmaIssuers);
    mbar_init(never, 1);
    abort_flag[0] = 0;
    abort_flag[1] = static_cast<int>(p.wait_limit_us);
    *skip_s = p.skip_on_error && *reinterpret_cast<volatile const int*>(&p.ctrl->error) != 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total_units = *skip_s ? 0 : tstart_s[E] * NT;

  if (warp >= 8) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kControlRegs));
  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;              // bit s: stage s has a load in flight
      uint32_t issued_phase = 0;        // bit s: phase of that load
      for (int u = blockIdx.x; u < total_units; u += gridDim.x) {
        const Unit c = decode_unit(u, tstart_s, counts_s, E, NT);
        const int b_row0 = c.e * p.b_rows_per_expert +
                           (kMode == kGemm1 ? c.n * (kTileN / 2) : c.n * kTileN);
        const int b_row1 = kMode == kGemm1 ? b_row0 + p.inter : b_row0 + kTileN / 2;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.ctrl, 1)) goto producer_done;
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          uint8_t* a_dst = sA + stage * kStageABytes;
          uint8_t* b_dst = sB + stage * kStageBBytes;
          tma_load_2d(a_dst, &tm_a, &full[stage], kb * kBlockK, c.row0);
          tma_load_2d(b_dst, &tm_b, &full[stage], kb * kBlockK, b_row0);
          tma_load_2d(b_dst + kStageBBytes / 2, &tm_b, &full[stage], kb * kBlockK, b_row1);
          issued |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:
      // Every load this thread issued lands before the CTA can exit, also
      // when a consumer gave up on its stage (abort raised at any time).
      for (int s = 0; s < kStages; ++s)
        if (issued & (1u << s)) drain_wait(&full[s], (issued_phase >> s) & 1u);
    }
  } else if (warp == 9 || warp == 10) {
    // ------------------------------------------------------------ MMA issuers
    // Warp 9 issues every scale group that writes TMEM buffer 0, warp 10 every
    // group that writes buffer 1.  Each issuer waits only on its own buffer's
    // "released" barrier and visits the stages in K order, so no barrier it
    // waits on is ever more than one phase ahead (the parity waits need that),
    // and the cost of issuing is split over two sub-partitions.
    if constexpr (kMode == kGemm2Bf16) {
      // bf16 operands carry no block scales: warp 9 accumulates a unit's whole K
      // range into one TMEM buffer (unit parity), four K=16 MMAs per 128-byte
      // stage, and commits the buffer once per unit; warp 10 only joins the
      // drain.
      if (lane == 0 && warp == 9) {
        const uint32_t idesc = umma_idesc_bf16_f32(kTileM, kTileN);
        const uint64_t a_desc0 = umma_desc_sw128(smem_u32(sA));
        const uint64_t b_desc0 = umma_desc_sw128(smem_u32(sB));
        int stage = 0;
        uint32_t phase = 0;
        uint32_t ui = 0;
        for (int u = blockIdx.x; u < total_units; u += gridDim.x, ++ui) {
          const uint32_t buf = ui & 1u;
          if (!mbar_wait(&tempty[buf], ((ui >> 1) & 1u) ^ 1u, abort_flag, p.ctrl, 7))
            goto mma_done;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + buf * kTileN;
#pragma unroll 1
          for (int kb = 0; kb < KB; ++kb) {
            const uint64_t a_d = a_desc0 + ((static_cast<uint32_t>(stage) * kStageABytes) >> 4);
            const uint64_t b_d = b_desc0 + ((static_cast<uint32_t>(stage) * kStageBBytes) >> 4);
            if (!mbar_wait(&full[stage], phase, abort_flag, p.ctrl, 8)) goto mma_done;
            tc_fence_after();
            umma_bf16_x4(d_tmem, a_d, b_d, idesc, kb > 0 ? 1u : 0u);
            umma_commit(&empty[stage]);
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
          umma_commit(&tfull[buf]);
        }
      }
    } else if (lane == 0) {
      constexpr int kGroups = kMode == kGemm1 ? 1 : 2;   // scale blocks per K block
      constexpr int kMmaPerGroup = (kBlockK / 32) / kGroups;
      const uint32_t me = static_cast<uint32_t>(warp - 9);   // = the buffer it fills
      const uint32_t idesc = umma_idesc_e4m3_f32(kTileM, kTileN);
      const uint32_t d_tmem = tmem_base + me * kTileN;
      const uint64_t a_desc0 = umma_desc_sw128(smem_u32(sA));
      const uint64_t b_desc0 = umma_desc_sw128(smem_u32(sB));
      int stage = 0;
      uint32_t phase = 0;
      uint32_t g = 0;
      if (kMode == kGemm1 && p.stall && me == 0 &&
          !mbar_wait(never, 0, abort_flag, p.ctrl, 9))
        goto mma_done;
      for (int u = blockIdx.x; u < total_units; u += gridDim.x) {
        for (int kb = 0; kb < KB; ++kb) {
          bool have_stage = false;
#pragma unroll
          for (int gi = 0; gi < kGroups; ++gi, ++g) {
            if ((g & 1u) != me) continue;
            // Descriptors of this group's K slices: the start-address field is
            // the low bits, so slices and stages are plain offsets (>> 4).
            uint64_t a_d[kMmaPerGroup], b_d[kMmaPerGroup];
#pragma unroll
            for (int kk = 0; kk < kMmaPerGroup; ++kk) {
              const uint32_t koff = static_cast<uint32_t>((gi * kMmaPerGroup + kk) * 32);
              a_d[kk] = a_desc0 + ((static_cast<uint32_t>(stage) * kStageABytes + koff) >> 4);
              b_d[kk] = b_desc0 + ((static_cast<uint32_t>(stage) * kStageBBytes + koff) >> 4);
              materialize(a_d[kk]);
              materialize(b_d[kk]);
            }
            if (!have_stage) {
              if (!mbar_wait(&full[stage], phase, abort_flag, p.ctrl, 2)) goto mma_done;
              have_stage = true;
            }
            if (!mbar_wait(&tempty[me], ((g >> 1) & 1u) ^ 1u, abort_flag, p.ctrl, 3))
              goto mma_done;
            tc_fence_after();
            umma_f8_group<kMmaPerGroup>(d_tmem, a_d, b_d, idesc);
            umma_commit(&tfull[me]);
            umma_commit(&empty[stage]);
          }
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    if (lane == 0) {
    mma_done:
      // Commits of one issuer arrive in order; once both issuers' drain
      // commits have landed, every MMA and barrier arrival is done and TMEM /
      // shared memory can be released.
      umma_commit(drain);
      drain_wait(drain, 0);
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kEpilogueRegs));
    // ------------------------------------------------------------ promotion + epilogue
    const int q = warp & 3, h = warp >> 2;
    const int r = q * 32 + lane;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    const int kb_rows = p.hidden / kBlockK;          // H/128
    const int ib_rows = p.inter / kBlockK;           // I/128
    uint32_t g = 0;
    for (int u = blockIdx.x; u < total_units; u += gridDim.x) {
      const Unit c = decode_unit(u, tstart_s, counts_s, E, NT);
      // Whether the next group's partial is already known to be complete:
      // checked right after a buffer is released, so that the check's
      // latency overlaps the FMAs that follow instead of stalling the warp.
      bool next_ready = false;
      const bool warp_active = q * 32 < c.nrows;
      const bool row_valid = r < c.nrows;
      const int64_t grow = static_cast<int64_t>(c.row0) + r;
      float acc[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) acc[i] = 0.f;

      if constexpr (kMode == kGemm1) {
        // W1 scale [E, 2I/128, H/128]: gate block n, SiLU block I/128 + n.
        const float* ws = p.b_scale + static_cast<int64_t>(c.e) * (2 * ib_rows) * KB;
        const float* ws_x1 = ws + static_cast<int64_t>(c.n) * KB;
        const float* ws_x2 = ws + static_cast<int64_t>(ib_rows + c.n) * KB;
        // Activation scales of K block kb+2 are loaded while block kb is
        // promoted: they come from DRAM (the permute's row copies push them
        // out of L2), and a load issued one K block ahead stalled every
        // group's first multiply (clock64 traces: ~300 of ~1000 cycles per
        // group).
        // The weight scales are the same for the whole warp: lane i holds K
        // block 32c + i of the current 32-block chunk c (and of the next), and
        // each K block takes its value with a shuffle, so the loop issues
        // their loads once per 32 K blocks instead of twice per K block.
        const float* sa_p = p.a_scale + grow;
        float w1_c = lane < KB ? __ldg(ws_x1 + lane) : 0.f;
        float w2_c = lane < KB ? __ldg(ws_x2 + lane) : 0.f;
        float w1_cn = lane + 32 < KB ? __ldg(ws_x1 + 32 + lane) : 0.f;
        float w2_cn = lane + 32 < KB ? __ldg(ws_x2 + 32 + lane) : 0.f;
        float sa_n = warp_active ? __ldg(sa_p) : 0.f;
        float sa_nn = warp_active && KB > 1 ? __ldg(sa_p + p.npad) : 0.f;
        for (int kb = 0; kb < KB; ++kb) {
          if ((kb & 31) == 0 && kb > 0) {
            w1_c = w1_cn;
            w2_c = w2_cn;
            const int nk = kb + 32 + lane;
            w1_cn = nk < KB ? __ldg(ws_x1 + nk) : 0.f;
            w2_cn = nk < KB ? __ldg(ws_x2 + nk) : 0.f;
          }
          const float s1 = sa_n * __shfl_sync(0xffffffffu, w1_c, kb & 31);
          const float s2 = sa_n * __shfl_sync(0xffffffffu, w2_c, kb & 31);
          sa_n = sa_nn;
          if (kb + 2 < KB && warp_active) sa_nn = __ldg(sa_p + static_cast<int64_t>(kb + 2) * p.npad);
          const uint32_t buf = g & 1u;
          if (!next_ready && !mbar_wait(&tfull[buf], (g >> 1) & 1u, abort_flag, p.ctrl, 4))
            goto epi_done;
          tc_fence_after();
          if (warp_active) {
            const uint32_t tb = t_lane + buf * kTileN;
            float v[64];
            // X1 columns 64h..64h+63, then X2 columns 128+64h..; the buffer is
            // released as soon as the last columns are in registers, before
            // their FMAs (the hold time bounds the tensor core, see above).
            tmem_ld32(tb + 64u * h, v);
            tmem_ld32(tb + 64u * h + 32, v + 32);
            tmem_ld_wait();
            fma_pairs(acc, v, s1);
            tmem_ld32(tb + 128u + 64u * h, v);
            tmem_ld32(tb + 128u + 64u * h + 32, v + 32);
            tmem_ld_wait();
            release_buffer(&tempty[buf], lane);
            next_ready = mbar_test_wait(&tfull[buf ^ 1u], ((g + 1) >> 1) & 1u);
            fma_pairs(acc + 64, v, s2);
          } else {
            release_buffer(&tempty[buf], lane);
            next_ready = false;
          }
          ++g;
        }
        // SwiGLU + 1x64 requant (kernel.py:128-151).  The MMA is stalled while
        // this runs (two groups ahead at most), so silu(x) = x / (1 + exp(-x))
        // uses the fast division (reciprocal approximation and multiply, within
        // 2 ulp of the IEEE quotient; the accumulators themselves differ from
        // the reference's in summation order by far more) and the requant one
        // IEEE reciprocal of the scale per row instead of 64 divisions.  The
        // IEEE-rounded reciprocal per element cost 8-9% of GEMM1 at T=8192-16384.
        if (warp_active) {
          float amax = 0.f;
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            const float x1 = acc[j], x2 = acc[64 + j];
            const float cval = __fdividef(x2, 1.0f + __expf(-x2)) * x1;
            acc[j] = cval;
            amax = fmaxf(amax, fabsf(cval));
          }
          const float sc = fmaxf(amax / 448.0f, 1e-12f);
          const float inv = 1.0f / sc;
          uint8_t* stg = xpose + warp * kXposeBytesPerWarp;
          if (p.inter_bf16 != nullptr) {
            // For the bf16 GEMM2: the same FP8 codes, dequantised (code * scale)
            // and rounded to bf16; 128 bytes per row, through the staging tile
            // in two passes of 32 values.
#pragma unroll
            for (int pass = 0; pass < 2; ++pass) {
#pragma unroll
              for (int q16 = 0; q16 < 4; ++q16) {
                uint32_t w4[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const float* a2 = acc + 32 * pass + 8 * q16 + 2 * j;
                  const __nv_fp8x2_storage_t codes =
                      static_cast<__nv_fp8x2_storage_t>(pack_e4m3x2(a2[0] * inv, a2[1] * inv));
                  const float2 f =
                      __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(codes, __NV_E4M3)));
                  const __nv_bfloat162 b = __floats2bfloat162_rn(f.x * sc, f.y * sc);
                  w4[j] = *reinterpret_cast<const uint32_t*>(&b);
                }
                *reinterpret_cast<uint4*>(stg + xpose_off(lane, q16)) =
                    make_uint4(w4[0], w4[1], w4[2], w4[3]);
              }
              __syncwarp();
              uint8_t* dstb = reinterpret_cast<uint8_t*>(p.inter_bf16) +
                              2 * (static_cast<int64_t>(c.row0 + q * 32) * p.inter +
                                   c.n * (kTileN / 2) + 64 * h + 32 * pass) +
                              16 * (lane & 3);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int rr = 8 * i + (lane >> 2);
                if (q * 32 + rr < c.nrows)
                  *reinterpret_cast<uint4*>(dstb + 2 * static_cast<int64_t>(rr) * p.inter) =
                      *reinterpret_cast<const uint4*>(stg + xpose_off(rr, lane & 3));
              }
              __syncwarp();
            }
          } else {
          // Each lane's 64 FP8 codes go through the warp's staging tile; the
          // stores then write 64 contiguous bytes of 8 rows per instruction
          // instead of 16 bytes of 32 rows.
#pragma unroll
          for (int q16 = 0; q16 < 4; ++q16) {
            uint32_t w4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float* a4 = acc + 16 * q16 + 4 * j;
              w4[j] = pack_e4m3x2(a4[0] * inv, a4[1] * inv) |
                      (pack_e4m3x2(a4[2] * inv, a4[3] * inv) << 16);
            }
            *reinterpret_cast<uint4*>(stg + xpose_off(lane, q16)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
          }
          __syncwarp();
          uint8_t* dst = p.inter_out + static_cast<int64_t>(c.row0 + q * 32) * p.inter +
                         c.n * (kTileN / 2) + 64 * h + 16 * (lane & 3);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int rr = 8 * i + (lane >> 2);
            if (q * 32 + rr < c.nrows)
              *reinterpret_cast<uint4*>(dst + static_cast<int64_t>(rr) * p.inter) =
                  *reinterpret_cast<const uint4*>(stg + xpose_off(rr, lane & 3));
          }
          __syncwarp();
          if (row_valid) p.inter_scale[static_cast<int64_t>(2 * c.n + h) * p.npad + grow] = sc;
          }
        }
      } else {
        if constexpr (kMode == kGemm2Bf16) {
          // The unit's whole K range was accumulated in TMEM buffer (unit
          // parity): one wait, 128 columns read, the buffer released.
          const uint32_t buf = g & 1u;
          if (!mbar_wait(&tfull[buf], (g >> 1) & 1u, abort_flag, p.ctrl, 6)) goto epi_done;
          tc_fence_after();
          if (warp_active) {
            const uint32_t tb = t_lane + buf * kTileN + 128u * h;
            tmem_ld32(tb, acc);
            tmem_ld32(tb + 32, acc + 32);
            tmem_ld_wait();
            tmem_ld32(tb + 64, acc + 64);
            tmem_ld32(tb + 96, acc + 96);
            tmem_ld_wait();
          }
          release_buffer(&tempty[buf], lane);
          ++g;
        } else {
        // W2 scale [E, H/128, I/128]: row block 2n + h of this thread's columns.
        const float* ws = p.b_scale + (static_cast<int64_t>(c.e) * kb_rows + 2 * c.n + h) * KB;
        // Both intermediate scales of K block kb+2 and its weight scale are
        // loaded at the top of K block kb, two K blocks (four groups) ahead of
        // their use, as in GEMM1.
        const float* sa_p = p.a_scale + grow;
        float sa0_n = warp_active ? __ldg(sa_p) : 0.f;
        float sa1_n = warp_active ? __ldg(sa_p + p.npad) : 0.f;
        float sw_n = __ldg(ws);
        float sa0_nn = 0.f, sa1_nn = 0.f, sw_nn = 0.f;
        if (KB > 1) {
          if (warp_active) {
            sa0_nn = __ldg(sa_p + 2 * p.npad);
            sa1_nn = __ldg(sa_p + 3 * p.npad);
          }
          sw_nn = __ldg(ws + 1);
        }
        for (int kb = 0; kb < KB; ++kb) {
          const float sg0 = sa0_n * sw_n, sg1 = sa1_n * sw_n;
          sa0_n = sa0_nn;
          sa1_n = sa1_nn;
          sw_n = sw_nn;
          if (kb + 2 < KB) {
            if (warp_active) {
              sa0_nn = __ldg(sa_p + static_cast<int64_t>(2 * kb + 4) * p.npad);
              sa1_nn = __ldg(sa_p + static_cast<int64_t>(2 * kb + 5) * p.npad);
            }
            sw_nn = __ldg(ws + kb + 2);
          }
#pragma unroll
          for (int gi = 0; gi < 2; ++gi) {
            const float s = gi == 0 ? sg0 : sg1;
            const uint32_t buf = g & 1u;
            if (!next_ready && !mbar_wait(&tfull[buf], (g >> 1) & 1u, abort_flag, p.ctrl, 5))
              goto epi_done;
            tc_fence_after();
            if (warp_active) {
              const uint32_t tb = t_lane + buf * kTileN + 128u * h;
              float v[64];
              tmem_ld32(tb, v);
              tmem_ld32(tb + 32, v + 32);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 64; ++i) acc[i] = fmaf(v[i], s, acc[i]);
              tmem_ld32(tb + 64, v);
              tmem_ld32(tb + 96, v + 32);
              tmem_ld_wait();
              release_buffer(&tempty[buf], lane);
              next_ready = mbar_test_wait(&tfull[buf ^ 1u], ((g + 1) >> 1) & 1u);
#pragma unroll
              for (int i = 0; i < 64; ++i) acc[64 + i] = fmaf(v[i], s, acc[64 + i]);
            } else {
              release_buffer(&tempty[buf], lane);
              next_ready = false;
            }
            ++g;
          }
        }
        }
        // Routing-weighted scatter-add into out[token] (kernel.py:236-250).
        // Every row goes to a different token, so a lane-per-row red.v4
        // touches 32 rows x 16 B per instruction.  The weighted values go
        // through the warp's staging tile 16 columns at a time instead, and
        // each red.v4 instruction then adds 64 contiguous bytes to 8 rows.
        // Deterministic combine: the same values are stored to the row's own
        // line of rows_out instead, and a gather adds them in a fixed order.
        if (warp_active) {
          const float w = row_valid ? p.row_weight[grow] : 0.f;
          const int tok = row_valid ? p.row_token[grow] : 0;
          const bool store_rows = p.rows_out != nullptr;
          float* stg = reinterpret_cast<float*>(xpose + warp * kXposeBytesPerWarp);
          float* dst_i[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int rr = 8 * i + (lane >> 2);
            const int t_i = __shfl_sync(0xffffffffu, tok, rr);
            const int64_t line = store_rows ? static_cast<int64_t>(c.row0) + q * 32 + rr
                                            : static_cast<int64_t>(t_i);
            float* base = store_rows ? p.rows_out : p.out_f32;
            dst_i[i] = q * 32 + rr < c.nrows
                           ? base + line * p.hidden + c.n * kTileN + 128 * h + 4 * (lane & 3)
                           : nullptr;
          }
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float* a4 = acc + 16 * ch + 4 * j;
              *reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(stg) + xpose_off(lane, j)) =
                  make_float4(a4[0] * w, a4[1] * w, a4[2] * w, a4[3] * w);
            }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int rr = 8 * i + (lane >> 2);
              const float4 v4 = *reinterpret_cast<const float4*>(
                  reinterpret_cast<const uint8_t*>(stg) + xpose_off(rr, lane & 3));
              if (dst_i[i]) {
                if (store_rows)
                  *reinterpret_cast<float4*>(dst_i[i] + 16 * ch) = v4;
                else
                  red_add_v4(dst_i[i] + 16 * ch, v4.x, v4.y, v4.z, v4.w);
              }
            }
            __syncwarp();
          }
        }
      }
    }
  epi_done:;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

int gemm_set_smem_attrs() {
  const int smem = gemm_smem_bytes();
  if (cudaFuncSetAttribute(moe_gemm_kernel<kGemm1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           smem) != cudaSuccess)
    return MOE_ERR_CUDA;
  if (cudaFuncSetAttribute(moe_gemm_kernel<kGemm2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           smem) != cudaSuccess)
    return MOE_ERR_CUDA;
  if (cudaFuncSetAttribute(moe_gemm_kernel<kGemm2Bf16>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return MOE_ERR_CUDA;
  return MOE_OK;
}

int launch_gemm(int mode, const CUtensorMap& tm_a, const CUtensorMap& tm_b, const GemmParams& p,
                int grid, cudaStream_t stream) {
  const int smem = gemm_smem_bytes();
  if (mode == kGemm1)
    moe_gemm_kernel<kGemm1><<<grid, kGemmThreads, smem, stream>>>(tm_a, tm_b, p);
  else if (mode == kGemm2)
    moe_gemm_kernel<kGemm2><<<grid, kGemmThreads, smem, stream>>>(tm_a, tm_b, p);
  else
    moe_gemm_kernel<kGemm2Bf16><<<grid, kGemmThreads, smem, stream>>>(tm_a, tm_b, p);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

}  // namespace moe
