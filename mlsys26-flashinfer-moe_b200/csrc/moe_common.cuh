// Device-side building blocks for the sm_100a MoE kernels: mbarriers with
// bounded waits, TMA tile loads, tcgen05 (UMMA) descriptors / MMA / TMEM
// access, and a few numeric helpers.  Everything here is inline PTX written
// for compute_100a; nothing falls back to older tensor-core paths.
#pragma once

#include <cstdint>
#include <utility>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp8.h>
#include <cuda_bf16.h>

#include "../../include/moe_b200.h"

namespace moe {

// ---------------------------------------------------------------------------
// error reporting shared by all kernels
// ---------------------------------------------------------------------------

// Control block at the start of the workspace.  `done` is the arrival counter
// of the routing kernel's last-block scan; `error` holds the first device-side
// error code (MOE_ERR_TIMEOUT) and `error_info` where it happened; `gemm_done`
// counts finished CTAs of the decode GEMM2.  Zeroed before every forward.
struct CtrlBlock {
  unsigned int done;
  int error;
  int error_info;
  unsigned int gemm_done;   // decode GEMM2 CTAs finished (bf16 output by the last)
  int pad[60];
};

// Bounded waits give up after this many nanoseconds of %globaltimer unless the
// caller set another limit (MoeFwdArgs.wait_limit_ns).  Normal waits last
// microseconds; only a broken pipeline reaches the limit.  Drains after an
// abort (letting copies and MMAs already in flight land before shared memory
// and TMEM are released) always use this default.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

// The limit as the kernels keep it: whole microseconds, at least one.
__host__ __device__ constexpr unsigned int wait_limit_us(unsigned long long ns) {
  return ns == 0 ? static_cast<unsigned int>(kWaitLimitNs / 1000)
         : ns >= 1000ull * 0x7fffffffull ? 0x7fffffffu
                                         : static_cast<unsigned int>((ns + 999) / 1000);
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report_error(CtrlBlock* ctrl, int code, int info) {
  if (atomicCAS(&ctrl->error, 0, code) == 0) ctrl->error_info = info;
}

// ---------------------------------------------------------------------------
// programmatic dependent launch
// ---------------------------------------------------------------------------

// Lets the next kernel in the stream (launched with programmatic stream
// serialization) start its prologue once every CTA of this grid has issued
// this or exited.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launches `kern` so that it may start while the previous kernel in the
// stream finishes (programmatic stream serialization): it must call
// griddep_wait() before reading anything that kernel writes.
template <typename... Params, typename... Args>
inline cudaError_t launch_programmatic(void (*kern)(Params...), dim3 grid, dim3 block, size_t smem,
                                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Waits until the previous kernel in the stream has completed and its memory
// operations are visible; returns at once when this grid was launched without
// programmatic serialization.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------------------------
// shared-memory addresses and mbarriers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// A thread whose try_wait finds the phase incomplete is suspended until the
// phase completes or this many nanoseconds pass, whichever comes first: waiting
// threads neither spin (which takes issue slots from the promotion warps on the
// same sub-partition) nor sleep past the completion (which delays the hand-off).
constexpr uint32_t kSuspendHintNs = 10000000u;

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity,
                                              uint32_t hint_ns = kSuspendHintNs) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Non-blocking check of a phase: issued early, its latency hides behind work
// that does not depend on the answer.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Suspend-time hint of the retries after a first unsuccessful try_wait: how
// often a thread in an abnormally long wait looks at the abort flag and the
// clock.
constexpr uint32_t kRetryHintNs = 1000000u;

// Wait until the phase with the given parity of `bar` has completed.  Gives up
// when `abort[0]` is raised by another warp or when abort[1] microseconds (the
// CTA's wait limit, kept in the shared word after the flag and read only on
// this slow path, so that it costs the hot loops no register) have passed
// since the first try_wait returned; then it raises `abort[0]`, records
// MOE_ERR_TIMEOUT with `where` and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          CtrlBlock* ctrl, int where) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (;;) {
    if (mbar_try_wait(bar, parity, kRetryHintNs)) return true;
    if (*abort) return false;
    if (globaltimer() - t0 > 1000ull * static_cast<unsigned int>(abort[1])) {
      *abort = 1;
      report_error(ctrl, MOE_ERR_TIMEOUT, where);
      return false;
    }
  }
}

// 4-byte global -> shared copy that completes asynchronously (no register is
// held while the load is in flight); each thread waits for its own copies.
__device__ __forceinline__ void cp_async4(uint32_t dst_smem, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst_smem), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMA
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load of one box into shared memory; completion is signalled on
// `bar` as transaction bytes.  x is the inner (contiguous) coordinate.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 / TMEM
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored in the
// canonical 128-byte-swizzled layout: rows of 128 bytes, 8-row atoms of
// 1024 bytes laid out contiguously (stride byte offset 1024).  The tile base
// must be 1024-byte aligned; advancing along K inside the 128-byte row is done
// by adding the byte offset to the start address.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);          // start address
  d |= static_cast<uint64_t>(1u) << 16;                              // LBO (unused, =16 B)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;                      // SBO
  d |= static_cast<uint64_t>(1u) << 46;                              // descriptor version
  d |= static_cast<uint64_t>(2u) << 61;                              // SWIZZLE_128B
  return d;
}

// Instruction descriptor: e4m3 x e4m3 -> fp32, both operands K-major.
__host__ __device__ constexpr uint32_t umma_idesc_e4m3_f32(int m, int n) {
  return (1u << 4)                                  // D format f32
         | (0u << 7) | (0u << 10)                   // A, B = e4m3
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

// Instruction descriptor: bf16 x bf16 -> fp32 (kind::f16), both operands K-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16_f32(int m, int n) {
  return (1u << 4)                                  // D format f32
         | (1u << 7) | (1u << 10)                   // A, B = bf16
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

// Four bf16 MMAs of K=16 each (one 128-byte row of the swizzled K-major tiles:
// the descriptors of the slices are the stage's plus 32 bytes each, i.e. +2 in
// the start-address field), D (+)= A*B^T; `accumulate` = 0 starts D over with
// the first of them.
__device__ __forceinline__ void umma_bf16_x4(uint32_t d_tmem, uint64_t a, uint64_t b,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred f, t;\n\t.reg .b64 a1, a2, a3, b1, b2, b3;\n\t"
      "setp.ne.b32 f, %4, 0;\n\t"
      "setp.eq.b32 t, %3, %3;\n\t"
      "add.s64 a1, %1, 2;\n\tadd.s64 a2, %1, 4;\n\tadd.s64 a3, %1, 6;\n\t"
      "add.s64 b1, %2, 2;\n\tadd.s64 b2, %2, 4;\n\tadd.s64 b3, %2, 6;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, f;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a1, b1, %3, t;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a2, b2, %3, t;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a3, b3, %3, t;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by a single thread.
__device__ __forceinline__ void umma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// One scale group of MMAs, D = A0*B0^T + A1*B1^T (+ ...), issued from one asm
// block with descriptors computed beforehand.  The issuing thread shares its
// sub-partition with promotion warps that stream FMAs and win most issue
// slots, so every instruction between "buffer free" and the last MMA costs
// far more than its latency; this keeps that window to the MMAs themselves.
template <int kCount>
__device__ __forceinline__ void umma_f8_group(uint32_t d_tmem, const uint64_t* a, const uint64_t* b,
                                              uint32_t idesc) {
  static_assert(kCount == 2 || kCount == 4, "groups of 2 or 4 MMAs");
  if constexpr (kCount == 2) {
    asm volatile(
        "{\n\t.reg .pred f, t;\n\t"
        "setp.ne.b32 f, %5, %5;\n\t"
        "setp.eq.b32 t, %5, %5;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %3, %5, f;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %2, %4, %5, t;\n\t}" ::"r"(d_tmem),
        "l"(a[0]), "l"(a[1]), "l"(b[0]), "l"(b[1]), "r"(idesc)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred f, t;\n\t"
        "setp.ne.b32 f, %9, %9;\n\t"
        "setp.eq.b32 t, %9, %9;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %5, %9, f;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %2, %6, %9, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %3, %7, %9, t;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %4, %8, %9, t;\n\t}" ::"r"(d_tmem),
        "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]),
        "r"(idesc)
        : "memory");
  }
}

// Forces values to be computed at this point of the program (before the
// volatile asm that follows, e.g. a barrier wait).
__device__ __forceinline__ void materialize(uint64_t v) { asm volatile("" ::"l"(v)); }

// Arrive on `bar` once every tcgen05 operation issued so far by this thread
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Each thread of the warp reads 32 consecutive fp32 columns of its TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Each thread of the warp reads 16 consecutive fp32 columns of its TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// numerics
// ---------------------------------------------------------------------------

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

// Two fp32 -> two e4m3 bytes (round to nearest even, saturating), x in the low byte.
__device__ __forceinline__ uint32_t pack_e4m3x2(float x, float y) {
  return static_cast<uint32_t>(
      __nv_cvt_float2_to_fp8x2(make_float2(x, y), __NV_SATFINITE, __NV_E4M3));
}

}  // namespace moe
