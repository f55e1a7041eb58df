// Shared device helpers for the sm_100a MoE kernels: error flags, bounded
// mbarrier waits, TMA tile loads and the tcgen05 (5th-gen tensor core / TMEM)
// instruction wrappers.  Everything here is inline PTX written for sm_100a.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define MOE_DEV __device__ __forceinline__

namespace moe {

// Device-side status codes written to the plan's error word.  The host reads
// the word after a forward (moe_status) and maps it to MOE_ERR_TIMEOUT /
// MOE_ERR_DEVICE.  Kernels never trap: a wait that runs out of time records a
// code and the kernel drains and returns.
enum DevErr : int {
  DEV_OK = 0,
  DEV_TIMEOUT_FULL = 1,      // MMA waited too long for a TMA stage
  DEV_TIMEOUT_EMPTY = 2,     // producer waited too long for a free stage
  DEV_TIMEOUT_TMEM_FULL = 3, // epilogue waited too long for an accumulator
  DEV_TIMEOUT_TMEM_EMPTY = 4,// MMA waited too long for an accumulator buffer
  DEV_TIMEOUT_CONV = 5,      // int8 converter waited too long
  DEV_BAD_TILE = 6,          // tile list entry out of range
  DEV_BAD_ROUTE = 7,         // router produced an expert id out of range
  DEV_RANGE = 8,             // an activation does not fit an f16 operand or output
  DEV_TILE_OVERFLOW = 9,     // a tile list needs more entries than the workspace holds
  DEV_TIMEOUT_PEER = 10,     // a peer GPU's epoch flag did not arrive in time
};

// f16 conversion of v stays finite (|v| rounds to at most 65504); false for NaN too.
MOE_DEV bool fits_f16(float v) { return fabsf(v) < 65520.f; }

// ~1 s at the B200 boost clock.  Legitimate waits in these kernels are
// microseconds; this bound only ends a wait that can no longer complete.
constexpr long long kWaitLimitCycles = 2000000000LL;

MOE_DEV void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

MOE_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- launch chaining
// Every forward kernel is launched with programmatic stream serialisation, so
// its launch and on-chip prologue overlap the tail of the kernel before it.
// pdl_release lets the next kernel of the stream start launching; pdl_wait
// blocks until the previous kernel has completed and its writes are visible.
// Kernels call both before their first global-memory access (a no-op when the
// launch did not ask for chaining).
MOE_DEV void pdl_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
MOE_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
MOE_DEV void pdl_enter() {
  pdl_release();
  pdl_wait();
}

// ---------------------------------------------------------------- mbarrier
MOE_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

MOE_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

MOE_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

MOE_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

MOE_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity; false if the wait ran out of time
// (`limit` cycles) or the CTA was told to abort (another role already timed out).
// Every waiting thread polls on its own: parking threads with a suspend-time
// hint, or letting one lane poll for its warp, both measured slower (the INT8
// decode GEMM's converter warps sit on this path once per k-block).
MOE_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                               long long limit = kWaitLimitCycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - start > limit) return false;
  }
}

// Same bound, but not cut short by the abort flag: used when a role drains its
// own in-flight copies / MMAs before the CTA releases shared memory and TMEM.
MOE_DEV bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > kWaitLimitCycles) return false;
  }
  return true;
}

// ---------------------------------------------------------------- TMA
MOE_DEV void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Contiguous bulk load global -> shared (this CTA): both addresses 16-byte aligned,
// bytes a multiple of 16; completion counted in bytes on bar.
MOE_DEV void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2D tiled load global -> shared (this CTA), completion counted in bytes on bar.
// c0 is the innermost (K) coordinate in elements, c1 the row coordinate.
MOE_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* map, int32_t c0, int32_t c1,
                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
MOE_DEV void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
MOE_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
MOE_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
MOE_DEV void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
MOE_DEV void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, f16 inputs, f32 accumulate.
MOE_DEV void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, f16 inputs, f32 accumulate.  A (M = 128
// rows) sits in TMEM lane m = row m, two f16 per 32-bit column in K order (the
// lower half the even k): one K = 16 step spans 8 columns from a_tmem.
MOE_DEV void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on bar when every tcgen05.mma issued so far by this thread completes.
MOE_DEV void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
MOE_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 bit, 32 consecutive columns per thread.
MOE_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 bit, 16 consecutive columns per thread, written back to TMEM.
MOE_DEV void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 bit, 32 consecutive columns per thread (no wait: the caller
// issues tcgen05.wait::st after its last store).
MOE_DEV void tmem_st32_nowait(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
      "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]),
      "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]),
      "r"(v[30]), "r"(v[31])
      : "memory");
}
MOE_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Generic-proxy writes to shared memory become visible to the async proxy (TMA,
// tensor core operand reads) after this fence.
MOE_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major tile written by TMA with
// 128-byte swizzle: rows of 128 B, 8-row atoms 1024 B apart (SBO), tile base
// 1024-byte aligned.  Layout code 2 = SWIZZLE_128B, version bits [46,48) = 1.
MOE_DEV uint64_t sw128_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(1) << 16;              // LBO (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;      // SBO
  d |= static_cast<uint64_t>(1) << 46;              // version
  d |= static_cast<uint64_t>(2) << 61;              // SWIZZLE_128B
  return d;
}

// Instruction descriptor: f16 x f16 -> f32, both operands K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n) {
  return (1u << 4)                                  // D format f32
         | (0u << 7) | (0u << 10)                   // A, B = f16
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

// SwiGLU's silu in the GEMM epilogue (its f16 output rounds far above the
// intrinsics' error); the exponent is clamped so the fast divide never sees a
// denominator beyond 2^126.
MOE_DEV float silu_f(float g) { return __fdividef(g, 1.0f + __expf(fminf(-g, 80.f))); }
MOE_DEV float sigmoid_f(float v) { return 1.0f / (1.0f + expf(-v)); }

}  // namespace moe
