// Shared device/host helpers for the smelb sm_100a kernels: error plumbing, bf16 helpers and thin PTX
// wrappers for mbarrier, TMA (cp.async.bulk.tensor) and the 5th-gen tensor core (tcgen05 + TMEM).
//
// Every wait on an mbarrier is bounded: after SMELB_WAIT_NS nanoseconds of spinning the waiting thread records
// an error code in a device status word and gives up, so a logic error shows up as a status code on the host
// instead of a hung GPU.
#pragma once

#include <cstdint>
#include <cstdio>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#ifndef SMELB_WAIT_NS
#define SMELB_WAIT_NS 2000000000ull  // 2 s: no single pipeline wait legitimately takes this long
#endif

namespace smelb {

// ------------------------------------------------------------------------------------------- status codes
enum Status : int {
  kOk = 0,
  kErrShape = -1,        // bad shape / size / alignment
  kErrDtype = -2,        // unsupported dtype or format
  kErrWorkspace = -3,    // workspace too small
  kErrTimeout = -4,      // a device-side wait gave up
  kErrCuda = -5,         // a CUDA runtime/driver call failed
  kErrArg = -6,          // bad argument (null pointer, unknown activation, ...)
};

void set_last_error(const char* fmt, ...);

#define SMELB_CHECK_ARG(cond, code, ...)   \
  do {                                     \
    if (!(cond)) {                         \
      ::smelb::set_last_error(__VA_ARGS__); \
      return (code);                       \
    }                                      \
  } while (0)

#define SMELB_CUDA(call)                                                                    \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess) {                                                                \
      ::smelb::set_last_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, \
                              __LINE__);                                                    \
      return ::smelb::kErrCuda;                                                             \
    }                                                                                       \
  } while (0)

// Device-side status: word 0 holds the first failure code (atomicCAS, first one wins); words 1-3 the block, tile and
// k-block index where it happened.
enum DevErr : int {
  kDevErrNone = 0,
  kDevErrWaitFull = 1,       // MMA waiting for a token tile
  kDevErrWaitEmpty = 2,      // token producer waiting for a free slot
  kDevErrWaitAccFull = 3,    // epilogue waiting for an accumulator
  kDevErrWaitAccEmpty = 4,   // MMA waiting for a free accumulator
  kDevErrTmaDrain = 5,       // a producer waiting for its last copies at exit
  kDevErrTooManyGroups = 6,
  kDevErrBadIndex = 7,       // expert index out of range in the dispatch plan
  kDevErrWaitAFull = 8,      // MMA waiting for a weight tile
  kDevErrWaitQFull = 9,      // dequant waiting for staged nibbles
  kDevErrWaitAEmptyDeq = 10, // dequant waiting for a free weight slot
  kDevErrWaitAEmptyTma = 11, // weight producer waiting for a free weight slot
  kDevErrWaitQEmpty = 12,    // staging producer waiting for a consumed stage
};
constexpr int kStatusWords = 4;

using bf16 = __nv_bfloat16;

__device__ __forceinline__ void dev_fail(int* err, int code) {
  if (err && atomicCAS(err, 0, code) == 0) {
    err[1] = blockIdx.x;
    err[2] = -1;
    err[3] = -1;
  }
}

__device__ __forceinline__ void dev_fail_at(int* err, int code, int tile, int kb) {
  if (err && atomicCAS(err, 0, code) == 0) {
    err[1] = blockIdx.x;
    err[2] = tile;
    err[3] = kb;
  }
}

// ------------------------------------------------------------------------------------------- timers
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------------------------------- smem address
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// arrive `count` times at once
__device__ __forceinline__ void mbar_arrive_n(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// raise the current phase's expected transaction bytes without arriving
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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

// try_wait that may suspend the thread for up to `hint_ns` while the phase is incomplete; the thread resumes when
// the phase completes. Waiting warps then leave the issue slots to the warps that work.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
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

#ifndef SMELB_BACKOFF_MAX_NS
#define SMELB_BACKOFF_MAX_NS 512u
#endif
#ifndef SMELB_SUSPEND_NS
#define SMELB_SUSPEND_NS 100000u  // upper bound of one suspended try_wait (100 us); the wake-up is on completion
#endif

// Wait until the phase with the given parity has completed. Returns false (and records `code` with the location in
// the status words) when the wait gives up after SMELB_WAIT_NS. The fast path is a single try_wait; the slow path
// (out of line) suspends in try_wait instead of spinning, and checks the clock between suspensions.
static __device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, int* err, int code, int tile, int kb) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t sleep_ns = 0;
  while (true) {
    if (mbar_try_wait_suspend(bar, parity, SMELB_SUSPEND_NS)) return true;
    if (globaltimer_ns() - t0 > SMELB_WAIT_NS) {
      dev_fail_at(err, code, tile, kb);
      return false;
    }
    // back off so that a waiting warp leaves its scheduler's issue slots to the warps that work: a few quick polls,
    // then sleeps growing to SMELB_BACKOFF_MAX_NS
    if (sleep_ns) __nanosleep(sleep_ns);
    sleep_ns = sleep_ns ? min(2 * sleep_ns, (uint32_t)SMELB_BACKOFF_MAX_NS) : 32u;
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code, int tile = -1,
                                          int kb = -1) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, err, code, tile, kb);
}

// The whole warp waits (every lane polls; the result is made warp-uniform).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int* err, int code, int tile = -1,
                                               int kb = -1) {
  const bool ok = mbar_wait(bar, parity, err, code, tile, kb);
  return __all_sync(0xffffffffu, ok);
}

// ------------------------------------------------------------------------------------------- proxy fences
// Make generic-proxy shared-memory writes visible to the async proxy (TMA, tcgen05.mma operand reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 2-D tiled load global -> shared, completion counted on `bar` (complete_tx bytes).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* m, int32_t x, int32_t y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled load global -> shared, completion counted on `bar` (complete_tx bytes).
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* m, int32_t x, int32_t y, int32_t z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// ------------------------------------------------------------------------------------------- tcgen05 / TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 inputs, fp32 accumulate), issued by one thread.
// No "memory" clobber: operand visibility is ordered by the mbarrier waits and tcgen05 fences, and a clobber would
// make the compiler reload every memory-resident value (kernel parameters included) after each MMA.
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T: A is read from tensor memory (row m of the tile in lane m, two bf16 of
// consecutive k per 32-bit column, 8 columns per K=16 step), so only B is read from shared memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// One lane of the (converged) warp is elected; tcgen05.mma is issued from warp-uniform code through it, which keeps
// the operands in uniform registers (a lone divergent thread issues several times slower).
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// Arrive on `bar` once all tcgen05 operations issued so far by this thread have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets row (lane base + i), columns c..c+31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 16 (x8) consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns from registers: thread i of the warp writes row (lane base + i).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05 format): start address, LBO, SBO (all >>4), version 1, swizzle mode.
// layout 2 = 128-byte swizzle.
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;  // descriptor version for sm_100
  d |= (uint64_t)2u << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16: bf16 x bf16 -> fp32, M=128, N=n, A/B major as given (0 = K, 1 = MN).
__device__ __forceinline__ uint32_t make_idesc_bf16(uint32_t n, uint32_t a_mn_major, uint32_t b_mn_major) {
  uint32_t d = 0;
  d |= 1u << 4;                   // D format F32
  d |= 1u << 7;                   // A format BF16
  d |= 1u << 10;                  // B format BF16
  d |= (a_mn_major & 1u) << 15;   // A major
  d |= (b_mn_major & 1u) << 16;   // B major
  d |= ((n >> 3) & 0x3Fu) << 17;  // N >> 3
  d |= ((128u >> 4) & 0x1Fu) << 24;  // M >> 4
  return d;
}

// ------------------------------------------------------------------------------------------- numerics
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

// ------------------------------------------------------------------------------------------- int4 expansion
// A group takes the bf16x2 fast path when every value q*s + z (q in 0..15) is exactly representable in fp32: then
// rounding the exact value once to bf16 (fma.rn.bf16x2) equals the reference's fp32 dequant followed by a bf16
// cast. Other groups (extreme scale/zero exponent gaps, subnormals, non-finite) are expanded in fp32.
__device__ __forceinline__ bool dq_fast_ok(uint32_t sz) {
  const uint32_t s = sz & 0xFFFFu, z = sz >> 16;
  if ((z & 0x7FFFu) == 0 || (s & 0x7FFFu) == 0) return true;
  const int es = (s >> 7) & 0xFF, ez = (z >> 7) & 0xFF;
  if (es < 32 || ez < 32 || es == 0xFF || ez == 0xFF) return false;
  const int d = ez - es;
  return d <= 15 && d >= -11;
}

__device__ __forceinline__ uint32_t bf162_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __nv_bfloat162 bits_bf162(uint32_t v) { return *reinterpret_cast<__nv_bfloat162*>(&v); }

// One 32-bit word = 8 nibbles, byte j holding element 2j (low nibble) and 2j+1 (high nibble) -> 8 bf16.
// (0x4300 | n) is the bf16 encoding of 128 + n, so subtracting 128 recovers n exactly.
__device__ __forceinline__ uint4 dq8_fast(uint32_t w, __nv_bfloat162 s2, __nv_bfloat162 z2) {
  const uint32_t y = w >> 4;
  const __nv_bfloat162 c128 = bits_bf162(0x43004300u);
  const uint32_t p0 = (__byte_perm(w, y, 0x0400) & 0x000F000Fu) | 0x43004300u;
  const uint32_t p1 = (__byte_perm(w, y, 0x0501) & 0x000F000Fu) | 0x43004300u;
  const uint32_t p2 = (__byte_perm(w, y, 0x0602) & 0x000F000Fu) | 0x43004300u;
  const uint32_t p3 = (__byte_perm(w, y, 0x0703) & 0x000F000Fu) | 0x43004300u;
  uint4 r;
  r.x = bf162_bits(__hfma2(__hsub2(bits_bf162(p0), c128), s2, z2));
  r.y = bf162_bits(__hfma2(__hsub2(bits_bf162(p1), c128), s2, z2));
  r.z = bf162_bits(__hfma2(__hsub2(bits_bf162(p2), c128), s2, z2));
  r.w = bf162_bits(__hfma2(__hsub2(bits_bf162(p3), c128), s2, z2));
  return r;
}

__device__ __forceinline__ uint4 dq8_exact(uint32_t w, float s, float z) {
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t b = (w >> (8 * j)) & 0xFFu;
    o[j] = bf162_bits(__floats2bfloat162_rn(fmaf((float)(b & 0xFu), s, z), fmaf((float)(b >> 4), s, z)));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// ------------------------------------------------------------------------------------------- activations
// Activations in fp32 on the bf16-rounded pre-activation, as the reference's bf16 `act` (smel/moe.py:91-107), using
// the hardware exp2 / reciprocal / tanh approximations: their relative error (~1e-6, and 2^-11 for tanh) is far below
// the bf16 rounding that follows. Short and inline so the unrolled epilogue columns overlap.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// act: 0 SiLU, 1 GELU-tanh (SMELB_ACT_*)
__device__ __forceinline__ float act_fwd(float x, int act) {
  if (act == 0) return __fdividef(x, 1.0f + __expf(-x));
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  return 0.5f * x * (1.0f + tanh_approx(k0 * (x + k1 * x * x * x)));
}


}  // namespace smelb
