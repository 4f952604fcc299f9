// Shared helpers of the sm_100a INT4 MoE kernels: error plumbing, dtype
// traits, and inline-PTX wrappers (cp.async, TMA bulk copies, mbarriers,
// mma.sync).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string>

#include "../../include/hydranet_b200.h"

namespace hn {

// ----------------------------------------------------------------------------
// Host-side error handling
// ----------------------------------------------------------------------------
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int check_cuda(cudaError_t e, const char* what);
int sm_count_current();

#define HN_REQUIRE(cond, msg)                                  \
  do {                                                         \
    if (!(cond)) return ::hn::fail(HN_ERR_INVALID, (msg));     \
  } while (0)
#define HN_REQUIRE_SUPPORTED(cond, msg)                        \
  do {                                                         \
    if (!(cond)) return ::hn::fail(HN_ERR_UNSUPPORTED, (msg)); \
  } while (0)
#define HN_CUDA(call)                                          \
  do {                                                         \
    int _rc = ::hn::check_cuda((call), #call);                 \
    if (_rc) return _rc;                                       \
  } while (0)

// Device error codes written into a workspace's error word.
enum : int { DEV_ERR_NONE = 0, DEV_ERR_WAIT_TIMEOUT = 1, DEV_ERR_BAD_INDEX = 2 };

// ----------------------------------------------------------------------------
// Activation dtype traits.  Dequantisation uses the exponent-magic trick
// (Kim et al., 2022, "Who Says Elephants Can't Run: Bringing Large Scale MoE
// Models into Cloud Scale Production"; also FasterTransformer): OR-ing a
// nibble n into the mantissa of a power of two gives the exact value 2^e + n.
// ----------------------------------------------------------------------------
struct BF16 {
  using T = __nv_bfloat16;
  using T2 = __nv_bfloat162;
  // 0x4300 = 128.0: low nibble -> 128 + n; nibble at bits 3..6 -> 128 + 8n.
  static constexpr uint32_t kMagic = 0x43004300u;
  static constexpr float kOddScale = 0.125f;   // B operand of odd k is x/8
  static constexpr float kCorrEven = 136.0f;   // (128 + n) - (n - 8)
  static constexpr float kCorrOdd = 24.0f;     // (16 + n) - (n - 8)
  static __device__ __forceinline__ float to_f(T v) { return __bfloat162float(v); }
  static __device__ __forceinline__ T from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    T2 p = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&p);
  }
};

struct F16 {
  using T = __half;
  using T2 = __half2;
  // 0x6400 = 1024.0: low nibble -> 1024 + n; nibble at bits 4..7 -> 1024 + 16n.
  static constexpr uint32_t kMagic = 0x64006400u;
  static constexpr float kOddScale = 0.0625f;  // B operand of odd k is x/16
  static constexpr float kCorrEven = 1032.0f;  // (1024 + n) - (n - 8)
  static constexpr float kCorrOdd = 72.0f;     // (64 + n) - (n - 8)
  static __device__ __forceinline__ float to_f(T v) { return __half2float(v); }
  static __device__ __forceinline__ T from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    T2 p = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&p);
  }
};

// ----------------------------------------------------------------------------
// PTX wrappers
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

template <uint32_t kMask>
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t c) {
  // (a & kMask) | c  -- one LOP3
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(d) : "r"(a), "n"(kMask), "r"(c));
  return d;
}

// cp.async 16 bytes global -> shared, L1 bypass, 256-byte L2 prefetch hint.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: the waiting thread is suspended in
// hardware until the phase completes or about hint_ns pass, instead of
// re-issuing polls that take issue slots from the other warps of its SMSP.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: gives up after kWaitLimitNs, records DEV_ERR_WAIT_TIMEOUT in
// *err and returns false, so a kernel whose partner never arrives still ends.
// Once any thread of the launch has recorded an error, every later wait of
// every thread gives up at once (it polls *err), so a failing launch finishes
// within about one wait limit instead of one limit per wait.
constexpr uint64_t kWaitLimitNs = 2000000000ull;
__device__ __forceinline__ int ld_volatile_s32(const int* p) {
  int v;
  asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
constexpr uint32_t kSuspendHintNs = 20000;
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  if (err && ld_volatile_s32(err) != 0) return false;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 8; ++i)
      if (mbar_try_wait_sleep(bar, parity, kSuspendHintNs)) return true;
    if (err && ld_volatile_s32(err) != 0) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
  if (err) atomicExch(err, DEV_ERR_WAIT_TIMEOUT);
  return false;
}

// TMA bulk copy (non-tensor) global -> shared, completion on an mbarrier.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Named barrier among a subset of warps.
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// D = A * B + C, m16n8k16, fp32 accumulate.
template <typename Tr>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);

template <>
__device__ __forceinline__ void mma16816<BF16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<F16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float ld_cg_f32(const float* p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ld_cg_f32x4(const float4* p) {
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + __expf(-v)); }

}  // namespace hn

namespace hn {
// ----------------------------------------------------------------------------
// tcgen05 (5th-generation tensor core) wrappers.  Formats follow the PTX ISA
// for sm_100a: instruction descriptor for .kind::f16 (D f32 at bits 4-5, A/B
// format at 7-9 / 10-12, N>>3 at 17-22, M>>4 at 24-28) and the shared-memory
// matrix descriptor (start>>4 at 0-13, LBO>>4 at 16-29, SBO>>4 at 32-45,
// version 1 at 46-47, layout type at 61-63; 0 = no swizzle).
// ----------------------------------------------------------------------------
template <typename Tr, int M, int N>
__host__ __device__ constexpr uint32_t umma_idesc() {
  constexpr uint32_t ab = (Tr::kMagic == 0x43004300u) ? 1u : 0u;  // 1 = bf16, 0 = f16
  return (1u << 4) | (ab << 7) | (ab << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ uint64_t umma_sdesc_noswizzle(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;  // descriptor version for sm_100
  return d;                 // base offset 0, legacy LBO mode, layout SWIZZLE_NONE (0)
}

__device__ __forceinline__ void tmem_alloc(uint32_t smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_dst), "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem desc], one elected thread; enable_d = 0 overwrites D.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t enable_d) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      :
      : "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(enable_d), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
// One k-group of one matrix: eight K=16 steps D (+)= A[a + 8s] * B[desc + s*step]
// (the first overwrites D) and the correction step D += A[a_corr] * B[desc_c].
// The WHOLE warp executes this with warp-uniform operands and elect.sync picks
// the one issuing lane inside the asm: issued that way an MMA costs about 18
// cycles at N <= 32, against about 46 when one lane issues it from a divergent
// branch.  Descriptors are passed as their 32-bit halves: the low half holds
// the start address and LBO, the high half SBO and the version.
template <int kStepB>
__device__ __forceinline__ void umma_group9(uint32_t d, uint32_t a, uint32_t b_lo, uint32_t b_hi, uint32_t idesc,
                                            uint32_t c_lo, uint32_t a_corr, uint32_t idesc_c) {
  asm volatile(
      "{\n\t.reg .pred pf, pt, e;\n\t.reg .b64 bd;\n\t.reg .b32 al, bl;\n\t"
      "setp.ne.b32 pf, %3, %3;\n\t"
      "setp.eq.b32 pt, %3, %3;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "mov.b64 bd, {%2, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], bd, %4, pf;\n\t"
      "add.u32 al, %1, 8;\n\tadd.u32 bl, %2, %5;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, bl, %5;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, bl, %5;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, bl, %5;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, bl, %5;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, bl, %5;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, bl, %5;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "mov.b64 bd, {%6, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%7], bd, %8, pt;\n\t}"
      :
      : "r"(d), "r"(a), "r"(b_lo), "r"(b_hi), "r"(idesc), "n"(kStepB), "r"(c_lo), "r"(a_corr), "r"(idesc_c)
      : "memory");
}

// Same k-group with the B operand in the K-major 128B-swizzle layout: k-step
// s reads half s/4 of the tile (N rows of 128 B each) at byte 32*(s%4), i.e.
// start = b_lo + (s/4)*8N + (s%4)*2 in 16-byte units.  The correction step has
// its own descriptor (no swizzle) with high half c_hi.
template <int N>
__device__ __forceinline__ void umma_group9_sw128(uint32_t d, uint32_t a, uint32_t b_lo, uint32_t b_hi,
                                                  uint32_t idesc, uint32_t c_lo, uint32_t c_hi, uint32_t a_corr,
                                                  uint32_t idesc_c) {
  asm volatile(
      "{\n\t.reg .pred pf, pt, e;\n\t.reg .b64 bd;\n\t.reg .b32 al, bl;\n\t"
      "setp.ne.b32 pf, %3, %3;\n\t"
      "setp.eq.b32 pt, %3, %3;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "mov.b64 bd, {%2, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], bd, %4, pf;\n\t"
      "add.u32 al, %1, 8;\n\tadd.u32 bl, %2, 2;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, %2, 4;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, %2, 6;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, %2, %5;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, bl, 2;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, bl, 2;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, bl, 2;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "mov.b64 bd, {%6, %7};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%8], bd, %9, pt;\n\t}"
      :
      : "r"(d), "r"(a), "r"(b_lo), "r"(b_hi), "r"(idesc), "n"(8 * N), "r"(c_lo), "r"(c_hi), "r"(a_corr),
        "r"(idesc_c)
      : "memory");
}

// tcgen05.commit from one elected lane of a converged warp (the lane that
// issued the MMAs through umma_group9's elect.sync: elect.sync picks the same
// lane, the lowest active one, every time).
__device__ __forceinline__ void umma_commit_elect(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar)
      : "memory");
}

// Arrive on an mbarrier once every previously issued tcgen05 async op of this thread completes.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
// Waits for this thread's prior tcgen05.st and keeps the two 16-word source
// arrays live (as asm inputs) until then, so their registers are not reused
// while a store may still be reading them.
__device__ __forceinline__ void tc_wait_st_keep(const uint32_t (&a)[16], const uint32_t (&b)[16]) {
  asm volatile(
      "tcgen05.wait::st.sync.aligned;" ::"r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]),
      "r"(a[6]), "r"(a[7]), "r"(a[8]), "r"(a[9]), "r"(a[10]), "r"(a[11]), "r"(a[12]), "r"(a[13]), "r"(a[14]),
      "r"(a[15]), "r"(b[0]), "r"(b[1]), "r"(b[2]), "r"(b[3]), "r"(b[4]), "r"(b[5]), "r"(b[6]), "r"(b[7]), "r"(b[8]),
      "r"(b[9]), "r"(b[10]), "r"(b[11]), "r"(b[12]), "r"(b[13]), "r"(b[14]), "r"(b[15])
      : "memory");
}

// tcgen05.ld writes its destination registers asynchronously; they are valid
// only after tcgen05.wait::ld.  tmem_ld8 issues the load; tmem_ld_wait8 waits
// AND names the registers as outputs, so the compiler cannot schedule any use
// of them before the wait.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tmem_ld_wait8(uint32_t (&r)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7])
               :
               : "memory");
}
__device__ __forceinline__ void reg_dep16(uint32_t (&r)[16]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}
// Orders later uses of r after a preceding (asm volatile) tcgen05.wait::ld.
__device__ __forceinline__ void reg_dep8(uint32_t (&r)[8]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}
// (a0, a1) += s * (d0, d1) with one packed fp32x2 FMA (sm_100).
__device__ __forceinline__ void ffma2(float& a0, float& a1, float s, uint32_t d0, uint32_t d1) {
  asm("{\n\t.reg .b64 ta, ts, td;\n\t"
      "mov.b64 ta, {%0, %1};\n\t"
      "mov.b64 ts, {%2, %2};\n\t"
      "mov.b64 td, {%3, %4};\n\t"
      "fma.rn.f32x2 ta, ts, td, ta;\n\t"
      "mov.b64 {%0, %1}, ta;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(s), "r"(d0), "r"(d1));
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Dequantise one 32-bit word (8 nibbles of k = 8w..8w+7) into 4 TMEM columns of
// bf16/f16 pairs: (n0,n4) (n2,n6) as 2^e+n, (n1,n5) (n3,n7) as 2^e+8n (bf16) or
// 2^e+16n (f16).
// Right shifts done on the FMA pipe: w >> k == mulhi(w, 2^(32-k)).  The
// multipliers are passed in registers loaded from kernel arguments so the
// compiler cannot turn them back into shifts, which would put all of the
// dequantisation on the (half-rate) integer ALU pipe.
struct ShiftMul {
  uint32_t m1, m8, m9;  // 2^31, 2^24, 2^23
};
__device__ __forceinline__ uint32_t mulhi_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.hi.u32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
template <typename Tr>
__device__ __forceinline__ void dequant_word_fma(uint32_t w, uint32_t* o, const ShiftMul& sm) {
  const uint32_t M = Tr::kMagic;
  const uint32_t w8 = mulhi_u32(w, sm.m8);
  o[0] = lop3_and_or<0x000F000Fu>(w, M);
  o[1] = lop3_and_or<0x000F000Fu>(w8, M);
  if constexpr (Tr::kMagic == BF16::kMagic) {
    o[2] = lop3_and_or<0x00780078u>(mulhi_u32(w, sm.m1), M);
    o[3] = lop3_and_or<0x00780078u>(mulhi_u32(w, sm.m9), M);
  } else {
    o[2] = lop3_and_or<0x00F000F0u>(w, M);
    o[3] = lop3_and_or<0x00F000F0u>(w8, M);
  }
}

template <typename Tr>
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t* o) {
  const uint32_t M = Tr::kMagic;
  o[0] = lop3_and_or<0x000F000Fu>(w, M);
  o[1] = lop3_and_or<0x000F000Fu>(w >> 8, M);
  if constexpr (Tr::kMagic == BF16::kMagic) {
    o[2] = lop3_and_or<0x00780078u>(w >> 1, M);
    o[3] = lop3_and_or<0x00780078u>(w >> 9, M);
  } else {
    o[2] = lop3_and_or<0x00F000F0u>(w, M);
    o[3] = lop3_and_or<0x00F000F0u>(w >> 8, M);
  }
}

}  // namespace hn
