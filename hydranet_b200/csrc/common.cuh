// Shared helpers of the sm_100a INT4 MoE kernels: error plumbing, dtype
// traits, and inline-PTX wrappers (cp.async, TMA bulk copies, mbarriers,
// tcgen05, programmatic dependent launch).
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
// hn_int4_linear and its workspace size with segments of at most 8*max_nt
// tokens (hn_int4_linear itself allows 128).
size_t int4_linear_workspace_nt(int64_t M, int64_t N, int64_t K, int max_nt);
// Address of hn_int4_linear_static's scratch array on the current device.
int static_scratch_address(void** out);
int int4_linear_nt(const void* x, int64_t ldx, int dtype, int64_t M, int64_t K, const uint8_t* w_packed,
                   const uint16_t* w_scales, int64_t N, int group_size, void* out, int64_t ldo, void* workspace,
                   size_t workspace_bytes, void* stream, int max_nt);

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
// Activation dtype traits (kMagic, the bit pattern of 1024.0 or 128.0 in the
// type, also tells the tensor-core instruction descriptor which type it is).
// ----------------------------------------------------------------------------
struct BF16 {
  using T = __nv_bfloat16;
  using T2 = __nv_bfloat162;
  static constexpr uint32_t kMagic = 0x43004300u;
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
  static constexpr uint32_t kMagic = 0x64006400u;
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
// Arrive once for the whole (converged) warp: one elected lane arrives.
__device__ __forceinline__ void mbar_arrive_elect(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b64 st;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
      : "memory");
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
// A wait first polls the barrier alone (kQuietPolls suspending try_waits, at
// most kQuietPolls * kSuspendHintNs): reading *err is a global-memory round
// trip, and a wait that branched on it before polling would pay that latency
// even when the phase completes a few cycles later.  Past the quiet polls it
// reads *err every kQuietPolls polls, so once any thread of the launch has
// recorded an error every other wait gives up within a few milliseconds, and
// a failing launch finishes within about one wait limit.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Records a device error code in the workspace's error word and, when bytes
// 8..15 of the workspace hold the address of a host-mapped int32 (pinned
// host memory; NULL: none), in that word too, so the host can see the error
// with a plain memory read, without synchronising.  Only failure paths call
// this.
__device__ __forceinline__ void record_error(int* err, int code) {
  if (!err) return;
  atomicExch(err, code);
  int* mirror = *reinterpret_cast<int* volatile*>(reinterpret_cast<char*>(err) + 8);
  if (mirror) {
    *reinterpret_cast<volatile int*>(mirror) = code;
    __threadfence_system();
  }
}
constexpr int kQuietPolls = 16;
__device__ __forceinline__ int ld_volatile_s32(const int* p) {
  int v;
  asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
constexpr uint32_t kSuspendHintNs = 20000;
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
#pragma unroll 1
  for (int i = 0; i < kQuietPolls; ++i)
    if (mbar_try_wait_sleep(bar, parity, kSuspendHintNs)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (err && ld_volatile_s32(err) != 0) return false;
#pragma unroll 1
    for (int i = 0; i < kQuietPolls; ++i)
      if (mbar_try_wait_sleep(bar, parity, kSuspendHintNs)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
  record_error(err, DEV_ERR_WAIT_TIMEOUT);
  return false;
}

// Bounded wait for a partner that is usually far away (an epilogue waiting
// for the end of a piece): poll, then sleep sleep_ns between polls, so the
// waiting warp takes almost no issue slots from the warps of its SMSP.
// Reads *err every 64 polls; same time limit and error reporting as mbar_wait.
__device__ __forceinline__ bool mbar_wait_backoff(uint32_t bar, uint32_t parity, int* err, uint32_t sleep_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    __nanosleep(sleep_ns);
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (err && ld_volatile_s32(err) != 0) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
  }
  record_error(err, DEV_ERR_WAIT_TIMEOUT);
  return false;
}

// Programmatic dependent launch: griddepcontrol.wait blocks until the
// preceding grid of the stream has completed and its memory is visible (it
// returns at once when the launch had no programmatic dependency);
// launch_dependents lets the next grid of the stream start launching.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
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

// One 128-wide k-group on the tensor core: eight K=16 steps with A = the
// 128 x 128 float16 weight tile in TMEM (8 columns per step) and B = the
// K-major SW128 token tile (two 64-k halves; step s starts at half s / 4,
// byte 32 * (s % 4); the second half is 8N 16-byte units after the first).
// The first step adds to D only when acc != 0.  One elected lane issues.
template <int N>
__device__ __forceinline__ void umma_group8_sw128(uint32_t d, uint32_t a, uint32_t b_lo, uint32_t b_hi,
                                                  uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p0, pt, e;\n\t.reg .b64 bd;\n\t.reg .b32 al, bl;\n\t"
      "setp.ne.b32 p0, %5, 0;\n\t"
      "setp.eq.b32 pt, %5, %5;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "mov.b64 bd, {%2, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], bd, %4, p0;\n\t"
      "add.u32 al, %1, 8;\n\tadd.u32 bl, %2, 2;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, %2, 4;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, %2, 6;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, %2, %6;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, bl, 2;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, bl, 2;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t"
      "add.u32 al, al, 8;\n\tadd.u32 bl, bl, 2;\n\tmov.b64 bd, {bl, %3};\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [al], bd, %4, pt;\n\t}"
      :
      : "r"(d), "r"(a), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(acc), "n"(8 * N)
      : "memory");
}

// tcgen05.commit from one elected lane of a converged warp (the lane that
// issued the MMAs through umma_group8_sw128's elect.sync: elect.sync picks the same
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
// Orders later uses of r after a preceding (asm volatile) tcgen05.wait::ld.
__device__ __forceinline__ void reg_dep8(uint32_t (&r)[8]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7])
               :
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
// wait::ld for two 16-column loads; both arrays become available after it.
__device__ __forceinline__ void tmem_ld_wait16x2(uint32_t (&r)[16], uint32_t (&q)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                 "+r"(q[0]), "+r"(q[1]), "+r"(q[2]), "+r"(q[3]), "+r"(q[4]), "+r"(q[5]), "+r"(q[6]), "+r"(q[7]),
                 "+r"(q[8]), "+r"(q[9]), "+r"(q[10]), "+r"(q[11]), "+r"(q[12]), "+r"(q[13]), "+r"(q[14]), "+r"(q[15])
               :
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
// Eight packed nibbles (one 32-bit word: k = 8c..8c+7, the even k in the low
// nibble of each byte) to four float16 pairs (n - 8) * s in the staged order
// {(k0,k4), (k2,k6), (k1,k5), (k3,k7)}.  Exponent-magic conversion (Kim et
// al., 2022, "Who Says Elephants Can't Run"; also FasterTransformer): OR-ing
// a nibble into the mantissa of 1024.0 gives 1024 + n (bits 0..3) or
// 1024 + 16n (bits 4..7) exactly;
// subtracting 1032, or scaling by 1/16 and subtracting 72, gives the integer
// n - 8 exactly, and the single rounding of its product with the float16
// scale pair s2 = (s, s) is the reference's `w_int.to(tl.float16) * scales`
// (kernels/int4_expert_mlp.py:83-90).  Thirteen instructions per word.
__device__ __forceinline__ void dequant_word_f16(uint32_t w, uint32_t s2, uint32_t* o) {
  const uint32_t w8 = w >> 8;
  uint32_t t0 = lop3_and_or<0x000F000Fu>(w, 0x64006400u);
  uint32_t t1 = lop3_and_or<0x000F000Fu>(w8, 0x64006400u);
  uint32_t t2 = lop3_and_or<0x00F000F0u>(w, 0x64006400u);
  uint32_t t3 = lop3_and_or<0x00F000F0u>(w8, 0x64006400u);
  asm("add.rn.f16x2 %0, %0, %1;" : "+r"(t0) : "r"(0xE408E408u));                   // - 1032
  asm("add.rn.f16x2 %0, %0, %1;" : "+r"(t1) : "r"(0xE408E408u));
  asm("fma.rn.f16x2 %0, %0, %1, %2;" : "+r"(t2) : "r"(0x2C002C00u), "r"(0xD480D480u));  // / 16 - 72
  asm("fma.rn.f16x2 %0, %0, %1, %2;" : "+r"(t3) : "r"(0x2C002C00u), "r"(0xD480D480u));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[0]) : "r"(t0), "r"(s2));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[1]) : "r"(t1), "r"(s2));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[2]) : "r"(t2), "r"(s2));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[3]) : "r"(t3), "r"(s2));
}

}  // namespace hn
