// hn_int4_linear_static: hn_int4_linear with its scratch in a device array
// compiled into the library, for callers that cannot provide device memory.
//
// The array is a file-scope __device__ variable, so the CUDA runtime creates
// one zero-filled copy per device when it loads this module there; nothing is
// allocated at call time.  Host code cannot use the array's name as a device
// address: every call looks the address up for the current device and
// context (cudaGetSymbolAddress, a host-side table lookup once the module is
// loaded), so a context that was reset or replaced never leaves a stale
// address behind.  The computation is the unchanged hn_int4_linear entry
// point, given that array as its workspace.
#include <string>

#include "common.cuh"

namespace hn {
namespace {

constexpr size_t kStaticScratchBytes = HN_INT4_LINEAR_STATIC_SCRATCH_BYTES;
// The widest token segments (at most 32 rows) whose scratch fits the array:
// the stream-K partials grow with the segment width (the 64- and 128-row
// segments hn_int4_linear uses above M = 64 need 19-39 MiB of partials
// alone).
constexpr int kStaticMaxNt = 4;
static_assert(kStaticScratchBytes % 256 == 0, "static scratch size must keep 256-byte granularity");

__device__ __align__(256) unsigned char g_linear_scratch[kStaticScratchBytes];

}  // namespace

// Address of the current device's copy of g_linear_scratch.
int static_scratch_address(void** out) {
  void* p = nullptr;
  HN_CUDA(cudaGetSymbolAddress(&p, g_linear_scratch));
  HN_REQUIRE(p && ((uintptr_t)p & 255) == 0, "int4_linear_static: static scratch is not 256-byte aligned");
  *out = p;
  return HN_OK;
}

// Segment cap (tokens / 8) for a static call: 4, 2 or 1, the first whose
// scratch fits; the cap with the smallest scratch when none does.
int static_max_nt(int64_t M, int64_t N, int64_t K) {
  for (int nt = kStaticMaxNt; nt > 1; nt /= 2)
    if (int4_linear_workspace_nt(M, N, K, nt) <= kStaticScratchBytes) return nt;
  return 1;
}

}  // namespace hn

extern "C" size_t hn_int4_linear_static_scratch_size(int64_t M, int64_t N, int64_t K) {
  return hn::int4_linear_workspace_nt(M, N, K, hn::static_max_nt(M, N, K));
}

extern "C" int hn_int4_linear_static(const void* x, int64_t ldx, int dtype, int64_t M, int64_t K,
                                     const uint8_t* w_packed, const uint16_t* w_scales, int64_t N, int group_size,
                                     void* out, int64_t ldo, void* stream) {
  const int max_nt = hn::static_max_nt(M, N, K);
  const size_t need = hn::int4_linear_workspace_nt(M, N, K, max_nt);
  if (need == 0) return hn::fail(HN_ERR_INVALID, "int4_linear_static: need M, N >= 1 and K >= 128");
  if (need > hn::kStaticScratchBytes)
    return hn::fail(HN_ERR_WORKSPACE, "int4_linear_static: M=" + std::to_string(M) + " N=" + std::to_string(N) +
                                          " K=" + std::to_string(K) + " needs " + std::to_string(need) +
                                          " bytes of scratch, more than the " +
                                          std::to_string(hn::kStaticScratchBytes) +
                                          " bytes compiled into the library; call hn_int4_linear with a workspace");
  void* ws = nullptr;
  const int rc = hn::static_scratch_address(&ws);
  if (rc) return rc;
  return hn::int4_linear_nt(x, ldx, dtype, M, K, w_packed, w_scales, N, group_size, out, ldo, ws,
                            hn::kStaticScratchBytes, stream, max_nt);
}

// The array's error word (its first 4 bytes), read on 'stream' and cleared.
extern "C" int hn_int4_linear_static_error(int* error_code, void* stream) {
  HN_REQUIRE(error_code, "hn_int4_linear_static_error: error_code is NULL");
  void* ws = nullptr;
  const int rc = hn::static_scratch_address(&ws);
  if (rc) return rc;
  return hn_workspace_error(ws, hn::kStaticScratchBytes, error_code, stream);
}
