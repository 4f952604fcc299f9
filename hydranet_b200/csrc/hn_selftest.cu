// hn_selftest_wait_timeout: the failure path of the library's bounded waits,
// on demand.  One CTA sets up an mbarrier that nothing ever arrives at and
// lets two warps wait on it with the same wait functions the engine uses
// (mbar_wait, mbar_wait_backoff).  The first wait to pass the time limit
// records DEV_ERR_WAIT_TIMEOUT in the workspace's error word; the other sees
// the word and gives up; the launch ends, and the context stays usable.  A
// test reads the word back with hn_workspace_error (or, when the self-test ran
// on hn_int4_linear_static's array, with hn_int4_linear_static_error).
#include "common.cuh"

namespace hn {
namespace {

__global__ void __launch_bounds__(64) wait_timeout_kernel(int* err, int mode) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);  // one arrival expected, none ever made
    fence_barrier_init();
  }
  __syncthreads();
  if ((threadIdx.x & 31) != 0) return;
  // phase 0 of a fresh barrier never completes here
  if (threadIdx.x == 0 && mode == 0)
    mbar_wait(b, 0, err);
  else
    mbar_wait_backoff(b, 0, err, 2000);
}

}  // namespace
}  // namespace hn

extern "C" int hn_selftest_wait_timeout(void* workspace, size_t workspace_bytes, int mode, void* stream) {
  HN_REQUIRE(mode == 0 || mode == 1, "hn_selftest_wait_timeout: mode is 0 or 1");
  if (!workspace) {
    // the error word of hn_int4_linear_static's array
    const int rc = hn::static_scratch_address(&workspace);
    if (rc) return rc;
    workspace_bytes = HN_INT4_LINEAR_STATIC_SCRATCH_BYTES;
  }
  HN_REQUIRE(workspace_bytes >= 512, "hn_selftest_wait_timeout: need a workspace of >= 512 bytes");
  hn::wait_timeout_kernel<<<1, 64, 0, (cudaStream_t)stream>>>(reinterpret_cast<int*>(workspace), mode);
  HN_CUDA(cudaGetLastError());
  return HN_OK;
}
