// Error plumbing, device queries, the INT4 packer/unpacker/dequantiser and the
// elementwise SiLU*mul kernel.
#include <atomic>
#include <cstdio>
#include <mutex>
#include <unordered_map>

#include "common.cuh"

namespace hn {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return HN_OK;
  std::string m = std::string(what) + ": " + cudaGetErrorString(e);
  cudaGetLastError();  // clear a sticky launch error so the next call starts clean
  return fail(HN_ERR_CUDA, m);
}

static std::atomic<int> g_sm_limit{0};  // hn_set_sm_limit (0: none)

static int sm_count_device() {
  static std::mutex mu;
  static std::unordered_map<int, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  cache[dev] = n;
  return n;
}

// SMs the engines size their grids for: the device's, or fewer under hn_set_sm_limit.
int sm_count_current() {
  const int n = sm_count_device();
  const int lim = g_sm_limit.load(std::memory_order_relaxed);
  return (n > 0 && lim > 0 && lim < n) ? lim : n;
}

// ---------------------------------------------------------------------------
// Packer: one warp per (row, 128-column group); each lane owns 4 columns.
// Arithmetic follows ExpertWeightPacker.quantize_tensor
// (preprocess/pack_weights.py:156-181) in the input dtype: absmax, /7 (IEEE
// division, rounded to the input dtype), clamp(min=1e-10) in that dtype,
// w/scale (rounded to the input dtype), round-half-even, clip to [-8, 7], +8.
// ---------------------------------------------------------------------------
template <typename In>
__device__ __forceinline__ float load_w(const In* p);
template <>
__device__ __forceinline__ float load_w<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float load_w<__half>(const __half* p) { return __half2float(*p); }

template <typename In>
__device__ __forceinline__ float to_in_dtype(float v);
template <>
__device__ __forceinline__ float to_in_dtype<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_in_dtype<__half>(float v) { return __half2float(__float2half_rn(v)); }

template <typename In>
__global__ void quantize_kernel(const In* __restrict__ w, int64_t rows, int64_t cols, uint8_t* __restrict__ packed,
                                uint16_t* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const int64_t groups = cols / 128;
  const int64_t task = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (task >= rows * groups) return;
  const int64_t r = task / groups, g = task % groups;
  const In* src = w + r * cols + g * 128 + lane * 4;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = load_w<In>(src + i);
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  float scale = to_in_dtype<In>(__fdiv_rn(amax, 7.0f));
  scale = fmaxf(scale, to_in_dtype<In>(1e-10f));
  uint32_t q[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float t = rintf(to_in_dtype<In>(__fdiv_rn(v[i], scale)));
    t = fminf(fmaxf(t, -8.0f), 7.0f);
    // an all-zero fp16 group divides 0 by 0; the result NaN is stored as nibble 0
    q[i] = (t != t) ? 0u : (uint32_t)(int)(t + 8.0f);
  }
  uint16_t two = (uint16_t)((q[0] | (q[1] << 4)) | ((q[2] | (q[3] << 4)) << 8));
  *reinterpret_cast<uint16_t*>(packed + r * (cols / 2) + g * 64 + lane * 2) = two;
  if (lane == 0) {
    __half hs = __float2half_rn(scale);
    scales[r * groups + g] = *reinterpret_cast<uint16_t*>(&hs);
  }
}

__global__ void unpack_kernel(const uint8_t* __restrict__ packed, int64_t nbytes, uint8_t* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nbytes; i += (int64_t)gridDim.x * blockDim.x) {
    uint8_t b = packed[i];
    out[2 * i] = b & 0xF;
    out[2 * i + 1] = b >> 4;
  }
}

__global__ void dequant_kernel(const uint8_t* __restrict__ packed, const __half* __restrict__ scales, int64_t rows,
                               int64_t cols, __half* __restrict__ out) {
  const int64_t n = rows * cols / 2;
  const int64_t groups = cols / 128;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (cols / 2), c = (i % (cols / 2)) * 2;
    const __half s = scales[r * groups + c / 128];
    const uint8_t b = packed[i];
    out[r * cols + c] = __hmul(__int2half_rn((int)(b & 0xF) - 8), s);
    out[r * cols + c + 1] = __hmul(__int2half_rn((int)(b >> 4) - 8), s);
  }
}

template <typename Tr>
__global__ void silu_mul_kernel(const typename Tr::T* __restrict__ g, const typename Tr::T* __restrict__ u,
                                typename Tr::T* __restrict__ o, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float a = Tr::to_f(g[i]);
    o[i] = Tr::from_f(a / (1.0f + expf(-a)) * Tr::to_f(u[i]));
  }
}

static int grid_for(int64_t work, int block) {
  int64_t sms = sm_count_current();
  if (sms <= 0) sms = 148;
  int64_t g = (work + block - 1) / block;
  return (int)std::max<int64_t>(1, std::min<int64_t>(g, sms * 16));
}

}  // namespace hn

using namespace hn;

extern "C" {

int hn_abi_version(void) { return HN_ABI_VERSION; }

const char* hn_last_error(void) { return g_last_error.c_str(); }

int hn_device_sm_count(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int hn_set_sm_limit(int max_sms) {
  if (max_sms < 0) return -1;
  return hn::g_sm_limit.exchange(max_sms);
}

int hn_quantize_int4(const void* w, int w_dtype, int64_t rows, int64_t cols, int group_size, uint8_t* packed,
                     uint16_t* scales, void* stream) {
  HN_REQUIRE(w && packed && scales, "hn_quantize_int4: null pointer");
  HN_REQUIRE(rows >= 0 && cols >= 0, "hn_quantize_int4: negative shape");
  HN_REQUIRE(group_size > 0 && cols % group_size == 0,
             "hn_quantize_int4: in_features must be divisible by group_size");
  HN_REQUIRE_SUPPORTED(group_size == 128, "hn_quantize_int4: only group_size 128 is implemented");
  if (rows == 0 || cols == 0) return HN_OK;
  const int64_t tasks = rows * (cols / 128);
  const int block = 256;
  const int64_t grid = (tasks + 7) / 8;
  HN_REQUIRE(grid < (int64_t)1 << 31, "hn_quantize_int4: matrix too large");
  cudaStream_t s = (cudaStream_t)stream;
  if (w_dtype == HN_DTYPE_F32)
    quantize_kernel<float><<<(unsigned)grid, block, 0, s>>>((const float*)w, rows, cols, packed, scales);
  else if (w_dtype == HN_DTYPE_F16)
    quantize_kernel<__half><<<(unsigned)grid, block, 0, s>>>((const __half*)w, rows, cols, packed, scales);
  else
    return fail(HN_ERR_UNSUPPORTED, "hn_quantize_int4: weight dtype must be float32 or float16");
  HN_CUDA(cudaGetLastError());
  return HN_OK;
}

int hn_unpack_int4(const uint8_t* packed, int64_t rows, int64_t cols, uint8_t* out, void* stream) {
  HN_REQUIRE(packed && out, "hn_unpack_int4: null pointer");
  HN_REQUIRE(rows >= 0 && cols >= 0 && cols % 2 == 0, "hn_unpack_int4: cols must be even");
  const int64_t n = rows * cols / 2;
  if (n == 0) return HN_OK;
  unpack_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(packed, n, out);
  HN_CUDA(cudaGetLastError());
  return HN_OK;
}

int hn_dequant_int4(const uint8_t* packed, const uint16_t* scales, int64_t rows, int64_t cols, int group_size,
                    uint16_t* out, void* stream) {
  HN_REQUIRE(packed && scales && out, "hn_dequant_int4: null pointer");
  HN_REQUIRE(rows >= 0 && cols >= 0 && group_size > 0 && cols % group_size == 0, "hn_dequant_int4: bad shape");
  HN_REQUIRE_SUPPORTED(group_size == 128, "hn_dequant_int4: only group_size 128 is implemented");
  const int64_t n = rows * cols / 2;
  if (n == 0) return HN_OK;
  dequant_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(packed, (const __half*)scales, rows, cols,
                                                                      (__half*)out);
  HN_CUDA(cudaGetLastError());
  return HN_OK;
}

int hn_silu_mul(const void* gate, const void* up, void* out, int64_t n, int dtype, void* stream) {
  HN_REQUIRE(gate && up && out, "hn_silu_mul: null pointer");
  HN_REQUIRE(n >= 0, "hn_silu_mul: negative size");
  if (n == 0) return HN_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == HN_DTYPE_BF16)
    silu_mul_kernel<BF16><<<grid_for(n, 256), 256, 0, s>>>((const __nv_bfloat16*)gate, (const __nv_bfloat16*)up,
                                                          (__nv_bfloat16*)out, n);
  else if (dtype == HN_DTYPE_F16)
    silu_mul_kernel<F16><<<grid_for(n, 256), 256, 0, s>>>((const __half*)gate, (const __half*)up, (__half*)out, n);
  else
    return fail(HN_ERR_UNSUPPORTED, "hn_silu_mul: dtype must be float16 or bfloat16");
  HN_CUDA(cudaGetLastError());
  return HN_OK;
}

}  // extern "C"
