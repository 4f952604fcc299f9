// Expert-parallel exchange kernels: the device side of a dispatch/combine in
// which every rank owns a contiguous block of E/W experts.
//
// A rank's T tokens are sent at most once to each destination rank, with the
// token's top-k list rewritten for that rank (local expert id where the pick
// lives there, -1 elsewhere).  Block d of the send buffer holds one fixed row
// per token t -- [activations (H x 2 bytes) | k local ids (int32) | k weights
// (float32)] padded to 16 bytes -- so the block has T rows whatever the
// routing, one all-to-all with equal splits delivers it, and no count ever
// has to reach the host.  A row whose token has no pick on d keeps only its
// ids (all -1); the receiving grouped kernel skips such rows.
//
//   hn_ep_pack     x, routing -> send [W][T][row]
//   hn_ep_unpack   recv [W][T][row] -> rows [W*T][H], ids [W*T][k], weights [W*T][k]
//   hn_ep_combine  back [W][T][H] (per-destination partial sums) -> out [T][H],
//                  summed in rank order in fp32 over the ranks that had picks
#include <string>

#include "common.cuh"

namespace hn {
namespace {

__host__ __device__ inline size_t ep_row_bytes(int64_t H, int top_k) {
  return ((size_t)H * 2 + (size_t)top_k * 8 + 15) & ~(size_t)15;
}

// one CTA per (destination, token) row
__global__ void __launch_bounds__(256) ep_pack_kernel(const uint8_t* x, int T, int H, int K, const int32_t* idx,
                                                      const float* w, int per, uint8_t* send, size_t rb) {
  const int row = blockIdx.x, d = row / T, t = row - d * T;
  uint8_t* dst = send + (size_t)row * rb;
  __shared__ int s_any;
  if (threadIdx.x == 0) s_any = 0;
  __syncthreads();
  if (threadIdx.x < K) {
    const int e = idx[(int64_t)t * K + threadIdx.x];
    const bool mine = e >= d * per && e < (d + 1) * per;
    reinterpret_cast<int32_t*>(dst + (size_t)H * 2)[threadIdx.x] = mine ? e - d * per : -1;
    reinterpret_cast<float*>(dst + (size_t)H * 2 + (size_t)K * 4)[threadIdx.x] =
        mine ? w[(int64_t)t * K + threadIdx.x] : 0.f;
    if (mine) s_any = 1;
  }
  __syncthreads();
  if (!s_any) return;  // nothing of this token runs on d: its activations are not needed there
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * H * 2);
  uint4* o = reinterpret_cast<uint4*>(dst);
  for (int i = threadIdx.x; i < H / 8; i += 256) o[i] = __ldg(src + i);
}

__global__ void __launch_bounds__(256) ep_unpack_kernel(const uint8_t* recv, int H, int K, size_t rb, uint8_t* x_out,
                                                        int32_t* idx_out, float* w_out) {
  const int row = blockIdx.x;
  const uint8_t* src = recv + (size_t)row * rb;
  __shared__ int s_any;
  if (threadIdx.x == 0) s_any = 0;
  __syncthreads();
  if (threadIdx.x < K) {
    const int e = reinterpret_cast<const int32_t*>(src + (size_t)H * 2)[threadIdx.x];
    idx_out[(int64_t)row * K + threadIdx.x] = e;
    w_out[(int64_t)row * K + threadIdx.x] = reinterpret_cast<const float*>(src + (size_t)H * 2 + (size_t)K * 4)[threadIdx.x];
    if (e >= 0) s_any = 1;
  }
  __syncthreads();
  if (!s_any) return;  // an unused row: the grouped kernel skips it, its activations are never read
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  uint4* o = reinterpret_cast<uint4*>(x_out + (size_t)row * H * 2);
  for (int i = threadIdx.x; i < H / 8; i += 256) o[i] = s4[i];
}

// out[t, :] = sum over ranks d (in order) holding a pick of token t of back[d][t][:]
template <typename Tr>
__global__ void __launch_bounds__(256) ep_combine_kernel(const void* back, int T, int H, int K, const int32_t* idx,
                                                         int per, int W, void* out) {
  const int t = blockIdx.x;
  __shared__ unsigned s_mask;
  if (threadIdx.x == 0) s_mask = 0;
  __syncthreads();
  if (threadIdx.x < K) {
    const int e = idx[(int64_t)t * K + threadIdx.x];
    if (e >= 0 && e < per * W) atomicOr(&s_mask, 1u << (e / per));
  }
  __syncthreads();
  const unsigned mask = s_mask;
  const typename Tr::T* b = reinterpret_cast<const typename Tr::T*>(back);
  typename Tr::T* o = reinterpret_cast<typename Tr::T*>(out) + (int64_t)t * H;
  for (int h = threadIdx.x; h < H; h += 256) {
    float acc = 0.f;
    for (int d = 0; d < W; ++d)
      if (mask >> d & 1u) acc += Tr::to_f(b[((int64_t)d * T + t) * H + h]);
    o[h] = Tr::from_f(acc);
  }
}

int check_ep(int dtype, int64_t T, int64_t H, int top_k, int64_t E, int world) {
  HN_REQUIRE(dtype == HN_DTYPE_BF16 || dtype == HN_DTYPE_F16, "ep: activations must be float16 or bfloat16");
  HN_REQUIRE(T >= 1 && T <= (1 << 20) && H >= 8 && H % 8 == 0, "ep: bad token count or hidden size");
  HN_REQUIRE(top_k >= 1 && top_k <= 32, "ep: top_k must be 1..32");
  HN_REQUIRE(world >= 1 && world <= 32, "ep: world size must be 1..32");
  HN_REQUIRE(E >= world && E % world == 0, "ep: experts must split evenly over the ranks");
  HN_REQUIRE((int64_t)world * T <= (1 << 24), "ep: too many rows");
  return HN_OK;
}

}  // namespace
}  // namespace hn

using namespace hn;

extern "C" {

size_t hn_ep_row_bytes(int64_t H, int top_k) {
  if (H < 8 || top_k < 1) return 0;
  return ep_row_bytes(H, top_k);
}

int hn_ep_pack(const void* x, int dtype, int64_t T, int64_t H, int top_k, const int32_t* topk_idx,
               const float* topk_w, int64_t E, int world, void* send, void* stream) {
  int rc = check_ep(dtype, T, H, top_k, E, world);
  if (rc) return rc;
  HN_REQUIRE(x && topk_idx && topk_w && send, "hn_ep_pack: null pointer");
  HN_REQUIRE((((uintptr_t)x | (uintptr_t)send) & 15) == 0, "hn_ep_pack: x and send must be 16-byte aligned");
  ep_pack_kernel<<<(unsigned)(world * T), 256, 0, (cudaStream_t)stream>>>(
      static_cast<const uint8_t*>(x), (int)T, (int)H, top_k, topk_idx, topk_w, (int)(E / world),
      static_cast<uint8_t*>(send), ep_row_bytes(H, top_k));
  HN_CUDA(cudaGetLastError());
  return HN_OK;
}

int hn_ep_unpack(const void* recv, int dtype, int64_t rows, int64_t H, int top_k, void* x_out, int32_t* idx_out,
                 float* w_out, void* stream) {
  int rc = check_ep(dtype, rows, H, top_k, 1, 1);
  if (rc) return rc;
  HN_REQUIRE(recv && x_out && idx_out && w_out, "hn_ep_unpack: null pointer");
  HN_REQUIRE((((uintptr_t)recv | (uintptr_t)x_out) & 15) == 0, "hn_ep_unpack: recv and x_out must be 16-byte aligned");
  ep_unpack_kernel<<<(unsigned)rows, 256, 0, (cudaStream_t)stream>>>(static_cast<const uint8_t*>(recv), (int)H,
                                                                     top_k, ep_row_bytes(H, top_k),
                                                                     static_cast<uint8_t*>(x_out), idx_out, w_out);
  HN_CUDA(cudaGetLastError());
  return HN_OK;
}

int hn_ep_combine(const void* back, int dtype, int64_t T, int64_t H, int top_k, const int32_t* topk_idx, int64_t E,
                  int world, void* out, void* stream) {
  int rc = check_ep(dtype, T, H, top_k, E, world);
  if (rc) return rc;
  HN_REQUIRE(back && topk_idx && out, "hn_ep_combine: null pointer");
  const int per = (int)(E / world);
  if (dtype == HN_DTYPE_BF16)
    ep_combine_kernel<BF16><<<(unsigned)T, 256, 0, (cudaStream_t)stream>>>(back, (int)T, (int)H, top_k, topk_idx,
                                                                         per, world, out);
  else
    ep_combine_kernel<F16><<<(unsigned)T, 256, 0, (cudaStream_t)stream>>>(back, (int)T, (int)H, top_k, topk_idx,
                                                                        per, world, out);
  HN_CUDA(cudaGetLastError());
  return HN_OK;
}

}  // extern "C"
