// INT4 mixture-of-experts decode path for sm_100a.
//
//   route_prep_kernel   one CTA per token: router logits / top-k / weights
//                       (or caller-given routing), the token's activations
//                       staged as float16 in MMA operand order, and -- in the
//                       last CTA to finish -- the dispatch plan (per-expert
//                       token lists cut into segments of at most 8*nt tokens).
//   tc_engine_kernel    persistent grouped INT4 GEMV/GEMM on the tcgen05 tensor
//                       cores over (weight-row tile x segment) tiles, k-split
//                       "stream-K" style so every CTA streams the same number
//                       of 128-wide k-groups.
//                       KIND_GATEUP: gate+up rows together, SiLU(gate)*up in
//                       the epilogue, written as the next phase's operand.
//                       KIND_DOWN: down projection; EPI_COMBINE scales by the
//                       routing weight and sums the top-k choices per token,
//                       EPI_STORE writes rows straight to the output.
//
// Arithmetic follows the reference kernel (kernels/int4_expert_mlp.py:55-93):
// weights are dequantised to float16 as (n - 8) * scale with one rounding,
// activations enter as float16, and products accumulate in fp32.  The
// dequantised tile is written to tensor memory and used as the A operand of
// tcgen05.mma (M = 128 weight rows), the tokens are the B operand (N = 16 or
// 32) in shared memory, and each piece of a tile accumulates in TMEM.
#include <algorithm>
#include <atomic>
#include <type_traits>
#include <cstring>
#include <string>
#include <cuda.h>

#include "common.cuh"

namespace hn {

constexpr int kChunk = 256;  // bytes per (token, k-group): 16 units of 16 B (128 float16)
constexpr int kMaxExperts = 1024;
constexpr int kMaxTopK = 32;
constexpr int kPlanSmemEntries = 4096;  // routing entries the plan builder copies into shared memory
// Routings of up to this many (token, slot) entries are planned by the prep
// kernel's last CTA, which counts each assignment's rank directly; larger
// ones by plan_kernel (one CTA per expert), whose cost does not grow with
// experts x tokens.
constexpr int kPlanRankEntries = 1024;

enum { KIND_GATEUP = 0, KIND_DOWN = 1 };
enum { EPI_COMBINE = 0, EPI_STORE = 1 };
enum { ROUTE_COMPUTE = 0, ROUTE_GIVEN = 1, ROUTE_IDENTITY = 2 };

struct Plan {
  int* err;
  int* route_ctr;
  int* counts;   // [E]
  int* n_segs;   // [1]
  int4* segs;    // [max_segs] {expert, first assignment, tokens, 0}
  int* n_segs2;  // [1] a second cut of the same lists into seg2-token segments (down phase), or NULL
  int4* segs2;   // [max_segs2]
  int seg2;      // 0: no second cut
  int* a_tok;    // [T*K] token of assignment p
  int* a_tk;     // [T*K] t*K + slot of assignment p (inverse of pos)
  float* a_w;    // [T*K] routing weight of assignment p
  int* pos;      // [T*K] assignment index of (t, k)
  int* idx;      // [T*K] top-k expert ids
  float* wts;    // [T*K] top-k weights (rounded to the activation dtype)
  int* nval;     // [T] slots of each token that hold an expert (caller routing may leave slots -1)
  int* n_assign; // [1] assignments planned (T*K less the -1 slots)
  uint8_t* xp;   // [T][K_in/128][kChunk]    staged activations (token-major)
  uint8_t* hp;   // [T*K][F/128][kChunk]     staged SiLU(gate)*up (assignment-major)
  float* corr_x; // [T][K_in/128]  offset staging: per (token, k-group) correction of the mma.sync engine
  float* corr_h; // [T*K][F/128]   the same for hp
  uint8_t* xs;   // [T*K][K_in/128][kChunk]  staged activations in assignment order (large routings), or NULL
  float* part1;  // stream-K partial tiles, phase 1
  float* part2;  // stream-K partial tiles, phase 2
  float* R;      // [T*K][H] weighted expert outputs (EPI_COMBINE)
  float* rlog;   // [T][E] router logits of a large batch (router_logits_kernel), or NULL
  int* ctr1;     // per phase-1 tile arrival counters
  int* ctr2;     // per phase-2 tile arrival counters
  int* rtctr;    // [row tiles][T] contributions summed into (row tile, token) so far
  int n_ctr;     // words from ctr1 to the end of the counter section (zeroed by the prep kernel)
};

__host__ __device__ constexpr int seg_tokens(int nt) { return 8 * nt; }

// ---------------------------------------------------------------------------
// Activation staging.  For k-group g and token t a 256-byte chunk holds 16
// units of 16 bytes; unit c covers x[128*g + 8*c + i], i = 0..7, as float16
// pairs in the order
//   { (x0, x4), (x2, x6), (x1, x5), (x3, x7) },
// the order in which dequant_word_f16 produces the same 8 nibbles of a packed
// 32-bit word, so TMEM column 4c + i of a dequantised weight row and 32-bit
// word i of unit c hold the same two k.  A unit is one 16-byte row of a
// K-major core matrix of the tensor-core B operand.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  return (uint32_t)__half_as_ushort(__float2half_rn(lo)) | ((uint32_t)__half_as_ushort(__float2half_rn(hi)) << 16);
}
__device__ __forceinline__ uint4 pack_unit(const float (&v)[8]) {
  return make_uint4(pack_h2(v[0], v[4]), pack_h2(v[2], v[6]), pack_h2(v[1], v[5]), pack_h2(v[3], v[7]));
}
// Offset staging for the mma.sync engine: it feeds the tensor core the
// exponent-magic values 1024 + n (even k) and 1024 + 16n (odd k) as they
// are, so the odd k of the tokens are staged divided by 16 and each
// (token, k-group) carries the sum the offsets add:
//   sum_k (w_k - 8) b_k = MMA - (1032 * sum_even b + 1152 * sum_odd b)
// with b the staged float16 values (odd ones already divided by 16).
__device__ __forceinline__ float gv_offset_correction(float sum_even, float sum_odd) {
  return 1032.f * sum_even + 1152.f * sum_odd;
}

// Byte offset of k (0..127) inside a staged chunk: unit k / 8, then the
// position of i = k % 8 in the order above (i with its three bits reversed).
__device__ __forceinline__ int staged_offset(int k) {
  const int i = k & 7;
  return (k >> 3) * 16 + (((i & 1) << 2) | (i & 2) | (i >> 2)) * 2;
}


// ---------------------------------------------------------------------------
// Router + staging + plan
// ---------------------------------------------------------------------------
struct RouteArgs {
  const void* x;
  int64_t ldx;
  int T, H, E, K;
  int mode;
  int kind;
  const void* rw;
  int rw_dtype;
  int logits_act;
  const float* bonus;
  float thr;
  const float* bias;
  int norm;
  float scaling;
  int n_group, topk_group;  // group-limited selection (sigmoid) when n_group > 1 && topk_group > 0
  const int32_t* given_idx;
  const float* given_w;
  int32_t* out_idx;
  float* out_w;
  float* out_logits;
  int seg;
  int gv_stage;  // 1: stage for the mma.sync engine (odd k divided by 16, per-group corrections)
  const float* pre_logits;  // [T][E] router logits from router_logits_kernel, or NULL: computed here
  int wbuf_off;    // byte offset of the router-weight chunk in dynamic shared memory
  int plan_here;   // 1: the last CTA builds the plan; 0: plan_kernel runs after this kernel
  Plan plan;
};

__device__ __forceinline__ float load_any(const void* p, int dtype, int64_t i) {
  if (dtype == HN_DTYPE_F32) return reinterpret_cast<const float*>(p)[i];
  if (dtype == HN_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

// Router weights are brought into shared memory in chunks of whole expert rows
// (at most kRouteChunkBytes) by one bulk async copy each, so a chunk costs one
// memory round trip.  The kernel body is kept free of large unrolled blocks:
// at small T one CTA runs it once, and every instruction it executes is
// fetched into the instruction cache once.
constexpr int kRouteChunkBytes = 64 * 1024;

__host__ __device__ inline int route_esize(int dtype) { return dtype == HN_DTYPE_F32 ? 4 : 2; }
__host__ __device__ inline int route_chunk_experts(int H, int E, int dtype) {
  const int per = kRouteChunkBytes / (H * route_esize(dtype));
  return per < 1 ? 1 : (per < E ? per : E);
}

template <typename Tr>
__global__ void __launch_bounds__(256) route_prep_kernel(const RouteArgs a) {
  extern __shared__ __align__(16) float rsm[];
  float* xs = rsm;                 // [H]
  float* lg = xs + a.H;            // [E]
  float* scs = lg + a.E;           // [E] selection scores
  // plan copies of the routing follow scs (see the plan section); the router
  // weight chunk sits at the end of the dynamic shared memory
  __shared__ int s_last;
  __shared__ int s_wsum[3][8];  // per-warp totals of the plan's scans
  __shared__ int s_idx[kMaxTopK];
  __shared__ float s_w[kMaxTopK];
  __shared__ __align__(8) uint64_t s_wbar;
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const typename Tr::T* xrow = reinterpret_cast<const typename Tr::T*>(a.x) + (int64_t)t * a.ldx;
  const int esz = route_esize(a.rw_dtype);
  const int CE = route_chunk_experts(a.H, a.E, a.rw_dtype);
  const bool bulk = a.mode == ROUTE_COMPUTE && !a.pre_logits && (reinterpret_cast<uintptr_t>(a.rw) & 15) == 0;
  uint8_t* wbuf = reinterpret_cast<uint8_t*>(rsm) + a.wbuf_off;
  if (bulk && tid == 0) {
    mbar_init(smem_u32(&s_wbar), 1);
    fence_barrier_init();
    const uint32_t bytes = (uint32_t)(min(CE, a.E) * a.H * esz);
    mbar_arrive_expect_tx(smem_u32(&s_wbar), bytes);
    bulk_g2s(smem_u32(wbuf), a.rw, bytes, smem_u32(&s_wbar));
  }
  // The engine's arrival counters start every call at zero, whatever an
  // earlier call of another shape left in this part of the workspace.
  for (int i = t * 256 + tid; i < a.plan.n_ctr; i += gridDim.x * 256) a.plan.ctr1[i] = 0;
  if ((reinterpret_cast<uintptr_t>(xrow) & 15) == 0) {
    const uint4* xv = reinterpret_cast<const uint4*>(xrow);
    for (int i = tid; i < a.H / 8; i += 256) {
      const uint4 v = __ldg(xv + i);
      const typename Tr::T2* h2 = reinterpret_cast<const typename Tr::T2*>(&v);
      for (int u = 0; u < 4; ++u) {
        xs[8 * i + 2 * u] = Tr::to_f(h2[u].x);
        xs[8 * i + 2 * u + 1] = Tr::to_f(h2[u].y);
      }
    }
  } else {
    for (int i = tid; i < a.H; i += 256) xs[i] = Tr::to_f(xrow[i]);
  }
  __syncthreads();

  // 1. staged activations.  For the mma.sync engine (gv_stage) the odd k are
  // stored divided by 16 and each k-group gets its offset correction
  // (gv_offset_correction): the engine multiplies by 1024 + n and 1024 + 16n.
  // Lanes 16h..16h+15 of a warp hold the 16 units of one k-group.
  for (int u0 = 0; u0 < a.H / 8; u0 += 256) {
    const int u = u0 + tid;
    const bool ok = u < a.H / 8;
    const int g = u >> 4, ch = u & 15;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = ok ? xs[g * 128 + ch * 8 + i] : 0.f;
    if (a.gv_stage) {
      float ce = 0.f, co = 0.f;
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        v[i + 1] *= 0.0625f;
        ce += __half2float(__float2half_rn(v[i]));
        co += __half2float(__float2half_rn(v[i + 1]));
      }
      float c = gv_offset_correction(ce, co);
      for (int o = 8; o; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
      if (ok && ch == 0) a.plan.corr_x[(int64_t)t * (a.H / 128) + g] = c;
    }
    if (ok) *reinterpret_cast<uint4*>(a.plan.xp + ((int64_t)t * (a.H / 128) + g) * kChunk + ch * 16) = pack_unit(v);
  }

  // 2. routing for this token
  if (a.mode == ROUTE_COMPUTE) {
    if (a.pre_logits) {
      // logits of a large batch come from router_logits_kernel
      for (int e = tid; e < a.E; e += 256) {
        const float v = __ldg(a.pre_logits + (int64_t)t * a.E + e);
        lg[e] = a.logits_act ? Tr::to_f(Tr::from_f(v)) : v;
      }
      __syncthreads();
    }
    // router logits, one warp per expert row of the chunk in shared memory
    for (int c0 = 0; c0 < (a.pre_logits ? 0 : a.E); c0 += CE) {
      const int ce = min(CE, a.E - c0);
      if (bulk) mbar_wait(smem_u32(&s_wbar), (uint32_t)((c0 / CE) & 1), a.plan.err);
      for (int r = warp; r < ce; r += 8) {
        const int e = c0 + r;
        float acc = 0.f;
        if (bulk) {
          const uint8_t* row = wbuf + (size_t)r * a.H * esz;
          if (esz == 4) {
            for (int i = lane; i < a.H / 4; i += 32) {
              const float4 w = reinterpret_cast<const float4*>(row)[i];
              acc = fmaf(xs[4 * i], w.x, acc);
              acc = fmaf(xs[4 * i + 1], w.y, acc);
              acc = fmaf(xs[4 * i + 2], w.z, acc);
              acc = fmaf(xs[4 * i + 3], w.w, acc);
            }
          } else {
            const bool bf = a.rw_dtype == HN_DTYPE_BF16;
            for (int i = lane; i < a.H / 8; i += 32) {
              const uint4 w = reinterpret_cast<const uint4*>(row)[i];
              const uint32_t q[4] = {w.x, w.y, w.z, w.w};
              for (int c = 0; c < 4; ++c) {
                float lo, hi;
                if (bf) {
                  lo = __uint_as_float(q[c] << 16);
                  hi = __uint_as_float(q[c] & 0xFFFF0000u);
                } else {
                  const __half2 hh = *reinterpret_cast<const __half2*>(&q[c]);
                  lo = __low2float(hh);
                  hi = __high2float(hh);
                }
                acc = fmaf(xs[8 * i + 2 * c], lo, acc);
                acc = fmaf(xs[8 * i + 2 * c + 1], hi, acc);
              }
            }
          }
        } else {
          for (int i = lane; i < a.H; i += 32) acc += xs[i] * load_any(a.rw, a.rw_dtype, (int64_t)e * a.H + i);
        }
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) lg[e] = a.logits_act ? Tr::to_f(Tr::from_f(acc)) : acc;
      }
      __syncthreads();
      if (bulk && c0 + CE < a.E && tid == 0) {
        // every warp has finished with the chunk (its values were consumed
        // before the barrier above), so the buffer can be refilled
        const uint32_t bytes = (uint32_t)(min(CE, a.E - c0 - CE) * a.H * esz);
        mbar_arrive_expect_tx(smem_u32(&s_wbar), bytes);
        bulk_g2s(smem_u32(wbuf), reinterpret_cast<const uint8_t*>(a.rw) + (size_t)(c0 + CE) * a.H * esz, bytes,
                 smem_u32(&s_wbar));
      }
    }
    if (warp == 0) {
      // optional cache-affinity bonus (model/router.py:132-175)
      if (a.kind == HN_ROUTER_SOFTMAX_TOPK && a.bonus) {
        float mx = -INFINITY;
        for (int e = lane; e < a.E; e += 32) mx = fmaxf(mx, lg[e]);
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float se = 0.f;
        for (int e = lane; e < a.E; e += 32) se += expf(lg[e] - mx);
        for (int o = 16; o; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
        float ent = 0.f;
        for (int e = lane; e < a.E; e += 32) {
          const float p = expf(lg[e] - mx) / se;
          ent -= p * logf(p + 1e-10f);
        }
        for (int o = 16; o; o >>= 1) ent += __shfl_xor_sync(0xffffffffu, ent, o);
        const bool on = ent / logf((float)a.E) > a.thr;
        __syncwarp();
        if (on)
          for (int e = lane; e < a.E; e += 32) lg[e] += a.bonus[e];
        __syncwarp();
      }
      if (a.out_logits)
        for (int e = lane; e < a.E; e += 32) a.out_logits[(int64_t)t * a.E + e] = lg[e];
      // selection scores in shared memory; ties resolve to the lower index
      for (int e = lane; e < a.E; e += 32) {
        float v = lg[e];
        if (a.kind == HN_ROUTER_SIGMOID_TOPK) {
          v = 1.0f / (1.0f + expf(-v));
          if (a.bias) v += a.bias[e];
        }
        if (v != v) v = -INFINITY;  // a NaN score never wins a slot
        scs[e] = v;
      }
      __syncwarp();
      // group-limited routing (model/glm4.py:285-297): lane g scores group g
      // by its best selection score; the topk_group best groups stay, the
      // other experts' scores become 0
      unsigned keep = 0xffffffffu;
      const bool grouped = a.kind == HN_ROUTER_SIGMOID_TOPK && a.n_group > 1 && a.topk_group > 0;
      const int gsz = grouped ? a.E / a.n_group : a.E;
      if (grouped) {
        float gm = -INFINITY;
        if (lane < a.n_group)
          for (int i = 0; i < gsz; ++i) gm = fmaxf(gm, scs[lane * gsz + i]);
        keep = 0u;
        for (int j = 0; j < a.topk_group; ++j) {
          float bv = lane < a.n_group && !((keep >> lane) & 1u) ? gm : -INFINITY;
          int bi = lane < a.n_group && !((keep >> lane) & 1u) ? lane : 0x7fffffff;
          for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
              bv = ov;
              bi = oi;
            }
          }
          if (bi < a.n_group) keep |= 1u << bi;
        }
        for (int e = lane; e < a.E; e += 32)
          if (!((keep >> (e / gsz)) & 1u)) scs[e] = 0.f;
        __syncwarp();
      }
#pragma unroll 1
      for (int k = 0; k < a.K; ++k) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int e = lane; e < a.E; e += 32) {
          const float v = scs[e];
          if (v > bv || (v == bv && e < bi)) {
            bv = v;
            bi = e;
          }
        }
        for (int o = 16; o; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
          }
        }
        if (bi >= a.E) bi = 0;  // unreachable for finite scores; keeps the index in range
        if (lane == 0) {
          s_idx[k] = bi;
          scs[bi] = -INFINITY;
        }
        __syncwarp();
      }
      if (lane == 0) {
        // weights are built in shared memory (s_w)
        if (a.kind == HN_ROUTER_SOFTMAX_TOPK) {
          // softmax over the selected logits (model/router.py:114), renormalised (:117)
          float mx = -INFINITY;
          for (int k = 0; k < a.K; ++k) mx = fmaxf(mx, lg[s_idx[k]]);
          float sum = 0.f;
          for (int k = 0; k < a.K; ++k) {
            s_w[k] = expf(lg[s_idx[k]] - mx);
            sum += s_w[k];
          }
          float s2 = 0.f;
          for (int k = 0; k < a.K; ++k) {
            s_w[k] = s_w[k] / sum;
            s2 += s_w[k];
          }
          for (int k = 0; k < a.K; ++k) s_w[k] = s_w[k] / s2;
        } else {
          // sigmoid scores of the selected experts, unbiased (model/glm4.py:300-307);
          // an expert of a dropped group (only when top_k exceeds the kept
          // experts) carries its masked score, 0
          float sum = 0.f;
          for (int k = 0; k < a.K; ++k) {
            const bool kept = (keep >> (s_idx[k] / gsz)) & 1u;
            s_w[k] = kept ? 1.0f / (1.0f + expf(-lg[s_idx[k]])) : 0.f;
            sum += s_w[k];
          }
          for (int k = 0; k < a.K; ++k) {
            if (a.norm) s_w[k] = s_w[k] / (sum + 1e-9f);
            s_w[k] = s_w[k] * a.scaling;
          }
        }
        for (int k = 0; k < a.K; ++k) s_w[k] = Tr::to_f(Tr::from_f(s_w[k]));  // cast to the activation dtype
      }
      __syncwarp();
    }
    __syncthreads();
  } else if (tid == 0) {
    for (int k = 0; k < a.K; ++k) {
      if (a.mode == ROUTE_GIVEN) {
        // -1 marks an unused slot: it takes no expert work and adds nothing
        // to the combine; a token with only unused slots is left out entirely
        int e = a.given_idx[(int64_t)t * a.K + k];
        float w = a.given_w[(int64_t)t * a.K + k];
        if (e == -1) {
          w = 0.f;
        } else if (e < 0 || e >= a.E) {
          record_error(a.plan.err, DEV_ERR_BAD_INDEX);
          e = 0;
        }
        s_idx[k] = e;
        s_w[k] = w;
      } else {
        s_idx[k] = 0;
        s_w[k] = 1.0f;
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    int nv = 0;
    for (int k = 0; k < a.K; ++k) nv += s_idx[k] >= 0;
    a.plan.nval[t] = nv;
  }
  if (tid < a.K) {
    a.plan.idx[(int64_t)t * a.K + tid] = s_idx[tid];
    a.plan.wts[(int64_t)t * a.K + tid] = s_w[tid];
    if (a.out_idx) a.out_idx[(int64_t)t * a.K + tid] = s_idx[tid];
    if (a.out_w) a.out_w[(int64_t)t * a.K + tid] = s_w[tid];
  }

  // 3. the last CTA to finish builds the plan (small routings; larger ones
  // are planned by plan_kernel, launched after this kernel)
  if (!a.plan_here) return;
  // A single token's CTA holds the whole routing already: no election, and
  // the plan reads it from shared memory instead of back from global memory.
  const bool solo = gridDim.x == 1;
  if (solo) {
    __syncthreads();
  } else {
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(a.plan.route_ctr, 1) == a.T - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
  }
  int* cnt = reinterpret_cast<int*>(rsm);  // reuse (>= E ints available: H >= 128 floats)
  int* off = cnt + a.E;
  const int TK = a.T * a.K;
  // every token's routing, read once into shared memory when it fits
  const bool in_smem = TK <= kPlanSmemEntries;
  int* pidx = reinterpret_cast<int*>(rsm + a.H + 2 * a.E);
  float* pwts = reinterpret_cast<float*>(pidx + (in_smem ? TK : 0));
  for (int e = tid; e < a.E; e += 256) cnt[e] = 0;
  if (in_smem)
    for (int i = tid; i < TK; i += 256) {
      pidx[i] = solo ? s_idx[i] : __ldcg(a.plan.idx + i);
      pwts[i] = solo ? s_w[i] : __ldcg(a.plan.wts + i);
    }
  __syncthreads();
  for (int i = tid; i < TK; i += 256) {
    const int e = in_smem ? pidx[i] : __ldcg(a.plan.idx + i);
    if (e >= 0) atomicAdd(&cnt[e], 1);  // -1: a skipped token's slot
  }
  __syncthreads();
  // Offsets and segments of every expert by a block-wide exclusive scan over
  // the experts (thread i owns experts [i*c, (i+1)*c)): each thread cuts its
  // own experts' segments, in expert order, at the positions the scan gives.
  {
    const int c = (a.E + 255) / 256, e0 = tid * c, e1 = min(a.E, e0 + c);
    int n = 0, ns = 0, ns2 = 0;
    for (int e = e0; e < e1; ++e) {
      const int m = cnt[e];
      n += m;
      ns += (m + a.seg - 1) / a.seg;
      if (a.plan.seg2) ns2 += (m + a.plan.seg2 - 1) / a.plan.seg2;
    }
    int incl[3] = {n, ns, ns2};
#pragma unroll
    for (int v = 0; v < 3; ++v)
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl[v], o);
        if (lane >= o) incl[v] += y;
      }
    if (lane == 31)
      for (int v = 0; v < 3; ++v) s_wsum[v][warp] = incl[v];
    __syncthreads();
    int base[3];
    for (int v = 0; v < 3; ++v) {
      base[v] = 0;
      for (int w = 0; w < warp; ++w) base[v] += s_wsum[v][w];
    }
    int o = base[0] + incl[0] - n, sg = base[1] + incl[1] - ns, sg2 = base[2] + incl[2] - ns2;
    for (int e = e0; e < e1; ++e) {
      const int m = cnt[e];
      off[e] = o;
      for (int j = 0; j < m; j += a.seg) a.plan.segs[sg++] = make_int4(e, o + j, min(a.seg, m - j), 0);
      if (a.plan.seg2)
        for (int j = 0; j < m; j += a.plan.seg2)
          a.plan.segs2[sg2++] = make_int4(e, o + j, min(a.plan.seg2, m - j), 0);
      o += m;
      a.plan.counts[e] = m;
    }
    if (tid == 255) {
      *a.plan.n_segs = sg;
      if (a.plan.seg2) *a.plan.n_segs2 = sg2;
      *a.plan.route_ctr = 0;
      *a.plan.n_assign = o;
      s_idx[0] = o;  // assignments planned (skipped tokens' slots excluded)
    }
  }
  __syncthreads();
  // positions past the planned assignments (left by skipped tokens) name
  // token 0, so a copy over all T*K positions stays in bounds
  for (int p = s_idx[0] + tid; p < TK; p += 256) a.plan.a_tok[p] = 0;
  // per-expert assignment order: by token, then by top-k slot -- the rank of
  // assignment i among its expert's is the count of earlier ones with the
  // same expert (a token listing an expert twice gets two slots); routings
  // planned here hold at most kPlanRankEntries entries, all in shared memory
  for (int i = tid; i < TK; i += 256) {
    const int e = pidx[i];
    if (e < 0) continue;
    int r = 0;
    for (int j = 0; j < i; ++j) r += pidx[j] == e;
    const int p = off[e] + r;
    a.plan.pos[i] = p;
    a.plan.a_tok[p] = i / a.K;
    a.plan.a_tk[p] = i;
    a.plan.a_w[p] = pwts[i];
  }
}

// ---------------------------------------------------------------------------
// Router logits of a large batch, logits[t, e] = sum_h x[t, h] * W[e, h] in
// fp32 (the reference's `F.linear(h.float(), W.float())`, model/glm4.py:279;
// the Mixtral gate's model-dtype rounding is applied by the prep kernel).
// One CTA computes a 64-token x 64-expert tile, each thread 4 x 4 outputs,
// over 32-wide chunks of h staged in shared memory; every output sums h in
// order, so the result does not depend on the launch shape.  The per-token
// path in route_prep_kernel reads the whole router matrix once per token,
// which is what a batch of thousands of tokens cannot afford.
// ---------------------------------------------------------------------------
constexpr int kRgM = 64, kRgN = 64, kRgK = 32;
constexpr int kRouterGemmMinT = 256;  // batches from this size route through router_logits_kernel

// Tile loads: x as one 16-byte vector (8 activations) per thread, W as one
// 16-byte vector (4 fp32 or 8 half) per thread per 32-wide row chunk; the
// next chunk is loaded into registers while the current one is multiplied.
template <typename Tr>
__global__ void __launch_bounds__(256) router_logits_kernel(const void* x, int64_t ldx, int T, int H, int E,
                                                            const void* rw, int rw_dtype, float* out) {
  __shared__ __align__(16) float xs[kRgK][kRgM + 4];  // [k][token]
  __shared__ __align__(16) float ws[kRgK][kRgN + 4];  // [k][expert]
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int t0 = blockIdx.x * kRgM, e0 = blockIdx.y * kRgN;
  const typename Tr::T* xp = reinterpret_cast<const typename Tr::T*>(x);
  const bool w32 = rw_dtype == HN_DTYPE_F32;
  // this thread's loads: x row xt, k offset xk (8 values); W row(s) and k offsets
  const int xt = tid >> 2, xk = (tid & 3) * 8;
  const bool xok = t0 + xt < T;
  auto load_x = [&](int k0) -> uint4 {
    return xok ? __ldg(reinterpret_cast<const uint4*>(xp + (int64_t)(t0 + xt) * ldx + k0 + xk))
               : make_uint4(0u, 0u, 0u, 0u);
  };
  // fp32 W: 2 vectors of 4 (rows tid>>3 and 32 + (tid>>3), k (tid&7)*4); 16-bit W: 1 vector of 8
  auto load_w = [&](int k0, int q) -> uint4 {
    int e, k;
    if (w32) {
      e = e0 + q * 32 + (tid >> 3);
      k = (tid & 7) * 4;
      return e < E ? __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(rw) + (int64_t)e * H + k0 + k))
                   : make_uint4(0u, 0u, 0u, 0u);
    }
    e = e0 + (tid >> 2);
    k = (tid & 3) * 8;
    return (q == 0 && e < E)
               ? __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(rw) + (int64_t)e * H + k0 + k))
               : make_uint4(0u, 0u, 0u, 0u);
  };
  auto put = [&](uint4 xv, uint4 w0, uint4 w1) {
    const typename Tr::T2* x2 = reinterpret_cast<const typename Tr::T2*>(&xv);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xs[xk + 2 * i][xt] = Tr::to_f(x2[i].x);
      xs[xk + 2 * i + 1][xt] = Tr::to_f(x2[i].y);
    }
    if (w32) {
      const float* f0 = reinterpret_cast<const float*>(&w0);
      const float* f1 = reinterpret_cast<const float*>(&w1);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ws[(tid & 7) * 4 + i][tid >> 3] = f0[i];
        ws[(tid & 7) * 4 + i][32 + (tid >> 3)] = f1[i];
      }
    } else {
      const uint32_t* h = reinterpret_cast<const uint32_t*>(&w0);
      const bool bf = rw_dtype == HN_DTYPE_BF16;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float lo, hi;
        if (bf) {
          lo = __uint_as_float(h[i] << 16);
          hi = __uint_as_float(h[i] & 0xFFFF0000u);
        } else {
          const __half2 hh = *reinterpret_cast<const __half2*>(&h[i]);
          lo = __low2float(hh);
          hi = __high2float(hh);
        }
        ws[(tid & 3) * 8 + 2 * i][tid >> 2] = lo;
        ws[(tid & 3) * 8 + 2 * i + 1][tid >> 2] = hi;
      }
    }
  };
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  uint4 xv = load_x(0), w0 = load_w(0, 0), w1 = load_w(0, 1);
  for (int k0 = 0; k0 < H; k0 += kRgK) {
    put(xv, w0, w1);
    __syncthreads();
    if (k0 + kRgK < H) {
      xv = load_x(k0 + kRgK);
      w0 = load_w(k0 + kRgK, 0);
      w1 = load_w(k0 + kRgK, 1);
    }
#pragma unroll 8
    for (int kk = 0; kk < kRgK; ++kk) {
      const float4 av = *reinterpret_cast<const float4*>(&xs[kk][ty * 4]);
      const float4 bv = *reinterpret_cast<const float4*>(&ws[kk][tx * 4]);
      const float a4[4] = {av.x, av.y, av.z, av.w}, b4[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a4[i], b4[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + ty * 4 + i;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = e0 + tx * 4 + j;
      if (t < T && e < E) out[(int64_t)t * E + e] = acc[i][j];
    }
  }
}

// ---------------------------------------------------------------------------
// Router logits of a large bf16 batch on the tensor cores (mma.sync
// m16n8k16, bf16 operands, fp32 accumulation).  The tokens are exact in
// bf16; the router weight is split into nsplit bf16 parts whose sum is the
// weight exactly (three for fp32, whose 24-bit significand bf16 takes 8 bits
// at a time; two for fp16; one for bf16), and the parts' products accumulate
// into one fp32 sum, so the logits keep fp32-level accuracy (the reference
// computes them as `F.linear(h.float(), W.float())`, model/glm4.py:279).
// Each 64-wide chunk of h accumulates on the tensor core in a fresh fragment
// that is then added to the running sum in fp32 (round to nearest): the
// tensor core's own accumulation over all of h drifts several times further
// from the exact sum than an fp32 matrix product does.
// CTA tile 64 tokens x 128 experts over 64-wide chunks of h, double-buffered
// in shared memory; warp tile 32 tokens x 32 experts (2 x 4 MMA tiles).
// Every output sums its chunks in h order, whatever the launch shape.
// ---------------------------------------------------------------------------
constexpr int kRtM = 64, kRtN = 128, kRtK = 64, kRtLd = kRtK + 8;  // row pitch 144 B (16-byte aligned rows)
constexpr size_t kRtSmem = (size_t)2 * (kRtM + 3 * kRtN) * kRtLd * 2;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// v = hi + mid + lo exactly (bf16 parts; each residual is exact in fp32)
__device__ __forceinline__ void split3_bf16(float v, uint16_t& hi, uint16_t& mid, uint16_t& lo) {
  const __nv_bfloat16 h = __float2bfloat16_rn(v);
  const float r1 = v - __bfloat162float(h);
  const __nv_bfloat16 m = __float2bfloat16_rn(r1);
  const __nv_bfloat16 l = __float2bfloat16_rn(r1 - __bfloat162float(m));
  hi = __bfloat16_as_ushort(h);
  mid = __bfloat16_as_ushort(m);
  lo = __bfloat16_as_ushort(l);
}

__global__ void __launch_bounds__(256) router_logits_tc_kernel(const __nv_bfloat16* x, int64_t ldx, int T, int H,
                                                               int E, const void* rw, int rw_dtype, float* out) {
  extern __shared__ __align__(16) uint16_t rts[];  // [2][kRtM][kRtLd] tokens, then [2][3][kRtN][kRtLd] weight parts
  uint16_t* const xs = rts;
  uint16_t* const ws = rts + 2 * kRtM * kRtLd;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t0 = blockIdx.x * kRtM, e0 = blockIdx.y * kRtN;
  const int nsplit = rw_dtype == HN_DTYPE_F32 ? 3 : (rw_dtype == HN_DTYPE_F16 ? 2 : 1);
  // global -> registers: 2 token vectors (8 bf16) and 8 weight vectors (4 fp32 or, 16-bit, 4 of 8) per thread
  uint4 xr[2], wr[8];
  auto load = [&](int k0) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int v = tid + 256 * i, t = t0 + (v >> 3), k = k0 + (v & 7) * 8;
      xr[i] = t < T ? __ldg(reinterpret_cast<const uint4*>(x + (int64_t)t * ldx + k)) : make_uint4(0u, 0u, 0u, 0u);
    }
    if (rw_dtype == HN_DTYPE_F32) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int v = tid + 256 * i, e = e0 + (v >> 4), k = k0 + (v & 15) * 4;
        wr[i] = e < E ? __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(rw) + (int64_t)e * H + k))
                      : make_uint4(0u, 0u, 0u, 0u);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int v = tid + 256 * i, e = e0 + (v >> 3), k = k0 + (v & 7) * 8;
        wr[i] = e < E ? __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(rw) + (int64_t)e * H + k))
                      : make_uint4(0u, 0u, 0u, 0u);
      }
    }
  };
  // registers -> shared buffer b (weight parts split here)
  auto store = [&](int b) {
    uint16_t* xb = xs + b * kRtM * kRtLd;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int v = tid + 256 * i;
      *reinterpret_cast<uint4*>(xb + (v >> 3) * kRtLd + (v & 7) * 8) = xr[i];
    }
    uint16_t* wb = ws + b * 3 * kRtN * kRtLd;
    if (rw_dtype == HN_DTYPE_F32) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int v = tid + 256 * i, row = v >> 4, col = (v & 15) * 4;
        const float f[4] = {__uint_as_float(wr[i].x), __uint_as_float(wr[i].y), __uint_as_float(wr[i].z),
                            __uint_as_float(wr[i].w)};
        uint16_t p[3][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) split3_bf16(f[j], p[0][j], p[1][j], p[2][j]);
#pragma unroll
        for (int q = 0; q < 3; ++q)
          *reinterpret_cast<uint2*>(wb + (q * kRtN + row) * kRtLd + col) =
              make_uint2((uint32_t)p[q][0] | ((uint32_t)p[q][1] << 16), (uint32_t)p[q][2] | ((uint32_t)p[q][3] << 16));
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int v = tid + 256 * i, row = v >> 3, col = (v & 7) * 8;
        if (rw_dtype == HN_DTYPE_BF16) {
          *reinterpret_cast<uint4*>(wb + row * kRtLd + col) = wr[i];
        } else {
          const uint16_t* h = reinterpret_cast<const uint16_t*>(&wr[i]);
          uint16_t p[3][8];
#pragma unroll
          for (int j = 0; j < 8; ++j) split3_bf16(__half2float(__ushort_as_half(h[j])), p[0][j], p[1][j], p[2][j]);
#pragma unroll
          for (int q = 0; q < 2; ++q)
            *reinterpret_cast<uint4*>(wb + (q * kRtN + row) * kRtLd + col) =
                make_uint4((uint32_t)p[q][0] | ((uint32_t)p[q][1] << 16), (uint32_t)p[q][2] | ((uint32_t)p[q][3] << 16),
                           (uint32_t)p[q][4] | ((uint32_t)p[q][5] << 16), (uint32_t)p[q][6] | ((uint32_t)p[q][7] << 16));
        }
      }
    }
  };
  float acc[2][4][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[i][j][r] = 0.f;
  const int wm = warp & 1, wn = warp >> 1;  // warp tile: tokens 32*wm.., experts 32*wn..
  // ldmatrix row addresses of this lane: A (tokens) rows (l & 15), k half (l >> 4);
  // B (weights) rows (l & 7) + 8 * (l >> 4), k half ((l >> 3) & 1)
  const int a_row = lane & 15, a_k = (lane >> 4) * 8;
  const int b_row = (lane & 7) + 8 * (lane >> 4), b_k = ((lane >> 3) & 1) * 8;
  const int nk = H / kRtK;
  load(0);
  store(0);
  __syncthreads();
  for (int c = 0; c < nk; ++c) {
    const int b = c & 1;
    if (c + 1 < nk) load((c + 1) * kRtK);
    const uint32_t xb = smem_u32(xs + b * kRtM * kRtLd);
    const uint32_t wb = smem_u32(ws + b * 3 * kRtN * kRtLd);
    float tg[2][4][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r) tg[i][j][r] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kRtK; kk += 16) {
      uint32_t af[2][4];
#pragma unroll
      for (int mi = 0; mi < 2; ++mi)
        ldsm_x4(xb + ((wm * 32 + mi * 16 + a_row) * kRtLd + kk + a_k) * 2, af[mi][0], af[mi][1], af[mi][2], af[mi][3]);
      for (int q = 0; q < nsplit; ++q) {
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t b0, b1, b2, b3;  // n tiles 2np (b0, b1) and 2np+1 (b2, b3)
          ldsm_x4(wb + ((q * kRtN + wn * 32 + np * 16 + b_row) * kRtLd + kk + b_k) * 2, b0, b1, b2, b3);
#pragma unroll
          for (int mi = 0; mi < 2; ++mi) {
            mma_bf16(tg[mi][2 * np], af[mi], b0, b1);
            mma_bf16(tg[mi][2 * np + 1], af[mi], b2, b3);
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[i][j][r] += tg[i][j][r];
    if (c + 1 < nk) store(b ^ 1);
    __syncthreads();
  }
  const int g = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int mi = 0; mi < 2; ++mi)
#pragma unroll
    for (int ni = 0; ni < 4; ++ni)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int t = t0 + wm * 32 + mi * 16 + g + 8 * (r >> 1);
        const int e = e0 + wn * 32 + ni * 8 + 2 * tq + (r & 1);
        if (t < T && e < E) out[(int64_t)t * E + e] = acc[mi][ni][r];
      }
}

// ---------------------------------------------------------------------------
// Router logits of a small batch whose router matrix spans several of the
// prep kernel's 64 KB chunks (GLM-4.5: 128 experts x 4096 fp32 = 2 MB): the
// per-token prep CTA would stream the whole matrix chunk by chunk, one round
// trip each.  Here CTA (b, c) stages kRgvE expert rows in shared memory (as
// fp32) and each of its warps dots them with one of tokens 8c..8c+7; a lane
// sums h = 8*lane + 256*i in order and the warp reduces by xor-shuffle, so
// the result does not depend on the launch shape.  logits[t, e] is fp32 (the
// prep kernel applies the Mixtral gate's model-dtype rounding).
// ---------------------------------------------------------------------------
constexpr int kRgvE = 2;
// Taken when the router has more than 32 Ki weights (64 KB at 16 bits):
// decided on the weight count, not on the dtype, so a host-only query can
// tell without knowing the router's dtype.
__host__ __device__ inline bool router_gemv_wanted(int64_t H, int64_t E) {
  return E * H * 2 > (int64_t)kRouteChunkBytes;
}
template <typename Tr>
__global__ void __launch_bounds__(256) router_gemv_kernel(const void* x, int64_t ldx, int T, int H, int E,
                                                          const void* rw, int rw_dtype, float* out) {
  extern __shared__ __align__(16) float wsm[];  // [kRgvE][H]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int e0 = blockIdx.x * kRgvE, ne = min(kRgvE, E - e0);
  // the rows in 16-byte vectors, four loads in flight per thread before any store
  const int n = ne * H;
  if (rw_dtype == HN_DTYPE_F32 && (reinterpret_cast<uintptr_t>(rw) & 15) == 0) {
    const float4* src = reinterpret_cast<const float4*>(rw) + (int64_t)e0 * H / 4;
    for (int i0 = tid; i0 < n / 4; i0 += 4 * 256) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i0 + u * 256 < n / 4) v[u] = __ldg(src + i0 + u * 256);
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i0 + u * 256 < n / 4) reinterpret_cast<float4*>(wsm)[i0 + u * 256] = v[u];
    }
  } else if (rw_dtype != HN_DTYPE_F32 && (reinterpret_cast<uintptr_t>(rw) & 15) == 0) {
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(rw) + (int64_t)e0 * H);
    const bool bf = rw_dtype == HN_DTYPE_BF16;
    for (int i0 = tid; i0 < n / 8; i0 += 4 * 256) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i0 + u * 256 < n / 8) v[u] = __ldg(src + i0 + u * 256);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (i0 + u * 256 >= n / 8) continue;
        const uint32_t q[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        float* d = wsm + (i0 + u * 256) * 8;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (bf) {
            d[2 * c] = __uint_as_float(q[c] << 16);
            d[2 * c + 1] = __uint_as_float(q[c] & 0xFFFF0000u);
          } else {
            const __half2 hh = *reinterpret_cast<const __half2*>(&q[c]);
            d[2 * c] = __low2float(hh);
            d[2 * c + 1] = __high2float(hh);
          }
        }
      }
    }
  } else {
    for (int i = tid; i < n; i += 256) wsm[i] = load_any(rw, rw_dtype, (int64_t)e0 * H + i);
  }
  __syncthreads();
  const typename Tr::T* xp = reinterpret_cast<const typename Tr::T*>(x);
  const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && (ldx % 8 == 0);
  // CTA row blockIdx.y takes 8 tokens, one per warp; a lane's 16-byte loads
  // of its token are issued kRgvBatch at a time before any is used
  const int t = blockIdx.y * 8 + warp;
  if (t >= T) return;
  float acc[kRgvE];
#pragma unroll
  for (int e = 0; e < kRgvE; ++e) acc[e] = 0.f;
  const typename Tr::T* xr = xp + (int64_t)t * ldx;
  constexpr int kRgvBatch = 8;
  for (int h0 = lane * 8; h0 < H; h0 += 256 * kRgvBatch) {
    float xv[kRgvBatch][8];
#pragma unroll
    for (int b = 0; b < kRgvBatch; ++b) {
      const int h = h0 + b * 256;
      if (h >= H) continue;
      if (vec) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(xr + h));
        const typename Tr::T2* h2 = reinterpret_cast<const typename Tr::T2*>(&v);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          xv[b][2 * u] = Tr::to_f(h2[u].x);
          xv[b][2 * u + 1] = Tr::to_f(h2[u].y);
        }
      } else {
#pragma unroll
        for (int u = 0; u < 8; ++u) xv[b][u] = Tr::to_f(xr[h + u]);
      }
    }
#pragma unroll
    for (int b = 0; b < kRgvBatch; ++b) {
      const int h = h0 + b * 256;
      if (h >= H) continue;
#pragma unroll
      for (int e = 0; e < kRgvE; ++e) {
        const float4 w0 = *reinterpret_cast<const float4*>(wsm + e * H + h);
        const float4 w1 = *reinterpret_cast<const float4*>(wsm + e * H + h + 4);
        acc[e] = fmaf(xv[b][0], w0.x, acc[e]);
        acc[e] = fmaf(xv[b][1], w0.y, acc[e]);
        acc[e] = fmaf(xv[b][2], w0.z, acc[e]);
        acc[e] = fmaf(xv[b][3], w0.w, acc[e]);
        acc[e] = fmaf(xv[b][4], w1.x, acc[e]);
        acc[e] = fmaf(xv[b][5], w1.y, acc[e]);
        acc[e] = fmaf(xv[b][6], w1.z, acc[e]);
        acc[e] = fmaf(xv[b][7], w1.w, acc[e]);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < kRgvE; ++e)
    for (int o = 16; o; o >>= 1) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
  if (lane < ne) out[(int64_t)t * E + e0 + lane] = lane == 0 ? acc[0] : acc[kRgvE > 1 ? 1 : 0];
}

// ---------------------------------------------------------------------------
// Dispatch plan for large routings (T*K above kPlanSmemEntries): one CTA per
// expert e.  Each CTA histograms every expert's assignments (so no counters
// cross CTAs), takes its offset and segment base from the prefix over the
// experts before it, writes its segments, then lists its assignments in
// (token, slot) order -- the order the single-CTA builder above produces --
// with a block scan over contiguous per-thread chunks of the routing.
// ---------------------------------------------------------------------------
struct PlanArgs {
  int T, K, E, seg;
  Plan plan;
};

// Gate/up operand of a large routing in assignment order: row p of xs is the
// staged row of token a_tok[p], so the engine reads each segment as
// consecutive rows (TMA boxes) instead of gathering token by token.  One
// warp per row; 8 rows per block.
// Rows past the planned assignments (the -1 slots of a caller routing) are
// not copied: no segment covers them.
__global__ void __launch_bounds__(256) stage_rows_kernel(const int* a_tok, const int* n_assign, int n_rows,
                                                         const uint8_t* xp, uint8_t* xs, int64_t row_bytes) {
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= n_rows || r >= __ldcg(n_assign)) return;
  const int u = (int)(row_bytes / 16);
  const uint4* src = reinterpret_cast<const uint4*>(xp + (int64_t)a_tok[r] * row_bytes);
  uint4* dst = reinterpret_cast<uint4*>(xs + (int64_t)r * row_bytes);
#pragma unroll 4
  for (int w = lane; w < u; w += 32) dst[w] = __ldcg(src + w);
}

// One CTA per expert.  Both passes over the routing read it with 16-byte
// loads through L1; the second gives every thread a contiguous run of
// (token, slot) entries, so one block-wide scan of the per-thread match
// counts orders the expert's assignments by (token, slot) with no barrier
// inside the loops.
__global__ void __launch_bounds__(256) plan_kernel(const PlanArgs a) {
  extern __shared__ int psm[];
  int* cnt = psm;  // [E]
  __shared__ int s_base[2];  // assignment offset, segment offset of this expert
  __shared__ int s_wsum[8];
  const int e = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int64_t TK = (int64_t)a.T * a.K;
  const int64_t n4 = TK >> 2;  // plan.idx is 256-byte aligned
  const int4* idx4 = reinterpret_cast<const int4*>(a.plan.idx);
  for (int i = tid; i < a.E; i += 256) cnt[i] = 0;
  __syncthreads();
  for (int64_t i = tid; i < n4; i += 256) {
    const int4 v = idx4[i];
    if (v.x >= 0) atomicAdd(&cnt[v.x], 1);  // -1: a skipped token's slot
    if (v.y >= 0) atomicAdd(&cnt[v.y], 1);
    if (v.z >= 0) atomicAdd(&cnt[v.z], 1);
    if (v.w >= 0) atomicAdd(&cnt[v.w], 1);
  }
  for (int64_t i = 4 * n4 + tid; i < TK; i += 256) {
    const int x = a.plan.idx[i];
    if (x >= 0) atomicAdd(&cnt[x], 1);
  }
  __syncthreads();
  if (tid == 0) {
    const int s2 = a.plan.seg2;
    int o = 0, ns = 0, ns2 = 0;
    for (int x = 0; x < e; ++x) {
      o += cnt[x];
      ns += (cnt[x] + a.seg - 1) / a.seg;
      if (s2) ns2 += (cnt[x] + s2 - 1) / s2;
    }
    s_base[0] = o;
    s_base[1] = ns;
    const int m = cnt[e];
    for (int j = 0; j < m; j += a.seg) a.plan.segs[ns++] = make_int4(e, o + j, min(a.seg, m - j), 0);
    if (s2)
      for (int j = 0; j < m; j += s2) a.plan.segs2[ns2++] = make_int4(e, o + j, min(s2, m - j), 0);
    a.plan.counts[e] = m;
    if (e == a.E - 1) {
      *a.plan.n_segs = ns;
      if (s2) *a.plan.n_segs2 = ns2;
      *a.plan.n_assign = o + m;
    }
  }
  __syncthreads();
  if (e == a.E - 1)
    // positions past the planned assignments (skipped tokens' slots) name
    // token 0, so a copy over all T*K positions stays in bounds
    for (int64_t q = s_base[0] + cnt[e] + tid; q < TK; q += 256) a.plan.a_tok[q] = 0;
  // this thread's entries: [lo, hi), a multiple of 4 long except at the end
  const int64_t run = ((TK + 255) / 256 + 3) & ~(int64_t)3;
  const int64_t lo = min(TK, (int64_t)tid * run), hi = min(TK, lo + run);
  auto match = [&](int64_t i, int x) { return x == e ? 1 : 0; };
  int mine = 0;
  for (int64_t i = lo; i < hi; i += 4) {
    if (i + 4 <= hi) {
      const int4 v = idx4[i >> 2];
      mine += match(i, v.x) + match(i, v.y) + match(i, v.z) + match(i, v.w);
    } else {
      for (int64_t j = i; j < hi; ++j) mine += match(j, a.plan.idx[j]);
    }
  }
  int incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_wsum[wid] = incl;
  __syncthreads();
  int p = s_base[0] + incl - mine;
  for (int w = 0; w < wid; ++w) p += s_wsum[w];
  if (mine == 0) return;
  for (int64_t i = lo; i < hi; ++i) {
    if (a.plan.idx[i] != e) continue;
    a.plan.pos[i] = p;
    a.plan.a_tok[p] = (int)(i / a.K);
    a.plan.a_tk[p] = (int)i;
    a.plan.a_w[p] = a.plan.wts[i];
    ++p;
  }
}

// ---------------------------------------------------------------------------
// Grouped GEMV engine
// ---------------------------------------------------------------------------
// 2-D TMA descriptors of one expert's packed matrices (uint8, [rows, K/2]):
// gate/up boxes are 128 B x 128 rows, down boxes 128 B x 256 rows; 128B swizzle.
struct ExpertMaps {
  CUtensorMap gate, up, down;
};
static_assert(sizeof(ExpertMaps) == 384, "ExpertMaps layout");

struct EngineArgs {
  int K;     // reduction length (multiple of 128)
  int G;     // K / 128
  int N;     // weight rows
  int n_rt;  // row tiles
  int T, topk;
  const int4* segs;
  const int* n_segs;
  const int* a_tok;
  const int* a_tk;
  const float* a_w;
  const int* pos;
  const hn_expert_ptrs* table;
  hn_expert_ptrs single;
  const ExpertMaps* maps;  // device array [E] of tensor maps, or NULL: use single_maps
  ExpertMaps single_maps;
  const uint8_t* bsrc;  // staged tokens, [row][group][kChunk]
  int64_t b_rstride;    // bytes per staged row (groups * kChunk)
  int64_t b_rows;       // staged rows (KIND_DOWN tensor map)
  int b_use_tok;
  CUtensorMap bmap;     // KIND_DOWN: bsrc as uint8 [b_rows, b_rstride], 128 B x N boxes, 128B swizzle
  uint8_t* hp;
  int64_t hp_rstride;
  float* R;
  void* out;
  int64_t ldo;
  float* part;
  int* tile_ctr;
  int* rt_ctr;
  const int* nval;  // [T] slots per token that hold an expert (the combine's completion count)
  const int* tidx;  // [T*K] expert of each slot, -1 = unused (skipped by the combine)
  int* err;
  int P;
  int early;  // KIND_DOWN after a gate/up launch: only the token producer waits for it
  int defer_combine;  // EPI_COMBINE: leave the top-k sum to combine_kernel (large routings)
  int allow_rr;       // whole tiles round-robin over the CTAs when there are >= 4 per CTA (prefill sizes)
  int64_t max_segs;   // segments the plan can hold (bounds the tiles of an mma.sync engine CTA)
  int max_nt;         // tokens per segment / 8
  int gv;             // this call runs on the mma.sync engine (decided once for all its phases)
  float* corr_x;      // offset corrections of the staged activations / SiLU(gate)*up (mma.sync engine)
  float* corr_h;
};

template <int KIND>
struct TileMap {
  // GATEUP tiles are segment-major; DOWN tiles row-tile-major (a row tile's
  // segments finish together for the in-kernel combine), or segment-major
  // when segmaj (round-robin tiles: a wave of CTAs then shares one segment's
  // tokens and the row tiles of few experts in L2).
  static __device__ __forceinline__ void split(int tile, int n_rt, int n_segs, int& seg, int& rt, bool segmaj) {
    if (KIND == KIND_GATEUP || segmaj) {
      seg = tile / n_rt;
      rt = tile - seg * n_rt;
    } else {
      rt = tile / n_segs;
      seg = tile - rt * n_segs;
    }
  }
};

// Shared-memory plan of the tcgen05 engine (base rounded up to 1024 B).
//   weight ring: ST stages of 32 KB = one 2-D TMA box pair (A0 rows, A1 rows)
//     x 128 B (two 128-wide k-groups), 128B-swizzled: the 16-byte chunk c of
//     row r sits at chunk c ^ (r & 7) of the row.
//   token ring: SB stages of [2 halves][N tokens][128 B], 128B-swizzled
//     (the 16-byte unit u of token row r at u ^ (r & 7)): half h holds units
//     8h..8h+7 (k 64h..64h+63) of the k-group; the K-major SW128 operand of
//     MMA k-step s starts at half s/4, byte 32*(s%4), with SBO = 1024 bytes
//     (8 token rows).
template <int N, int ST, int SB>
struct TcSmem {
  static constexpr int kHdr = N <= 32 ? 1024 : 2048;  // barriers + per-token flags of the combine
  static constexpr int kWStage = 32768;
  static constexpr int kW = ST * kWStage;
  static constexpr int kBStage = 2 * N * 128;  // a multiple of 1024: stages stay swizzle-aligned
  static constexpr int kB = SB * kBStage;
  static constexpr int kTotal = 1024 /* alignment slack */ + kHdr + kW + kB;
  static_assert(kBStage % 1024 == 0, "token stages must stay 1024-byte aligned");
};

// Warp roles (a warp runs on SMSP warp % 4): dequant warps, epilogue warps,
// then one role warp on each SMSP.
constexpr int kTmemCols = 512;
constexpr int kKSplit = 2;                       // dequant warps per (matrix, TMEM lane quarter)
constexpr int kDeqWarps = 8 * kKSplit;
constexpr int kEpiWarps = 4;                     // one per TMEM lane quarter
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kTokWarp = kDeqWarps + kEpiWarps;  // token producer (SMSP 0)
constexpr int kMmaWarp0 = kTokWarp + 1;          // MMA issuer of matrix 0 (SMSP 1), allocates TMEM
constexpr int kWgtWarp = kTokWarp + 2;           // weight producer (SMSP 2)
constexpr int kMmaWarp1 = kTokWarp + 3;          // MMA issuer of matrix 1 (SMSP 3)
constexpr int kTcThreads = (kTokWarp + 4) * 32;
static_assert(kTokWarp % 4 == 0, "the four role warps must sit on the four SMSPs");

// TMEM columns: SA weight stages of {A0, A1} x 64 columns (128 k as float16
// pairs) from column 0, then SD piece accumulators of {A0, A1} x N fp32
// columns (with two, the MMA fills one while the epilogue drains the other).
// N = 16: 3 x 128 + 2 x 32; N = 32: 3 x 128 + 2 x 64; N = 64: 2 x 128 +
// 2 x 128; N = 128: 2 x 128 + 1 x 256.
template <int N>
struct TmemPlan {
  static constexpr int kDCols = 2 * N;
  static constexpr int SD = (2 * kDCols + 2 * 128 <= kTmemCols) ? 2 : 1;
  static constexpr int kFit = (kTmemCols - SD * kDCols) / 128;
  static constexpr int SA = kFit > 4 ? 4 : kFit;
  static constexpr int kD0 = SA * 128;
  static_assert(SA >= 2 && kD0 + SD * kDCols <= kTmemCols, "TMEM plan exceeds 512 columns");
};

// Segment, row tile, token count and first assignment of a tile.
struct TileInfo {
  int seg, rt, m, p0;
};
template <int KIND>
__device__ __forceinline__ TileInfo tile_info(const EngineArgs& a, int tile, int n_segs, bool segmaj) {
  TileInfo v;
  TileMap<KIND>::split(tile, a.n_rt, n_segs, v.seg, v.rt, segmaj);
  const int4 sg = a.segs[v.seg];
  v.m = sg.z;
  v.p0 = sg.y;
  return v;
}
template <int KIND>
__device__ __forceinline__ int tile_expert(const EngineArgs& a, int tile, int n_segs, bool segmaj) {
  int seg, rt;
  TileMap<KIND>::split(tile, a.n_rt, n_segs, seg, rt, segmaj);
  return __ldg(&a.segs[seg].x);
}
// Scale matrix of (expert e, matrix j) and the offset of row r's scale row in
// a tile; rows past N read row N-1's scales and are never stored.
template <int KIND>
__device__ __forceinline__ const uint16_t* scale_base(const EngineArgs& a, int e, int j) {
  const hn_expert_ptrs* ep = a.table ? a.table + e : &a.single;
  return KIND == KIND_GATEUP ? (j ? ep->up_scales : ep->gate_scales) : ep->down_scales;
}
template <int KIND>
__device__ __forceinline__ int64_t scale_off(const EngineArgs& a, int tile, int n_segs, int j, int r, bool segmaj) {
  int seg, rt;
  TileMap<KIND>::split(tile, a.n_rt, n_segs, seg, rt, segmaj);
  const int row = KIND == KIND_GATEUP ? rt * 128 + r : rt * 256 + j * 128 + r;
  return (int64_t)min(row, a.N - 1) * a.G;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// The same load with an L2 cache policy (createpolicy): weights are read
// once per layer, so they are loaded evict-first and leave L2 to what is
// reused (staged tokens, scales, routing plan, router weights, code).
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
      "%3}], [%4], %5;" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Stage index and phase bit of a ring of S mbarrier-guarded stages, advanced
// once per use.  A consumer waits on full[idx] with parity `phase`; a producer
// waits on empty[idx] with parity `phase ^ 1`, which a freshly initialised
// barrier already satisfies, so the first round needs no special case.
template <int S>
struct Ring {
  int idx = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next() {
    if (++idx == S) {
      idx = 0;
      phase ^= 1u;
    }
  }
};

// Persistent grouped GEMV/GEMM on the 5th-generation tensor cores.
//
// Work items are (tile, k-group pair); CTA c owns items [c*NI/P, (c+1)*NI/P)
// (stream-K), so every CTA streams the same number of weight bytes.  A tile's
// k-groups that one CTA runs (a "piece") accumulate in one TMEM accumulator.
// Warp roles (a warp runs on SMSP warp % 4):
//   warps 0-15   dequant warps: warp w dequantises matrix j = (w >> 2) & 1 for
//                TMEM lanes 32*(w&3).. (its 32 rows), k-half w >> 3 (64 k) of
//                each group, as float16 (n - 8) * scale, into the A stage;
//   warps 16-19  epilogue warps (one per lane quarter, both matrices): at the
//                end of each piece they drain the accumulator, write the
//                stream-K partial or run the epilogue;
//   warp 20      token producer: the token ring (TMA boxes for the down
//                phase, per-lane cp.async gathers for gate/up);
//   warps 21, 23 MMA issuers for matrix 0 and matrix 1: per k-group eight K=16
//                steps with the dequantised weights (TMEM) as A and the tokens
//                (SMEM) as B into the piece's accumulator; the two matrices use
//                separate columns, so two warps on two SMSPs issue them
//                independently;
//   warp 22      weight producer: one 32 KB 2-D TMA box pair per item.
// All hand-offs are mbarriers with bounded waits.
template <typename Tr, int N, int KIND, int EPI, int ST, int SB>
__global__ void __launch_bounds__(kTcThreads, 1) tc_engine_kernel(const __grid_constant__ EngineArgs a) {
  using L = TcSmem<N, ST, SB>;
  constexpr int SA = TmemPlan<N>::SA, SD = TmemPlan<N>::SD, D0 = TmemPlan<N>::kD0, DC = TmemPlan<N>::kDCols;
  // The token producer signals stage k after issuing group k + LOOK (its
  // copies then had LOOK groups of time to land); issuing k + LOOK needs the
  // MMA of k + LOOK - SB to be done, so SB - LOOK groups of slack remain.
  constexpr int LOOK = N <= 32 ? 3 : 2;
  static_assert(LOOK >= 1 && SB - LOOK >= 2 && SA <= 4 && SB <= 16 && ST <= 8 && N % 16 == 0 && N <= 128,
                "stage counts");
  constexpr uint32_t IDESC = umma_idesc<F16, 128, N>();
  constexpr uint32_t kDescHiSW128 = (1024u >> 4) | (1u << 14) | (2u << 29);  // SBO 1024 B, version 1, SWIZZLE_128B
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint64_t* a_full = bars;        // [SA][2] dequant warps of matrix j -> its MMA warp
  uint64_t* a_empty = bars + 8;   // [SA][2] MMA commit (matrix j) -> its dequant warps
  uint64_t* d_full = bars + 16;   // [SD] both MMA warps' commits at a piece end -> epilogue warps
  uint64_t* d_empty = bars + 20;  // [SD] epilogue warps -> MMA warps
  uint64_t* b_full = bars + 24;   // [SB] token producer -> MMA warps
  uint64_t* b_empty = bars + 40;  // [SB] both MMA warps' commits -> token producer
  uint64_t* w_full = bars + 56;   // [ST] weight TMA -> dequant warps
  uint64_t* w_empty = bars + 64;  // [ST] dequant warps -> weight producer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 72);
  int* bcast = reinterpret_cast<int*>(bars + 73);
  uint8_t* wst = smem + L::kHdr;
  uint8_t* bst = wst + L::kW;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < 2 * SA; ++s) {
      mbar_init(smem_u32(&a_full[s]), 4 * kKSplit);  // the dequant warps of one matrix
      mbar_init(smem_u32(&a_empty[s]), 1);
    }
    for (int s = 0; s < SD; ++s) {
      mbar_init(smem_u32(&d_full[s]), 2);
      mbar_init(smem_u32(&d_empty[s]), kEpiWarps);
    }
    for (int s = 0; s < SB; ++s) {
      // KIND_DOWN fills a stage with TMA (one arrival + bytes), KIND_GATEUP
      // with per-lane cp.async (one arrival per lane)
      mbar_init(smem_u32(&b_full[s]), (KIND == KIND_DOWN || !a.b_use_tok) ? 1 : 32);
      mbar_init(smem_u32(&b_empty[s]), 2);
    }
    for (int s = 0; s < ST; ++s) {
      mbar_init(smem_u32(&w_full[s]), 1);
      mbar_init(smem_u32(&w_empty[s]), kDeqWarps);
    }
    fence_barrier_init();
  }
  if (warp == kMmaWarp0) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  // Programmatic dependent launch: everything above runs while the previous
  // kernel of the stream finishes.  The gate/up phase reads the routing plan
  // and the staged tokens of the prep kernel, so it waits here, then lets the
  // down phase launch.  A down phase that follows a gate/up launch (a.early)
  // needs only the plan for its weight and dequant pipeline -- the plan was
  // complete and visible before that gate/up launch let it start -- and its
  // token producer waits for the gate/up results itself; any other launch
  // waits here for its predecessor.
  if (KIND == KIND_GATEUP || !a.early) griddep_wait();
  if (KIND == KIND_GATEUP) griddep_launch_dependents();
  const int n_segs = *a.n_segs;
  const int n_tiles = a.n_rt * n_segs;
  const int GP = (a.G + 1) >> 1;  // k-group pairs per tile
  const int64_t NI = (int64_t)n_tiles * GP;
  const int64_t P = min((int64_t)a.P, NI);
  const int64_t c = blockIdx.x;
  // Stream-K (items [c*NI/P, (c+1)*NI/P), tiles split across CTAs and
  // finished by the last arriver) balances a handful of tiles; with at least
  // four tiles per CTA, whole tiles go round-robin (tile c, c+P, ...), so the
  // CTAs of a wave work on neighbouring tiles and share their data in L2.
  const bool rr = a.allow_rr && n_tiles >= 4 * P;
  const int tstep = rr ? (int)P : 1;
  const int64_t b0 = c * NI / P, b1 = (c + 1) * NI / P;
  auto cta_of = [&](int64_t i) -> int64_t { return ((i + 1) * P - 1) / NI; };
  auto begin_of = [&](int64_t cc) -> int64_t { return cc * NI / P; };
  // Items are walked with 32-bit counters: (tile0, gp0) is the first item.
  const int rr_tiles = rr ? (int)((n_tiles - c + P - 1) / P) : 0;
  const int n_items = rr ? rr_tiles * GP : (int)(b1 - b0);
  const int tile0 = rr ? (int)c : (int)(b0 / GP), gp0 = rr ? 0 : (int)(b0 - (int64_t)tile0 * GP);
  const int tile_last = rr ? (int)c + (rr_tiles - 1) * (int)P : (int)((b1 - 1) / GP);

  const bool active = NI > 0 && c < P;

  if (!active) {
    // no work for this CTA: straight to the teardown
  } else if (warp == kWgtWarp) {
    // ------------------------- weight producer (2-D TMA) -------------------------
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      Ring<ST> rw;
      int tile = tile0, gp = gp0;
      for (int i = 0; i < n_items; ++i) {
        int seg, rt;
        TileMap<KIND>::split(tile, a.n_rt, n_segs, seg, rt, rr);
        const int e = a.segs[seg].x;
        const ExpertMaps* em = a.maps ? a.maps + e : &a.single_maps;
        mbar_wait(smem_u32(&w_empty[rw.idx]), rw.phase ^ 1u, a.err);
        const uint32_t bar = smem_u32(&w_full[rw.idx]);
        mbar_arrive_expect_tx(bar, L::kWStage);
        const uint32_t dst = smem_u32(wst + rw.idx * L::kWStage);
        // decode streams each weight once (evict-first); round-robin tiles
        // reuse an expert's weights across its segments (default policy)
        if (KIND == KIND_GATEUP) {
          if (rr) {
            tma_load_2d(dst, &em->gate, gp * 128, rt * 128, bar);
            tma_load_2d(dst + 16384, &em->up, gp * 128, rt * 128, bar);
          } else {
            tma_load_2d_hint(dst, &em->gate, gp * 128, rt * 128, bar, pol);
            tma_load_2d_hint(dst + 16384, &em->up, gp * 128, rt * 128, bar, pol);
          }
        } else {
          if (rr)
            tma_load_2d(dst, &em->down, gp * 128, rt * 256, bar);
          else
            tma_load_2d_hint(dst, &em->down, gp * 128, rt * 256, bar, pol);
        }
        rw.next();
        if (++gp == GP) {
          gp = 0;
          tile += tstep;
        }
      }
    }
    __syncwarp();
  } else if (warp == kTokWarp) {
    // ------------------------- token producer -------------------------
    int k = 0, tile = tile0, gp = gp0;
    if (KIND == KIND_DOWN || !a.b_use_tok) {
      // Rows of a segment are consecutive (assignment order): each k-group is
      // two TMA boxes of N rows x 128 B (128B swizzle); rows past the end are
      // zero-filled.
      Ring<SB> rb;
      if (lane == 0) {
        griddep_wait();  // the staged rows are the previous kernel's output
        for (int i = 0; i < n_items; ++i) {
          int seg, rt;
          TileMap<KIND>::split(tile, a.n_rt, n_segs, seg, rt, rr);
          const int row0 = a.segs[seg].y;
          const int ng = min(2, a.G - 2 * gp);
          for (int gi = 0; gi < ng; ++gi, ++k) {
            const int grp = 2 * gp + gi;
            mbar_wait(smem_u32(&b_empty[rb.idx]), rb.phase ^ 1u, a.err);
            const uint32_t bar = smem_u32(&b_full[rb.idx]);
            mbar_arrive_expect_tx(bar, (uint32_t)(2 * N * 128));
            const uint32_t dst = smem_u32(bst + rb.idx * L::kBStage);
            tma_load_2d(dst, &a.bmap, grp * kChunk, row0, bar);
            tma_load_2d(dst + N * 128, &a.bmap, grp * kChunk + 128, row0, bar);
            rb.next();
          }
          if (++gp == GP) {
            gp = 0;
            tile += tstep;
          }
        }
      }
      __syncwarp();
    } else {
      // Gathered tokens: lane l copies tokens l, l+32, ... of the segment with
      // cp.async into the swizzled rows; a stage is signalled (after its
      // copies landed and a proxy fence) LOOK groups later.
      constexpr int TPL = (N + 31) / 32;  // tokens per lane
      Ring<SB> rb, rs;  // rb: stage being filled; rs: next stage to signal (LOOK behind)
      for (int i = 0; i < n_items; ++i) {
        int seg, rt;
        TileMap<KIND>::split(tile, a.n_rt, n_segs, seg, rt, rr);
        const int4 sg = a.segs[seg];
        const uint8_t* src_tok[TPL];
#pragma unroll
        for (int q = 0; q < TPL; ++q) {
          const int tk = lane + 32 * q;
          src_tok[q] = nullptr;
          if (tk < sg.z) {
            const int row = a.b_use_tok ? a.a_tok[sg.y + tk] : sg.y + tk;
            src_tok[q] = a.bsrc + (int64_t)row * a.b_rstride;
          }
        }
        const int ng = min(2, a.G - 2 * gp);
        for (int gi = 0; gi < ng; ++gi, ++k) {
          const int grp = 2 * gp + gi;
          mbar_wait(smem_u32(&b_empty[rb.idx]), rb.phase ^ 1u, a.err);
#pragma unroll
          for (int q = 0; q < TPL; ++q) {
            if (src_tok[q]) {
              const int tk = lane + 32 * q;
              const uint32_t dst = smem_u32(bst + rb.idx * L::kBStage + tk * 128);
              const uint8_t* src = src_tok[q] + (int64_t)grp * kChunk;
              const int sw = tk & 7;
#pragma unroll
              for (int u = 0; u < 16; ++u)
                cp_async16(dst + (u >> 3) * (N * 128) + (((u & 7) ^ sw) << 4), src + u * 16);
            }
          }
          cp_async_commit();
          rb.next();
          if (k >= LOOK) {
            cp_async_wait<LOOK>();
            fence_proxy_async_smem();  // generic-proxy writes -> read by the tensor core (async proxy)
            mbar_arrive(smem_u32(&b_full[rs.idx]));
            rs.next();
          }
        }
        if (++gp == GP) {
          gp = 0;
          tile += tstep;
        }
      }
      cp_async_wait<0>();
      fence_proxy_async_smem();
      for (int r = 0; r < min(k, LOOK); ++r) {
        mbar_arrive(smem_u32(&b_full[rs.idx]));
        rs.next();
      }
    }
  } else if (warp == kMmaWarp0 || warp == kMmaWarp1) {
    // ------------------------------ MMA issuers ------------------------------
    // The whole warp runs this loop (operands stay warp-uniform); the MMAs and
    // commits are issued by one elected lane.
    const int mj = warp == kMmaWarp0 ? 0 : 1;
    Ring<SA> ra;
    Ring<SB> rb;
    Ring<SD> rd;
    // per-warp constants: barrier addresses (stage s at +8*s, A stages at
    // +16*s for this matrix), the B ring's descriptor start, TMEM columns
    const uint32_t afull_m = smem_u32(&a_full[mj]), aempty_m = smem_u32(&a_empty[mj]);
    const uint32_t bfull0 = smem_u32(&b_full[0]), bempty0 = smem_u32(&b_empty[0]);
    const uint32_t dfull0 = smem_u32(&d_full[0]), dempty0 = smem_u32(&d_empty[0]);
    // B descriptor (32-bit halves): K-major SW128 tile (start, LBO ignored =
    // 1, SBO 1024 B, layout SWIZZLE_128B); stage sb starts kBStage/16 units on
    constexpr uint32_t kBStep = L::kBStage >> 4;
    const uint32_t b_lo0 = ((smem_u32(bst) >> 4) & 0x3FFFu) | (1u << 16);
    const uint32_t a_col = tbase + mj * 64, d_col = tbase + D0 + mj * N;
    uint32_t acc = 0;  // 0: the next group starts a piece (overwrites the accumulator)
    auto group = [&](bool end) {
      const int sa = ra.idx, sb = rb.idx;
      if (acc == 0) mbar_wait(dempty0 + 8 * rd.idx, rd.phase ^ 1u, a.err);
      mbar_wait(bfull0 + 8 * sb, rb.phase, a.err);
      mbar_wait(afull_m + 16 * sa, ra.phase, a.err);
      tc_fence_after();
      umma_group8_sw128<N>(d_col + rd.idx * DC, a_col + sa * 128, b_lo0 + sb * kBStep, kDescHiSW128, IDESC, acc);
      umma_commit_elect(aempty_m + 16 * sa);
      umma_commit_elect(bempty0 + 8 * sb);
      if (end) {
        umma_commit_elect(dfull0 + 8 * rd.idx);
        rd.next();
      }
      acc = end ? 0u : 1u;
      ra.next();
      rb.next();
    };
    int gp = gp0;
    for (int i = 0; i < n_items; ++i) {
      const int ng = min(2, a.G - 2 * gp);
      const bool last_item = i == n_items - 1;
      group((2 * gp == a.G - 1) || (last_item && ng == 1));
      if (ng == 2) group((2 * gp + 1 == a.G - 1) || last_item);
      if (++gp == GP) gp = 0;
    }
    __syncwarp();
  } else if (warp < kDeqWarps) {
    // ------------------------------ dequant warps ------------------------------
    constexpr int kC = 4 / kKSplit;  // 16-byte chunks (32 k each) of a group per thread
    const int q = warp & 3, j = (warp >> 2) & 1, h = warp >> 3, r = q * 32 + lane;
    const uint32_t tlane = tbase + ((uint32_t)(q * 32) << 16);
    const uint8_t* wrow = wst + (j * 128 + r) * 128;  // this thread's row inside a weight stage
    const int swz = r & 7;
    // Scale prefetch cursor, two items ahead of the dequantisation: fetch()
    // loads the two group scales of the item at (ptile, pgp) and advances.
    // The scale row of the next tile (its base pointer) and the expert of the
    // tile after it are loaded a whole tile ahead, so no load result is
    // consumed soon after it was issued.
    int ptile = tile0, pgp = gp0, pleft = n_items;
    const uint16_t* sp =
        scale_base<KIND>(a, tile_expert<KIND>(a, ptile, n_segs, rr), j) + scale_off<KIND>(a, ptile, n_segs, j, r, rr);
    const uint16_t* nb =
        ptile + tstep <= tile_last ? scale_base<KIND>(a, tile_expert<KIND>(a, ptile + tstep, n_segs, rr), j) : sp;
    int nne = ptile + 2 * tstep <= tile_last ? tile_expert<KIND>(a, ptile + 2 * tstep, n_segs, rr) : 0;
    auto fetch = [&](uint32_t& s0, uint32_t& s1) {
      if (pleft <= 0) return;
      s0 = __ldg(sp + 2 * pgp);
      s1 = 2 * pgp + 1 < a.G ? __ldg(sp + 2 * pgp + 1) : 0u;
      if (--pleft > 0 && ++pgp == GP) {
        pgp = 0;
        ptile += tstep;
        sp = nb + scale_off<KIND>(a, ptile, n_segs, j, r, rr);
        nb = ptile + tstep <= tile_last ? scale_base<KIND>(a, nne, j) : sp;
        nne = ptile + 2 * tstep <= tile_last ? tile_expert<KIND>(a, ptile + 2 * tstep, n_segs, rr) : 0;
      }
    };
    uint32_t sc0 = 0, sc1 = 0, n10 = 0, n11 = 0, n20 = 0, n21 = 0;  // scales of items it, it+1, it+2
    fetch(sc0, sc1);
    fetch(n10, n11);
    fetch(n20, n21);
    // Per-thread constants: swizzled offsets of this row's 16-byte chunks for
    // the two groups of a weight stage, this matrix's A-stage barriers (stage
    // sa at +16*sa bytes) and TMEM column.
    int choff[2][kC];
#pragma unroll
    for (int g = 0; g < 2; ++g)
#pragma unroll
      for (int i = 0; i < kC; ++i) choff[g][i] = ((g * 4 + h * kC + i) ^ swz) << 4;
    const uint32_t afull_j = smem_u32(&a_full[j]), aempty_j = smem_u32(&a_empty[j]);
    const uint32_t tcol_j = tlane + j * 64 + h * (16 * kC);
    Ring<ST> rw;
    Ring<SA> ra;
    // One group: load this thread's chunks, wait for the A stage, dequantise
    // into TMEM, wait for the stores, signal (and release the weight stage
    // after the item's last group: the refill is an async-proxy write that is
    // not ordered after shared loads still in flight).
    auto group = [&](const uint8_t* wrow_p, int gi, uint32_t sv, bool last, uint32_t wempty) {
      const int sa = ra.idx;
      uint4 W[kC];
#pragma unroll
      for (int i = 0; i < kC; ++i) W[i] = *reinterpret_cast<const uint4*>(wrow_p + choff[gi][i]);
      const uint32_t s2 = __byte_perm(sv, sv, 0x1010);
      mbar_wait(aempty_j + 16 * sa, ra.phase ^ 1u, a.err);
      tc_fence_after();
      const uint32_t acol = tcol_j + sa * 128;
#pragma unroll
      for (int i = 0; i < kC; ++i) {
        uint32_t o[16];
        dequant_word_f16(W[i].x, s2, o + 0);
        dequant_word_f16(W[i].y, s2, o + 4);
        dequant_word_f16(W[i].z, s2, o + 8);
        dequant_word_f16(W[i].w, s2, o + 12);
        tmem_st16(acol + 16 * i, o);
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      mbar_arrive_elect(afull_j + 16 * sa);
      if (last) mbar_arrive_elect(wempty);
      ra.next();
    };
    int gp = gp0;
#pragma unroll 1
    for (int it = 0; it < n_items; ++it) {
      const int ng = min(2, a.G - 2 * gp);
      const int ws = rw.idx;
      mbar_wait(smem_u32(&w_full[ws]), rw.phase, a.err);
      const uint8_t* wrow_p = wrow + ws * L::kWStage;
      const uint32_t wempty = smem_u32(&w_empty[ws]);
      group(wrow_p, 0, sc0, ng == 1, wempty);
      if (ng == 2) group(wrow_p, 1, sc1, true, wempty);
      rw.next();
      if (++gp == GP) gp = 0;
      sc0 = n10;
      sc1 = n11;
      n10 = n20;
      n11 = n21;
      fetch(n20, n21);
    }
  } else {
    // ------------------------------ epilogue warps ------------------------------
    const int q = warp & 3, r = q * 32 + lane;
    const int et = threadIdx.x - kDeqWarps * 32;  // 0 .. kEpiThreads-1
    const uint32_t tlane = tbase + ((uint32_t)(q * 32) << 16);
    // One 16-token chunk of the piece's result: v0 = matrix 0 (gate rows, or
    // the first 128 down rows), v1 = matrix 1 (up rows, or down rows 128..255).
    auto emit = [&](const TileInfo& ti, int hc, const float (&v0)[16], const float (&v1)[16]) {
      if (KIND == KIND_GATEUP) {
        // SiLU(gate) * up as float16 into the down phase's staged operand:
        // row r of row tile rt is k = r of k-group rt
        uint8_t* dstp = a.hp + (int64_t)ti.rt * kChunk + staged_offset(r);
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          const int tok = hc * 16 + n;
          if (tok < ti.m) {
            const float hv = silu_f(v0[n]) * v1[n];
            *reinterpret_cast<__half*>(dstp + (int64_t)(ti.p0 + tok) * a.hp_rstride) = __float2half_rn(hv);
          }
        }
      } else {
        // rows r and r + 128 of the 256-row tile, per token
        const int row0 = ti.rt * 256 + r;
        const bool ok0 = row0 < a.N, ok1 = row0 + 128 < a.N;
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          const int tok = hc * 16 + n;
          if (tok < ti.m) {
            const int p = ti.p0 + tok;
            if (EPI == EPI_STORE) {
              typename Tr::T* o = reinterpret_cast<typename Tr::T*>(a.out) + (int64_t)a.a_tok[p] * a.ldo + row0;
              if (ok0) o[0] = Tr::from_f(v0[n]);
              if (ok1) o[128] = Tr::from_f(v1[n]);
            } else {
              const float w = a.a_w[p];
              float* o = a.R + (int64_t)a.a_tk[p] * a.N + row0;
              if (ok0) o[0] = v0[n] * w;
              if (ok1) o[128] = v1[n] * w;
            }
          }
        }
      }
    };
    // Top-k combine, spread over the tiles: R holds weight * y for every
    // (token, slot) row; each (row tile, token) counts the contributions
    // written so far, and the tile that writes a token's last one sums its
    // slots in slot order (the same order whichever tile does it) into the
    // output.  The counter is reset by that tile.
    auto combine = [&](const TileInfo& ti) {
      __threadfence();
      named_bar_sync(1, kEpiThreads);
      if (et < ti.m) {
        const int t = a.a_tok[ti.p0 + et];
        int* ctr = a.rt_ctr + (int64_t)ti.rt * a.T + t;
        const bool last = atomicAdd(ctr, 1) == __ldcg(a.nval + t) - 1;
        if (last) *ctr = 0;
        bcast[2 + et] = last ? t : -1;
      }
      named_bar_sync(1, kEpiThreads);
      __threadfence();
      const int r0 = ti.rt * 256 + 2 * et;
      if (r0 < a.N) {  // N is a multiple of 128: rows r0, r0 + 1
        const float* Rb = a.R + r0;
        typename Tr::T* ob = reinterpret_cast<typename Tr::T*>(a.out) + r0;
#pragma unroll 4
        for (int i = 0; i < ti.m; ++i) {
          const int t = bcast[2 + i];
          if (t >= 0) {
            float x = 0.f, y = 0.f;
            for (int kk = 0; kk < a.topk; ++kk) {
              if (__ldcg(a.tidx + (int64_t)t * a.topk + kk) < 0) continue;  // an unused slot: no row was written
              const float2 v = __ldcg(reinterpret_cast<const float2*>(Rb + (int64_t)(t * a.topk + kk) * a.N));
              x += v.x;
              y += v.y;
            }
            ob[(int64_t)t * a.ldo] = Tr::from_f(x);
            ob[(int64_t)t * a.ldo + 1] = Tr::from_f(y);
          }
        }
      }
    };
    Ring<SD> rd;
#pragma unroll 1
    for (int tile = tile0; tile <= tile_last; tile += tstep) {
      const TileInfo ti = tile_info<KIND>(a, tile, n_segs, rr);
      const int64_t ts = (int64_t)tile * GP, te = ts + GP;
      const uint32_t dcol = tlane + D0 + rd.idx * DC;
      mbar_wait_backoff(smem_u32(&d_full[rd.idx]), rd.phase, a.err, 256);
      tc_fence_after();
      bool own = true;
      if (rr || (b0 <= ts && b1 >= te)) {
        // the whole tile ran here: epilogue straight from the accumulator
#pragma unroll 1
        for (int hc = 0; hc < N / 16; ++hc) {
          if (hc * 16 < ti.m) {
            uint32_t d0[16], d1[16];
            tmem_ld16(dcol + hc * 16, d0);
            tmem_ld16(dcol + N + hc * 16, d1);
            tmem_ld_wait16x2(d0, d1);
            float v0[16], v1[16];
#pragma unroll
            for (int n = 0; n < 16; ++n) {
              v0[n] = __uint_as_float(d0[n]);
              v1[n] = __uint_as_float(d1[n]);
            }
            emit(ti, hc, v0, v1);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&d_empty[rd.idx]));
      } else {
        // Every piece of a split tile (the last arriver's own too) goes
        // through its partial slot; the last arriver sums the slots in CTA
        // order, so the result does not depend on which CTA finishes last.
        const int slot = (ts <= b0) ? 0 : 1;
        float* dst = a.part + ((((int64_t)c * 2 + slot) * 2 * kEpiWarps + q) * N) * 32 + lane;
#pragma unroll 1
        for (int hc = 0; hc < N / 16; ++hc) {
          if (hc * 16 < ti.m) {
            uint32_t d0[16], d1[16];
            tmem_ld16(dcol + hc * 16, d0);
            tmem_ld16(dcol + N + hc * 16, d1);
            tmem_ld_wait16x2(d0, d1);
#pragma unroll
            for (int n = 0; n < 16; ++n) {
              dst[(hc * 16 + n) * 32] = __uint_as_float(d0[n]);
              dst[(kEpiWarps * N + hc * 16 + n) * 32] = __uint_as_float(d1[n]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&d_empty[rd.idx]));
        __threadfence();
        named_bar_sync(1, kEpiThreads);
        const int64_t c0 = cta_of(ts), c1 = cta_of(te - 1);
        if (et == 0) bcast[0] = (atomicAdd(&a.tile_ctr[tile], 1) == (int)(c1 - c0));
        named_bar_sync(1, kEpiThreads);
        own = bcast[0] != 0;
        if (own) {
          __threadfence();
#pragma unroll 1
          for (int hc = 0; hc < N / 16; ++hc) {
            if (hc * 16 < ti.m) {
              float v0[16], v1[16];
#pragma unroll
              for (int n = 0; n < 16; ++n) v0[n] = v1[n] = 0.f;
              for (int64_t cc = c0; cc <= c1; ++cc) {
                const int64_t bc = begin_of(cc);
                const int sl = (bc >= ts && bc < te) ? 0 : 1;
                const float* src = a.part + ((((int64_t)cc * 2 + sl) * 2 * kEpiWarps + q) * N) * 32 + lane;
#pragma unroll
                for (int n = 0; n < 16; ++n) {
                  v0[n] += ld_cg_f32(src + (hc * 16 + n) * 32);
                  v1[n] += ld_cg_f32(src + (kEpiWarps * N + hc * 16 + n) * 32);
                }
              }
              emit(ti, hc, v0, v1);
            }
          }
          if (et == 0) a.tile_ctr[tile] = 0;
        }
      }
      if (KIND == KIND_DOWN && EPI == EPI_COMBINE && own && !a.defer_combine) combine(ti);
      rd.next();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp0) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

#include "hn_gv.cuh"

// ---------------------------------------------------------------------------
// Top-k combine of a large routing: out[t, :] = sum over slots k, in slot
// order, of R[t*K + k, :] (each row already scaled by its routing weight), in
// fp32, stored in the activation dtype.  Bandwidth-bound: one pass over R.
// Decode-size routings combine inside the down-phase epilogue instead.
// ---------------------------------------------------------------------------
template <typename Tr>
__global__ void __launch_bounds__(256) combine_kernel(const float* R, const int* tidx, int T, int K, int H, void* out,
                                                      int64_t ldo) {
  const int64_t n4 = (int64_t)T * (H / 4);
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n4; i += (int64_t)gridDim.x * 256) {
    const int t = (int)(i / (H / 4)), h = (int)(i - (int64_t)t * (H / 4)) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < K; ++k) {
      if (__ldg(tidx + (int64_t)t * K + k) < 0) continue;  // an unused slot: no row was written
      const float4 v = __ldcs(reinterpret_cast<const float4*>(R + ((int64_t)t * K + k) * H + h));
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    typename Tr::T* o = reinterpret_cast<typename Tr::T*>(out) + (int64_t)t * ldo + h;
    o[0] = Tr::from_f(acc.x);
    o[1] = Tr::from_f(acc.y);
    o[2] = Tr::from_f(acc.z);
    o[3] = Tr::from_f(acc.w);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// Tokens per segment = N of the MMA, 8*nt: 16 or 32 for decode-size steps
// (T <= 64); for larger steps by the mean assignments per expert, T*K/E, up
// to 128 (prefill), so each dequantised weight tile serves more tokens.
static int pick_nt(int64_t T, int64_t K, int64_t E) {
  if (T <= 8) return 1;
  if (T <= 64) {
    // decode: 8-token segments while experts get at most 2 assignments on
    // average (GLM-4.5 at 32 tokens: hardly any expert reaches 9), 16-token
    // ones up to 4 on average (or T <= 16), else 32 tokens
    const int64_t avg = T * K / std::max<int64_t>(E, 1);
    if (avg <= 2) return 1;
    return (avg <= 4 || T <= 16) ? 2 : 4;
  }
  const int64_t avg = T * K / std::max<int64_t>(E, 1);
  if (avg >= 96) return 16;
  if (avg >= 48) return 8;
  return 4;
}

// Weight stages (32 KB each) and token stages per tile width N; the totals
// stay within 227 KB of shared memory.
template <int N>
struct TcTune {
  static constexpr int ST = N <= 32 ? 5 : (N == 64 ? 4 : 3);
  static constexpr int SB = N <= 32 ? 8 : (N == 64 ? 5 : 4);
};

static int encode_token_map(CUtensorMap* data, const void* base, int64_t rows, int64_t row_bytes, int box_rows);

// Which engine runs a phase: segments of at most 16 tokens go to the
// register-dequant mma.sync engine (gv_kernel) unless hn_set_decode_engine
// chose the tcgen05 engine; larger segments always run on tcgen05, whose
// tensor pipe is four times wider (at 24-32 tokens per segment the mma.sync
// pipe, not HBM, would bound the phase).
static std::atomic<int> g_decode_engine{HN_ENGINE_AUTO};
static int gv_nt(int nt) { return nt <= 1 ? 1 : 2; }
// CTAs of an mma.sync engine launch (two per SM)
static int gv_grid(int nt) {
  const int sms = sm_count_current();
  (void)nt;
  return (sms > 0 ? sms : 148) * GvCfg<1>::kCtasPerSm;
}
static int gv_warps(int nt) {
  (void)nt;
  return GvCfg<1>::W;
}
// Tiles one CTA's step range can touch at most: the engine caches their
// metadata in shared memory (kGvMaxTiles entries).
static bool gv_fits(int nt, int64_t max_segs, int64_t rows, bool gateup) {
  const int64_t tile_rows = (gateup ? 16 : 32) * (int64_t)gv_warps(nt);
  const int64_t tiles = max_segs * ((rows + tile_rows - 1) / tile_rows);
  return tiles / gv_grid(nt) + 3 <= kGvMaxTiles;
}
static bool use_gv(int nt) { return nt <= 2 && g_decode_engine.load(std::memory_order_relaxed) != HN_ENGINE_TCGEN05; }
// Bytes of stream-K partials an mma.sync engine launch may write.
static size_t gv_part_bytes(int nt) {
  return (size_t)gv_grid(nt) * 2 * gv_warps(nt) * 2 * gv_nt(nt) * 32 * 16;
}

template <typename Tr, int NT, int KIND, int EPI>
static int launch_gv_t(const GvArgs& a, cudaStream_t s) {
  using C = GvCfg<NT>;
  auto kern = gv_kernel<Tr, NT, KIND, EPI>;
  static std::atomic<bool> attr_set[64] = {};  // per instantiation and device; setting it twice is harmless
  int dev = 0;
  HN_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !attr_set[dev].load(std::memory_order_acquire)) {
    HN_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kTotal));
    if (dev >= 0 && dev < 64) attr_set[dev].store(true, std::memory_order_release);
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)gv_grid(NT));
  cfg.blockDim = dim3((unsigned)C::kThreads);
  cfg.dynamicSmemBytes = C::kTotal;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  HN_CUDA(cudaLaunchKernelEx(&cfg, kern, a));
  return HN_OK;
}

template <typename Tr, int KIND, int EPI>
static int launch_gv(int nt, const GvArgs& a, cudaStream_t s) {
  if (nt <= 1) return launch_gv_t<Tr, 1, KIND, EPI>(a, s);
  return launch_gv_t<Tr, 2, KIND, EPI>(a, s);
}

// The mma.sync engine's arguments for the phase the tcgen05 engine's
// arguments describe (same plan, same staged rows, same outputs).
static GvArgs gv_args(const EngineArgs& e, int KIND) {
  GvArgs g{};
  g.K = e.K;
  g.G = e.G;
  g.rows = e.N;
  const int tile_rows = (KIND == KIND_GATEUP ? 16 : 32) * gv_warps(gv_nt(e.max_nt));
  g.tps = (e.N + tile_rows - 1) / tile_rows;
  g.T = e.T;
  g.topk = e.topk;
  g.segs = e.segs;
  g.n_segs = e.n_segs;
  g.a_tok = e.a_tok;
  g.a_tk = e.a_tk;
  g.a_w = e.a_w;
  g.table = e.table;
  g.single = e.single;
  g.bsrc = e.bsrc;
  g.b_rstride = e.b_rstride;
  g.b_by_token = KIND == KIND_GATEUP ? 1 : e.b_use_tok;  // gate/up reads x by token (xp), down its own rows
  g.corr_b = g.b_by_token ? e.corr_x : e.corr_h;          // offset corrections of those staged rows
  g.corr_out = KIND == KIND_GATEUP ? e.corr_h : nullptr;  // gate/up stages hp and its corrections
  g.hp = e.hp;
  g.hp_rstride = e.hp_rstride;
  g.R = e.R;
  g.out = e.out;
  g.ldo = e.ldo;
  g.part = e.part;
  g.tile_ctr = e.tile_ctr;
  g.rt_ctr = e.rt_ctr;
  g.nval = e.nval;
  g.tidx = e.tidx;
  g.defer_combine = e.defer_combine;
  g.early = e.early;
  g.P = e.P;
  return g;
}

template <typename Tr, int N, int KIND, int EPI>
static int launch_engine_t(const EngineArgs& a, cudaStream_t s) {
  using TU = TcTune<N>;
  using L = TcSmem<N, TU::ST, TU::SB>;
  static_assert(2 * L::kTotal > 228 * 1024, "one engine CTA per SM: it allocates all 512 TMEM columns");
  static_assert(L::kTotal <= 227 * 1024, "engine shared memory exceeds the per-CTA limit");
  auto kern = tc_engine_kernel<Tr, N, KIND, EPI, TU::ST, TU::SB>;
  EngineArgs e = a;
  if (KIND == KIND_DOWN || !e.b_use_tok) {
    const int rc = encode_token_map(&e.bmap, e.bsrc, e.b_rows, e.b_rstride, N);
    if (rc) return rc;
  }
  static bool attr_set[64] = {};  // per instantiation and device
  int dev = 0;
  HN_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    HN_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal));
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  // Programmatic stream serialisation: the launch may start while the
  // previous kernel of the stream finishes (see griddep_wait in the kernel).
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)e.P);
  cfg.blockDim = dim3((unsigned)kTcThreads);
  cfg.dynamicSmemBytes = L::kTotal;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  HN_CUDA(cudaLaunchKernelEx(&cfg, kern, e));
  return HN_OK;
}

template <typename Tr, int KIND, int EPI>
static int launch_engine(int nt, const EngineArgs& a, cudaStream_t s) {
  if (a.gv) return launch_gv<Tr, KIND, EPI>(nt, gv_args(a, KIND), s);
  if (nt <= 2) return launch_engine_t<Tr, 16, KIND, EPI>(a, s);
  if (nt <= 4) return launch_engine_t<Tr, 32, KIND, EPI>(a, s);
  if (nt <= 8) return launch_engine_t<Tr, 64, KIND, EPI>(a, s);
  return launch_engine_t<Tr, 128, KIND, EPI>(a, s);
}

// A workspace has a counter section at its FRONT and a data section at its
// BACK.  The error word (offset 0) and the prep kernel's arrival counter
// (offset 256) must be zero when a call starts; the error word is only ever
// set by a failing wait, and the route counter is reset by the kernel that
// reads its final value.  No data section reaches below offset 512 (every
// layout's counter section is at least 1280 bytes and the data section sits
// above it), so those two words survive calls of any shape.  The engine
// counters after them are zeroed by the prep kernel at the start of every
// call, because another shape's data section may have covered them.
struct Layout {
  size_t err, route_ctr, ctr1, ctr2, rtctr, counters;                                     // front
  size_t counts, n_segs, segs, n_segs2, segs2, a_tok, a_tk, a_w, pos, idx, wts, nval, n_assign, corr_x, corr_h, xp, hp, xs, part1, part2, R,
      rlog, data;  // back (relative)
  bool has_rlog, has_xs;
  bool gv;           // the call runs on the mma.sync engine (every phase, offset staging)
  int seg2;          // second segment cut for the down phase (0: none)
  int64_t max_segs;  // segments the plan can hold
  size_t total() const { return counters + data; }
};

static size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// T tokens of width Kin, top-k over E experts; phase 1 rows F (0: no phase 1),
// phase 2 rows N2.
static Layout make_layout(int64_t T, int64_t Kin, int64_t E, int topk, int64_t F, int64_t N2, int nt, int P,
                          bool combine) {
  Layout l{};
  const int64_t TK = T * topk;
  const int64_t seg = seg_tokens(nt);
  const int64_t max_segs = std::min<int64_t>(E, TK) + (TK + seg - 1) / seg;
  l.max_segs = max_segs;
  const int64_t n_rt2 = (N2 + 255) / 256;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o = align256(o + std::max<size_t>(bytes, 4));
    return at;
  };
  l.err = take(4);
  l.route_ctr = take(4);
  l.ctr1 = take(F ? 4 * max_segs * (F / 128) : 0);
  l.ctr2 = take(4 * max_segs * n_rt2);
  l.rtctr = take(combine ? 4 * n_rt2 * T : 4);
  l.counters = o;
  o = 0;
  l.counts = take(4 * E);
  l.n_segs = take(4);
  l.segs = take(16 * max_segs);
  // 128-token segments of a routed layer: the down phase runs 64-token tiles
  // (two accumulator stages), cut from the same assignment lists
  l.seg2 = (F && nt >= 16) ? seg_tokens(8) : 0;
  const int64_t max_segs2 = l.seg2 ? std::min<int64_t>(E, TK) + (TK + l.seg2 - 1) / l.seg2 : 0;
  l.n_segs2 = take(4);
  l.segs2 = take(16 * max_segs2);
  l.a_tok = take(4 * TK);
  l.a_tk = take(4 * TK);
  l.a_w = take(4 * TK);
  l.pos = take(4 * TK);
  l.idx = take(4 * TK);
  l.wts = take(4 * TK);
  l.nval = take(4 * T);
  l.n_assign = take(4);
  l.corr_x = take((size_t)4 * (Kin / 128) * T);
  l.corr_h = take(F ? (size_t)4 * (F / 128) * TK : 0);
  l.xp = take((size_t)(Kin / 128) * T * kChunk);
  l.hp = take(F ? (size_t)(F / 128) * TK * kChunk : 0);
  // routed gate/up tokens staged in assignment order, read by TMA instead of
  // gathered token by token: pays for its extra copy from a mean of 12
  // assignments per expert (e.g. Mixtral at 64 tokens) and 32-token segments
  // one engine for every phase of a call: the mma.sync engine when each
  // phase's tile table fits it (its staging differs from the tcgen05 engine's)
  l.gv = use_gv(nt) && gv_fits(nt, max_segs, N2, false) && (!F || gv_fits(nt, max_segs, F, true));
  l.has_xs = F && combine && nt >= 4 && TK >= 12 * E && !l.gv;
  l.xs = take(l.has_xs ? (size_t)(Kin / 128) * TK * kChunk : 0);
  // tcgen05 engine: [CTA][2 slots][fold warp][N][32] fp32 with N >= 16; the
  // mma.sync engine: [CTA][2 slots][warp][2 MMA tiles][NT][32 lanes][4] fp32
  size_t part = (size_t)P * 2 * 8 * (8 * std::max(nt, 2)) * 32 * 4;
  if (use_gv(nt)) part = std::max(part, gv_part_bytes(nt));
  l.part1 = take(F ? part : 0);
  l.part2 = take(part);
  l.R = take(combine ? (size_t)TK * N2 * 4 : 0);
  // router logits from router_logits_kernel (T >= kRouterGemmMinT) or from
  // router_gemv_kernel (routers of more than one prep chunk): T*E floats
  l.has_rlog = true;
  l.rlog = take(l.has_rlog ? (size_t)T * E * 4 : 0);
  l.data = o;
  return l;
}

static Plan plan_at(void* ws, size_t ws_bytes, const Layout& l) {
  uint8_t* b = static_cast<uint8_t*>(ws);
  uint8_t* d = b + ((ws_bytes - l.data) & ~(size_t)255);  // data section, 256-byte aligned, at the back
  Plan p;
  p.err = reinterpret_cast<int*>(b + l.err);
  p.route_ctr = reinterpret_cast<int*>(b + l.route_ctr);
  p.ctr1 = reinterpret_cast<int*>(b + l.ctr1);
  p.ctr2 = reinterpret_cast<int*>(b + l.ctr2);
  p.rtctr = reinterpret_cast<int*>(b + l.rtctr);
  p.n_ctr = (int)((l.counters - l.ctr1) / 4);
  p.counts = reinterpret_cast<int*>(d + l.counts);
  p.n_segs = reinterpret_cast<int*>(d + l.n_segs);
  p.segs = reinterpret_cast<int4*>(d + l.segs);
  p.seg2 = l.seg2;
  p.n_segs2 = l.seg2 ? reinterpret_cast<int*>(d + l.n_segs2) : nullptr;
  p.segs2 = l.seg2 ? reinterpret_cast<int4*>(d + l.segs2) : nullptr;
  p.a_tok = reinterpret_cast<int*>(d + l.a_tok);
  p.a_tk = reinterpret_cast<int*>(d + l.a_tk);
  p.a_w = reinterpret_cast<float*>(d + l.a_w);
  p.pos = reinterpret_cast<int*>(d + l.pos);
  p.idx = reinterpret_cast<int*>(d + l.idx);
  p.wts = reinterpret_cast<float*>(d + l.wts);
  p.nval = reinterpret_cast<int*>(d + l.nval);
  p.n_assign = reinterpret_cast<int*>(d + l.n_assign);
  p.corr_x = reinterpret_cast<float*>(d + l.corr_x);
  p.corr_h = reinterpret_cast<float*>(d + l.corr_h);
  p.xp = d + l.xp;
  p.hp = d + l.hp;
  p.xs = l.has_xs ? d + l.xs : nullptr;
  p.part1 = reinterpret_cast<float*>(d + l.part1);
  p.part2 = reinterpret_cast<float*>(d + l.part2);
  p.R = reinterpret_cast<float*>(d + l.R);
  p.rlog = l.has_rlog ? reinterpret_cast<float*>(d + l.rlog) : nullptr;
  return p;
}

// The workspace must hold both sections with 256 bytes of slack for aligning
// the data section; its base must be 256-byte aligned.
static int check_ws(const void* ws, size_t bytes, const Layout& l) {
  HN_REQUIRE(((uintptr_t)ws & 255) == 0, "workspace must be 256-byte aligned");
  if (bytes < l.total() + 256) return fail(HN_ERR_WORKSPACE, "workspace too small");
  return HN_OK;
}

static int grid_p(int nt) {
  (void)nt;
  const int sms = sm_count_current();
  return sms > 0 ? sms : 148;  // one persistent engine CTA per SM
}

template <typename Tr>
static int launch_route(const RouteArgs& ra, cudaStream_t s) {
  const int64_t TK = (int64_t)ra.T * ra.K;
  RouteArgs r = ra;
  // the routing copy of the last CTA's planner (routings it plans)
  size_t sm = (size_t)(ra.H + 2 * ra.E) * 4 + (TK <= kPlanRankEntries ? (size_t)TK * 8 : 0);
  sm = std::max(sm, (size_t)(2 * ra.E) * 4);
  sm = (sm + 15) & ~(size_t)15;
  r.wbuf_off = (int)sm;
  // the GEMM's 16-byte vector loads need aligned rows of x and of the router matrix
  const bool gemm = ra.mode == ROUTE_COMPUTE && ra.T >= kRouterGemmMinT && ra.plan.rlog &&
                    ((uintptr_t)ra.x & 15) == 0 && ra.ldx % 8 == 0 && ((uintptr_t)ra.rw & 15) == 0;
  // small batches whose router matrix spans several prep chunks: logits by router_gemv_kernel
  const bool gemv = ra.mode == ROUTE_COMPUTE && !gemm && ra.plan.rlog && router_gemv_wanted(ra.H, ra.E);
  if (ra.mode == ROUTE_COMPUTE && !gemm && !gemv)
    sm += (size_t)route_chunk_experts(ra.H, ra.E, ra.rw_dtype) * ra.H * route_esize(ra.rw_dtype);
  HN_REQUIRE(sm <= 227 * 1024, "router: hidden size too large for the shared-memory plan");
  if (sm > 48 * 1024)
    HN_CUDA(cudaFuncSetAttribute(route_prep_kernel<Tr>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  r.plan_here = TK <= kPlanRankEntries;
  if (gemm && std::is_same<Tr, BF16>::value && ra.H % kRtK == 0) {
    static std::atomic<bool> attr_tc[64] = {};  // per device; setting it twice is harmless
    int dev = 0;
    HN_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !attr_tc[dev].load(std::memory_order_acquire)) {
      HN_CUDA(cudaFuncSetAttribute(router_logits_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRtSmem));
      if (dev >= 0 && dev < 64) attr_tc[dev].store(true, std::memory_order_release);
    }
    router_logits_tc_kernel<<<dim3((unsigned)((ra.T + kRtM - 1) / kRtM), (unsigned)((ra.E + kRtN - 1) / kRtN)), 256,
                              kRtSmem, s>>>(static_cast<const __nv_bfloat16*>(ra.x), ra.ldx, ra.T, ra.H, ra.E, ra.rw,
                                            ra.rw_dtype, ra.plan.rlog);
    HN_CUDA(cudaGetLastError());
    r.pre_logits = ra.plan.rlog;
  } else if (gemm) {
    router_logits_kernel<Tr><<<dim3((unsigned)((ra.T + kRgM - 1) / kRgM), (unsigned)((ra.E + kRgN - 1) / kRgN)), 256, 0, s>>>(
        ra.x, ra.ldx, ra.T, ra.H, ra.E, ra.rw, ra.rw_dtype, ra.plan.rlog);
    HN_CUDA(cudaGetLastError());
    r.pre_logits = ra.plan.rlog;
  } else if (gemv) {
    const size_t gsm = (size_t)kRgvE * ra.H * 4;
    HN_REQUIRE(gsm <= 227 * 1024, "router: hidden size too large for the router GEMV");
    if (gsm > 48 * 1024)
      HN_CUDA(cudaFuncSetAttribute(router_gemv_kernel<Tr>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gsm));
    const dim3 grid((unsigned)((ra.E + kRgvE - 1) / kRgvE), (unsigned)((ra.T + 7) / 8));
    router_gemv_kernel<Tr><<<grid, 256, gsm, s>>>(ra.x, ra.ldx, ra.T, ra.H, ra.E, ra.rw, ra.rw_dtype, ra.plan.rlog);
    HN_CUDA(cudaGetLastError());
    r.pre_logits = ra.plan.rlog;
  }
  route_prep_kernel<Tr><<<ra.T, 256, sm, s>>>(r);
  HN_CUDA(cudaGetLastError());
  if (!r.plan_here) {
    HN_REQUIRE(ra.E <= kMaxExperts, "too many experts for the plan kernel");
    PlanArgs pa{ra.T, ra.K, ra.E, ra.seg, ra.plan};
    plan_kernel<<<ra.E, 256, (size_t)ra.E * 4, s>>>(pa);
    HN_CUDA(cudaGetLastError());
  }
  if (ra.plan.xs) {
    stage_rows_kernel<<<(unsigned)((TK + 7) / 8), 256, 0, s>>>(ra.plan.a_tok, ra.plan.n_assign, (int)TK,
                                                                ra.plan.xp, ra.plan.xs,
                                                                (int64_t)(ra.H / 128) * kChunk);
    HN_CUDA(cudaGetLastError());
  }
  return HN_OK;
}

static int check_router(const hn_router_params* r, int64_t E) {
  HN_REQUIRE(r, "router params are NULL");
  HN_REQUIRE(r->kind == HN_ROUTER_SOFTMAX_TOPK || r->kind == HN_ROUTER_SIGMOID_TOPK, "unknown router kind");
  HN_REQUIRE(r->weight, "router weight is NULL");
  HN_REQUIRE(r->weight_dtype >= HN_DTYPE_F32 && r->weight_dtype <= HN_DTYPE_BF16, "bad router weight dtype");
  HN_REQUIRE(r->top_k >= 1 && r->top_k <= E && r->top_k <= kMaxTopK, "top_k out of range");
  if (r->kind == HN_ROUTER_SIGMOID_TOPK && r->n_group > 1 && r->topk_group > 0) {
    HN_REQUIRE(r->n_group <= 32 && E % r->n_group == 0, "n_group must divide the experts and be at most 32");
    HN_REQUIRE(r->topk_group <= r->n_group, "topk_group exceeds n_group");
  }
  return HN_OK;
}

// ---------------------------------------------------------------------------
// 2-D TMA descriptors.  cuTensorMapEncodeTiled is fetched from the driver at
// run time (cudaGetDriverEntryPoint) so the library needs no -lcuda.
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  // looked up once, thread-safely (a function-local static's initialiser runs once)
  static const EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(p);
    cudaGetLastError();
    return static_cast<EncodeTiledFn>(nullptr);
  }();
  return fn;
}

// uint8 matrix [rows, row_bytes] read as boxes of 128 bytes x box_rows, 128B swizzle.
static int encode_rows_map(CUtensorMap* m, const void* base, int64_t rows, int64_t row_bytes, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(HN_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (no CUDA driver)");
  HN_REQUIRE(base && ((uintptr_t)base & 15) == 0, "packed weights must be non-null and 16-byte aligned");
  HN_REQUIRE(row_bytes % 16 == 0 && rows >= 1, "bad packed weight shape");
  cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1u, 1u};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HN_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  return HN_OK;
}

// Staged token rows (uint8 [rows, row_bytes]) for the down-phase token ring:
// 128 B x box_rows boxes with 128B swizzle.
static int encode_token_map(CUtensorMap* data, const void* base, int64_t rows, int64_t row_bytes, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(HN_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (no CUDA driver)");
  HN_REQUIRE(base && ((uintptr_t)base & 255) == 0 && row_bytes % 16 == 0 && rows >= 1,
             "staged token rows must be 256-byte aligned with 16-byte multiple rows");
  cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t es[2] = {1u, 1u};
  cuuint32_t box_d[2] = {128u, (cuuint32_t)box_rows};
  CUresult r = fn(data, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box_d, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HN_ERR_CUDA, "cuTensorMapEncodeTiled (tokens) failed: " + std::to_string((int)r));
  return HN_OK;
}

static int encode_expert_maps(ExpertMaps* out, const hn_expert_ptrs& p, int64_t H, int64_t F) {
  memset(out, 0, sizeof(*out));
  int rc = HN_OK;
  if (p.gate_packed && (rc = encode_rows_map(&out->gate, p.gate_packed, F, H / 2, 128))) return rc;
  if (p.up_packed && (rc = encode_rows_map(&out->up, p.up_packed, F, H / 2, 128))) return rc;
  if (p.down_packed && (rc = encode_rows_map(&out->down, p.down_packed, H, F / 2, 256))) return rc;
  return HN_OK;
}

struct MoECall {
  const void* x;
  int64_t ldx;
  int dtype;
  int64_t T, H, F, E;
  int topk;
  int route_mode;
  const hn_router_params* router;
  const int32_t* given_idx;
  const float* given_w;
  const hn_expert_ptrs* table;
  hn_expert_ptrs single;
  const ExpertMaps* maps;  // device array [E] of tensor maps, or NULL: use single_maps
  ExpertMaps single_maps;
  void* out;
  int64_t ldo;
  int32_t* out_idx;
  float* out_w;
  float* out_logits;
  void* ws;
  size_t ws_bytes;
  cudaStream_t stream;
  bool run_experts;
  int phase;  // 0: all; 1: prep only; 2: gate/up engine only; 3: down engine only
  int64_t expected;  // caller routing: slots expected to hold an expert (0: all T*topk)
};

// Segment width of a call: from the tokens whose slots are expected to hold an
// expert (a caller-routed block of which only some slots are this call's).
static int call_nt(int64_t T, int topk, int64_t E, int64_t expected) {
  const int64_t t_eff = expected > 0 ? std::max<int64_t>(1, std::min<int64_t>(T, expected / topk)) : T;
  return pick_nt(t_eff, topk, E);
}

template <typename Tr>
static int run_moe(const MoECall& m) {
  const int64_t TK = m.T * m.topk;
  const int nt = call_nt(m.T, m.topk, m.E, m.expected);
  const int P = grid_p(nt);
  // routed calls always scale by the routing weight and combine; the identity
  // plan of a single expert MLP stores rows directly
  const bool combine = m.route_mode != ROUTE_IDENTITY;
  const Layout l = make_layout(m.T, m.H, m.E, m.topk, m.F, m.H, nt, P, combine);
  int rc0 = check_ws(m.ws, m.ws_bytes, l);
  if (rc0) return rc0;
  const Plan plan = plan_at(m.ws, m.ws_bytes, l);

  RouteArgs ra{};
  ra.x = m.x;
  ra.ldx = m.ldx;
  ra.T = (int)m.T;
  ra.H = (int)m.H;
  ra.E = (int)m.E;
  ra.K = m.topk;
  ra.mode = m.route_mode;
  if (m.router) {
    ra.kind = m.router->kind;
    ra.rw = m.router->weight;
    ra.rw_dtype = m.router->weight_dtype;
    ra.logits_act = m.router->logits_in_act_dtype;
    ra.bonus = m.router->affinity_bonus;
    ra.thr = m.router->entropy_threshold;
    ra.bias = m.router->kind == HN_ROUTER_SIGMOID_TOPK ? m.router->correction_bias : nullptr;
    ra.norm = m.router->norm_topk_prob;
    ra.scaling = m.router->routed_scaling_factor;
    ra.n_group = m.router->n_group;
    ra.topk_group = m.router->topk_group;
  }
  ra.given_idx = m.given_idx;
  ra.given_w = m.given_w;
  ra.out_idx = m.out_idx;
  ra.out_w = m.out_w;
  ra.out_logits = m.out_logits;
  ra.seg = seg_tokens(nt);
  ra.plan = plan;
  ra.gv_stage = m.run_experts && l.gv;
  // a route-only call (hn_moe_route) runs no expert phase, so nothing would
  // read the assignment-ordered copy of the tokens: skip making it
  if (!m.run_experts) ra.plan.xs = nullptr;
  int rc = HN_OK;
  if (m.phase == 0 || m.phase == 1) rc = launch_route<Tr>(ra, m.stream);
  if (rc || !m.run_experts || m.phase == 1) return rc;

  EngineArgs e1{};
  e1.K = (int)m.H;
  e1.G = (int)(m.H / 128);
  e1.N = (int)m.F;
  e1.n_rt = (int)(m.F / 128);
  e1.T = (int)m.T;
  e1.topk = m.topk;
  e1.segs = plan.segs;
  e1.n_segs = plan.n_segs;
  e1.a_tok = plan.a_tok;
  e1.a_tk = plan.a_tk;
  e1.a_w = plan.a_w;
  e1.pos = plan.pos;
  e1.table = m.table;
  e1.single = m.single;
  e1.maps = static_cast<const ExpertMaps*>(m.maps);
  if (!m.table) {
    rc = encode_expert_maps(&e1.single_maps, m.single, m.H, m.F);
    if (rc) return rc;
  }
  // gate/up tokens: gathered per token from xp, or read as consecutive rows
  // (TMA) when they are already in assignment order -- the identity plan of
  // a single expert, or xs staged by the plan kernel of a large routing
  e1.b_rstride = (m.H / 128) * kChunk;
  if (m.route_mode == ROUTE_IDENTITY) {
    e1.bsrc = plan.xp;
    e1.b_use_tok = 0;
    e1.b_rows = m.T;
  } else if (plan.xs) {
    e1.bsrc = plan.xs;
    e1.b_use_tok = 0;
    e1.b_rows = TK;
  } else {
    e1.bsrc = plan.xp;
    e1.b_use_tok = 1;
  }
  e1.hp = plan.hp;
  e1.hp_rstride = (m.F / 128) * kChunk;
  e1.part = plan.part1;
  e1.tile_ctr = plan.ctr1;
  e1.err = plan.err;
  e1.P = P;
  e1.allow_rr = nt >= 8;
  e1.max_segs = l.max_segs;
  e1.max_nt = nt;
  e1.nval = plan.nval;
  e1.tidx = plan.idx;
  e1.gv = l.gv;
  e1.corr_x = plan.corr_x;
  e1.corr_h = plan.corr_h;
  if (m.phase == 0 || m.phase == 2) rc = launch_engine<Tr, KIND_GATEUP, EPI_COMBINE>(nt, e1, m.stream);
  if (rc || m.phase == 2) return rc;

  EngineArgs e2 = e1;
  e2.K = (int)m.F;
  e2.G = (int)(m.F / 128);
  e2.N = (int)m.H;
  e2.n_rt = (int)((m.H + 255) / 256);
  e2.bsrc = plan.hp;
  e2.b_rstride = (m.F / 128) * kChunk;
  e2.b_use_tok = 0;
  e2.b_rows = TK;
  e2.R = plan.R;
  e2.out = m.out;
  e2.ldo = m.ldo;
  e2.part = plan.part2;
  e2.tile_ctr = plan.ctr2;
  e2.rt_ctr = plan.rtctr;
  e2.early = 1;
  int nt2 = nt;
  if (plan.seg2) {
    // 64-token tiles for the down phase: two accumulator stages instead of one
    e2.segs = plan.segs2;
    e2.n_segs = plan.n_segs2;
    nt2 = plan.seg2 / 8;
    e2.allow_rr = nt2 >= 8;
  }
  if (!combine) return launch_engine<Tr, KIND_DOWN, EPI_STORE>(nt2, e2, m.stream);
  // large routings: the epilogue only writes the weighted rows, one
  // bandwidth-bound pass sums them afterwards
  e2.defer_combine = TK > kPlanSmemEntries;
  rc = launch_engine<Tr, KIND_DOWN, EPI_COMBINE>(nt2, e2, m.stream);
  if (rc || !e2.defer_combine) return rc;
  const int64_t n4 = m.T * (m.H / 4);
  const int blocks = (int)std::min<int64_t>((n4 + 255) / 256, (int64_t)grid_p(nt) * 8);
  combine_kernel<Tr><<<blocks, 256, 0, m.stream>>>(plan.R, plan.idx, (int)m.T, m.topk, (int)m.H, m.out, m.ldo);
  HN_CUDA(cudaGetLastError());
  return HN_OK;
}

static int dispatch_moe(const MoECall& m) {
  if (m.dtype == HN_DTYPE_BF16) return run_moe<BF16>(m);
  if (m.dtype == HN_DTYPE_F16) return run_moe<F16>(m);
  return fail(HN_ERR_UNSUPPORTED, "activation dtype must be float16 or bfloat16");
}

static int check_dims(int64_t T, int64_t H, int64_t F, int64_t E) {
  HN_REQUIRE(T >= 1, "need at least one token");
  HN_REQUIRE(T <= (1 << 20), "too many tokens");
  HN_REQUIRE(H >= 128 && H % 128 == 0, "hidden dim must be a positive multiple of 128");
  HN_REQUIRE(F >= 128 && F % 128 == 0, "intermediate dim must be a positive multiple of 128");
  HN_REQUIRE(E >= 1 && E <= kMaxExperts, "number of experts out of range");
  HN_REQUIRE(H <= 32768 && F <= (1 << 18), "dims too large");
  return HN_OK;
}

}  // namespace hn

using namespace hn;

extern "C" {

size_t hn_moe_workspace_size(int64_t T, int64_t H, int64_t F, int64_t E, int top_k) {
  return hn_moe_experts_workspace_size_expected(T, H, F, E, top_k, 0);
}

size_t hn_moe_experts_workspace_size_expected(int64_t T, int64_t H, int64_t F, int64_t E, int top_k,
                                              int64_t expected_assignments) {
  if (T < 1 || H < 128 || F < 128 || E < 1 || top_k < 1 || expected_assignments < 0) return 0;
  const int nt = call_nt(T, top_k, E, expected_assignments);
  return make_layout(T, H, E, top_k, F, H, nt, grid_p(nt), true).total() + 256;
}

int hn_moe_layer_launches(int64_t T, int64_t H, int64_t F, int64_t E, int top_k) {
  if (T < 1 || H < 128 || F < 128 || E < 1 || top_k < 1) return 0;
  const int nt = pick_nt(T, top_k, E);
  const Layout l = make_layout(T, H, E, top_k, F, H, nt, grid_p(nt), true);
  const bool big = T * top_k > kPlanSmemEntries;
  int n = 3;  // route_prep_kernel, the gate/up engine, the down engine
  // router_logits_kernel (from kRouterGemmMinT tokens, when x and the router
  // rows are 16-byte aligned) or router_gemv_kernel (routers of more than 32 Ki weights)
  n += T >= kRouterGemmMinT || router_gemv_wanted(H, E);
  n += T * top_k > kPlanRankEntries;  // plan_kernel
  n += l.has_xs;    // stage_rows_kernel
  n += big;         // combine_kernel
  return n;
}

size_t hn_expert_mlp_workspace_size(int64_t T, int64_t H, int64_t F) {
  if (T < 1 || H < 128 || F < 128) return 0;
  const int nt = pick_nt(T, 1, 1);
  return make_layout(T, H, 1, 1, F, H, nt, grid_p(nt), false).total() + 256;
}

size_t hn_int4_linear_workspace_size(int64_t M, int64_t N, int64_t K) {
  return hn::int4_linear_workspace_nt(M, N, K, 16);
}

static int moe_layer_call(int phase, const void* x, int dtype, int64_t T, int64_t H, int64_t F, int64_t E,
                          const hn_router_params* router, const hn_expert_ptrs* experts, const void* expert_maps,
                          void* out, int32_t* topk_idx, float* topk_w, float* logits, void* workspace,
                          size_t workspace_bytes, void* stream);

int hn_moe_layer_int4(const void* x, int dtype, int64_t T, int64_t H, int64_t F, int64_t E,
                      const hn_router_params* router, const hn_expert_ptrs* experts, const void* expert_maps,
                      void* out, int32_t* topk_idx,
                      float* topk_w, float* logits, void* workspace, size_t workspace_bytes, void* stream) {
  return moe_layer_call(0, x, dtype, T, H, F, E, router, experts, expert_maps, out, topk_idx, topk_w, logits,
                        workspace, workspace_bytes, stream);
}

int hn_moe_layer_int4_phase(int phase, const void* x, int dtype, int64_t T, int64_t H, int64_t F, int64_t E,
                            const hn_router_params* router, const hn_expert_ptrs* experts, const void* expert_maps,
                            void* out, int32_t* topk_idx, float* topk_w, float* logits, void* workspace,
                            size_t workspace_bytes, void* stream) {
  HN_REQUIRE(phase >= 1 && phase <= 3, "hn_moe_layer_int4_phase: phase must be 1, 2 or 3");
  return moe_layer_call(phase, x, dtype, T, H, F, E, router, experts, expert_maps, out, topk_idx, topk_w, logits,
                        workspace, workspace_bytes, stream);
}

static int moe_layer_call(int phase, const void* x, int dtype, int64_t T, int64_t H, int64_t F, int64_t E,
                          const hn_router_params* router, const hn_expert_ptrs* experts, const void* expert_maps,
                          void* out, int32_t* topk_idx, float* topk_w, float* logits, void* workspace,
                          size_t workspace_bytes, void* stream) {
  int rc = check_dims(T, H, F, E);
  if (rc) return rc;
  rc = check_router(router, E);
  if (rc) return rc;
  HN_REQUIRE(x && experts && expert_maps && out && workspace, "hn_moe_layer_int4: null pointer");
  HN_REQUIRE(((uintptr_t)expert_maps & 63) == 0, "expert_maps must be 64-byte aligned");
  MoECall m{};
  m.x = x;
  m.ldx = H;
  m.dtype = dtype;
  m.T = T;
  m.H = H;
  m.F = F;
  m.E = E;
  m.topk = router->top_k;
  m.route_mode = ROUTE_COMPUTE;
  m.phase = phase;
  m.router = router;
  m.table = experts;
  m.maps = static_cast<const ExpertMaps*>(expert_maps);
  m.out = out;
  m.ldo = H;
  m.out_idx = topk_idx;
  m.out_w = topk_w;
  m.out_logits = logits;
  m.ws = workspace;
  m.ws_bytes = workspace_bytes;
  m.stream = (cudaStream_t)stream;
  m.run_experts = true;
  return dispatch_moe(m);
}

int hn_moe_experts_int4(const void* x, int dtype, int64_t T, int64_t H, int64_t F, int64_t E, int top_k,
                        const int32_t* topk_idx, const float* topk_w, const hn_expert_ptrs* experts,
                        const void* expert_maps, void* out,
                        void* workspace, size_t workspace_bytes, void* stream) {
  return hn_moe_experts_int4_expected(x, dtype, T, H, F, E, top_k, topk_idx, topk_w, experts, expert_maps, out, 0,
                                      workspace, workspace_bytes, stream);
}

int hn_moe_experts_int4_expected(const void* x, int dtype, int64_t T, int64_t H, int64_t F, int64_t E, int top_k,
                                 const int32_t* topk_idx, const float* topk_w, const hn_expert_ptrs* experts,
                                 const void* expert_maps, void* out, int64_t expected_assignments,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_dims(T, H, F, E);
  if (rc) return rc;
  HN_REQUIRE(expected_assignments >= 0, "expected_assignments must be >= 0");
  HN_REQUIRE(top_k >= 1 && top_k <= E && top_k <= kMaxTopK, "top_k out of range");
  HN_REQUIRE(x && topk_idx && topk_w && experts && expert_maps && out && workspace,
             "hn_moe_experts_int4: null pointer");
  HN_REQUIRE(((uintptr_t)expert_maps & 63) == 0, "expert_maps must be 64-byte aligned");
  MoECall m{};
  m.x = x;
  m.ldx = H;
  m.dtype = dtype;
  m.T = T;
  m.H = H;
  m.F = F;
  m.E = E;
  m.topk = top_k;
  m.route_mode = ROUTE_GIVEN;
  m.given_idx = topk_idx;
  m.given_w = topk_w;
  m.table = experts;
  m.maps = static_cast<const ExpertMaps*>(expert_maps);
  m.out = out;
  m.ldo = H;
  m.ws = workspace;
  m.ws_bytes = workspace_bytes;
  m.stream = (cudaStream_t)stream;
  m.run_experts = true;
  m.expected = expected_assignments;
  return dispatch_moe(m);
}

int hn_moe_route(const void* x, int dtype, int64_t T, int64_t H, int64_t E, const hn_router_params* router,
                 int32_t* topk_idx, float* topk_w, float* logits, void* workspace, size_t workspace_bytes,
                 void* stream) {
  int rc = check_dims(T, H, 128, E);
  if (rc) return rc;
  rc = check_router(router, E);
  if (rc) return rc;
  HN_REQUIRE(x && workspace, "hn_moe_route: null pointer");
  MoECall m{};
  m.x = x;
  m.ldx = H;
  m.dtype = dtype;
  m.T = T;
  m.H = H;
  m.F = 128;
  m.E = E;
  m.topk = router->top_k;
  m.route_mode = ROUTE_COMPUTE;
  m.router = router;
  m.out_idx = topk_idx;
  m.out_w = topk_w;
  m.out_logits = logits;
  m.ws = workspace;
  m.ws_bytes = workspace_bytes;
  m.stream = (cudaStream_t)stream;
  m.run_experts = false;
  return dispatch_moe(m);
}

int hn_expert_mlp_int4(const void* x, int dtype, int64_t T, int64_t H, int64_t F, const uint8_t* gate_packed,
                       const uint16_t* gate_scales, const uint8_t* up_packed, const uint16_t* up_scales,
                       const uint8_t* down_packed, const uint16_t* down_scales, int group_size, void* out,
                       void* workspace, size_t workspace_bytes, void* stream) {
  HN_REQUIRE_SUPPORTED(group_size == 128, "only group_size 128 is implemented");
  int rc = check_dims(T, H, F, 1);
  if (rc) return rc;
  HN_REQUIRE(x && gate_packed && gate_scales && up_packed && up_scales && down_packed && down_scales && out &&
                 workspace,
             "hn_expert_mlp_int4: null pointer");
  HN_REQUIRE((((uintptr_t)gate_packed | (uintptr_t)up_packed | (uintptr_t)down_packed) & 15) == 0,
             "hn_expert_mlp_int4: packed weights must be 16-byte aligned");
  MoECall m{};
  m.x = x;
  m.ldx = H;
  m.dtype = dtype;
  m.T = T;
  m.H = H;
  m.F = F;
  m.E = 1;
  m.topk = 1;
  m.route_mode = ROUTE_IDENTITY;
  m.single = hn_expert_ptrs{gate_packed, gate_scales, up_packed, up_scales, down_packed, down_scales};
  m.out = out;
  m.ldo = H;
  m.ws = workspace;
  m.ws_bytes = workspace_bytes;
  m.stream = (cudaStream_t)stream;
  m.run_experts = true;
  return dispatch_moe(m);
}

int hn_int4_linear(const void* x, int64_t ldx, int dtype, int64_t M, int64_t K, const uint8_t* w_packed,
                   const uint16_t* w_scales, int64_t N, int group_size, void* out, int64_t ldo, void* workspace,
                   size_t workspace_bytes, void* stream) {
  return hn::int4_linear_nt(x, ldx, dtype, M, K, w_packed, w_scales, N, group_size, out, ldo, workspace,
                            workspace_bytes, stream, 16);
}

}  // extern "C"

namespace hn {

size_t int4_linear_workspace_nt(int64_t M, int64_t N, int64_t K, int max_nt) {
  if (M < 1 || N < 1 || K < 128) return 0;
  const int nt = std::min(pick_nt(M, 1, 1), max_nt);
  return make_layout(M, K, 1, 1, 0, N, nt, grid_p(nt), false).total() + 256;
}

// hn_int4_linear with segments of at most 8*max_nt tokens (the static-scratch
// entry caps them at 32, which keeps its stream-K partials small).
int int4_linear_nt(const void* x, int64_t ldx, int dtype, int64_t M, int64_t K, const uint8_t* w_packed,
                   const uint16_t* w_scales, int64_t N, int group_size, void* out, int64_t ldo, void* workspace,
                   size_t workspace_bytes, void* stream, int max_nt) {
  HN_REQUIRE_SUPPORTED(group_size == 128, "only group_size 128 is implemented");
  HN_REQUIRE(M >= 1 && N >= 1 && K >= 128 && K % 128 == 0, "int4_linear: need M, N >= 1 and K a multiple of 128");
  HN_REQUIRE(M <= (1 << 20) && N <= (1 << 20) && K <= 32768, "int4_linear: dims too large");
  HN_REQUIRE(((uintptr_t)w_packed & 15) == 0, "int4_linear: packed weights must be 16-byte aligned");
  HN_REQUIRE(ldx >= K && ldo >= N, "int4_linear: bad row stride");
  HN_REQUIRE(x && w_packed && w_scales && out && workspace, "int4_linear: null pointer");
  const int nt = std::min(pick_nt(M, 1, 1), max_nt);
  const int P = grid_p(nt);
  const Layout l = make_layout(M, K, 1, 1, 0, N, nt, P, false);
  int rc0 = check_ws(workspace, workspace_bytes, l);
  if (rc0) return rc0;
  const Plan plan = plan_at(workspace, workspace_bytes, l);
  cudaStream_t s = (cudaStream_t)stream;
  RouteArgs ra{};
  ra.x = x;
  ra.ldx = ldx;
  ra.T = (int)M;
  ra.H = (int)K;
  ra.E = 1;
  ra.K = 1;
  ra.mode = ROUTE_IDENTITY;
  ra.seg = seg_tokens(nt);
  ra.plan = plan;
  ra.gv_stage = l.gv;
  EngineArgs e{};
  e.K = (int)K;
  e.G = (int)(K / 128);
  e.N = (int)N;
  e.n_rt = (int)((N + 255) / 256);
  e.T = (int)M;
  e.topk = 1;
  e.segs = plan.segs;
  e.n_segs = plan.n_segs;
  e.a_tok = plan.a_tok;
  e.a_tk = plan.a_tk;
  e.a_w = plan.a_w;
  e.pos = plan.pos;
  e.table = nullptr;
  e.single = hn_expert_ptrs{nullptr, nullptr, nullptr, nullptr, w_packed, w_scales};
  e.maps = nullptr;
  {
    const int mrc = encode_rows_map(&e.single_maps.down, w_packed, N, K / 2, 256);
    if (mrc) return mrc;
  }
  e.bsrc = plan.xp;
  e.b_rstride = (K / 128) * kChunk;
  e.b_use_tok = 1;
  e.b_rows = M;
  e.out = out;
  e.ldo = ldo;
  e.part = plan.part2;
  e.tile_ctr = plan.ctr2;
  e.rt_ctr = plan.rtctr;
  e.err = plan.err;
  e.P = P;
  e.allow_rr = nt >= 8;
  e.max_segs = l.max_segs;
  e.max_nt = nt;
  e.nval = plan.nval;
  e.tidx = plan.idx;
  e.gv = l.gv;
  e.corr_x = plan.corr_x;
  e.corr_h = plan.corr_h;
  int rc;
  if (dtype == HN_DTYPE_BF16) {
    rc = launch_route<BF16>(ra, s);
    if (!rc) rc = launch_engine<BF16, KIND_DOWN, EPI_STORE>(nt, e, s);
  } else if (dtype == HN_DTYPE_F16) {
    rc = launch_route<F16>(ra, s);
    if (!rc) rc = launch_engine<F16, KIND_DOWN, EPI_STORE>(nt, e, s);
  } else {
    return fail(HN_ERR_UNSUPPORTED, "int4_linear: activation dtype must be float16 or bfloat16");
  }
  return rc;
}

}  // namespace hn

extern "C" {

size_t hn_expert_maps_bytes(void) { return sizeof(ExpertMaps); }

int hn_expert_maps_encode(const hn_expert_ptrs* host_table, int64_t E, int64_t H, int64_t F, void* host_out) {
  HN_REQUIRE(host_table && host_out, "hn_expert_maps_encode: null pointer");
  HN_REQUIRE(E >= 1 && H >= 128 && H % 128 == 0 && F >= 128 && F % 128 == 0, "hn_expert_maps_encode: bad shape");
  HN_REQUIRE(((uintptr_t)host_out & 63) == 0, "hn_expert_maps_encode: output must be 64-byte aligned");
  ExpertMaps* out = static_cast<ExpertMaps*>(host_out);
  for (int64_t e = 0; e < E; ++e) {
    const int rc = encode_expert_maps(&out[e], host_table[e], H, F);
    if (rc) return rc;
  }
  return HN_OK;
}

int hn_set_decode_engine(int engine) {
  if (engine != HN_ENGINE_AUTO && engine != HN_ENGINE_TCGEN05) {
    fail(HN_ERR_INVALID, "hn_set_decode_engine: unknown engine " + std::to_string(engine));
    return -1;
  }
  return g_decode_engine.exchange(engine);
}

int hn_workspace_error(const void* workspace, size_t workspace_bytes, int* error_code, void* stream) {
  HN_REQUIRE(workspace && error_code && workspace_bytes >= 4, "hn_workspace_error: bad arguments");
  HN_CUDA(cudaMemcpyAsync(error_code, workspace, 4, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
  HN_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  if (*error_code != 0) HN_CUDA(cudaMemsetAsync(const_cast<void*>(workspace), 0, 4, (cudaStream_t)stream));
  return HN_OK;
}

}  // extern "C"
