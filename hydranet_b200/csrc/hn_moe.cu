// INT4 mixture-of-experts decode path for sm_100a.
//
//   route_prep_kernel   one CTA per token: router logits / top-k / weights
//                       (or caller-given routing), the token's activations
//                       staged into MMA-fragment order, and -- in the last CTA
//                       to finish -- the dispatch plan (per-expert token lists
//                       cut into segments of at most 8*NT tokens).
//   engine_kernel       persistent grouped INT4 GEMV/GEMM over (weight-row
//                       tile x segment) tiles, k-split "stream-K" style so every
//                       CTA streams the same number of 128-wide k-groups.
//                       KIND_GATEUP: gate+up rows together, SiLU(gate)*up in
//                       the epilogue, written as the next phase's operand.
//                       KIND_DOWN: down projection; EPI_COMBINE scales by the
//                       routing weight and sums the top-k choices per token,
//                       EPI_STORE writes rows straight to the output.
//
// Weight tiles are streamed by per-thread cp.async into a per-warp ring; the
// activation chunk of each k-group (shared by all warps) arrives by TMA bulk
// copies issued by a producer warp and tracked by mbarriers.  The MMA is
// mma.sync m16n8k16 with the WEIGHTS as the 16-row A operand and tokens as
// the 8-column B operand.
//
// Dequantisation without subtraction: a nibble n OR-ed into the mantissa of
// 2^e gives 2^e + n exactly (bf16: 128+n for a low nibble, 128+8n for a nibble
// in bits 3..6; fp16: 1024+n / 1024+16n).  The B operand of odd k is
// pre-divided by 8 (bf16) or 16 (fp16), so for every k the MMA computes
// (n - 8 + c_k) * x_k with c_k = 136 / 24 (bf16) or 1032 / 72 (fp16).  The
// constant part, C = sum_k c_k x_k per (token, group), is computed once when
// the activations are staged and subtracted before the group scale is
// applied: acc += scale[row, group] * (mma_partial - C).  Weights therefore
// enter the MMA as the exact integers n - 8, and the scale multiplies in fp32.
#include <algorithm>
#include <cstring>
#include <string>
#include <cuda.h>

#include "common.cuh"

namespace hn {

constexpr int kChunk = 272;  // bytes per (token, k-group): 16 B correction unit + 16 units of 16 B
constexpr int kMaxExperts = 1024;
constexpr int kMaxTopK = 32;
constexpr int kPlanSmemEntries = 4096;  // routing entries the plan builder copies into shared memory

enum { KIND_GATEUP = 0, KIND_DOWN = 1 };
enum { EPI_COMBINE = 0, EPI_STORE = 1 };
enum { ROUTE_COMPUTE = 0, ROUTE_GIVEN = 1, ROUTE_IDENTITY = 2 };

struct Plan {
  int* err;
  int* route_ctr;
  int* counts;   // [E]
  int* n_segs;   // [1]
  int4* segs;    // [max_segs] {expert, first assignment, tokens, 0}
  int* a_tok;    // [T*K] token of assignment p
  float* a_w;    // [T*K] routing weight of assignment p
  int* pos;      // [T*K] assignment index of (t, k)
  int* idx;      // [T*K] top-k expert ids
  float* wts;    // [T*K] top-k weights (rounded to the activation dtype)
  uint8_t* xp;   // [T][K_in/128][kChunk]    staged activations (token-major)
  uint8_t* hp;   // [T*K][F/128][kChunk]     staged SiLU(gate)*up (assignment-major)
  float* part1;  // stream-K partial tiles, phase 1
  float* part2;  // stream-K partial tiles, phase 2
  float* R;      // [T*K][H] weighted expert outputs (EPI_COMBINE)
  int* ctr1;     // per phase-1 tile arrival counters
  int* ctr2;     // per phase-2 tile arrival counters
  int* rtctr;    // per output row-tile segment counters
  int n_ctr;     // words from ctr1 to the end of the counter section (zeroed by the prep kernel)
};

__host__ __device__ constexpr int seg_tokens(int nt) { return 8 * nt; }

// ---------------------------------------------------------------------------
// Activation staging.  For k-group g and token t a 272-byte chunk holds the
// correction unit followed by 16 data units of 16 bytes.
// Data unit c (at byte 16 + 16c) covers x[128*g + 8*c + i], i = 0..7, packed
// as bf16/f16 pairs
//   { (x0, x4), (x2, x6), (x1*s, x5*s), (x3*s, x7*s) }   (s = odd-k scale)
// i.e. logical k 8c..8c+7 of the MMA, matching the TMEM columns the weight
// dequantiser writes for the same 8 nibbles (dequant_word).  A unit is one
// 16-byte row of a K-major core matrix of the tensor-core B operand.
// The correction unit (byte 0) holds C = sum_k c_k x_k of the group as three
// bf16 values whose sum is exactly the fp32 C, then five bf16 zeros; the
// engine multiplies it by a constant A column of -1s in the same MMA chain,
// so the accumulator already holds sum_k (n_k - 8) x_k.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 correction_unit(float c) {
  const __nv_bfloat16 h0 = __float2bfloat16_rn(c);
  const float r1 = c - __bfloat162float(h0);  // exact
  const __nv_bfloat16 h1 = __float2bfloat16_rn(r1);
  const float r2 = r1 - __bfloat162float(h1);  // exact, at most 8 significant bits
  const __nv_bfloat16 h2 = __float2bfloat16_rn(r2);
  uint4 u;
  u.x = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
  u.y = (uint32_t)__bfloat16_as_ushort(h2);
  u.z = 0u;
  u.w = 0u;
  return u;
}
template <typename Tr>
__device__ __forceinline__ void pack_unit(const float (&v)[8], uint4& out, float& cpart) {
  const float s = Tr::kOddScale;
  uint4 u;
  u.x = Tr::pack(v[0], v[4]);
  u.y = Tr::pack(v[2], v[6]);
  u.z = Tr::pack(v[1] * s, v[5] * s);
  u.w = Tr::pack(v[3] * s, v[7] * s);
  // effective odd values are what the MMA actually sees (times 1/s, exact)
  const typename Tr::T2* oz = reinterpret_cast<const typename Tr::T2*>(&u.z);
  const typename Tr::T2* ow = reinterpret_cast<const typename Tr::T2*>(&u.w);
  float2 fz = make_float2(Tr::to_f(oz->x), Tr::to_f(oz->y));
  float2 fw = make_float2(Tr::to_f(ow->x), Tr::to_f(ow->y));
  const float inv = 1.0f / s;
  cpart = Tr::kCorrEven * (((v[0] + v[2]) + v[4]) + v[6]) + Tr::kCorrOdd * inv * (((fz.x + fw.x) + fz.y) + fw.y);
  out = u;
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
  const int32_t* given_idx;
  const float* given_w;
  int32_t* out_idx;
  float* out_w;
  float* out_logits;
  int seg;
  int wbuf_off;  // byte offset of the router-weight chunk in dynamic shared memory
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
  float* cpart = lg + a.E;         // [H/8]
  float* scs = cpart + a.H / 8;    // [E] selection scores
  // plan copies of the routing follow scs (see the plan section); the router
  // weight chunk sits at the end of the dynamic shared memory
  __shared__ int s_last;
  __shared__ int s_idx[kMaxTopK];
  __shared__ float s_w[kMaxTopK];
  __shared__ __align__(8) uint64_t s_wbar;
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const typename Tr::T* xrow = reinterpret_cast<const typename Tr::T*>(a.x) + (int64_t)t * a.ldx;
  const int esz = route_esize(a.rw_dtype);
  const int CE = route_chunk_experts(a.H, a.E, a.rw_dtype);
  const bool bulk = a.mode == ROUTE_COMPUTE && (reinterpret_cast<uintptr_t>(a.rw) & 15) == 0;
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

  // 1. staged activations + per-group correction C
  const int units = a.H / 8;
  for (int u = tid; u < units; u += 256) {
    const int g = u >> 4, ch = u & 15;
    const int k0 = g * 128 + ch * 8;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = xs[k0 + i];
    uint4 packed;
    float cp;
    pack_unit<Tr>(v, packed, cp);
    *reinterpret_cast<uint4*>(a.plan.xp + ((int64_t)t * (a.H / 128) + g) * kChunk + 16 + ch * 16) = packed;
    cpart[u] = cp;
  }
  __syncthreads();
  for (int g = tid; g < a.H / 128; g += 256) {
    float c = 0.f;
    for (int u = 0; u < 16; ++u) c += cpart[g * 16 + u];
    *reinterpret_cast<uint4*>(a.plan.xp + ((int64_t)t * (a.H / 128) + g) * kChunk) = correction_unit(c);
  }

  // 2. routing for this token
  if (a.mode == ROUTE_COMPUTE) {
    // router logits, one warp per expert row of the chunk in shared memory
    for (int c0 = 0; c0 < a.E; c0 += CE) {
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
          // sigmoid scores of the selected experts, unbiased (model/glm4.py:300-307)
          float sum = 0.f;
          for (int k = 0; k < a.K; ++k) {
            s_w[k] = 1.0f / (1.0f + expf(-lg[s_idx[k]]));
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
        int e = a.given_idx[(int64_t)t * a.K + k];
        if (e < 0 || e >= a.E) {
          atomicExch(a.plan.err, DEV_ERR_BAD_INDEX);
          e = 0;
        }
        s_idx[k] = e;
        s_w[k] = a.given_w[(int64_t)t * a.K + k];
      } else {
        s_idx[k] = 0;
        s_w[k] = 1.0f;
      }
    }
  }
  __syncthreads();
  if (tid < a.K) {
    a.plan.idx[(int64_t)t * a.K + tid] = s_idx[tid];
    a.plan.wts[(int64_t)t * a.K + tid] = s_w[tid];
    if (a.out_idx) a.out_idx[(int64_t)t * a.K + tid] = s_idx[tid];
    if (a.out_w) a.out_w[(int64_t)t * a.K + tid] = s_w[tid];
  }

  // 3. the last CTA to finish builds the plan
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicAdd(a.plan.route_ctr, 1) == a.T - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  int* cnt = reinterpret_cast<int*>(rsm);  // reuse (>= E ints available: H >= 128 floats)
  int* off = cnt + a.E;
  const int TK = a.T * a.K;
  // every token's routing, read once into shared memory when it fits
  const bool in_smem = TK <= kPlanSmemEntries;
  int* pidx = reinterpret_cast<int*>(rsm + a.H + 2 * a.E + a.H / 8);
  float* pwts = reinterpret_cast<float*>(pidx + (in_smem ? TK : 0));
  for (int e = tid; e < a.E; e += 256) cnt[e] = 0;
  if (in_smem)
    for (int i = tid; i < TK; i += 256) {
      pidx[i] = __ldcg(a.plan.idx + i);
      pwts[i] = __ldcg(a.plan.wts + i);
    }
  __syncthreads();
  for (int i = tid; i < TK; i += 256) atomicAdd(&cnt[in_smem ? pidx[i] : __ldcg(a.plan.idx + i)], 1);
  __syncthreads();
  if (tid == 0) {
    int o = 0, ns = 0;
    for (int e = 0; e < a.E; ++e) {
      off[e] = o;
      const int m = cnt[e];
      for (int j = 0; j < m; j += a.seg) a.plan.segs[ns++] = make_int4(e, o + j, min(a.seg, m - j), 0);
      o += m;
      a.plan.counts[e] = m;
    }
    *a.plan.n_segs = ns;
    *a.plan.route_ctr = 0;
  }
  __syncthreads();
  // per-expert assignment order: by token, then by top-k slot (ballot over 32
  // tokens at a time); a token listing the same expert twice gets two slots
  for (int e = warp; e < a.E; e += 8) {
    int base = 0;
    for (int t0 = 0; t0 < a.T; t0 += 32) {
      const int tt = t0 + lane;
      for (int k = 0; k < a.K; ++k) {
        const int64_t at = (int64_t)tt * a.K + k;
        const bool hit = tt < a.T && (in_smem ? pidx[at] : __ldcg(a.plan.idx + at)) == e;
        const unsigned bal = __ballot_sync(0xffffffffu, hit);
        if (hit) {
          const int p = off[e] + base + __popc(bal & ((1u << lane) - 1u));
          a.plan.pos[(int64_t)tt * a.K + k] = p;
          a.plan.a_tok[p] = tt;
          a.plan.a_w[p] = in_smem ? pwts[at] : __ldcg(a.plan.wts + at);
        }
        base += __popc(bal);
      }
    }
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
  ShiftMul shm;  // 2^31, 2^24, 2^23 (see dequant_word_fma)
  int K;     // reduction length (multiple of 128)
  int G;     // K / 128
  int N;     // weight rows
  int n_rt;  // row tiles
  int T, topk;
  const int4* segs;
  const int* n_segs;
  const int* a_tok;
  const float* a_w;
  const int* pos;
  const hn_expert_ptrs* table;
  hn_expert_ptrs single;
  const ExpertMaps* maps;  // device array [E] of tensor maps, or NULL: use single_maps
  ExpertMaps single_maps;
  const uint8_t* bsrc;  // staged tokens, [row][group][kChunk]
  int64_t b_rstride;    // bytes per staged row (groups * kChunk)
  int64_t b_rows;       // staged rows (KIND_DOWN tensor maps)
  int b_use_tok;
  CUtensorMap bmap;     // KIND_DOWN: bsrc as uint8 [rows, b_rstride], 128 B x N boxes, 128B swizzle
  CUtensorMap cmap;     // KIND_DOWN: same tensor, 16 B x N boxes (correction units), no swizzle
  uint8_t* hp;
  int64_t hp_rstride;
  float* R;
  void* out;
  int64_t ldo;
  float* part;
  int* tile_ctr;
  int* rt_ctr;
  int* err;
  int P;
};

template <int KIND>
struct TileMap {
  // GATEUP tiles are segment-major, DOWN tiles row-tile-major.
  static __device__ __forceinline__ void split(int tile, int n_rt, int n_segs, int& seg, int& rt) {
    if (KIND == KIND_GATEUP) {
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
//     (the 16-byte unit u of token row r at u ^ (r & 7)): half h holds data
//     units 8h..8h+7 (logical k 64h..64h+63) of the k-group; the K-major
//     SW128 operand of MMA k-step s starts at half s/4, byte 32*(s%4), with
//     SBO = 1024 bytes (8 token rows);
//   correction ring: SB stages of [N tokens][16 B] correction units followed
//     by N x 16 zero bytes (the second K half of the correction step);
//   htile / cpart: epilogue staging.
template <int N, int ST, int SB>
struct TcSmem {
  static constexpr int kHdr = 1024;
  static constexpr int kWStage = 32768;
  static constexpr int kW = ST * kWStage;
  static constexpr int kBStage = 2 * N * 128;  // a multiple of 1024: stages stay swizzle-aligned
  static constexpr int kB = SB * kBStage;
  static constexpr int kCStage = 2 * N * 16;
  static constexpr int kC = SB * kCStage;
  static constexpr int kH = 128 * (N + 1) * 4 + N * 16 * 4;
  static constexpr int kTotal = 1024 /* alignment slack */ + kHdr + kW + kB + kC + kH;
  static_assert(kBStage % 1024 == 0, "token stages must stay 1024-byte aligned");
};

// TMEM columns: SA weight stages of {A0, A1} x 64 columns (128 k as bf16/f16
// pairs) from column 0, SD accumulator stages of {A0, A1} x N fp32 columns
// after them, and the 8-column constant A block of the correction step.
// N = 16: 3 x 128 + 3 x 32 + 8; N = 32: 2 x 128 + 3 x 64 + 8.
constexpr int kTmemCols = 512;
// Warp roles (a warp runs on SMSP warp % 4): dequant warps, fold warps, then
// one role warp on each SMSP.
constexpr int kDeqWarps = 8;
constexpr int kFoldWarps = 8;
constexpr int kTokWarp = 16;   // token producer (SMSP 0)
constexpr int kMmaWarp0 = 17;  // MMA issuer of matrix 0 (SMSP 1), allocates TMEM
constexpr int kWgtWarp = 18;   // weight producer (SMSP 2)
constexpr int kMmaWarp1 = 19;  // MMA issuer of matrix 1 (SMSP 3)
constexpr int kTcThreads = 20 * 32;
template <int N>
struct TmemPlan {
  static constexpr int SA = (N == 16) ? 3 : 2;
  static constexpr int SD = 3;
  static constexpr int kD0 = SA * 128;
  static constexpr int kCorr = kD0 + SD * 2 * N;
  static_assert(kCorr + 8 <= kTmemCols, "TMEM plan exceeds 512 columns");
};

// Per-thread view of the tile: thread (matrix j, row r).
struct RowView {
  int seg, rt, m, p0, e;
  const uint16_t* s;  // this thread's scale row (+ group)
};

template <int KIND>
__device__ __forceinline__ void load_rowview(const EngineArgs& a, int tile, int n_segs, int j, int r, RowView& v) {
  TileMap<KIND>::split(tile, a.n_rt, n_segs, v.seg, v.rt);
  const int4 sg = a.segs[v.seg];
  v.m = sg.z;
  v.p0 = sg.y;
  v.e = sg.x;
  const hn_expert_ptrs ep = a.table ? a.table[sg.x] : a.single;
  const uint16_t* S;
  int row;
  if (KIND == KIND_GATEUP) {
    S = j ? ep.up_scales : ep.gate_scales;
    row = v.rt * 128 + r;
  } else {
    S = ep.down_scales;
    row = v.rt * 256 + j * 128 + r;
  }
  row = min(row, a.N - 1);  // rows past N read row N-1's scales and are never stored
  v.s = S + (int64_t)row * a.G;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
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

// Persistent grouped GEMV on the 5th-generation tensor cores.
//
// Work items are (tile, k-group pair); CTA c owns items [c*NI/P, (c+1)*NI/P)
// (stream-K), so every CTA streams the same number of weight bytes.  Warp
// roles (a warp runs on SMSP warp % 4):
//   warps 0-7    dequant warps: warp w dequantises matrix j = w >> 2 for TMEM
//                lanes 32*(w&3).. (its 32 rows), all 128 k of each group, into
//                the A stage;
//   warps 8-15   fold warps: warp w owns the same rows of matrix (w >> 2) & 1
//                and folds each group's accumulator into fp32 registers,
//                acc += scale[row, group] * D, for all N tokens; they also run
//                the stream-K fix-up and the epilogue;
//   warp 16      token producer: cp.async of each group's token units;
//   warps 17, 19 MMA issuers for matrix 0 and matrix 1: per k-group eight
//                K=16 steps with the dequantised weights (TMEM) as A and the
//                tokens (SMEM) as B, then the correction step, into one TMEM
//                accumulator stage; the two matrices use separate columns, so
//                two warps on two SMSPs can issue them independently;
//   warp 18      weight producer: one 32 KB 2-D TMA box pair per item.
// Dequantising and folding are separate warps so that a warp never waits for
// a TMEM store and a TMEM load of two different groups one after the other.
// All hand-offs are mbarriers with bounded waits.
template <typename Tr, int N, int KIND, int EPI, int ST, int SB>
__global__ void __launch_bounds__(kTcThreads, 1) tc_engine_kernel(const __grid_constant__ EngineArgs a) {
  using L = TcSmem<N, ST, SB>;
  constexpr int SA = TmemPlan<N>::SA, SD = TmemPlan<N>::SD, D0 = TmemPlan<N>::kD0, CORR = TmemPlan<N>::kCorr;
  // The token producer signals stage k after issuing group k + LOOK (its
  // copies then had LOOK groups of time to land); issuing k + LOOK needs the
  // MMA of k + LOOK - SB to be done, so SB - LOOK groups of slack remain.
  constexpr int LOOK = 3;
  static_assert(LOOK >= 1 && SB - LOOK >= 4 && SA <= 4 && SD <= 4 && SB <= 16 && ST <= 8, "stage counts");
  constexpr uint32_t IDESC = umma_idesc<Tr, 128, N>();
  constexpr uint32_t IDESC_CORR = umma_idesc<BF16, 128, N>();
  constexpr uint32_t kDescHiSW128 = (1024u >> 4) | (1u << 14) | (2u << 29);  // SBO 1024 B, version 1, SWIZZLE_128B
  constexpr uint32_t kDescHiCorr = (128u >> 4) | (1u << 14);                 // SBO 128 B, version 1, no swizzle
  constexpr int kFoldThreads = kFoldWarps * 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint64_t* a_full = bars;        // [SA][2] dequant warps of matrix j -> its MMA warp
  uint64_t* a_empty = bars + 8;   // [SA][2] MMA commit (matrix j) -> its dequant warps
  uint64_t* d_full = bars + 16;   // [SD] both MMA warps' commits -> fold warps
  uint64_t* d_empty = bars + 20;  // [SD] fold warps -> MMA warps
  uint64_t* b_full = bars + 24;   // [SB] token producer -> MMA warps
  uint64_t* b_empty = bars + 40;  // [SB] both MMA warps' commits -> token producer
  uint64_t* w_full = bars + 56;   // [ST] weight TMA -> dequant warps
  uint64_t* w_empty = bars + 64;  // [ST] dequant warps -> weight producer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 72);
  int* bcast = reinterpret_cast<int*>(bars + 73);
  uint8_t* wst = smem + L::kHdr;
  uint8_t* bst = wst + L::kW;
  uint8_t* cst = bst + L::kB;
  float* htile = reinterpret_cast<float*>(cst + L::kC);
  float* cpart = htile + 128 * (N + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_segs = *a.n_segs;
  const int n_tiles = a.n_rt * n_segs;
  const int GP = (a.G + 1) >> 1;  // k-group pairs per tile
  const int64_t NI = (int64_t)n_tiles * GP;
  if (NI <= 0) return;
  const int64_t P = min((int64_t)a.P, NI);
  const int64_t c = blockIdx.x;
  if (c >= P) return;
  const int64_t b0 = c * NI / P, b1 = (c + 1) * NI / P;
  auto cta_of = [&](int64_t i) -> int64_t { return ((i + 1) * P - 1) / NI; };
  auto begin_of = [&](int64_t cc) -> int64_t { return cc * NI / P; };
  // Items are walked with 32-bit counters: (tile0, gp0) is the first item.
  const int n_items = (int)(b1 - b0);
  const int tile0 = (int)(b0 / GP), gp0 = (int)(b0 - (int64_t)tile0 * GP);

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2 * SA; ++s) {
      mbar_init(smem_u32(&a_full[s]), kDeqWarps / 2);  // the dequant warps of one matrix
      mbar_init(smem_u32(&a_empty[s]), 1);
    }
    for (int s = 0; s < SD; ++s) {
      mbar_init(smem_u32(&d_full[s]), 2);
      mbar_init(smem_u32(&d_empty[s]), kFoldWarps);
    }
    for (int s = 0; s < SB; ++s) {
      // KIND_DOWN fills a stage with TMA (one arrival + bytes), KIND_GATEUP
      // with per-lane cp.async (one arrival per lane)
      mbar_init(smem_u32(&b_full[s]), KIND == KIND_DOWN ? 1 : 32);
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
  // zero halves of the correction ring (read by the correction MMA, never written)
  for (int i = threadIdx.x; i < SB * N; i += kTcThreads)
    *reinterpret_cast<uint4*>(cst + (i / N) * L::kCStage + N * 16 + (i % N) * 16) = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == kWgtWarp) {
    // ------------------------- weight producer (2-D TMA) -------------------------
    if (lane == 0) {
      Ring<ST> rw;
      int tile = tile0, gp = gp0;
      for (int i = 0; i < n_items; ++i) {
        int seg, rt;
        TileMap<KIND>::split(tile, a.n_rt, n_segs, seg, rt);
        const int e = a.segs[seg].x;
        const ExpertMaps* em = a.maps ? a.maps + e : &a.single_maps;
        mbar_wait(smem_u32(&w_empty[rw.idx]), rw.phase ^ 1u, a.err);
        const uint32_t bar = smem_u32(&w_full[rw.idx]);
        mbar_arrive_expect_tx(bar, L::kWStage);
        const uint32_t dst = smem_u32(wst + rw.idx * L::kWStage);
        if (KIND == KIND_GATEUP) {
          tma_load_2d(dst, &em->gate, gp * 128, rt * 128, bar);
          tma_load_2d(dst + 16384, &em->up, gp * 128, rt * 128, bar);
        } else {
          tma_load_2d(dst, &em->down, gp * 128, rt * 256, bar);
        }
        rw.next();
        if (++gp == GP) {
          gp = 0;
          ++tile;
        }
      }
    }
    __syncwarp();
  } else if (warp == kTokWarp) {
    // ------------------------- token producer -------------------------
    // Lane l copies the 17 units of token l of the segment; a stage is
    // signalled (after its copies landed and a proxy fence) LOOK stages later.
    int k = 0, tile = tile0, gp = gp0;
    if (KIND == KIND_DOWN) {
      // Rows of a segment are consecutive (assignment order): each k-group is
      // three TMA boxes of N rows (two 128-byte data halves, 128B swizzle, and
      // the correction units); rows past the end are zero-filled.
      Ring<SB> rb;
      if (lane == 0) {
        for (int i = 0; i < n_items; ++i) {
          int seg, rt;
          TileMap<KIND>::split(tile, a.n_rt, n_segs, seg, rt);
          const int row0 = a.segs[seg].y;
          const int ng = min(2, a.G - 2 * gp);
          for (int gi = 0; gi < ng; ++gi, ++k) {
            const int grp = 2 * gp + gi;
            mbar_wait(smem_u32(&b_empty[rb.idx]), rb.phase ^ 1u, a.err);
            const uint32_t bar = smem_u32(&b_full[rb.idx]);
            mbar_arrive_expect_tx(bar, (uint32_t)(2 * N * 128 + N * 16));
            const uint32_t dst = smem_u32(bst + rb.idx * L::kBStage);
            tma_load_2d(dst, &a.bmap, grp * kChunk + 16, row0, bar);
            tma_load_2d(dst + N * 128, &a.bmap, grp * kChunk + 16 + 128, row0, bar);
            tma_load_2d(smem_u32(cst + rb.idx * L::kCStage), &a.cmap, grp * kChunk, row0, bar);
            rb.next();
          }
          if (++gp == GP) {
            gp = 0;
            ++tile;
          }
        }
      }
      __syncwarp();
    } else {
      // Gathered tokens: lane l copies token l of the segment with cp.async
      // into the swizzled rows; a stage is signalled (after its copies landed
      // and a proxy fence) LOOK groups later.
      Ring<SB> rb, rs;  // rb: stage being filled; rs: next stage to signal (LOOK behind)
      for (int i = 0; i < n_items; ++i) {
        int seg, rt;
        TileMap<KIND>::split(tile, a.n_rt, n_segs, seg, rt);
        const int4 sg = a.segs[seg];
        const uint8_t* src_tok = nullptr;
        if (lane < sg.z) {
          const int row = a.b_use_tok ? a.a_tok[sg.y + lane] : sg.y + lane;
          src_tok = a.bsrc + (int64_t)row * a.b_rstride;
        }
        const int ng = min(2, a.G - 2 * gp);
        for (int gi = 0; gi < ng; ++gi, ++k) {
          const int grp = 2 * gp + gi;
          mbar_wait(smem_u32(&b_empty[rb.idx]), rb.phase ^ 1u, a.err);
          if (src_tok) {
            const uint32_t dst = smem_u32(bst + rb.idx * L::kBStage + lane * 128);
            const uint8_t* src = src_tok + (int64_t)grp * kChunk;
            const int sw = lane & 7;
#pragma unroll
            for (int u = 0; u < 16; ++u)
              cp_async16(dst + (u >> 3) * (N * 128) + (((u & 7) ^ sw) << 4), src + 16 + u * 16);
            cp_async16(smem_u32(cst + rb.idx * L::kCStage + lane * 16), src);
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
          ++tile;
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
    Ring<SD> rd;
    Ring<SB> rb;
    int gp = gp0;
    for (int i = 0; i < n_items; ++i) {
      const int ng = min(2, a.G - 2 * gp);
      for (int gi = 0; gi < ng; ++gi) {
        const int sa = ra.idx, sd = rd.idx, sb = rb.idx;
        mbar_wait(smem_u32(&b_full[sb]), rb.phase, a.err);
        mbar_wait(smem_u32(&d_empty[sd]), rd.phase ^ 1u, a.err);
        mbar_wait(smem_u32(&a_full[2 * sa + mj]), ra.phase, a.err);
        tc_fence_after();
        // B descriptors (32-bit halves): data = K-major SW128 tile (start,
        // LBO ignored = 1, SBO 1024 B, layout SWIZZLE_128B); correction = K-major
        // no-swizzle tile (LBO = N*16 B to the zero half, SBO 128 B).
        const uint32_t b_lo = ((smem_u32(bst + sb * L::kBStage) >> 4) & 0x3FFFu) | (1u << 16);
        const uint32_t c_lo = ((smem_u32(cst + sb * L::kCStage) >> 4) & 0x3FFFu) | (uint32_t)(N << 16);
        umma_group9_sw128<N>(tbase + D0 + sd * 2 * N + mj * N, tbase + sa * 128 + mj * 64, b_lo, kDescHiSW128,
                             IDESC, c_lo, kDescHiCorr, tbase + CORR, IDESC_CORR);
        umma_commit_elect(smem_u32(&a_empty[2 * sa + mj]));
        umma_commit_elect(smem_u32(&b_empty[sb]));
        umma_commit_elect(smem_u32(&d_full[sd]));
        ra.next();
        rd.next();
        rb.next();
      }
      if (++gp == GP) gp = 0;
    }
    __syncwarp();
  } else if (warp < kDeqWarps) {
    // ------------------------------ dequant warps ------------------------------
    const int q = warp & 3, j = warp >> 2, r = q * 32 + lane;
    const uint32_t tlane = tbase + ((uint32_t)(q * 32) << 16);
    const uint8_t* wrow = wst + (j * 128 + r) * 128;  // this thread's row inside a weight stage
    const ShiftMul shm = a.shm;
    const int swz = r & 7;
    if (j == 0) {
      // constant A block of the correction step: k0..k2 = -1 (bf16), rest 0
      uint32_t cv8[8] = {0xBF80BF80u, 0x0000BF80u, 0u, 0u, 0u, 0u, 0u, 0u};
      tmem_st8(tlane + CORR, cv8);
      tc_wait_st();
      tc_fence_before();
    }
    // Each group: (at an item start) wait for the weight stage, load this
    // thread's 64 bytes of the group, wait for the A stage, dequantise into
    // TMEM, signal.  Nothing here waits on a later item, so a group's signal
    // never depends on the next weight stage having landed.
    Ring<ST> rw;
    Ring<SA> ra;
    int gp = gp0;
#pragma unroll 1
    for (int it = 0; it < n_items; ++it) {
      const int ng = min(2, a.G - 2 * gp);
      const int ws = rw.idx;
      mbar_wait(smem_u32(&w_full[ws]), rw.phase, a.err);
      const uint8_t* wrow_p = wrow + ws * L::kWStage;
#pragma unroll 1
      for (int gi = 0; gi < ng; ++gi) {
        const int sa = ra.idx;
        uint4 W[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) W[i] = *reinterpret_cast<const uint4*>(wrow_p + (((gi * 4 + i) ^ swz) << 4));
        mbar_wait(smem_u32(&a_empty[2 * sa + j]), ra.phase ^ 1u, a.err);
        tc_fence_after();
        const uint32_t acol = tlane + sa * 128 + j * 64;
        {
          uint32_t o0[16], o1[16];
          dequant_word_fma<Tr>(W[0].x, o0 + 0, shm);
          dequant_word_fma<Tr>(W[0].y, o0 + 4, shm);
          dequant_word_fma<Tr>(W[0].z, o0 + 8, shm);
          dequant_word_fma<Tr>(W[0].w, o0 + 12, shm);
          dequant_word_fma<Tr>(W[1].x, o1 + 0, shm);
          dequant_word_fma<Tr>(W[1].y, o1 + 4, shm);
          dequant_word_fma<Tr>(W[1].z, o1 + 8, shm);
          dequant_word_fma<Tr>(W[1].w, o1 + 12, shm);
          tmem_st16(acol, o0);
          tmem_st16(acol + 16, o1);
        }
        {
          uint32_t o2[16], o3[16];
          dequant_word_fma<Tr>(W[2].x, o2 + 0, shm);
          dequant_word_fma<Tr>(W[2].y, o2 + 4, shm);
          dequant_word_fma<Tr>(W[2].z, o2 + 8, shm);
          dequant_word_fma<Tr>(W[2].w, o2 + 12, shm);
          dequant_word_fma<Tr>(W[3].x, o3 + 0, shm);
          dequant_word_fma<Tr>(W[3].y, o3 + 4, shm);
          dequant_word_fma<Tr>(W[3].z, o3 + 8, shm);
          dequant_word_fma<Tr>(W[3].w, o3 + 12, shm);
          tmem_st16(acol + 32, o2);
          tmem_st16(acol + 48, o3);
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(smem_u32(&a_full[2 * sa + j]));
          // The weight stage is released only after every lane consumed its
          // shared loads (the dequant above read W): the refill is an
          // async-proxy write that is not ordered after loads still in flight.
          if (gi == ng - 1) mbar_arrive(smem_u32(&w_empty[ws]));
        }
        ra.next();
      }
      rw.next();
      if (++gp == GP) gp = 0;
    }
  } else if (warp < kDeqWarps + kFoldWarps) {
    // ------------------------------- fold warps -------------------------------
    const int fw = warp - kDeqWarps;
    const int q = fw & 3, j = fw >> 2, r = q * 32 + lane;
    const uint32_t tlane = tbase + ((uint32_t)(q * 32) << 16);
    int tile = tile0;
    RowView cv;
    load_rowview<KIND>(a, tile, n_segs, j, r, cv);
    float acc[N];
#pragma unroll
    for (int n = 0; n < N; ++n) acc[n] = 0.f;
    // Group scales of the current item, and of the next one when it is in the
    // same tile (loaded one item ahead so the loads never stall a group).
    auto load_scales = [&](int gp_, float (&sc)[2]) {
      const int g0 = 2 * gp_;
      sc[0] = __half2float(__ushort_as_half(__ldg(cv.s + g0)));
      sc[1] = g0 + 1 < a.G ? __half2float(__ushort_as_half(__ldg(cv.s + g0 + 1))) : 0.f;
    };
    float sc_cur[2], sc_nxt[2];
    load_scales(gp0, sc_nxt);
    Ring<SD> rd;
    int gp = gp0;
#pragma unroll 1
    for (int it = 0; it < n_items; ++it) {
      const int ng = min(2, a.G - 2 * gp);
      sc_cur[0] = sc_nxt[0];
      sc_cur[1] = sc_nxt[1];
      if (gp + 1 < GP && it + 1 < n_items) load_scales(gp + 1, sc_nxt);
#pragma unroll 1
      for (int gi = 0; gi < ng; ++gi) {
        const int grp = 2 * gp + gi;
        const int sd = rd.idx;
        const float scale = gi ? sc_cur[1] : sc_cur[0];
        const int m = cv.m;
        mbar_wait(smem_u32(&d_full[sd]), rd.phase, a.err);
        tc_fence_after();
#pragma unroll
        for (int h = 0; h < N / 16; ++h) {
          if (h * 16 < m) {
            uint32_t d[16];
            tmem_ld16(tlane + D0 + sd * 2 * N + j * N + h * 16, d);
            tmem_ld_wait16(d);
#pragma unroll
            for (int n = 0; n < 16; n += 2) ffma2(acc[h * 16 + n], acc[h * 16 + n + 1], scale, d[n], d[n + 1]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&d_empty[sd]));
        rd.next();
        const bool tile_end = (grp == a.G - 1) || (it == n_items - 1 && gi == ng - 1);
        if (!tile_end) continue;
        // ---------------- finish this CTA's piece of the tile ----------------
        const int64_t ts = (int64_t)tile * GP, te = ts + GP;
        bool own = true;
        if (!(b0 <= ts && b1 >= te)) {
          // Every piece (the last arriver's own too) goes through its partial
          // slot; the last arriver sums the slots in CTA order, so the result
          // does not depend on which CTA finishes last.
          const int slot = (ts <= b0) ? 0 : 1;
          float* dst = a.part + ((((int64_t)c * 2 + slot) * kFoldWarps + fw) * N) * 32 + lane;
#pragma unroll
          for (int n = 0; n < N; ++n) dst[n * 32] = acc[n];
          __threadfence();
          named_bar_sync(1, kFoldThreads);
          const int64_t c0 = cta_of(ts), c1 = cta_of(te - 1);
          if (fw == 0 && lane == 0) bcast[0] = (atomicAdd(&a.tile_ctr[tile], 1) == (int)(c1 - c0));
          named_bar_sync(1, kFoldThreads);
          own = bcast[0] != 0;
          if (own) {
            __threadfence();
#pragma unroll
            for (int n = 0; n < N; ++n) acc[n] = 0.f;
            for (int64_t cc = c0; cc <= c1; ++cc) {
              const int64_t bc = begin_of(cc);
              const int sl = (bc >= ts && bc < te) ? 0 : 1;
              const float* src = a.part + ((((int64_t)cc * 2 + sl) * kFoldWarps + fw) * N) * 32 + lane;
#pragma unroll
              for (int n = 0; n < N; ++n) acc[n] += ld_cg_f32(src + n * 32);
            }
            if (fw == 0 && lane == 0) a.tile_ctr[tile] = 0;
          }
        }
        if (own) {
          const int ft = threadIdx.x - kDeqWarps * 32;  // 0 .. kFoldThreads-1
          if (KIND == KIND_GATEUP) {
            if (j == 1) {
#pragma unroll
              for (int n = 0; n < N; ++n) htile[r * (N + 1) + n] = acc[n];
            }
            named_bar_sync(1, kFoldThreads);
            if (j == 0) {
#pragma unroll
              for (int n = 0; n < N; ++n) {
                const float hv = silu_f(acc[n]) * htile[r * (N + 1) + n];
                htile[r * (N + 1) + n] = Tr::to_f(Tr::from_f(hv));
              }
            }
            named_bar_sync(1, kFoldThreads);
            uint8_t* dstp = a.hp + (int64_t)cv.rt * kChunk;  // group rt of each staged row
            for (int task = ft; task < m * 16; task += kFoldThreads) {
              const int tok = task >> 4, ch = task & 15;
              float v[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) v[i] = htile[(ch * 8 + i) * (N + 1) + tok];
              uint4 pk;
              float cp;
              pack_unit<Tr>(v, pk, cp);
              *reinterpret_cast<uint4*>(dstp + (int64_t)(cv.p0 + tok) * a.hp_rstride + 16 + ch * 16) = pk;
              cpart[tok * 16 + ch] = cp;
            }
            named_bar_sync(1, kFoldThreads);
            if (ft < m) {
              float cs = 0.f;
              for (int u = 0; u < 16; ++u) cs += cpart[ft * 16 + u];
              *reinterpret_cast<uint4*>(dstp + (int64_t)(cv.p0 + ft) * a.hp_rstride) = correction_unit(cs);
            }
            named_bar_sync(1, kFoldThreads);
          } else {
            const int row = cv.rt * 256 + j * 128 + r;
            if (row < a.N) {
#pragma unroll
              for (int n = 0; n < N; ++n) {
                if (n < m) {
                  const int p = cv.p0 + n;
                  if (EPI == EPI_STORE)
                    reinterpret_cast<typename Tr::T*>(a.out)[(int64_t)a.a_tok[p] * a.ldo + row] = Tr::from_f(acc[n]);
                  else
                    a.R[(int64_t)p * a.N + row] = acc[n] * a.a_w[p];
                }
              }
            }
            if (EPI == EPI_COMBINE) {
              __threadfence();
              named_bar_sync(1, kFoldThreads);
              if (ft == 0) bcast[1] = (atomicAdd(&a.rt_ctr[cv.rt], 1) == n_segs - 1);
              named_bar_sync(1, kFoldThreads);
              if (bcast[1]) {
                __threadfence();
                const int r0 = cv.rt * 256, nr = min(256, a.N - r0);
                for (int task = ft; task < a.T * nr; task += kFoldThreads) {
                  const int t = task / nr, rr = r0 + task - t * nr;
                  float sacc = 0.f;
                  for (int kk = 0; kk < a.topk; ++kk)
                    sacc += ld_cg_f32(a.R + (int64_t)a.pos[t * a.topk + kk] * a.N + rr);
                  reinterpret_cast<typename Tr::T*>(a.out)[(int64_t)t * a.ldo + rr] = Tr::from_f(sacc);
                }
                if (ft == 0) a.rt_ctr[cv.rt] = 0;
              }
            }
          }
        }
#pragma unroll
        for (int n = 0; n < N; ++n) acc[n] = 0.f;
      }
      if (++gp == GP) {
        gp = 0;
        if (it + 1 < n_items) {
          ++tile;
          load_rowview<KIND>(a, tile, n_segs, j, r, cv);
          load_scales(0, sc_nxt);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp0) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// Tokens per segment = N of the MMA (16 or 32); 8*nt with nt in {2, 4}.
static int pick_nt(int64_t max_tokens_per_expert) { return max_tokens_per_expert <= 16 ? 2 : 4; }

// Weight stages (32 KB each) and token stages per tile width N; the totals
// stay within 227 KB of shared memory.
template <int N>
struct TcTune {
  static constexpr int ST = (N == 16) ? 5 : 4, SB = 8;
};

static int encode_token_maps(CUtensorMap* data, CUtensorMap* corr, const void* base, int64_t rows,
                             int64_t row_bytes, int box_rows);

template <typename Tr, int N, int KIND, int EPI>
static int launch_engine_t(const EngineArgs& a, cudaStream_t s) {
  using TU = TcTune<N>;
  using L = TcSmem<N, TU::ST, TU::SB>;
  static_assert(2 * L::kTotal > 228 * 1024, "one engine CTA per SM: it allocates all 512 TMEM columns");
  static_assert(L::kTotal <= 227 * 1024, "engine shared memory exceeds the per-CTA limit");
  auto kern = tc_engine_kernel<Tr, N, KIND, EPI, TU::ST, TU::SB>;
  EngineArgs e = a;
  if (KIND == KIND_DOWN) {
    const int rc = encode_token_maps(&e.bmap, &e.cmap, e.bsrc, e.b_rows, e.b_rstride, N);
    if (rc) return rc;
  }
  static bool attr_set[64] = {};  // per instantiation and device
  int dev = 0;
  HN_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    HN_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal));
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  kern<<<e.P, kTcThreads, L::kTotal, s>>>(e);
  HN_CUDA(cudaGetLastError());
  return HN_OK;
}

template <typename Tr, int KIND, int EPI>
static int launch_engine(int nt, const EngineArgs& a, cudaStream_t s) {
  if (nt <= 2) return launch_engine_t<Tr, 16, KIND, EPI>(a, s);
  return launch_engine_t<Tr, 32, KIND, EPI>(a, s);
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
  size_t counts, n_segs, segs, a_tok, a_w, pos, idx, wts, xp, hp, part1, part2, R, data;  // back (relative)
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
  l.rtctr = take(4 * n_rt2);
  l.counters = o;
  o = 0;
  l.counts = take(4 * E);
  l.n_segs = take(4);
  l.segs = take(16 * max_segs);
  l.a_tok = take(4 * TK);
  l.a_w = take(4 * TK);
  l.pos = take(4 * TK);
  l.idx = take(4 * TK);
  l.wts = take(4 * TK);
  l.xp = take((size_t)(Kin / 128) * T * kChunk);
  l.hp = take(F ? (size_t)(F / 128) * TK * kChunk : 0);
  const size_t part = (size_t)P * 2 * 8 * (8 * nt) * 32 * 4;  // [CTA][2 slots][fold warp][N][32] fp32
  l.part1 = take(F ? part : 0);
  l.part2 = take(part);
  l.R = take(combine ? (size_t)TK * N2 * 4 : 0);
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
  p.a_tok = reinterpret_cast<int*>(d + l.a_tok);
  p.a_w = reinterpret_cast<float*>(d + l.a_w);
  p.pos = reinterpret_cast<int*>(d + l.pos);
  p.idx = reinterpret_cast<int*>(d + l.idx);
  p.wts = reinterpret_cast<float*>(d + l.wts);
  p.xp = d + l.xp;
  p.hp = d + l.hp;
  p.part1 = reinterpret_cast<float*>(d + l.part1);
  p.part2 = reinterpret_cast<float*>(d + l.part2);
  p.R = reinterpret_cast<float*>(d + l.R);
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
  size_t sm = (size_t)(ra.H + 2 * ra.E + ra.H / 8) * 4 + (TK <= kPlanSmemEntries ? (size_t)TK * 8 : 0);
  sm = std::max(sm, (size_t)(2 * ra.E) * 4);
  sm = (sm + 15) & ~(size_t)15;
  r.wbuf_off = (int)sm;
  if (ra.mode == ROUTE_COMPUTE) sm += (size_t)route_chunk_experts(ra.H, ra.E, ra.rw_dtype) * ra.H * route_esize(ra.rw_dtype);
  HN_REQUIRE(sm <= 227 * 1024, "router: hidden size too large for the shared-memory plan");
  if (sm > 48 * 1024)
    HN_CUDA(cudaFuncSetAttribute(route_prep_kernel<Tr>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  route_prep_kernel<Tr><<<ra.T, 256, sm, s>>>(r);
  HN_CUDA(cudaGetLastError());
  return HN_OK;
}

static int check_router(const hn_router_params* r, int64_t E) {
  HN_REQUIRE(r, "router params are NULL");
  HN_REQUIRE(r->kind == HN_ROUTER_SOFTMAX_TOPK || r->kind == HN_ROUTER_SIGMOID_TOPK, "unknown router kind");
  HN_REQUIRE(r->weight, "router weight is NULL");
  HN_REQUIRE(r->weight_dtype >= HN_DTYPE_F32 && r->weight_dtype <= HN_DTYPE_BF16, "bad router weight dtype");
  HN_REQUIRE(r->top_k >= 1 && r->top_k <= E && r->top_k <= kMaxTopK, "top_k out of range");
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
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    else
      cudaGetLastError();
  }
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
// data halves as 128 B x box_rows boxes with 128B swizzle, correction units as
// 16 B x box_rows boxes without swizzle.
static int encode_token_maps(CUtensorMap* data, CUtensorMap* corr, const void* base, int64_t rows,
                             int64_t row_bytes, int box_rows) {
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
  cuuint32_t box_c[2] = {16u, (cuuint32_t)box_rows};
  r = fn(corr, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box_c, es,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HN_ERR_CUDA, "cuTensorMapEncodeTiled (corrections) failed: " + std::to_string((int)r));
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
};

template <typename Tr>
static int run_moe(const MoECall& m) {
  const int64_t TK = m.T * m.topk;
  const int nt = pick_nt(std::min<int64_t>(m.T, TK));
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
  }
  ra.given_idx = m.given_idx;
  ra.given_w = m.given_w;
  ra.out_idx = m.out_idx;
  ra.out_w = m.out_w;
  ra.out_logits = m.out_logits;
  ra.seg = seg_tokens(nt);
  ra.plan = plan;
  int rc = HN_OK;
  if (m.phase == 0 || m.phase == 1) rc = launch_route<Tr>(ra, m.stream);
  if (rc || !m.run_experts || m.phase == 1) return rc;

  EngineArgs e1{};
  e1.shm = ShiftMul{1u << 31, 1u << 24, 1u << 23};
  e1.K = (int)m.H;
  e1.G = (int)(m.H / 128);
  e1.N = (int)m.F;
  e1.n_rt = (int)(m.F / 128);
  e1.T = (int)m.T;
  e1.topk = m.topk;
  e1.segs = plan.segs;
  e1.n_segs = plan.n_segs;
  e1.a_tok = plan.a_tok;
  e1.a_w = plan.a_w;
  e1.pos = plan.pos;
  e1.table = m.table;
  e1.single = m.single;
  e1.maps = static_cast<const ExpertMaps*>(m.maps);
  if (!m.table) {
    rc = encode_expert_maps(&e1.single_maps, m.single, m.H, m.F);
    if (rc) return rc;
  }
  e1.bsrc = plan.xp;
  e1.b_rstride = (m.H / 128) * kChunk;
  e1.b_use_tok = 1;
  e1.hp = plan.hp;
  e1.hp_rstride = (m.F / 128) * kChunk;
  e1.part = plan.part1;
  e1.tile_ctr = plan.ctr1;
  e1.err = plan.err;
  e1.P = P;
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
  if (combine) return launch_engine<Tr, KIND_DOWN, EPI_COMBINE>(nt, e2, m.stream);
  return launch_engine<Tr, KIND_DOWN, EPI_STORE>(nt, e2, m.stream);
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
  if (T < 1 || H < 128 || F < 128 || E < 1 || top_k < 1) return 0;
  const int nt = pick_nt(std::min<int64_t>(T, T * top_k));
  return make_layout(T, H, E, top_k, F, H, nt, grid_p(nt), true).total() + 256;
}

size_t hn_expert_mlp_workspace_size(int64_t T, int64_t H, int64_t F) {
  if (T < 1 || H < 128 || F < 128) return 0;
  const int nt = pick_nt(T);
  return make_layout(T, H, 1, 1, F, H, nt, grid_p(nt), false).total() + 256;
}

size_t hn_int4_linear_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M < 1 || N < 1 || K < 128) return 0;
  const int nt = pick_nt(M);
  return make_layout(M, K, 1, 1, 0, N, nt, grid_p(nt), false).total() + 256;
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
  int rc = check_dims(T, H, F, E);
  if (rc) return rc;
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
  HN_REQUIRE_SUPPORTED(group_size == 128, "only group_size 128 is implemented");
  HN_REQUIRE(M >= 1 && N >= 1 && K >= 128 && K % 128 == 0, "int4_linear: need M, N >= 1 and K a multiple of 128");
  HN_REQUIRE(M <= (1 << 20) && N <= (1 << 20) && K <= 32768, "int4_linear: dims too large");
  HN_REQUIRE(((uintptr_t)w_packed & 15) == 0, "int4_linear: packed weights must be 16-byte aligned");
  HN_REQUIRE(ldx >= K && ldo >= N, "int4_linear: bad row stride");
  HN_REQUIRE(x && w_packed && w_scales && out && workspace, "int4_linear: null pointer");
  const int nt = pick_nt(M);
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
  EngineArgs e{};
  e.shm = ShiftMul{1u << 31, 1u << 24, 1u << 23};
  e.K = (int)K;
  e.G = (int)(K / 128);
  e.N = (int)N;
  e.n_rt = (int)((N + 255) / 256);
  e.T = (int)M;
  e.topk = 1;
  e.segs = plan.segs;
  e.n_segs = plan.n_segs;
  e.a_tok = plan.a_tok;
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

int hn_workspace_error(const void* workspace, size_t workspace_bytes, int* error_code, void* stream) {
  HN_REQUIRE(workspace && error_code && workspace_bytes >= 4, "hn_workspace_error: bad arguments");
  HN_CUDA(cudaMemcpyAsync(error_code, workspace, 4, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
  HN_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  if (*error_code != 0) HN_CUDA(cudaMemsetAsync(const_cast<void*>(workspace), 0, 4, (cudaStream_t)stream));
  return HN_OK;
}

}  // extern "C"
