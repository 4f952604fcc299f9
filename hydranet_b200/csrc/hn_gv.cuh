// Grouped INT4 GEMV for decode-size segments (at most 16 tokens per expert
// segment) on the warp-level tensor-core path (mma.sync m16n8k16, fp32
// accumulate), with the packed weights dequantised in registers.
//
// Why a second engine: at 1-16 tokens per expert the work per weight byte is
// tiny, so the layer is a weight stream that must run at HBM speed.  The
// tcgen05 engine (tc_engine_kernel) has to write every dequantised weight
// into tensor memory and hand it between warp roles through barriers; here
// each thread loads its own packed bytes with 128-bit loads, converts them to
// float16 in registers and feeds them to the tensor core directly as the A
// operand, so no dequantised value ever leaves the register file and no warp
// waits for another except at shared token-slice boundaries.
//
// Work decomposition (stream-K over k-groups):
//   tile   = (segment, block of rows): gate/up 128 rows of F (warp w owns rows
//            16w..16w+15 of BOTH the gate and the up matrix), down 256 rows
//            (warp w owns rows 32w..32w+31 as two 16-row MMA tiles);
//   step   = one 128-wide k-group of one tile;
//   CTA c  = steps [c*NS/P, (c+1)*NS/P) of the NS steps of all tiles, so every
//            SM streams the same number of weight bytes.  A tile whose steps
//            are split between CTAs is finished by the CTA that completes it
//            last (partials summed in CTA order: deterministic).
// Every warp of a CTA walks the same steps (on its own rows), so the tokens
// of the current k-groups are shared through shared memory: "slices" of up to
// 8 k-groups, double-buffered, loaded with cp.async from the staged rows.
//
// Per thread (lane = 4*g + t) and k-group: row g and row g+8 of each of its
// two 16-row MMA tiles; for each row the 16 bytes at 16*t of the group (k
// 32t..32t+31).  Word q of those bytes (k 32t+8q..+7) becomes the A
// registers of MMA k-steps 2q and 2q+1: OR-ing the nibbles into the mantissa
// of 1024.0 gives the float16 pairs (k0,k4), (k2,k6) = 1024 + n [low
// nibbles, even k] and (k1,k5), (k3,k7) = 1024 + 16n [high nibbles, odd k],
// exact integers, fed to the tensor core as they are (four instructions and
// a shift per word).  The staged tokens hold x at even k and b = x / 16 at
// odd k, so the products are (1024 + n) x = (n - 8) x + 1032 x and
// (1024 + 16n) b = (n - 8) x + 1152 b: the group's MMA sum exceeds the wanted
// sum by 1032 * sum_even x + 1152 * sum_odd b, the per-token correction
// staged beside the tokens (gv_offset_correction), subtracted in the fold.  The token operand is stored so that
// one 16-byte shared load per (q, 8 tokens) yields the matching B registers:
// unit (q, t) of a token is the staged unit 4t+q of its k-group (the pair
// order above), at [q][token][t] inside the group.  Each k-group's MMAs
// accumulate into a fresh fp32 fragment that is then folded into the
// running sum times the group's fp32 scale (one FMA per element): the
// weights enter the tensor core as exact integers and the per-group scale is
// applied in fp32, so no float16 rounding of (n - 8) * scale happens at all.
//
// The epilogues are those of the tcgen05 engine: SiLU(gate)*up as float16
// into the down phase's staged rows (assignment order), routing-weighted rows
// plus the per-(row tile, token) completion count for the top-k combine, or
// plain rows for the single-matrix / single-expert calls.
// Included by hn_moe.cu inside namespace hn, after the tcgen05 engine (it
// uses the plan, staging and epilogue helpers defined there).
#pragma once

constexpr int kGvStages = 4;     // weight ring stages per warp (one k-group each)
constexpr int kGvMaxTiles = 32;  // tiles of one CTA's step range whose metadata is cached in shared memory

// Launch shape and shared-memory plan per token-tile count NT (8*NT tokens
// per segment, NT = 1 or 2): 8 warps and two CTAs per SM, four warps per
// scheduler within 128 registers.
//   weight ring  [warp][stage][4 loads][32 lanes][16 B]  (each thread reads back only what it copied)
//   token slices 2 x [group][4 q][8NT tokens][4 t][16 B]
//   scale slices 2 x [group][warp][2 MMA tiles][8 g][2 h] fp16
//   tile table   kGvMaxTiles x GvTileMeta
template <int NT>
struct GvTileMeta {
  const uint8_t* pk[2];   // packed matrix of MMA tile 0 / 1
  const uint16_t* sc[2];  // its scales
  int first, m;           // segment: first assignment, tokens
  int rows[8 * NT];       // staged row of each token of the segment
};
template <int NT>
struct GvCfg {
  static_assert(NT == 1 || NT == 2, "the mma.sync engine runs segments of up to 16 tokens");
  static constexpr int W = 8;
  static constexpr int kCtasPerSm = 2;
  static constexpr int kThreads = W * 32;
  static constexpr int kSlice = NT == 1 ? 8 : 4;  // k-groups per token slice (16 KB of tokens)
  static constexpr int kStage = 2048;             // one warp's 32 rows x 64 B of a k-group
  static constexpr int kGroupBytes = 2048 * NT;
  static constexpr int kRows = W * 32;  // weight rows of a tile (both matrices): one per thread
  static constexpr int kWRing = W * kGvStages * kStage;
  static constexpr int kBBuf = kSlice * kGroupBytes;
  static constexpr int kSBuf = kSlice * kRows * 2;
  static constexpr int kMeta = kGvMaxTiles * (int)sizeof(GvTileMeta<NT>);
  static constexpr int kMisc = 256;
  static constexpr int kCBuf = kSlice * 8 * NT * 4;  // offset corrections of a slice's tokens
  static constexpr int kCRed = W * 8 * NT * 4;       // gate/up epilogue: per-warp correction partials
  static constexpr int kTotal = kWRing + 2 * kBBuf + 2 * kSBuf + kMeta + kMisc + 2 * kCBuf + kCRed;
  static_assert(kTotal * kCtasPerSm <= 227 * 1024, "gv shared-memory plan exceeds the SM");
};

static_assert(sizeof(hn_expert_ptrs) == 6 * sizeof(void*), "hn_expert_ptrs is read as six pointers");

struct GvArgs {
  int K, G;  // reduction length and its k-groups
  int rows;  // rows of each matrix (F for gate/up; output rows for down)
  int tps;   // tiles per segment
  int T, topk;
  const int4* segs;
  const int* n_segs;
  const int* a_tok;
  const int* a_tk;
  const float* a_w;
  const hn_expert_ptrs* table;  // device table, or NULL: single
  hn_expert_ptrs single;
  const uint8_t* bsrc;  // staged token rows, [row][group][kChunk]
  int64_t b_rstride;
  int b_by_token;  // 1: staged row of assignment p is a_tok[p] (gate/up reads x); 0: row p
  uint8_t* hp;     // gate/up output rows (assignment order)
  int64_t hp_rstride;
  float* R;
  void* out;
  int64_t ldo;
  float* part;
  int* tile_ctr;
  int* rt_ctr;
  const int* nval;  // [T] slots per token that hold an expert
  const int* tidx;  // [T*K] expert of each slot, -1 = unused
  int defer_combine;
  int early;  // KIND_DOWN right after a gate/up launch: the plan is visible at entry, the staged rows later
  const float* corr_b;  // [staged row][G] offset correction of each staged row's k-groups
  float* corr_out;      // KIND_GATEUP: [assignment][rows / 128] corrections of the staged SiLU(gate)*up
  int P;
};

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Same with C = 0 (the first k-step of a group).
__device__ __forceinline__ void mma_f16_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// Eight packed nibbles -> four float16 pairs n - 8 (exact) in the staged pair
// order {(k0,k4), (k2,k6), (k1,k5), (k3,k7)}: OR-ing a nibble into the
// mantissa of 1024.0 gives 1024 + n (bits 0..3) or 1024 + 16n (bits 4..7);
// minus 1032, or times 1/16 minus 72, leaves n - 8.  Nine instructions.
__device__ __forceinline__ void dq_word(uint32_t w, uint32_t (&o)[4]) {
  const uint32_t w8 = w >> 8;
  o[0] = lop3_and_or<0x000F000Fu>(w, 0x64006400u);
  o[1] = lop3_and_or<0x000F000Fu>(w8, 0x64006400u);
  o[2] = lop3_and_or<0x00F000F0u>(w, 0x64006400u);
  o[3] = lop3_and_or<0x00F000F0u>(w8, 0x64006400u);
  asm("add.rn.f16x2 %0, %0, %1;" : "+r"(o[0]) : "r"(0xE408E408u));
  asm("add.rn.f16x2 %0, %0, %1;" : "+r"(o[1]) : "r"(0xE408E408u));
  asm("fma.rn.f16x2 %0, %0, %1, %2;" : "+r"(o[2]) : "r"(0x2C002C00u), "r"(0xD480D480u));
  asm("fma.rn.f16x2 %0, %0, %1, %2;" : "+r"(o[3]) : "r"(0x2C002C00u), "r"(0xD480D480u));
}

// Eight packed nibbles -> the float16 pairs 1024 + n (even k) and 1024 + 16n
// (odd k) in the staged pair order, exact; the offsets are removed by the
// per-group correction.  Five instructions.
__device__ __forceinline__ void dq_word_offset(uint32_t w, uint32_t (&o)[4]) {
  const uint32_t w8 = w >> 8;
  o[0] = lop3_and_or<0x000F000Fu>(w, 0x64006400u);
  o[1] = lop3_and_or<0x000F000Fu>(w8, 0x64006400u);
  o[2] = lop3_and_or<0x00F000F0u>(w, 0x64006400u);
  o[3] = lop3_and_or<0x00F000F0u>(w8, 0x64006400u);
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}

// Weight stream: read once per layer, so it bypasses L1 and is evict-first in L2.
__device__ __forceinline__ uint4 ldg_stream(const void* p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}
__device__ __forceinline__ uint32_t ldg_u16(const uint16_t* p) {
  unsigned short v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ const void* ldg_ptr(const void* const* p) {
  return reinterpret_cast<const void*>(__ldg(reinterpret_cast<const unsigned long long*>(p)));
}

template <int W>
__device__ __forceinline__ uint32_t word_of(const uint4& v) {
  return W == 0 ? v.x : (W == 1 ? v.y : (W == 2 ? v.z : v.w));
}

// Owner CTA of step s and the first step of CTA c (stream-K split).
__device__ __forceinline__ int64_t gv_begin(int64_t NS, int c, int P) { return NS * c / P; }
__device__ __forceinline__ int gv_owner(int64_t NS, int64_t s, int P) {
  return (int)(((s + 1) * P + NS - 1) / NS) - 1;
}

// cp.async of 16 bytes with an L2 cache policy (the weight stream: evict-first).
__device__ __forceinline__ void cp_async16_pol(uint32_t dst, const void* src, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "l"(pol)
               : "memory");
}
// Wait until at most n (0..kGvStages-2) of this thread's newest cp.async groups are pending.
__device__ __forceinline__ void cp_async_wait_n(int n) {
  static_assert(kGvStages == 4, "cp_async_wait_n covers 0..2");
  if (n <= 0)
    cp_async_wait<0>();
  else if (n == 1)
    cp_async_wait<1>();
  else
    cp_async_wait<2>();
}

template <typename Tr, int NT, int KIND, int EPI>
__global__ void __launch_bounds__(GvCfg<NT>::kThreads, GvCfg<NT>::kCtasPerSm)
    gv_kernel(const __grid_constant__ GvArgs a) {
  using C = GvCfg<NT>;
  using Meta = GvTileMeta<NT>;
  constexpr int S = kGvStages;
  constexpr int W = C::W;
  extern __shared__ __align__(128) uint8_t gsm[];
  uint8_t* const bbuf = gsm + C::kWRing;
  uint8_t* const sbuf = bbuf + 2 * C::kBBuf;
  Meta* const meta = reinterpret_cast<Meta*>(sbuf + 2 * C::kSBuf);
  int* const s_misc = reinterpret_cast<int*>(sbuf + 2 * C::kSBuf + C::kMeta);  // [0] flag, [1] count, [2..] tokens
  float* const cbuf = reinterpret_cast<float*>(sbuf + 2 * C::kSBuf + C::kMeta + C::kMisc);  // [2][kSlice][8NT]
  float* const cred = cbuf + 2 * (C::kCBuf / 4);                                             // [W][8NT]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gl = lane >> 2, tq = lane & 3;
  const int c = blockIdx.x, P = gridDim.x;
  const uint64_t pol = l2_evict_first_policy();

  // The plan comes from the prep kernel.  A gate/up launch (or a down launch
  // straight after the prep kernel) waits for it here; a down launch that
  // follows a gate/up launch (a.early) needs no wait for the plan -- the
  // gate/up launch only let it start after the prep kernel had completed --
  // and waits below, before it reads the staged gate/up results.
  if (KIND == KIND_GATEUP || !a.early) griddep_wait();
  const int ns = __ldcg(a.n_segs);
  const int G = a.G;
  const int64_t NS = (int64_t)ns * a.tps * G;
  const int64_t sb = gv_begin(NS, c, P), se = gv_begin(NS, c + 1, P);
  griddep_launch_dependents();
  if (sb >= se) return;
  const int tile0 = (int)(sb / G);
  const int ntl = (int)((se - 1) / G) - tile0 + 1;  // at most kGvMaxTiles (the host checks the bound)

  // ---- metadata of this CTA's tiles: expert tensors, segment, token rows ----
  auto expert_ptr = [&](int e, int which) -> const void* {
    if (a.table) return ldg_ptr(reinterpret_cast<const void* const*>(a.table + e) + which);
    // the single expert of the call's arguments (kernel parameter space: read directly)
    return which == 0 ? (const void*)a.single.gate_packed : which == 1 ? (const void*)a.single.gate_scales
         : which == 2 ? (const void*)a.single.up_packed : which == 3 ? (const void*)a.single.up_scales
         : which == 4 ? (const void*)a.single.down_packed : (const void*)a.single.down_scales;
  };
  for (int i = tid; i < ntl; i += C::kThreads) {
    const int4 sg = __ldcg(&a.segs[(tile0 + i) / a.tps]);
    Meta& mi = meta[i];
    mi.first = sg.y;
    mi.m = sg.z;
    // hn_expert_ptrs order: gate_packed, gate_scales, up_packed, up_scales, down_packed, down_scales
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const int wi = KIND == KIND_GATEUP ? 2 * mt : 4;
      mi.pk[mt] = static_cast<const uint8_t*>(expert_ptr(sg.x, wi));
      mi.sc[mt] = static_cast<const uint16_t*>(expert_ptr(sg.x, wi + 1));
    }
  }
  __syncthreads();
  for (int u = tid; u < ntl * 8 * NT; u += C::kThreads) {
    const int i = u / (8 * NT), n = u - i * (8 * NT);
    const int p = meta[i].first + n;
    meta[i].rows[n] = n < meta[i].m ? (a.b_by_token ? __ldcg(a.a_tok + p) : p) : 0;
  }
  __syncthreads();

  // matrix row of (MMA tile mt, half h) for this thread in tile-row block rt
  auto wrow = [&](int rt, int mt, int h) {
    const int r = KIND == KIND_GATEUP ? rt * (16 * W) + warp * 16 + gl + 8 * h
                                      : rt * (32 * W) + warp * 32 + mt * 16 + gl + 8 * h;
    return min(r, a.rows - 1);  // rows past the matrix load its last row and are never stored
  };

  // Steps are counted from the CTA's first step (32-bit); a tile's steps are
  // its k-groups 0..G-1, and the first step sits at group g_start of tile0.
  const int n_steps = (int)(se - sb);
  const int g_start = (int)(sb - (int64_t)tile0 * G);

  // ---- weight prefetcher: relative step pf_r into ring stage pf_slot ----
  int pf_r = 0, pf_i = 0, pf_g = g_start, pf_slot = 0;
  const uint8_t* pfp[4];
  auto pf_set = [&]() {
    const int rt = (tile0 + pf_i) % a.tps;
#pragma unroll
    for (int k = 0; k < 4; ++k)
      pfp[k] = meta[pf_i].pk[k >> 1] + (int64_t)wrow(rt, k >> 1, k & 1) * (a.K / 2) + 16 * tq;
  };
  const uint32_t wbase = smem_u32(gsm) + (uint32_t)(warp * S * C::kStage + lane * 16);
  auto pf_issue = [&]() {  // always commits one group (empty past the range)
    if (pf_r < n_steps) {
      const uint32_t dst = wbase + pf_slot * C::kStage;
#pragma unroll
      for (int k = 0; k < 4; ++k) cp_async16_pol(dst + k * 512, pfp[k] + pf_g * 64, pol);
      ++pf_r;
      pf_slot = pf_slot + 1 == S ? 0 : pf_slot + 1;
      if (++pf_g == G) {
        pf_g = 0;
        ++pf_i;
        if (pf_r < n_steps) pf_set();
      }
    }
    cp_async_commit();
  };

  // ---- token and scale slices: up to kSlice k-groups of one tile, double-buffered ----
  // length of the slice that starts at relative step r, group g of its tile
  auto slice_len = [&](int r, int g) { return min(n_steps - r, min(G - g, C::kSlice - (g & (C::kSlice - 1)))); };
  // this thread's (token, 16-byte unit) pairs of a slice copy: no division per unit
  constexpr int kPairs = 8 * NT * 16;
  constexpr int kPairIters = (kPairs + C::kThreads - 1) / C::kThreads;
  // token rows of the slice at (tile ti, group g0, gs groups) -> token buffer bufi
  // (cp.async, committed by the caller)
  auto load_tokens = [&](int bufi, int ti, int g0, int gs) {
    const Meta& mi = meta[ti];
    const uint32_t dst0 = smem_u32(bbuf) + bufi * C::kBBuf;
#pragma unroll
    for (int it = 0; it < kPairIters; ++it) {
      const int idx = tid + it * C::kThreads;
      const int n = idx >> 4, cc = idx & 15;
      if (idx < kPairs && n < mi.m) {
        const uint8_t* src = a.bsrc + (int64_t)mi.rows[n] * a.b_rstride + (int64_t)g0 * kChunk + cc * 16;
        const uint32_t dst = dst0 + (cc & 3) * (512 * NT) + n * 64 + (cc >> 2) * 16;
#pragma unroll
        for (int gi = 0; gi < C::kSlice; ++gi)
          if (gi < gs) cp_async16(dst + gi * C::kGroupBytes, src + gi * kChunk);
      }
    }
    // the tokens' offset corrections of the slice's groups: [gi][n]
    if (tid < 8 * NT * C::kSlice) {
      const int n = tid / C::kSlice, gi = tid - n * C::kSlice;
      if (n < mi.m && gi < gs)
        cp_async4(smem_u32(cbuf + bufi * (C::kCBuf / 4) + gi * 8 * NT + n),
                  a.corr_b + (int64_t)mi.rows[n] * G + g0 + gi);
    }
  };
  // scales of a slice: thread tid holds tile row tid's scales in registers
  uint32_t sreg[C::kSlice];
  const int my_mt = lane >> 4, my_h = (lane >> 3) & 1, my_g = lane & 7;
  auto load_scales = [&](int ti, int g0, int gs) {
    const int rt = (tile0 + ti) % a.tps;
    int r = KIND == KIND_GATEUP ? rt * (16 * W) + warp * 16 + my_g + 8 * my_h
                                : rt * (32 * W) + warp * 32 + my_mt * 16 + my_g + 8 * my_h;
    r = min(r, a.rows - 1);
    const uint16_t* sp = meta[ti].sc[my_mt] + (int64_t)r * G + g0;
#pragma unroll
    for (int gi = 0; gi < C::kSlice; ++gi) sreg[gi] = gi < gs ? ldg_u16(sp + gi) : 0u;
  };
  auto store_scales = [&](int bufi) {
    uint16_t* sd = reinterpret_cast<uint16_t*>(sbuf + bufi * C::kSBuf) + ((warp * 2 + my_mt) * 8 + my_g) * 2 + my_h;
#pragma unroll
    for (int gi = 0; gi < C::kSlice; ++gi) sd[gi * C::kRows] = (uint16_t)sreg[gi];
  };

  // A down phase right after gate/up fills its weight ring before it waits:
  // the weights do not depend on the gate/up results.  Its first step then
  // waits for every group (the token slice is the newest).
  const bool wfirst = KIND == KIND_DOWN && a.early;
  pf_set();
  if (wfirst)
#pragma unroll
    for (int i = 0; i < S - 1; ++i) pf_issue();
  if (KIND == KIND_DOWN) griddep_wait();  // the gate/up results are complete and visible from here on
  // current slice: relative steps [sl_begin, sl_end); the next one starts at (nx_i, nx_g)
  int sl_begin = 0, sl_end = slice_len(0, g_start), sl_n = 0, sl_prev_len = S - 1;
  load_tokens(0, 0, g_start, sl_end);
  cp_async_commit();  // the first token slice
  load_scales(0, g_start, sl_end);
  if (!wfirst)
#pragma unroll
    for (int i = 0; i < S - 1; ++i) pf_issue();


  // ---- consumer ----
  float acc[2][NT][4];
  int cur_i = 0, cur_g = g_start, cur_slot = 0;
  int piece_g0 = cur_g;
  int seg_first = 0, seg_m = 0, nta = 0;
  auto begin_tile = [&]() {
    seg_first = meta[cur_i].first;
    seg_m = meta[cur_i].m;
    nta = (seg_m + 7) >> 3;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mt][j][e] = 0.f;
  };
  begin_tile();

  auto epilogue = [&](const float (&v)[2][NT][4], int tile) {
    const int rt = tile % a.tps;
    if (KIND == KIND_GATEUP) {
      // SiLU(gate)*up staged for the down phase as the prep kernel stages
      // tokens (odd k divided by 16), and per token the offset correction of
      // this tile's 128 rows -- one k-group of the down phase: the thread's
      // rows (all of k's parity, that of gl), the 8 lanes of its tq, then the
      // warps in order, so the sum does not depend on timing
      const int f0 = rt * (16 * W) + warp * 16 + gl;
      const bool odd = gl & 1;
      float cpart[NT][2];
#pragma unroll
      for (int j = 0; j < NT; ++j) cpart[j][0] = cpart[j][1] = 0.f;
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        if (j >= nta) break;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int n = 8 * j + 2 * tq + (e & 1);
          const int f = f0 + 8 * (e >> 1);
          if (n < seg_m && f < a.rows) {
            const float hv = silu_f(v[0][j][e]) * v[1][j][e];
            const __half h = __float2half_rn(odd ? hv * 0.0625f : hv);
            *reinterpret_cast<__half*>(a.hp + (int64_t)(seg_first + n) * a.hp_rstride + (f >> 7) * kChunk +
                                       staged_offset(f & 127)) = h;
            cpart[j][e & 1] += __half2float(h);
          }
        }
      }
      __syncthreads();  // cred of the previous tile has been read
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          float c = odd ? gv_offset_correction(0.f, cpart[j][u]) : gv_offset_correction(cpart[j][u], 0.f);
          for (int o = 4; o < 32; o <<= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
          if (gl == 0) cred[warp * 8 * NT + 8 * j + 2 * tq + u] = c;
        }
      __syncthreads();
      if (tid < seg_m) {
        float c = 0.f;
        for (int w = 0; w < W; ++w) c += cred[w * 8 * NT + tid];
        a.corr_out[(int64_t)(seg_first + tid) * (a.rows / 128) + rt] = c;
      }
    } else {
      const int r0 = rt * (32 * W) + warp * 32 + gl;
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        if (j >= nta) break;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int n = 8 * j + 2 * tq + (e & 1);
          if (n >= seg_m) continue;
          const int p = seg_first + n;
          if (EPI == EPI_STORE) {
            typename Tr::T* o = reinterpret_cast<typename Tr::T*>(a.out) + (int64_t)__ldcg(a.a_tok + p) * a.ldo;
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
              const int r = r0 + mt * 16 + 8 * (e >> 1);
              if (r < a.rows) o[r] = Tr::from_f(v[mt][j][e]);
            }
          } else {
            const float wgt = __ldcg(a.a_w + p);
            float* Rrow = a.R + (int64_t)__ldcg(a.a_tk + p) * a.rows;
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
              const int r = r0 + mt * 16 + 8 * (e >> 1);
              if (r < a.rows) Rrow[r] = wgt * v[mt][j][e];
            }
          }
        }
      }
      if (EPI == EPI_COMBINE && !a.defer_combine) {
        // the tile that completes a token's top-k contributions for this row
        // block sums them in slot order into the output (one thread per row)
        __threadfence();
        __syncthreads();
        if (tid == 0) s_misc[1] = 0;
        __syncthreads();
        if (tid < seg_m) {
          const int t = __ldcg(a.a_tok + seg_first + tid);
          if (atomicAdd(a.rt_ctr + (int64_t)rt * a.T + t, 1) == __ldcg(a.nval + t) - 1)
            s_misc[2 + atomicAdd(&s_misc[1], 1)] = t;
        }
        __syncthreads();
        __threadfence();
        const int nl = s_misc[1];
        const int r = rt * (32 * W) + tid;
        for (int li = 0; li < nl; ++li) {
          const int t = s_misc[2 + li];
          if (r < a.rows) {
            float sum = 0.f;
            for (int k = 0; k < a.topk; ++k)
              if (__ldcg(a.tidx + (int64_t)t * a.topk + k) >= 0)  // unused slots wrote no row
                sum += __ldcg(a.R + ((int64_t)t * a.topk + k) * a.rows + r);
            reinterpret_cast<typename Tr::T*>(a.out)[(int64_t)t * a.ldo + r] = Tr::from_f(sum);
          }
        }
        __syncthreads();
      }
    }
  };

  // end of a tile piece: direct epilogue, or partial + last-arriver fix-up
  auto finish_piece = [&](int tile, bool whole, float (&tot)[2][NT][4]) {
    if (whole) {
      epilogue(acc, tile);
      return;
    }
    const int slot = tile == tile0 ? 0 : 1;
    float4* mine = reinterpret_cast<float4*>(a.part) + (((int64_t)c * 2 + slot) * W + warp) * (2 * NT * 32);
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int j = 0; j < NT; ++j)
        __stcg(mine + (mt * NT + j) * 32 + lane, make_float4(acc[mt][j][0], acc[mt][j][1], acc[mt][j][2], acc[mt][j][3]));
    __threadfence();
    __syncthreads();
    const int64_t t0 = (int64_t)tile * G;
    const int c0 = gv_owner(NS, t0, P), c1 = gv_owner(NS, t0 + G - 1, P);
    if (tid == 0) {
      int pieces = 0;
      for (int cc = c0; cc <= c1; ++cc) pieces += gv_begin(NS, cc, P) < gv_begin(NS, cc + 1, P);
      s_misc[0] = atomicAdd(a.tile_ctr + tile, 1) == pieces - 1;
    }
    __syncthreads();
    if (!s_misc[0]) return;
    __threadfence();
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) tot[mt][j][e] = 0.f;
    // the pieces in CTA order, kU at a time with all their loads in flight
    // before the first add (a tile of a small step is split over up to ~10 CTAs)
    constexpr int kU = NT == 1 ? 4 : 2;
    for (int cb = c0; cb <= c1; cb += kU) {
      float4 q[kU][2][NT];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int cc = cb + u;
        const int64_t b0 = gv_begin(NS, cc, P);
        const bool other = cc <= c1 && cc != c && b0 < gv_begin(NS, cc + 1, P);
        const int sl = b0 / G == tile ? 0 : 1;
        const float4* src =
            reinterpret_cast<const float4*>(a.part) + (((int64_t)cc * 2 + sl) * W + warp) * (2 * NT * 32);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int j = 0; j < NT; ++j)
            q[u][mt][j] = other ? __ldcg(src + (mt * NT + j) * 32 + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int cc = cb + u;
        if (cc > c1 || gv_begin(NS, cc, P) >= gv_begin(NS, cc + 1, P)) continue;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            if (cc == c) {
              tot[mt][j][0] += acc[mt][j][0];
              tot[mt][j][1] += acc[mt][j][1];
              tot[mt][j][2] += acc[mt][j][2];
              tot[mt][j][3] += acc[mt][j][3];
            } else {
              tot[mt][j][0] += q[u][mt][j].x;
              tot[mt][j][1] += q[u][mt][j].y;
              tot[mt][j][2] += q[u][mt][j].z;
              tot[mt][j][3] += q[u][mt][j].w;
            }
          }
      }
    }
    epilogue(tot, tile);
  };

  const uint32_t wcons = smem_u32(gsm) + (uint32_t)(warp * S * C::kStage + lane * 16);
#pragma unroll 1
  for (int r = 0; r < n_steps; ++r) {
    if (r == sl_begin) {
      // a new slice: its tokens (and this step's weights) have landed; its
      // scales go to shared memory; after the barrier the buffers of the
      // slice before it are free and the next slice starts loading
      if (wfirst && r == 0)
        cp_async_wait<0>();
      else
        cp_async_wait_n(min(S - 2, sl_prev_len - 1));
      store_scales(sl_n & 1);
      __syncthreads();
      if (sl_end < n_steps) {
        // the next slice: the rest of this tile's slice-aligned groups, or the next tile
        int ni = cur_i, ng = cur_g + (sl_end - sl_begin);
        if (ng == G) {
          ++ni;
          ng = 0;
        }
        const int nl = slice_len(sl_end, ng);
        load_tokens((sl_n + 1) & 1, ni, ng, nl);  // committed with this step's weight group
        load_scales(ni, ng, nl);
      }
    } else {
      cp_async_wait<S - 2>();
    }
    pf_issue();

    const int gi = r - sl_begin;
    uint4 wv[2][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(wv[mt][h].x), "=r"(wv[mt][h].y), "=r"(wv[mt][h].z), "=r"(wv[mt][h].w)
                     : "r"(wcons + cur_slot * C::kStage + (2 * mt + h) * 512));
    uint32_t sc2[2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
      sc2[mt] = *reinterpret_cast<const uint32_t*>(sbuf + (sl_n & 1) * C::kSBuf + gi * (C::kRows * 2) +
                                                   ((warp * 2 + mt) * 8 + gl) * 4);
    const uint8_t* bg = bbuf + (sl_n & 1) * C::kBBuf + gi * C::kGroupBytes + lane * 16;
    float tg[2][NT][4];  // a k-group's fresh sums; fix-up scratch in finish_piece
    // dequantise, multiply and fold one k-group for the segment's NTA token
    // tiles (a compile-time count, so the MMA chains of all tiles interleave)
    auto consume = [&](auto nta_c) {
      constexpr int NTA = decltype(nta_c)::value;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 bv[NTA];
#pragma unroll
        for (int j = 0; j < NTA; ++j) bv[j] = *reinterpret_cast<const uint4*>(bg + q * (512 * NT) + j * 512);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          uint32_t lo[4], hi[4];
          dq_word_offset(q == 0 ? wv[mt][0].x : q == 1 ? wv[mt][0].y : q == 2 ? wv[mt][0].z : wv[mt][0].w, lo);
          dq_word_offset(q == 0 ? wv[mt][1].x : q == 1 ? wv[mt][1].y : q == 2 ? wv[mt][1].z : wv[mt][1].w, hi);
#pragma unroll
          for (int j = 0; j < NTA; ++j) {
            if (q == 0)
              mma_f16_z(tg[mt][j], lo[0], hi[0], lo[1], hi[1], bv[j].x, bv[j].y);
            else
              mma_f16(tg[mt][j], lo[0], hi[0], lo[1], hi[1], bv[j].x, bv[j].y);
            mma_f16(tg[mt][j], lo[2], hi[2], lo[3], hi[3], bv[j].z, bv[j].w);
          }
        }
      }
      // fold the group into the running sums: minus the tokens' offset
      // corrections, times the rows' fp32 scales
      const float* cg = cbuf + (sl_n & 1) * (C::kCBuf / 4) + gi * 8 * NT + 2 * tq;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const float s0 = __half2float(__ushort_as_half((unsigned short)(sc2[mt] & 0xFFFFu)));
        const float s1 = __half2float(__ushort_as_half((unsigned short)(sc2[mt] >> 16)));
#pragma unroll
        for (int j = 0; j < NTA; ++j) {
          const float2 cr = *reinterpret_cast<const float2*>(cg + 8 * j);
          acc[mt][j][0] = fmaf(s0, tg[mt][j][0] - cr.x, acc[mt][j][0]);
          acc[mt][j][1] = fmaf(s0, tg[mt][j][1] - cr.y, acc[mt][j][1]);
          acc[mt][j][2] = fmaf(s1, tg[mt][j][2] - cr.x, acc[mt][j][2]);
          acc[mt][j][3] = fmaf(s1, tg[mt][j][3] - cr.y, acc[mt][j][3]);
        }
      }
    };
    if (NT == 1 || nta <= 1)
      consume(std::integral_constant<int, 1>{});
    else
      consume(std::integral_constant<int, NT>{});
    cur_slot = cur_slot + 1 == S ? 0 : cur_slot + 1;
    if (r + 1 == sl_end && sl_end < n_steps) {
      sl_prev_len = sl_end - sl_begin;
      sl_begin = sl_end;
      const int ng = cur_g + 1 == G ? 0 : cur_g + 1;
      sl_end = sl_begin + slice_len(sl_begin, ng);
      ++sl_n;
    }
    if (++cur_g == G || r + 1 == n_steps) {
      finish_piece(tile0 + cur_i, piece_g0 == 0 && cur_g == G, tg);
      if (cur_g == G && r + 1 < n_steps) {
        ++cur_i;
        cur_g = 0;
        piece_g0 = 0;
        begin_tile();
      }
    }
  }
  cp_async_wait<0>();  // no copy may still target shared memory when the CTA exits
}
