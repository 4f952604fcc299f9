/*
 * hydranet_b200.h -- C ABI of the B200 (sm_100a) INT4 mixture-of-experts path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches asynchronously on that stream, never
 * synchronises and never allocates device memory.  Kernels that need scratch
 * take a caller-owned workspace whose size comes from the matching
 * *_workspace_size() query (query on the device that will run the call).
 * A workspace must be 256-byte aligned, and its first 512 bytes (an error
 * word and an arrival counter) must be zero before its first use; zero-filling
 * the whole buffer once when it is allocated is enough.  Bytes 8..15 may then
 * be set to the address of a host-mapped int32 (pinned host memory, which the
 * device reaches at the same address): a device error recorded in the error
 * word is copied there as well, so the host can notice it with a plain read
 * instead of hn_workspace_error's synchronising copy.  The kernels leave it
 * re-usable: the two words stay zero unless a bounded wait failed (see
 * hn_workspace_error), every other counter is zeroed by each call itself, so
 * one workspace may serve calls of any shape whose size query it satisfies.
 * One workspace must not be used by two launches that may overlap on the
 * device.
 *
 * Return value: HN_OK (0) or an HN_ERR_* code; hn_last_error() gives the
 * message of the last failing call on the calling host thread.
 *
 * Tensor conventions follow the reference's packed format
 * (preprocess/pack_weights.py:133-181, cache/packed_expert_store.py:77-108):
 *   packed  uint8  [N, K/2]   two nibbles per byte, low nibble = even k
 *   scales  fp16   [N, K/group_size]
 *   weight  W[n, k] = (nibble - 8) * scale[n, k / group_size]
 * Only group_size == 128 is implemented (HN_ERR_UNSUPPORTED otherwise).
 * Activations are fp16 or bf16 (HN_DTYPE_*), row-major with unit inner stride.
 */
#ifndef HYDRANET_B200_H
#define HYDRANET_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HN_ABI_VERSION 3

#if defined(__GNUC__)
#define HN_API __attribute__((visibility("default")))
#else
#define HN_API
#endif

enum hn_status {
  HN_OK = 0,
  HN_ERR_INVALID = 1,      /* bad pointer / shape / argument          */
  HN_ERR_UNSUPPORTED = 2,  /* valid, but not implemented on this path */
  HN_ERR_CUDA = 3,         /* a CUDA runtime call failed              */
  HN_ERR_WORKSPACE = 4     /* workspace smaller than required         */
};

enum hn_dtype { HN_DTYPE_F32 = 0, HN_DTYPE_F16 = 1, HN_DTYPE_BF16 = 2 };

/* Router kinds (see hn_moe_route). */
enum hn_router_kind {
  HN_ROUTER_SOFTMAX_TOPK = 0, /* Mixtral: model/router.py:73-130        */
  HN_ROUTER_SIGMOID_TOPK = 1  /* GLM-4.5: model/glm4.py:261-309         */
};

/* Device-memory pointer table of one expert: the six tensors of a
 * GpuExpertSlot (cache/packed_expert_store.py:136-162). */
typedef struct hn_expert_ptrs {
  const uint8_t* gate_packed;  /* [F, H/2] */
  const uint16_t* gate_scales; /* [F, H/128] fp16 */
  const uint8_t* up_packed;    /* [F, H/2] */
  const uint16_t* up_scales;   /* [F, H/128] fp16 */
  const uint8_t* down_packed;  /* [H, F/2] */
  const uint16_t* down_scales; /* [H, F/128] fp16 */
} hn_expert_ptrs;

HN_API int hn_abi_version(void);
HN_API const char* hn_last_error(void);

/* Number of SMs the library sizes its persistent grids for (device 'device'). */
HN_API int hn_device_sm_count(int device);

/* ---------------------------------------------------------------------------
 * Packing (replaces ExpertWeightPacker.quantize_tensor / dequantize_tensor,
 * preprocess/pack_weights.py:133-181 and :230-268).
 * ------------------------------------------------------------------------- */

/* w [rows, cols] (fp32 or fp16, w_dtype) -> packed [rows, cols/2], scales
 * [rows, cols/group] fp16.  Bit-identical to the reference packer. */
HN_API int hn_quantize_int4(const void* w, int w_dtype, int64_t rows, int64_t cols, int group_size,
                     uint8_t* packed, uint16_t* scales, void* stream);

/* Raw nibbles 0..15 as uint8 [rows, cols] (debug/parity helper). */
HN_API int hn_unpack_int4(const uint8_t* packed, int64_t rows, int64_t cols, uint8_t* out, void* stream);

/* fp16 dequantisation (nibble - 8) * scale, as GpuExpertSlot._dequant_tensor
 * (cache/packed_expert_store.py:287-315).  out: fp16 [rows, cols]. */
HN_API int hn_dequant_int4(const uint8_t* packed, const uint16_t* scales, int64_t rows, int64_t cols,
                    int group_size, uint16_t* out, void* stream);

/* ---------------------------------------------------------------------------
 * Drop-in kernels (kernels/int4_gemm.py, kernels/int4_expert_mlp.py)
 * ------------------------------------------------------------------------- */

/* silu(gate) * up, elementwise, fp32 math, output in dtype
 * (replaces fused_silu_mul, kernels/int4_gemm.py:196-208, and silu_mul,
 * kernels/int4_expert_mlp.py:189-210). */
HN_API int hn_silu_mul(const void* gate, const void* up, void* out, int64_t n, int dtype, void* stream);

/* out[M, N] = x[M, K] @ W^T with W given packed (replaces int4_linear,
 * kernels/int4_gemm.py:124-172 and kernels/int4_expert_mlp.py:99-156).
 * ldx / ldo are row strides in elements. */
HN_API size_t hn_int4_linear_workspace_size(int64_t M, int64_t N, int64_t K);
HN_API int hn_int4_linear(const void* x, int64_t ldx, int dtype, int64_t M, int64_t K,
                   const uint8_t* w_packed, const uint16_t* w_scales, int64_t N, int group_size,
                   void* out, int64_t ldo, void* workspace, size_t workspace_bytes, void* stream);

/* out[T, H] = down(silu(gate(x)) * up(x)) in one fused two-phase pass
 * (replaces expert_mlp_int4_fused, kernels/int4_gemm.py:211-254, and
 * expert_mlp_int4 / expert_mlp_int4_from_slot, kernels/int4_expert_mlp.py:213-272). */
HN_API size_t hn_expert_mlp_workspace_size(int64_t T, int64_t H, int64_t F);
HN_API int hn_expert_mlp_int4(const void* x, int dtype, int64_t T, int64_t H, int64_t F,
                       const uint8_t* gate_packed, const uint16_t* gate_scales,
                       const uint8_t* up_packed, const uint16_t* up_scales,
                       const uint8_t* down_packed, const uint16_t* down_scales, int group_size,
                       void* out, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Grouped MoE layer: router + dispatch + expert MLPs + weighted top-k combine
 * (replaces TopKRouter.forward / GLM4SigmoidRouter.forward and the per-expert
 * loops of MixtralMoELayer.forward, model/mixtral.py:259-370, and
 * GLM4MoELayer.forward, model/glm4.py:365-473, routed part).
 * ------------------------------------------------------------------------- */

typedef struct hn_router_params {
  int kind;                 /* hn_router_kind                                    */
  int top_k;
  const void* weight;       /* [E, H] router weight                              */
  int weight_dtype;         /* hn_dtype of weight                                */
  int logits_in_act_dtype;  /* 1: round logits to the activation dtype before use
                               (Mixtral gate Linear runs in the model dtype,
                               model/router.py:102); 0: float32 logits            */
  const float* affinity_bonus; /* [E] or NULL: cache-affinity bonus per expert,
                               applied when the normalised entropy exceeds
                               entropy_threshold (model/router.py:132-175)         */
  float entropy_threshold;
  const float* correction_bias; /* [E] or NULL (sigmoid only): added to the scores
                               for selection only                                  */
  int norm_topk_prob;       /* sigmoid only (model/glm4.py:302-304)              */
  float routed_scaling_factor; /* sigmoid only (model/glm4.py:307)                */
  int n_group;              /* sigmoid only: group-limited routing when n_group > 1
                               and topk_group > 0 (model/glm4.py:285-297): the E
                               experts form n_group equal groups (n_group <= 32),
                               each scored by its best selection score; only the
                               topk_group best groups' experts keep their scores,
                               the others score 0 (ties: lower group index)       */
  int topk_group;
} hn_router_params;

HN_API size_t hn_moe_workspace_size(int64_t T, int64_t H, int64_t F, int64_t E, int top_k);

/* Number of kernel launches one hn_moe_layer_int4 call of this shape makes
 * (host-only query, no GPU needed; 0 for invalid sizes).  Three always (the
 * route/plan kernel, gate/up, down), plus one router-logits kernel from 256
 * tokens (when x and the router rows are 16-byte aligned) or when the router
 * has more than 32 Ki weights (E * H > 32768, e.g. GLM-4.5's 128 x 4096), the
 * assignment-ordered token copy when experts get >= 12 assignments on average
 * on the tcgen05 engine, the multi-CTA planner above 1024 (token, slot)
 * pairs and the combine pass above 4096. */
HN_API int hn_moe_layer_launches(int64_t T, int64_t H, int64_t F, int64_t E, int top_k);

/* TMA descriptors of an expert table (what the grouped ops stream weights
 * with): hn_expert_maps_bytes() bytes per expert (384).  hn_expert_maps_encode
 * fills a 64-byte aligned HOST buffer of E entries from a HOST copy of the
 * pointer table; copy it to device memory and pass it as expert_maps.  The
 * descriptors embed the weight addresses: re-encode when a slot moves (a slot
 * refilled in place keeps its descriptors).  Host-only, launches nothing. */
HN_API size_t hn_expert_maps_bytes(void);
HN_API int hn_expert_maps_encode(const hn_expert_ptrs* host_table, int64_t E, int64_t H, int64_t F,
                                 void* host_out);

/* x [T, H] -> out [T, H] = sum_k w[t,k] * MLP_{idx[t,k]}(x[t]).
 * experts: DEVICE pointer to E hn_expert_ptrs; expert_maps: DEVICE pointer to
 * their E TMA descriptors (hn_expert_maps_encode).  Optional outputs (may be NULL):
 * topk_idx int32 [T, k], topk_w float32 [T, k] (already rounded to the
 * activation dtype, as model/router.py:120 and model/glm4.py:309 cast them),
 * logits float32 [T, E]. */
HN_API int hn_moe_layer_int4(const void* x, int dtype, int64_t T, int64_t H, int64_t F, int64_t E,
                      const hn_router_params* router, const hn_expert_ptrs* experts, const void* expert_maps,
                      void* out, int32_t* topk_idx, float* topk_w, float* logits,
                      void* workspace, size_t workspace_bytes, void* stream);

/* hn_moe_layer_int4 split into its three launches, for callers that put
 * work between them (communication of an expert-parallel layer) or time them
 * separately: phase 1 = routing, activation staging and the dispatch plan;
 * 2 = gate/up projections with SiLU(gate)*up; 3 = down projection and the
 * weighted combine into out.  The state between phases lives in the
 * workspace: issuing phases 1, 2, 3 in order on one stream with identical
 * arguments computes exactly what one hn_moe_layer_int4 call computes.
 * No counterpart in the reference (its layer is a Python loop). */
HN_API int hn_moe_layer_int4_phase(int phase, const void* x, int dtype, int64_t T, int64_t H, int64_t F, int64_t E,
                                   const hn_router_params* router, const hn_expert_ptrs* experts,
                                   const void* expert_maps, void* out, int32_t* topk_idx, float* topk_w,
                                   float* logits, void* workspace, size_t workspace_bytes, void* stream);

/* Same as hn_moe_layer_int4 but with routing supplied by the caller
 * (topk_idx int32 [T, k], topk_w float32 [T, k]); used for expert-parallel
 * shards and for callers that route on their own.  An index of -1 marks an
 * unused slot: it takes no expert work and adds nothing to its token's sum; a
 * token whose k slots are all -1 is skipped (its output row is left
 * unspecified).  Other indices outside [0, E) are read as expert 0 and set
 * error code 2 in the workspace's error word (hn_workspace_error). */
HN_API int hn_moe_experts_int4(const void* x, int dtype, int64_t T, int64_t H, int64_t F, int64_t E,
                        int top_k, const int32_t* topk_idx, const float* topk_w,
                        const hn_expert_ptrs* experts, const void* expert_maps, void* out,
                        void* workspace, size_t workspace_bytes, void* stream);

/* hn_moe_experts_int4 for a block of rows of which only some slots hold an
 * expert (no counterpart in the reference: the rows an expert-parallel
 * exchange delivers, where about T * top_k / W of the slots are this rank's):
 * expected_assignments (> 0) is the caller's estimate of the slots that hold
 * an expert, from which the token-segment width is chosen instead of
 * T * top_k (0: the same as hn_moe_experts_int4).  The result does not depend
 * on the estimate, only the speed; the workspace is sized by
 * hn_moe_experts_workspace_size_expected with the same estimate. */
HN_API size_t hn_moe_experts_workspace_size_expected(int64_t T, int64_t H, int64_t F, int64_t E, int top_k,
                                                     int64_t expected_assignments);
HN_API int hn_moe_experts_int4_expected(const void* x, int dtype, int64_t T, int64_t H, int64_t F, int64_t E,
                                        int top_k, const int32_t* topk_idx, const float* topk_w,
                                        const hn_expert_ptrs* experts, const void* expert_maps, void* out,
                                        int64_t expected_assignments, void* workspace, size_t workspace_bytes,
                                        void* stream);

/* Router only: writes topk_idx/topk_w (and logits if non-NULL). */
HN_API int hn_moe_route(const void* x, int dtype, int64_t T, int64_t H, int64_t E,
                 const hn_router_params* router, int32_t* topk_idx, float* topk_w, float* logits,
                 void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Expert-parallel exchange (no counterpart in the reference, which runs every
 * expert on one GPU; its roadmap lists expert parallelism, README.md:179).
 * Rank r of W owns experts [r*E/W, (r+1)*E/W).  A step is: hn_ep_pack ->
 * all-to-all of W equal blocks -> hn_ep_unpack -> hn_moe_experts_int4 over the
 * W*T received rows (top_k slots of local ids, -1 = not here) -> all-to-all of
 * the W*T output rows back -> hn_ep_combine.  Every block holds T fixed rows,
 * one per source token (sent at most once per destination rank), so nothing
 * depends on counts the host would have to read.
 * ------------------------------------------------------------------------- */

/* Bytes of one exchange row: H activations (2 bytes each), top_k int32 local
 * expert ids and top_k float32 weights, rounded up to 16 bytes. */
HN_API size_t hn_ep_row_bytes(int64_t H, int top_k);

/* send [W][T][row]: block d, row t = token t's activations (only when one of
 * its picks lives on rank d) and its top-k list as rank d's local ids (-1
 * where the pick lives elsewhere) with the routing weights (0 there).
 * topk_idx int32 [T, top_k] global expert ids (-1 = unused slot), topk_w
 * float32 [T, top_k].  x and send 16-byte aligned. */
HN_API int hn_ep_pack(const void* x, int dtype, int64_t T, int64_t H, int top_k, const int32_t* topk_idx,
                      const float* topk_w, int64_t E, int world, void* send, void* stream);

/* recv [rows][row] -> x_out [rows, H] (rows without a local pick are left
 * unwritten), idx_out int32 [rows, top_k], w_out float32 [rows, top_k]. */
HN_API int hn_ep_unpack(const void* recv, int dtype, int64_t rows, int64_t H, int top_k, void* x_out,
                        int32_t* idx_out, float* w_out, void* stream);

/* out [T, H] = sum over the ranks d holding a pick of token t (in rank order,
 * fp32) of back [d][t][H]; back rows of other ranks are never read. */
HN_API int hn_ep_combine(const void* back, int dtype, int64_t T, int64_t H, int top_k, const int32_t* topk_idx,
                         int64_t E, int world, void* out, void* stream);

/* ---------------------------------------------------------------------------
 * Allocation-free int4_linear.  No counterpart in the reference: its Python
 * kernels allocate through PyTorch on every call.
 *
 * hn_int4_linear_static computes what hn_int4_linear computes, with the same
 * arguments minus the workspace.  Its scratch is an array of
 * HN_INT4_LINEAR_STATIC_SCRATCH_BYTES (16 MiB) compiled into this library:
 * the CUDA runtime creates one zero-filled copy per device when it loads the
 * library's module there, and the call itself allocates nothing.  It is meant
 * for callers that have no device memory to hand over, for example a host
 * that binds only this C ABI through an FFI and owns no CUDA allocator, or a
 * serving runtime that has given all free HBM to its caches, so that a
 * cudaMalloc on the decode path would fail or wait for the whole device.
 *
 *  - Token segments are capped at the widest of 32, 16 or 8 rows whose
 *    scratch fits the array.  Shapes whose
 *    hn_int4_linear_static_scratch_size(M, N, K) is still larger than the
 *    array are refused with HN_ERR_WORKSPACE (for example M = 64 with
 *    K = 14336 fits; M = 4096 with K = 14336 does not).  The query is
 *    host-only and needs no GPU.
 *  - Every call looks up the array's address on the current device and
 *    context (cudaGetSymbolAddress; host code cannot use the array's name as
 *    a device address).  The first lookup on a device may load the library's
 *    module there, so make the first call on each device before any stream
 *    capture.  A failure there is returned as HN_ERR_CUDA.
 *  - What must be zero: the array's first 512 bytes (an error word and an
 *    arrival counter) when a call starts.  They are zero after loading and
 *    stay zero unless a bounded device wait of a call timed out (segments of
 *    up to 16 rows run on the mma.sync engine, which has no such wait; the
 *    tcgen05 engine's waits are bounded).  hn_int4_linear_static_error reads the error word and
 *    clears it; results of calls issued while it was set are undefined.
 *  - There is ONE array per device, shared by every caller of this function.
 *    Two calls that may overlap on the device (streams with no ordering
 *    between them, or host threads racing on different streams) overwrite
 *    each other's scratch and produce wrong results.  Issue them on one
 *    stream, or use hn_int4_linear with one workspace per stream.
 * ------------------------------------------------------------------------- */
#define HN_INT4_LINEAR_STATIC_SCRATCH_BYTES ((size_t)16 << 20)
HN_API int hn_int4_linear_static(const void* x, int64_t ldx, int dtype, int64_t M, int64_t K,
                                 const uint8_t* w_packed, const uint16_t* w_scales, int64_t N, int group_size,
                                 void* out, int64_t ldo, void* stream);
/* Scratch bytes hn_int4_linear_static needs for this shape (0 for invalid
 * sizes); calls whose need exceeds HN_INT4_LINEAR_STATIC_SCRATCH_BYTES are
 * refused.  Host-only. */
HN_API size_t hn_int4_linear_static_scratch_size(int64_t M, int64_t N, int64_t K);
/* The static array's device error word on the current device: copies 4 bytes
 * device->host on 'stream', synchronises that stream, and clears the word if
 * it was set (as hn_workspace_error does for a workspace). */
HN_API int hn_int4_linear_static_error(int* error_code, void* stream);

/* Engine for segments of at most 32 tokens per expert (decode sizes).  No
 * counterpart in the reference.  HN_ENGINE_AUTO (the default) runs them on
 * the register-dequant mma.sync engine; HN_ENGINE_TCGEN05 runs them on the
 * tcgen05 engine that larger segments always use.  Both compute the same
 * function (fp32 accumulation of float16 tokens times exact n - 8 weights;
 * they differ only in where the group scale is applied), so the switch exists
 * for side-by-side measurement and parity tests.  Process-wide; applies to
 * calls issued after it returns, including the workspace-size and launch
 * queries.  Returns the previous engine, or -1 with HN_ERR_INVALID recorded
 * in hn_last_error for an unknown value. */
enum hn_engine { HN_ENGINE_AUTO = 0, HN_ENGINE_TCGEN05 = 1 };
HN_API int hn_set_decode_engine(int engine);

/* Grids of the grouped kernels are sized for at most max_sms SMs from the
 * next call on (0: all of the device's; process-wide; returns the previous
 * limit, or -1 for a negative argument).  No counterpart in the reference.
 * The persistent kernels otherwise hold every SM for their whole run, so a
 * collective issued beside them (an expert-parallel exchange on NCCL's
 * stream) cannot start until they end; leaving a few SMs free lets it run
 * alongside.  Results do not depend on the limit; workspaces sized under one
 * limit serve calls under any smaller one. */
HN_API int hn_set_sm_limit(int max_sms);

/* ---------------------------------------------------------------------------
 * Expert slot residency (host only, launches nothing): which (layer, expert)
 * occupies which of num_slots device slots of an over-budget expert cache.
 * The reference keeps this bookkeeping in Python per layer
 * (cache/expert_cache.py, ExpertCacheManager's tiers); here one table serves
 * all layers.  hn_slots_admit makes the n given experts of `layer` resident
 * (ids < 0 are ignored, duplicates count once, processed in ascending id
 * order): it writes one (slot, expert) pair per expert to load into `loads`
 * and one (layer, expert) pair per evicted expert into `evicted` (each at
 * most 2 * num_slots ints), sets *n_evicted and returns the number of loads;
 * a call needing more experts than there are slots changes nothing and
 * returns -HN_ERR_WORKSPACE.  Eviction takes, among the slots the call does
 * not need, a free one, else the least frequently used (HN_SLOTS_LFU: a use
 * count per (layer, expert), halved every decay_every uses, ties to the least
 * recent) or the least recently used (HN_SLOTS_LRU); ties to the lower slot.
 * Thread-safe per handle.  No counterpart in the reference's C API.
 * ------------------------------------------------------------------------- */
enum hn_slots_policy { HN_SLOTS_LFU = 0, HN_SLOTS_LRU = 1 };
typedef struct hn_slots hn_slots;
HN_API hn_slots* hn_slots_create(int num_slots, int policy, int64_t decay_every);
HN_API void hn_slots_destroy(hn_slots* slots);
HN_API int hn_slots_admit(hn_slots* slots, int layer, const int32_t* experts, int n, int32_t* loads,
                          int32_t* evicted, int* n_evicted);
/* Slot of (layer, expert), or -1 when it is not resident. */
HN_API int hn_slots_lookup(hn_slots* slots, int layer, int expert);
/* hits, misses and evictions so far, into out3[0..2]. */
HN_API int hn_slots_stats(hn_slots* slots, int64_t* out3);

/* Device-side error word of a workspace (bounded waits that timed out set it).
 * Copies 4 bytes device->host on 'stream' and synchronises that stream. */
HN_API int hn_workspace_error(const void* workspace, size_t workspace_bytes, int* error_code, void* stream);

/* Self-test of the failure path (no reference counterpart).  Launches one CTA
 * whose bounded waits wait on a barrier that nothing arrives at (mode 0: the
 * engine's polling wait and its backoff wait; mode 1: two backoff waits).
 * After the wait limit (2 s) the kernel records the timeout (error code 1)
 * in the workspace's error word and ends; hn_workspace_error then reports it.
 * Needs a workspace of >= 512 bytes whose first 4 bytes are zero.  With
 * workspace NULL it uses the error word of hn_int4_linear_static's array on
 * the current device instead (read back with hn_int4_linear_static_error). */
HN_API int hn_selftest_wait_timeout(void* workspace, size_t workspace_bytes, int mode, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* HYDRANET_B200_H */
