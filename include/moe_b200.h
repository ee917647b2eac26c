/*
 * moe_b200.h — C ABI of the B200 (sm_100a) fused Mixture-of-Experts operator.
 *
 * Conventions (the contest online judge's CUDA C ABI for this operator,
 * xpuoj_data/evaluation_guide.md:79-97):
 *   - every tensor is a device pointer (`void*`) to contiguous, row-major memory on the current
 *     CUDA device; integers are int64_t; `stream` is a cudaStream_t (NULL = legacy default);
 *   - calls are stream-ordered and asynchronous: no entry point synchronises the device or the
 *     stream, except moe_device_status();
 *   - the caller owns every buffer, including the scratch `workspace` (size from the matching
 *     *_workspace_bytes query); outputs are the only memory written besides the workspace;
 *   - every entry point returns 0 on success or a negative moe_status_t, and never aborts; the
 *     message of the last failure on the calling thread is returned by moe_last_error();
 *   - the library holds no mutable state other than per-device launch-attribute flags, a
 *     per-device SM-count cache and the per-device status word below.
 *
 * Element types (`dtype` arguments): MOE_F16 / MOE_BF16 for activations, weights and outputs,
 * MOE_F32 / MOE_F16 / MOE_BF16 for routing weights, MOE_I32 / MOE_I64 for expert ids.
 */
#ifndef MOE_B200_H_
#define MOE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MOE_API __attribute__((visibility("default")))
#else
#define MOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  MOE_F16 = 0,
  MOE_BF16 = 1,
  MOE_F32 = 2,
  MOE_I32 = 3,
  MOE_I64 = 4,
  MOE_I8 = 5,
  MOE_F8E4M3 = 6
} moe_dtype_t;

typedef enum {
  MOE_OK = 0,
  MOE_ERR_INVALID_ARG = -1,  /* bad shape, count or dtype */
  MOE_ERR_UNSUPPORTED = -2,  /* valid request this build does not implement */
  MOE_ERR_ALIGNMENT = -3,    /* pointer or row pitch not 16-byte aligned */
  MOE_ERR_CUDA = -4,         /* a CUDA runtime/driver call failed */
  MOE_ERR_WORKSPACE = -5     /* workspace missing or smaller than the query returned */
} moe_status_t;

/* Library version string. */
MOE_API const char* moe_version(void);

/* Message of the last failed call on this thread ("" if none). */
MOE_API const char* moe_last_error(void);

/* Reads (and with `clear` != 0 resets) the device status word of the current device after
 * synchronising `stream`: bit 0 = a bounded pipeline wait gave up, bit 1 = an expert index
 * outside [0, E) was met, bit 2 = a route index outside [0, R), bit 3 = the single-kernel MoE's
 * Stage2 gave up waiting for its rows' Stage1 results. 0 means every kernel since the
 * last clear completed normally. No reference counterpart (the reference has no device-side
 * error reporting). */
MOE_API int moe_device_status(void* stream, int clear, uint32_t* status_out);

/* Profiling hook, no reference counterpart. While set on the calling thread, moe_fused and
 * moe_fused_int8 record the given cudaEvent_t handles on their stream at stage boundaries:
 *   [0] before alignment, [1] after alignment, [2] after the gather, [3] after Stage1,
 *   [4] after Stage2 (int8: [4] after the intermediate requantisation, [5] after Stage2).
 * Events beyond n are not recorded. events = NULL or n = 0 turns the hook off. */
MOE_API int moe_set_profile_events(void* const* events, int n);

/* Tuning hook, no reference counterpart (the reference picks TileLang tiles per shape in
 * _pick_tiles, 初审材料/源代码/submission.py:1990-2079). Selects the grouped-GEMM tile
 * configuration of `stage` (1 = gate/up, 2 = down, 0 = both) by name for all later calls in the
 * process, e.g. "256a4b5" (single CTA, 256 accumulator columns, A/B ring depths 4/5) or
 * "p256a6b8" (CTA pair, cta_group::2); NULL or "auto" restores the per-call choice. Unknown names
 * return MOE_ERR_INVALID_ARG. Configurations a call cannot run (e.g. shapes that do not split
 * into whole k-blocks) fall back to the stage's single-CTA default. */
MOE_API int moe_set_tile(int stage, const char* name);

/* Tuning hook, no reference counterpart (the reference's Stage1 reads the stacked token rows of
 * its caller). Selects how the fused entry points' Stage1 loads its token rows, for all later
 * calls in the process: "tma" (a gather kernel stacks the routed rows, TMA boxes read the
 * stack), "gather" (TMA tile::gather4 loads of the token rows inside Stage1, no stacked copy) or
 * "lsu" (cp.async gather inside Stage1); NULL or "auto" restores the default. The workspace a
 * call needs depends on the path (the *_workspace_bytes functions follow the selection), so
 * switch paths only between calls whose workspaces are sized after the switch. Unknown names
 * return MOE_ERR_INVALID_ARG. The expert-parallel peer-memory mode always stacks its rows. */
MOE_API int moe_set_a_path(const char* name);

/* Selects, for all later calls in the process, whether Stage1 and Stage2 of moe_run_kernel and
 * moe_fused run as one kernel: 0 = two launches, 1 = the single kernel wherever it applies, 2 =
 * automatic, the default (the single kernel where it applies and the call averages fewer than 1.8
 * routing blocks of 128 rows per expert; the environment variable MOE_B200_SINGLE_KERNEL=0|1|2
 * sets the initial mode). The reference fuses nothing across its two stages; its one attempt at a
 * single-kernel MoE is xpuoj_data/probe_v236_fused_single_kernel.py. The single kernel is one
 * cooperative launch: each SM moves on to Stage2 units as soon as its own Stage1 units are done,
 * and a Stage2 unit waits (bounded; status bit 3 on timeout) until every Stage1 column tile of
 * its rows has been stored. It applies where both stages would run their default single-CTA tiles
 * on the TMA path: 16-bit routes without the ordered combine or expert-parallel peer memory, with
 * no tile forced by moe_set_tile and the default A path; other calls keep the two launches. Other
 * values return MOE_ERR_INVALID_ARG. */
MOE_API int moe_set_single_kernel(int mode);

/* ------------------------------------------------------------------------------------------
 * Reference drop-in: the contest operator.
 * Replaces run_kernel(stacked_expert_tokens, gate_w, up_w, down_w, routed_expert_weights,
 * group_sizes, group_offsets, group_padded_offsets, group_idx_for_bx, out)
 * (初审材料/源代码/submission.py:2098-2184; problem statement xpuoj_data/problem1_contest5.json,
 * interface section), with the shape scalars the Python entry point reads from tensor shapes
 * (:2110-2115) passed explicitly, as the contest online judge's C ABI does for `int` arguments.
 *
 *   stacked_expert_tokens [P, H]  dtype   (expert-grouped, padded to 128 rows per expert)
 *   gate_w, up_w          [E, I, H] dtype
 *   down_w                [E, H, I] dtype
 *   routed_expert_weights [R]     routed_dtype (MOE_F32 or MOE_F16), real-token order
 *   group_sizes [E], group_offsets [E+1], group_padded_offsets [E+1], group_idx_for_bx [P/128]  int32
 *   out                   [P, H]  dtype   (written in full: pad rows = 0)
 * Empty inputs follow the reference (:2117-2153): P == 0 writes nothing, R == 0 zero-fills out.
 * Route indices are clamped to [0, R-1] as in :935-947.
 * Requirements: H % 8 == 0, I % 8 == 0, P == 128 * num_blocks_m, 16-byte aligned pointers.
 * workspace >= moe_run_kernel_workspace_bytes(P, I, dtype) (the reference's cached up_logits
 * [P, I] buffer, :2081-2095).
 * ---------------------------------------------------------------------------------------- */
MOE_API size_t moe_run_kernel_workspace_bytes(int64_t total_padded_tokens, int64_t intermediate, int dtype);

MOE_API int moe_run_kernel(const void* stacked_expert_tokens, const void* gate_w, const void* up_w, const void* down_w,
                   const void* routed_expert_weights, int routed_dtype, const int32_t* group_sizes,
                   const int32_t* group_offsets, const int32_t* group_padded_offsets,
                   const int32_t* group_idx_for_bx, void* out, int64_t total_padded_tokens, int64_t hidden,
                   int64_t intermediate, int64_t num_experts, int64_t total_valid_tokens, int64_t num_blocks_m,
                   int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* moe_run_kernel for callers that cannot allocate device memory. This entry point has no
 * counterpart in the reference. Some callers have no way to hand the operator a scratch buffer:
 * the contest online judge, which binds `run_kernel` through the C ABI, passes only the operator's
 * own tensors and integers (xpuoj_data/evaluation_guide.md:79-97), and calling cudaMalloc inside a
 * timed or captured loop is not an option. Here the Stage1 intermediate lives in a buffer of
 * MOE_NOALLOC_WORKSPACE_BYTES that the library itself holds in static device memory: every GPU
 * that loads the library keeps those 64 MiB until the process exits. The call allocates nothing.
 *   - Same arguments and results as moe_run_kernel, without workspace / workspace_bytes.
 *   - Problems needing more than MOE_NOALLOC_WORKSPACE_BYTES (moe_run_kernel_workspace_bytes of
 *     P and I; about P * I * 2 bytes, e.g. P <= 16384 padded rows at I = 2048) fail with
 *     MOE_ERR_WORKSPACE and a message giving both sizes.
 *   - The first call on a device looks up the buffer's device address (once per device, with that
 *     device current); make that first call before any stream capture.
 *   - All calls on a device share the one buffer, which keeps the previous call's contents
 *     (nothing in it needs to start at zero). Calls that overlap on the GPU (different streams,
 *     no ordering between them) race on it: order them, or use moe_run_kernel. */
#define MOE_NOALLOC_WORKSPACE_BYTES (64u * 1024u * 1024u)

MOE_API int moe_run_kernel_noalloc(const void* stacked_expert_tokens, const void* gate_w, const void* up_w,
                                   const void* down_w, const void* routed_expert_weights, int routed_dtype,
                                   const int32_t* group_sizes, const int32_t* group_offsets,
                                   const int32_t* group_padded_offsets, const int32_t* group_idx_for_bx, void* out,
                                   int64_t total_padded_tokens, int64_t hidden, int64_t intermediate,
                                   int64_t num_experts, int64_t total_valid_tokens, int64_t num_blocks_m, int dtype,
                                   void* stream);

/* ------------------------------------------------------------------------------------------
 * Routing alignment on the device.
 * Replaces the metadata construction the reference's callers run in torch before run_kernel
 * (初审材料/源代码/benchmark/remote_bench.py:82-101, race_stress2.py:65-69): histogram of the
 * flat top-k ids, cumsum, ceil to block_m, repeat_interleave — plus the row permutation
 * (sorted_route_ids, a stable argsort of the ids; route_slot, its inverse).
 *
 *   topk_ids [R] (ids_dtype MOE_I32 / MOE_I64); ids outside [0, E) are skipped
 *   group_sizes [E], group_offsets [E+1], group_padded_offsets [E+1]       int32
 *   group_idx_for_bx [moe_max_padded_rows(R,E,block_m) / block_m] int32 (may be NULL)
 *   sorted_route_ids [moe_max_padded_rows(R,E,block_m)] int32, pad rows hold R
 *   route_slot [R] int32 (-1 for skipped ids)
 *   meta [4] int32: {P, P / block_m, valid routes, 0}
 * Requirements: 1 <= E <= 1024, block_m >= 1.
 * ---------------------------------------------------------------------------------------- */
MOE_API int64_t moe_max_padded_rows(int64_t num_routes, int64_t num_experts, int64_t block_m);
MOE_API size_t moe_align_workspace_bytes(int64_t num_routes, int64_t num_experts);

MOE_API int moe_align(const void* topk_ids, int ids_dtype, int64_t num_routes, int64_t num_experts, int64_t block_m,
              int32_t* group_sizes, int32_t* group_offsets, int32_t* group_padded_offsets,
              int32_t* group_idx_for_bx, int32_t* sorted_route_ids, int32_t* route_slot, int32_t* meta,
              void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------
 * Fused MoE on token-major tensors (the routed expert MLP with routing, grouping and the top-k
 * combine included). Mathematically the reference operator (problem1_contest5.json, PyTorch
 * reference section) applied to the stacked layout that moe_align builds, followed by the
 * weighted sum over each token's top-k routes that the reference leaves to its caller:
 *   out[t] = sum_j topk_weights[t, j] * Down_e(silu(Gate_e x_t) * Up_e x_t),  e = topk_ids[t, j]
 *
 *   hidden_states [T, H] dtype;  w_gate_up [E, 2I, H] dtype (rows 0..I-1 gate, I..2I-1 up);
 *   w_down [E, H, I] dtype;  topk_ids [T, topk] ids_dtype;  topk_weights [T, topk] weights_dtype;
 *   out [T, H] dtype.
 * No device synchronisation: block counts stay on the device.
 * Requirements: H % 8 == 0, I % 8 == 0, 1 <= E <= 1024.
 * ---------------------------------------------------------------------------------------- */
MOE_API size_t moe_fused_workspace_bytes(int64_t num_tokens, int64_t topk, int64_t num_experts, int64_t hidden,
                                 int64_t intermediate, int dtype);

MOE_API int moe_fused(const void* hidden_states, const void* w_gate_up, const void* w_down, const void* topk_ids,
              int ids_dtype, const void* topk_weights, int weights_dtype, void* out, int64_t num_tokens,
              int64_t hidden, int64_t intermediate, int64_t num_experts, int64_t topk, int dtype,
              void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------
 * moe_fused_ordered: moe_fused with a deterministic top-k combine (no reference counterpart: the
 * reference writes the padded per-route rows and leaves the combine to its caller). Stage2 runs
 * in the reference's padded-store form (submission.py:317-357) into a workspace buffer, then
 * out[t] = sum over j = 0 .. topk-1 of those rows, accumulated in fp32 in route order and
 * rounded once: bitwise the same result on every run. Arguments as moe_fused; workspace:
 * moe_fused_ordered_workspace_bytes (moe_fused's plus P_max * H * 2 + T * topk * 4 bytes).
 * ---------------------------------------------------------------------------------------- */
MOE_API size_t moe_fused_ordered_workspace_bytes(int64_t num_tokens, int64_t topk, int64_t num_experts,
                                                 int64_t hidden, int64_t intermediate, int dtype);

MOE_API int moe_fused_ordered(const void* hidden_states, const void* w_gate_up, const void* w_down,
                              const void* topk_ids, int ids_dtype, const void* topk_weights, int weights_dtype,
                              void* out, int64_t num_tokens, int64_t hidden, int64_t intermediate,
                              int64_t num_experts, int64_t topk, int dtype, void* workspace, size_t workspace_bytes,
                              void* stream);

/* ------------------------------------------------------------------------------------------
 * Router: softmax top-k of router logits, the step that produces topk_ids / topk_weights for the
 * fused MoE (no reference counterpart: the reference receives its routing pre-built; the
 * synthetic workloads route by softmax -> top-k -> renormalise, as tests/golden/cases.py:118-129
 * does with torch).
 *
 * moe_router_topk: logits [T, E] logits_dtype (MOE_F32 / MOE_F16 / MOE_BF16) ->
 *   topk_ids [T, topk] int32 in descending logit order (equal logits: lower expert id first;
 *   the order of fp32 values, +0 above -0), topk_weights [T, topk] fp32 =
 *   softmax(logits)[ids], divided by their sum when renormalize != 0.
 *   Requirements: 1 <= topk <= min(E, 32), 1 <= E <= 1024; logits finite.
 * moe_fused_router: moe_router_topk followed by moe_fused on its output, with the router kernel
 *   also building the alignment's expert histogram (one pass fewer). topk_ids / topk_weights are
 *   caller buffers and hold the routing afterwards. Workspace: moe_fused_workspace_bytes.
 * ---------------------------------------------------------------------------------------- */
MOE_API int moe_router_topk(const void* logits, int logits_dtype, int64_t num_tokens, int64_t num_experts,
                            int64_t topk, int renormalize, int32_t* topk_ids, float* topk_weights, void* stream);

/* moe_router_grouped_topk: group-limited sigmoid routing (the DeepSeek-V3 router). s =
 *   sigmoid(logits); selection scores c = s + bias (bias [E] fp32, or NULL); the experts form
 *   n_group equal groups, each scored by the sum of its two largest c; the topk_group best groups
 *   stay eligible; topk_ids = the topk largest c among their experts (descending; same total order
 *   and tie rule as moe_router_topk); topk_weights = s at those ids, divided by their sum (+1e-20)
 *   when renormalize != 0, times scale.
 *   Requirements: 1 <= n_group <= 32, E % n_group == 0, 1 <= topk_group <= n_group,
 *   1 <= topk <= min(32, topk_group * E / n_group). */
MOE_API int moe_router_grouped_topk(const void* logits, int logits_dtype, const float* bias, int64_t num_tokens,
                                    int64_t num_experts, int64_t n_group, int64_t topk_group, int64_t topk,
                                    int renormalize, float scale, int32_t* topk_ids, float* topk_weights,
                                    void* stream);

MOE_API int moe_fused_router(const void* hidden_states, const void* w_gate_up, const void* w_down,
                             const void* logits, int logits_dtype, int renormalize, int32_t* topk_ids,
                             float* topk_weights, void* out, int64_t num_tokens, int64_t hidden,
                             int64_t intermediate, int64_t num_experts, int64_t topk, int dtype, void* workspace,
                             size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------
 * W8A8 int8 route. Semantics of the reference's int8 experiment
 * (xpuoj_data/submission_v322_int8_v2.py:164-205 weight quantisation, :207-232 activation
 * quantisation, :234-454 int8 GEMMs with int32 accumulation and dequantisation), with one scale
 * per weight output row and per token instead of per expert / fixed.
 *
 * moe_quantize_rows_int8: q[r, :] = round_half_away(w[r, :] * 127 / amax_r), scale[r] = amax_r/127,
 *   w [rows, K] dtype -> q [rows, K] int8, scale [rows] fp32. Used offline on the weights.
 * moe_fused_int8: as moe_fused, with w13_q [E, 2I, H] int8 + w13_scale [E*2I] fp32 and
 *   w2_q [E, H, I] int8 + w2_scale [E*H] fp32; activations quantised per token on the device;
 *   the Stage1 intermediate is re-quantised per row; int32 accumulation; `dtype` output.
 * Requirements: H % 16 == 0, I % 16 == 0, 1 <= E <= 1024.
 * ---------------------------------------------------------------------------------------- */
MOE_API int moe_quantize_rows_int8(const void* w, int dtype, int64_t rows, int64_t cols, void* q, float* scale,
                           void* stream);

MOE_API size_t moe_fused_int8_workspace_bytes(int64_t num_tokens, int64_t topk, int64_t num_experts, int64_t hidden,
                                      int64_t intermediate, int dtype);

MOE_API int moe_fused_int8(const void* hidden_states, const void* w13_q, const float* w13_scale, const void* w2_q,
                   const float* w2_scale, const void* topk_ids, int ids_dtype, const void* topk_weights,
                   int weights_dtype, void* out, int64_t num_tokens, int64_t hidden, int64_t intermediate,
                   int64_t num_experts, int64_t topk, int dtype, void* workspace, size_t workspace_bytes,
                   void* stream);

/* ------------------------------------------------------------------------------------------
 * W8A8 fp8 (e4m3) route: the int8 route's scheme with e4m3 values (no reference counterpart; the
 * reference probed fp8 MMA code generation only, xpuoj_data/probe_v209_fp8_mma.py:1).
 * moe_quantize_rows_fp8: scale[r] = amax_r / 448, q[r, :] = e4m3(w[r, :] * (448 / amax_r)),
 *   rounded to nearest even and saturated to +-448; q holds the e4m3 bytes.
 * moe_fused_fp8: as moe_fused_int8 with fp8 weights and per-token fp8 activations; tcgen05
 *   kind::f8f6f4 with fp32 accumulation. Runs on the TMA A path only.
 * Requirements: H % 16 == 0, I % 16 == 0, 1 <= E <= 1024.
 * ---------------------------------------------------------------------------------------- */
MOE_API int moe_quantize_rows_fp8(const void* w, int dtype, int64_t rows, int64_t cols, void* q, float* scale,
                                  void* stream);

MOE_API size_t moe_fused_fp8_workspace_bytes(int64_t num_tokens, int64_t topk, int64_t num_experts, int64_t hidden,
                                             int64_t intermediate, int dtype);

MOE_API int moe_fused_fp8(const void* hidden_states, const void* w13_q, const float* w13_scale, const void* w2_q,
                          const float* w2_scale, const void* topk_ids, int ids_dtype, const void* topk_weights,
                          int weights_dtype, void* out, int64_t num_tokens, int64_t hidden, int64_t intermediate,
                          int64_t num_experts, int64_t topk, int dtype, void* workspace, size_t workspace_bytes,
                          void* stream);

/* ------------------------------------------------------------------------------------------
 * Packed weights: one buffer holding an expert set in the layout the fused kernels read (no
 * reference counterpart: the reference takes gate_w, up_w [E, I, H] and down_w [E, H, I] as
 * separate tensors on every call, 初审材料/源代码/submission.py:2098-2109). Sections, each
 * starting on a 256-byte boundary, in this order:
 *   w13       [E, 2I, H] kind   expert e's gate rows (0..I-1) then its up rows (I..2I-1): one
 *                               TMA stream and one [gate | up] accumulator per tile
 *   w13_scale [E * 2I] fp32     8-bit kinds only: per-row scales
 *   w2        [E, H, I] kind
 *   w2_scale  [E * H] fp32      8-bit kinds only
 * kind = MOE_F16 / MOE_BF16 (the activation dtype, weights copied), MOE_I8 or MOE_F8E4M3
 * (quantised per row as moe_quantize_rows_int8 / _fp8 do). The layout depends only on (E, H, I,
 * kind), so a packed buffer can be written to a file and mapped back.
 * moe_packed_weights_layout: byte offsets of the four sections (absent scales: offset of the
 *   next section, size 0) and the total size; returns MOE_ERR_INVALID_ARG for a bad kind/shape.
 * moe_pack_weights: fills `packed` from the reference layout (gate_w, up_w, down_w in `dtype`).
 * moe_fused_packed: moe_fused / moe_fused_int8 / moe_fused_fp8 on the packed weights;
 *   workspace: moe_fused_packed_workspace_bytes.
 * ---------------------------------------------------------------------------------------- */
MOE_API int moe_packed_weights_layout(int64_t num_experts, int64_t hidden, int64_t intermediate, int kind,
                                      size_t offsets_out[4], size_t* total_bytes_out);

MOE_API int moe_pack_weights(const void* gate_w, const void* up_w, const void* down_w, int dtype,
                             int64_t num_experts, int64_t hidden, int64_t intermediate, int kind, void* packed,
                             size_t packed_bytes, void* stream);

MOE_API size_t moe_fused_packed_workspace_bytes(int64_t num_tokens, int64_t topk, int64_t num_experts,
                                                int64_t hidden, int64_t intermediate, int kind, int dtype);

MOE_API int moe_fused_packed(const void* hidden_states, const void* packed, int kind, const void* topk_ids,
                             int ids_dtype, const void* topk_weights, int weights_dtype, void* out,
                             int64_t num_tokens, int64_t hidden, int64_t intermediate, int64_t num_experts,
                             int64_t topk, int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------
 * Expert-parallel building blocks (no reference counterpart: the reference runs on one GPU;
 * these wrap the NCCL all-to-all exchange that muxi_race_b200/ep.py issues through
 * torch.distributed). Experts are owned by ranks: expert_rank [E], expert_local [E] int32.
 *
 * moe_ep_plan: pairs (token t, rank r) such that t routes to an expert of r, sorted by r then t.
 *   send_counts [W], send_offsets [W+1] int32; send_pairs [T*W] int32 (t*W + r of each send row);
 *   pair_slot [T*W] int32 (send row of pair t*W + r, or -1); meta [4] int32 = {n, n, n, 0},
 *   n = number of send rows. workspace >= moe_ep_plan_workspace_bytes(T, W).
 * moe_ep_pack: send row p < n gets the token row (send_x [T*W, H] dtype), its top-k expert ids
 *   rewritten to the destination's local ids or -1 (send_ids [T*W, topk] int32) and its weights
 *   (send_w [T*W, topk] fp32).
 * moe_ep_combine: out[t] = sum over r of y[pair_slot[t*W + r]] (y [n, H] dtype, fp32 sum).
 * Requirements: 1 <= W <= 1024, H % 8 == 0.
 * ---------------------------------------------------------------------------------------- */
MOE_API size_t moe_ep_plan_workspace_bytes(int64_t num_tokens, int64_t world);

MOE_API int moe_ep_plan(const void* topk_ids, int ids_dtype, int64_t num_tokens, int64_t topk,
                        const int32_t* expert_rank, int64_t num_experts, int64_t world, int32_t* send_counts,
                        int32_t* send_offsets, int32_t* send_pairs, int32_t* pair_slot, int32_t* meta,
                        void* workspace, size_t workspace_bytes, void* stream);

MOE_API int moe_ep_pack(const void* hidden_states, const void* topk_ids, int ids_dtype, const void* topk_weights,
                        int weights_dtype, const int32_t* expert_rank, const int32_t* expert_local,
                        int64_t num_experts, const int32_t* send_pairs, const int32_t* meta, int64_t num_tokens,
                        int64_t hidden, int64_t topk, int64_t world, int dtype, void* send_x, int32_t* send_ids,
                        float* send_w, void* stream);

MOE_API int moe_ep_combine(const void* y, const int32_t* pair_slot, int64_t num_tokens, int64_t hidden,
                           int64_t world, int dtype, void* out, void* stream);

/* ------------------------------------------------------------------------------------------
 * Expert parallelism over peer memory. No reference counterpart (the reference runs on one
 * device); the same operator as moe_fused, with its experts sharded over W ranks (one process per
 * GPU of one node, NVLink peer access), and no collectives library or host synchronisation on
 * the data path.
 *
 * Every rank owns one region of moe_ep_region_bytes(T_max, hidden, topk, W) bytes from
 * moe_ep_region_alloc (device memory, zeroed), exports it with moe_ep_ipc_get (a 64-byte CUDA IPC
 * handle) and maps every peer's region with moe_ep_ipc_open. `regions` below is a DEVICE array of
 * W uint64 addresses: rank q's region as mapped in this process (this rank's own at [rank]).
 * A forward on every rank, in this order, on one stream:
 *   moe_ep_p2p_stage    copy this rank's hidden_states [T, H], topk_ids [T, k] (int32/int64) and
 *                       topk_weights [T, k] (fp32/fp16/bf16) into its region (T <= T_max);
 *   moe_ep_p2p_barrier  epoch e (increasing by one per barrier, starting at 1);
 *   moe_ep_p2p_compute  (own_region = this rank's region, as allocated) route every rank's
 *                       (token, slot) pairs whose expert this rank owns to its
 *                       local experts (expert_rank / expert_local: [E] int32 device arrays),
 *                       gather those token rows from the peers, run Stage1 / Stage2 with the
 *                       local weights w_gate_up [E_local, 2I, H] / w_down [E_local, H, I], and
 *                       combine each token's local routes into this rank's region;
 *   moe_ep_p2p_barrier  epoch e + 1;
 *   moe_ep_p2p_combine  out [T, H] = for each token, the sum over the ranks owning its experts of
 *                       their partial rows (read from their regions, ascending rank order).
 * A rank's region must not be freed or staged again before every rank has passed the second
 * barrier of the forward. Requirements: 1 <= W <= 32, dtype MOE_F16 / MOE_BF16, H % 8 == 0.
 * Barrier waits are bounded (60 s, far above any legitimate skew between the ranks' host threads;
 * status bit 0 on timeout).
 * ---------------------------------------------------------------------------------------- */
MOE_API size_t moe_ep_region_bytes(int64_t max_tokens, int64_t hidden, int64_t topk, int64_t world);
MOE_API int moe_ep_region_alloc(size_t bytes, void** region);
MOE_API int moe_ep_region_free(void* region);
MOE_API int moe_ep_ipc_get(const void* region, void* handle_64_bytes);
MOE_API int moe_ep_ipc_open(const void* handle_64_bytes, void** region);
MOE_API int moe_ep_ipc_close(void* region);

MOE_API int moe_ep_p2p_stage(void* region, const void* hidden_states, const void* topk_ids, int ids_dtype,
                             const void* topk_weights, int weights_dtype, int64_t num_tokens, int64_t max_tokens,
                             int64_t hidden, int64_t topk, int64_t world, int dtype, void* stream);

MOE_API int moe_ep_p2p_barrier(const uint64_t* regions, int rank, int world, uint32_t epoch, void* stream);

MOE_API size_t moe_ep_p2p_workspace_bytes(int64_t max_tokens, int64_t topk, int64_t world, int64_t local_experts,
                                          int64_t hidden, int64_t intermediate, int dtype);

MOE_API int moe_ep_p2p_compute(const uint64_t* regions, void* own_region, int rank, int world, int64_t max_tokens,
                               int64_t hidden, int64_t intermediate, int64_t topk, const int32_t* expert_rank,
                               const int32_t* expert_local, int64_t num_experts, const void* w_gate_up_local,
                               const void* w_down_local, int64_t local_experts, int dtype, void* workspace,
                               size_t workspace_bytes, void* stream);

MOE_API int moe_ep_p2p_combine(const uint64_t* regions, int rank, int world, int64_t num_tokens, int64_t max_tokens,
                               int64_t hidden, int64_t topk, const int32_t* expert_rank, int64_t num_experts,
                               int dtype, void* out, void* stream);

/* Push combine (alternative to moe_ep_p2p_combine): Stage2's epilogue stores every route's weighted
 * row into its slot t * k + j of its token's home rank's y block over NVLink, overlapping the GEMM
 * (plain 16-byte stores: each slot has one writer), and fences at system scope before its kernel
 * ends. Per forward, on one stream:
 *   moe_ep_p2p_stage, moe_ep_p2p_push_prepare (argument checks; nothing needs clearing),
 *   moe_ep_p2p_barrier(epoch), moe_ep_p2p_compute_push, moe_ep_p2p_barrier(epoch + 1),
 *   moe_ep_p2p_push_finish (sums each own token's slots with an expert id in [0, num_experts), in
 *   slot order, fp32, into out).
 * Same arguments as moe_ep_p2p_compute / the region layout. */
MOE_API int moe_ep_p2p_push_prepare(void* own_region, int64_t num_tokens, int64_t max_tokens, int64_t hidden,
                                    int64_t topk, int world, int dtype, void* stream);
MOE_API int moe_ep_p2p_compute_push(const uint64_t* regions, void* own_region, int rank, int world,
                                    int64_t max_tokens, int64_t hidden, int64_t intermediate, int64_t topk,
                                    const int32_t* expert_rank, const int32_t* expert_local, int64_t num_experts,
                                    const void* w13_local, const void* w2_local, int64_t local_experts, int dtype,
                                    void* workspace, size_t workspace_bytes, void* stream);
MOE_API int moe_ep_p2p_push_finish(const void* own_region, int64_t num_tokens, int64_t max_tokens, int64_t hidden,
                                   int64_t topk, int world, int64_t num_experts, int dtype, void* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H_ */
