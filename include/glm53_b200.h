/*
 * glm53_b200.h -- C ABI of the B200 (sm_100a) FP8 block-scaled MoE hot path.
 *
 * Conventions
 *   - Every entry point is `extern "C"`, takes plain device pointers, sizes
 *     and a `cudaStream_t` passed as `void*` (NULL = legacy default stream),
 *     and returns an int status: GLM53_OK or one of the GLM53_ERR_* codes.
 *     glm53_last_error() returns a thread-local message for the last failure.
 *   - BF16 tensors are passed as `void*` (16-bit storage), E4M3 weights as
 *     `uint8_t*` codes, block scales (`weight_scale_inv`) as `float*` on the
 *     128x128 grid, expert ids as `uint32_t*`, route weights as `float*`.
 *   - All tensors are row-major contiguous.  No entry point allocates device
 *     memory: callers pass workspace sized by the *_workspace_bytes queries.
 *   - Status mapping used by the Python layer: GLM53_ERR_INVALID -> ValueError,
 *     GLM53_ERR_INDEX -> IndexError, GLM53_ERR_CUDA -> RuntimeError.
 *   - Device-side fail-closed signals (expert id >= expert count, a bounded
 *     wait that gave up) are OR-ed into an optional `uint32_t* status` word in
 *     device memory instead of trapping (bits GLM53_STATUS_*).
 *
 * Reference citations are paths inside kiojuvr/glm53-flash-mlx.
 */
#ifndef GLM53_B200_H_
#define GLM53_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GLM53_OK 0
#define GLM53_ERR_INVALID 1
#define GLM53_ERR_CUDA 2
#define GLM53_ERR_INDEX 3

#define GLM53_STATUS_BAD_EXPERT 1u
#define GLM53_STATUS_WAIT_TIMEOUT 2u
#define GLM53_STATUS_BAD_GEOMETRY 4u

/* `flags` bit: the caller guarantees that the E4M3 weights contain no code
 * 0x7F or 0xFF (true of every E4M3FN checkpoint, where those codes are NaN;
 * checked once at bind time with glm53_e4m3_scan).  The kernels then decode
 * with the hardware conversion.  Without it they decode with an exact bit
 * re-bias that also maps 0x7F/0xFF to +-480 as the reference table does. */
#define GLM53_FLAG_E4M3_FINITE 1u

/* `flags` bits of glm53_packed_decode_moe that split one decode into two
 * calls on the same workspace, so that the shared expert (which needs no
 * routing) can run on a second stream while the router runs:
 * GLM53_FLAG_SHARED_ONLY computes only the shared expert (expert_ids and
 * scores are not read) and leaves its down partial in the workspace;
 * GLM53_FLAG_SKIP_SHARED then computes the routed slots and the final reduce,
 * adding that partial.  The second call's down stage must be ordered after
 * the first call (e.g. an event join).  Together they give the same bits as
 * one call.  (Measured on B200 inside one CUDA graph with the router between
 * them, the fork/join edges cost more than the overlap gains; the split is for
 * callers that overlap the shared expert with longer work of their own.) */
#define GLM53_FLAG_SHARED_ONLY 2u
#define GLM53_FLAG_SKIP_SHARED 4u

/* `flags` bit of glm53_packed_decode_moe: the kernel launched just before this
 * call on the same stream is the glm53_router_topk that produced expert_ids
 * and scores (or a kernel that only converts them).  The gate/up stage is then
 * launched as a programmatic dependent of it: the shared expert's rows, which
 * need no routing, stream while the router still runs, and the routed rows
 * wait on the device for the router's results.  The caller guarantees that x
 * and the workspace are not written by that previous kernel.  Same bits as
 * without the flag; ignored together with the split flags. */
#define GLM53_FLAG_AFTER_ROUTER 8u

/* `flags` bit of glm53_grouped_moe (with GLM53_FLAG_E4M3_FINITE): run the
 * grouped GEMMs on the FP8 tensor-core kernel (tcgen05 kind::f8f6f4).  The
 * E4M3 weights feed the MMA directly; each activation row is held as two E4M3
 * terms hi + lo of x * 2^-e (row maximum scaled into [128, 256)), exact for
 * every element within 2^9 of its row maximum, and the hidden rows between
 * gate/up and down stay BF16.  Ignored without GLM53_FLAG_E4M3_FINITE or when
 * a projection's shape does not fit the kernel (K % 128, K <= 4096; SwiGLU
 * hidden % 128; plain outputs % 256), which then runs the kind::f16 kernel. */
#define GLM53_FLAG_F8_MMA 16u

/* Kernel ABI identity string (replaces glm53_flash_mlx/abi.py:3-15 for the
 * CUDA kernels; part of any cache identity that depends on kernel numerics). */
const char* glm53_kernel_abi(void);

/* Message describing the last non-OK status returned on this thread. */
const char* glm53_last_error(void);

/* y[M,N] (BF16) = x[M,K] (BF16) @ dequant(w[N,K] E4M3, scale_inv[ceil(N/128),
 * ceil(K/128)])^T with FP32 accumulation.
 * Replaces block_fp8_linear, glm53_flash_mlx/fp8.py:254-299 (kernels K1/K2,
 * fp8.py:41-116). */
int glm53_fp8_linear(const void* x, int64_t M, int64_t K, const uint8_t* w,
                     int64_t N, const float* scale_inv, void* y, uint32_t flags,
                     void* stream);

/* Workspace bytes of glm53_fp8_linear_ws for M rows of width K. */
size_t glm53_fp8_linear_workspace_bytes(int64_t M, int64_t K);

/* Workspace bytes of glm53_fp8_linear_ws for M x K rows and N outputs with
 * room for split-K partial sums: when the tcgen05 GEMM has fewer output tiles
 * (128 rows x 128 outputs) than half the SMs, each tile's K is cut into ranges
 * computed by different CTAs and the FP32 partials are added in range order
 * by a second kernel (deterministic; a valid FP32 summation order of the same
 * products).  A workspace of only glm53_fp8_linear_workspace_bytes runs
 * without the split. */
size_t glm53_fp8_linear_splitk_workspace_bytes(int64_t M, int64_t K, int64_t N);

/* glm53_fp8_linear with caller scratch: for M > 16 rows, K % 128 == 0, N % 8
 * == 0 and 16-byte aligned x / w / workspace it runs the tcgen05 GEMM (the
 * activations converted once to FP16 x 2^-e rows in the workspace; exact FP16
 * weight products, FP32 promotion per 128-K block); otherwise it is
 * glm53_fp8_linear.  `status` (device word) receives GLM53_STATUS_WAIT_TIMEOUT
 * if a bounded wait gave up.  Same results contract as glm53_fp8_linear.
 * Replaces block_fp8_linear at large M, glm53_flash_mlx/fp8.py:254-299 (K2,
 * fp8.py:73-116). */
int glm53_fp8_linear_ws(const void* x, int64_t M, int64_t K, const uint8_t* w, int64_t N,
                        const float* scale_inv, void* y, void* workspace, size_t workspace_bytes,
                        uint32_t* status, uint32_t flags, void* stream);

/* One replay of a captured decode step with host buffers, as one call:
 * copy x_bytes from x_host into the graph's static input x_dev, launch
 * graph_exec (a cudaGraphExec_t, e.g. a captured router + packed decode), and
 * copy out_bytes of its static output out_dev into out_host (skipped when
 * out_host is NULL), all stream-ordered on `stream`.  Pinned host buffers
 * keep the copies asynchronous.  Serves CapturedDecode's host-buffer step
 * (the per-token PackedFP8MoE call, glm53_flash_mlx/packed.py:896-923, with
 * the input and result on the host). */
int glm53_graph_step(void* graph_exec, const void* x_host, void* x_dev, size_t x_bytes, const void* out_dev,
                     void* out_host, size_t out_bytes, void* stream);

/* Count (into *nan_count, device memory, accumulated) the 4-byte words of
 * w[n] that hold an E4M3 code 0x7F or 0xFF; zero means GLM53_FLAG_E4M3_FINITE
 * may be passed for these weights.  w must be 16-byte aligned.
 * Counterpart of the bind-time fail-closed scan the reference's table
 * (glm53_flash_mlx/fp8.py:22-39, 0x7F/0xFF = +-480) calls for. */
int glm53_e4m3_scan(const uint8_t* w, int64_t n, uint32_t* nan_count, void* stream);

/* Workspace bytes needed by glm53_router_topk for T tokens and E experts. */
size_t glm53_router_workspace_bytes(int64_t T, int64_t E);

/* FP32 router: logits = f32(x[T,H]) @ w[E,H]^T; s = sigmoid(logits);
 * choice = s + bias; optional group mask (n_group/topk_group); top_k of
 * choice (slot order: descending choice, ties to the lower expert id);
 * scores = s[idx], normalised over the top_k when norm_topk_prob, times
 * routed_scaling_factor.  logits may be NULL.
 * Up to 64 tokens every logit is summed in FP64 (the products of BF16
 * activations and FP32 weights are exact there) and rounded once to FP32:
 * one CTA per expert row up to 8 tokens, FP64 tensor-core tiles of 8 experts
 * x 8 tokens for 9..64 (H a multiple of 1024, up to 8192), so a token routed
 * alone and in such a batch may differ in a logit's last FP32 bit.  Larger
 * batches use BF16-split tensor-core tiles with FP64 sums of the K ranges.
 * Replaces Float32Gate.__call__, glm53_flash_mlx/patch.py:131-142, and the
 * mlx-vlm group_expert_select it calls. */
int glm53_router_topk(const void* x, int64_t T, int64_t H, const float* w,
                      int64_t E, const float* bias, int top_k, int n_group,
                      int topk_group, int norm_topk_prob,
                      float routed_scaling_factor, uint32_t* indices,
                      float* scores, float* logits, void* workspace,
                      size_t workspace_bytes, void* stream);

/* Workspace bytes needed by glm53_packed_decode_moe (and its gate/up stage).
 * The workspace must be zero-filled before its first use; every call leaves
 * its completion counters at zero again. */
size_t glm53_packed_decode_workspace_bytes(int top_k, int64_t H, int64_t I, int64_t I_shared);

/* Byte offsets, inside that workspace, of the intermediates a call leaves
 * there: offsets[0] = the SwiGLU hidden rows (BF16 [top_k * I + I_shared],
 * slot-major, the shared expert last), offsets[1] = the down projections
 * before rounding (FP32 [(top_k + 1) * H], slot-major, the shared expert
 * last).  For inspection (the parity tests certify every rounding site from
 * them); no reference counterpart. */
int glm53_packed_decode_workspace_layout(int top_k, int64_t H, int64_t I, int64_t I_shared, size_t* offsets);

/* One-token packed decode MoE over a packed expert bank:
 *   bank: gate_up_w [E,2I,H] (gate rows [0,I), up rows [I,2I)),
 *         gate_up_s [E, 2*ceil(I/128), ceil(H/128)],
 *         down_w [E,H,I], down_s [E, ceil(H/128), ceil(I/128)];
 *   shared expert (all six pointers NULL and I_shared 0 when absent):
 *         gate/up [I_shared,H] + scales, down [H,I_shared] + scale.
 * out[H] = BF16(sum_j f32(down_j) * scores[j]) (+ shared, BF16 add), with the
 * exact BF16 SwiGLU rounding of the reference.
 * Replaces PackedFP8MoE.__call__ decode, glm53_flash_mlx/packed.py:896-923
 * (kernels K7/K6/K8/K9 at packed.py:66-235 and the shared down K1). */
int glm53_packed_decode_moe(const void* x, int64_t H, const uint32_t* expert_ids,
                            const float* scores, int top_k,
                            const uint8_t* gate_up_w, const float* gate_up_s,
                            const uint8_t* down_w, const float* down_s,
                            int64_t E, int64_t I, const uint8_t* shared_gate_w,
                            const float* shared_gate_s, const uint8_t* shared_up_w,
                            const float* shared_up_s, const uint8_t* shared_down_w,
                            const float* shared_down_s, int64_t I_shared,
                            float limit, void* out, void* workspace,
                            size_t workspace_bytes, uint32_t* status,
                            uint32_t flags, void* stream);

/* The same decode over separately allocated experts: gate_w[j], gate_s[j],
 * up_w[j], up_s[j] ([I,H] + [ceil(I/128), ceil(H/128)]) and down_w[j],
 * down_s[j] ([H,I] + scales) are host arrays of top_k device pointers, one
 * per routed slot, in slot order; no expert-id indirection on the device.
 * Replaces DirectFP8MoE's selected top-8 decode, glm53_flash_mlx/fp8.py:
 * 372-383 (kernels K3/K4, fp8.py:142-251). */
int glm53_selected_decode_moe(const void* x, int64_t H, const float* scores, int top_k,
                              const uint8_t* const* gate_w, const float* const* gate_s,
                              const uint8_t* const* up_w, const float* const* up_s,
                              const uint8_t* const* down_w, const float* const* down_s,
                              int64_t I, const uint8_t* shared_gate_w,
                              const float* shared_gate_s, const uint8_t* shared_up_w,
                              const float* shared_up_s, const uint8_t* shared_down_w,
                              const float* shared_down_s, int64_t I_shared, float limit,
                              void* out, void* workspace, size_t workspace_bytes,
                              uint32_t* status, uint32_t flags, void* stream);

/* glm53_packed_decode_moe followed by the layer's mHC post-expand, in the same
 * two launches: the final reduce writes, instead of the MoE row moe[h], the 4
 * branches of the next residual state,
 *   out_state[b][h] = BF16(post[b] * moe[h] + sum_s comb[s][b] * residual[s][h]),
 * with the FMA chain over the 4 sources and the rounded post product added
 * last -- bit for bit what glm53_packed_decode_moe then glm53_hc_expand give.
 * residual / out_state BF16 [4, H] (they may not alias), post FP32 [4], comb
 * FP32 [4][4] (comb[source][branch]).  The FFN half of a GLM-5.3 decode layer
 * (mlp, then hc_expand: scripts/trace_grouped_fp8_route_amplification.py:
 * 178-214; the expand of native_indexer_plan.metal:2362-2389) without a third
 * launch.  Tensor-core shapes only (H, I, I_shared multiples of 128); flags
 * as glm53_packed_decode_moe except GLM53_FLAG_SHARED_ONLY (no output). */
int glm53_packed_decode_moe_hc(const void* x, int64_t H, const uint32_t* expert_ids, const float* scores,
                               int top_k, const uint8_t* gate_up_w, const float* gate_up_s,
                               const uint8_t* down_w, const float* down_s, int64_t E, int64_t I,
                               const uint8_t* shared_gate_w, const float* shared_gate_s,
                               const uint8_t* shared_up_w, const float* shared_up_s,
                               const uint8_t* shared_down_w, const float* shared_down_s, int64_t I_shared,
                               float limit, const void* residual, const float* post, const float* comb,
                               void* out_state, void* workspace, size_t workspace_bytes, uint32_t* status,
                               uint32_t flags, void* stream);

/* Size of the fixed scratch area of glm53_packed_decode_moe_static_scratch:
 * 1 MiB of device memory on every device that loads the library, held until
 * the process exits. */
#define GLM53_STATIC_SCRATCH_BYTES (1u << 20)

/* glm53_packed_decode_moe without a workspace argument: it allocates no device
 * memory.  No counterpart in the reference; it exists for callers that cannot
 * allocate at call time (an engine whose own pool already holds all of device
 * memory, or a decode loop where an allocation's possible device
 * synchronisation is not acceptable).  Same arguments, layouts and results as
 * glm53_packed_decode_moe.  Its scratch is one fixed array per device of
 * GLM53_STATIC_SCRATCH_BYTES: a call whose glm53_packed_decode_workspace_bytes
 * (top_k, H, I, I_shared) exceeds that returns GLM53_ERR_INVALID (config 2,
 * top_k 8, H 4096, I = I_shared = 1536, needs 176 KiB).  The calling thread's
 * current device must own `stream` and the pointers; the first call on each
 * device looks up the array's address (cudaGetSymbolAddress), so make that
 * first call before any stream capture.  Each call clears the array's
 * completion counters on `stream` before its kernels run; because that clear
 * sits between a router and this decode on the stream, GLM53_FLAG_AFTER_ROUTER
 * is rejected with GLM53_ERR_INVALID (the other flags are honoured).  All
 * calls on one device share the array, so calls whose GPU work overlaps (other
 * streams, other host threads) race and must be serialised by the caller. */
int glm53_packed_decode_moe_static_scratch(const void* x, int64_t H, const uint32_t* expert_ids,
                                           const float* scores, int top_k,
                                           const uint8_t* gate_up_w, const float* gate_up_s,
                                           const uint8_t* down_w, const float* down_s,
                                           int64_t E, int64_t I, const uint8_t* shared_gate_w,
                                           const float* shared_gate_s, const uint8_t* shared_up_w,
                                           const float* shared_up_s, const uint8_t* shared_down_w,
                                           const float* shared_down_s, int64_t I_shared,
                                           float limit, void* out, uint32_t* status,
                                           uint32_t flags, void* stream);

/* One token through one packed MoE layer (router + packed decode), with the
 * input and the result in host memory: what PackedFP8MoE's per-token call
 * (glm53_flash_mlx/packed.py:896-923, gate at patch.py:131-142) computes for
 * a host row, as one library call.  `d` describes the layer and the caller's
 * device buffers (all pointers device memory unless stated).  The call
 *   1. copies H BF16 values from x_host into d->x: a kernel reads the host
 *      row through its device mapping when x_host is pinned (page-locked by
 *      the CUDA runtime), else cudaMemcpyAsync;
 *   2. runs glm53_router_topk on d->x into d->expert_ids / d->scores (launched
 *      as a programmatic dependent of the copy kernel, waiting for it);
 *   3. runs glm53_packed_decode_moe with GLM53_FLAG_AFTER_ROUTER, writing the
 *      result straight into out_host through its device mapping when out_host
 *      is pinned, else into d->out followed by a copy to out_host (or only
 *      into d->out when out_host is NULL).
 * x_host NULL: d->x already holds the input (no copy; the router waits for
 * nothing).  Results are those of the separate calls; every step is ordered
 * on `stream`.  Requires top_k == 8 and H, I (and I_shared when non-zero)
 * multiples of 128. */
typedef struct glm53_decode_step_desc {
  int64_t H, E, I, I_shared;
  int top_k, n_group, topk_group, norm_topk_prob;
  float routed_scaling_factor, limit;
  uint32_t flags;               /* GLM53_FLAG_E4M3_FINITE or 0 */
  const float* router_w;        /* [E, H] FP32 */
  const float* router_bias;     /* [E] FP32 */
  const uint8_t* gate_up_w;
  const float* gate_up_s;
  const uint8_t* down_w;
  const float* down_s;
  const uint8_t* shared_gate_w; /* shared expert, or NULL when I_shared == 0 */
  const float* shared_gate_s;
  const uint8_t* shared_up_w;
  const float* shared_up_s;
  const uint8_t* shared_down_w;
  const float* shared_down_s;
  void* x;                      /* [H] BF16: the step's input row */
  uint32_t* expert_ids;         /* [top_k] */
  float* scores;                /* [top_k] */
  void* out;                    /* [H] BF16 */
  void* router_workspace;
  size_t router_workspace_bytes;
  void* decode_workspace;
  size_t decode_workspace_bytes;
  uint32_t* status;
  uint32_t* status_host;        /* pinned host word or NULL: before its own kernels
                                   run, each call copies *status (the bits of every
                                   earlier call on the stream) into it */
} glm53_decode_step_desc;

int glm53_decode_step_host(const glm53_decode_step_desc* d, const void* x_host, void* out_host, void* stream);

/* Copies the device status word into `host_word`, a 4-byte word of pinned
 * (page-locked, device-mapped) host memory, in stream order: once the work
 * enqueued before this call has run, the host reads the fail-closed bits
 * (GLM53_STATUS_*) with a plain memory read, without synchronising the
 * device.  This is how the Python modules raise the reference's IndexError /
 * RuntimeError (glm53_flash_mlx/packed.py:868-876; the device-side
 * invalid-route counter of native_indexer_plan.metal:1880-1900) at their next
 * call rather than never.  GLM53_ERR_INVALID when host_word is not mapped. */
int glm53_status_mirror(const uint32_t* status, uint32_t* host_word, void* stream);

/* Bound, in nanoseconds of device time, of the expert-parallel peer waits
 * (glm53_ep_owner_decode_p2p's arrival wait, glm53_ep_combine_p2p's row
 * wait) for kernels launched after this call, process-wide; 0 restores the
 * default of two seconds; values outside [1 ms, 60 s] are GLM53_ERR_INVALID.
 * A wait that reaches the bound sets GLM53_STATUS_WAIT_TIMEOUT and its kernel
 * returns.  No reference counterpart (the reference runs on one device); it
 * lets a test make a wait run out in milliseconds. */
int glm53_set_wait_limit_ns(unsigned long long ns);

/* Workspace bytes needed by glm53_routes_decode for R route slots. */
size_t glm53_routes_decode_workspace_bytes(int64_t R, int64_t H, int64_t I);

/* Per-route decode, the expert owner's half of expert-parallel decode: for
 * every slot r, out_rows[r] = BF16 of expert expert_ids[r]'s
 * down(SwiGLU(gate . x_r, up . x_r)) (the K7 + K6 arithmetic of
 * glm53_packed_decode_moe for one slot, bit-identical to its per-slot value),
 * with x_r = x_rows[r] (BF16 [R,H]).  Slots whose id is 0xFFFFFFFF are empty
 * and skipped (their rows are left untouched); other ids >= E raise
 * GLM53_STATUS_BAD_EXPERT.  Bank layout as glm53_packed_decode_moe; H and I
 * multiples of 128.  Replaces the owner-side expert loop of the expert-
 * parallel layout the reference's Direct/packed modules run on one device
 * (glm53_flash_mlx/packed.py:896-923, per slot). */
int glm53_routes_decode(const void* x_rows, int64_t R, int64_t H, const uint32_t* expert_ids,
                        const uint8_t* gate_up_w, const float* gate_up_s,
                        const uint8_t* down_w, const float* down_s, int64_t E, int64_t I,
                        float limit, void* out_rows, void* workspace, size_t workspace_bytes,
                        uint32_t* status, uint32_t flags, void* stream);

/* Workspace bytes of glm53_routes_decode_coalesced for R slots over E experts. */
size_t glm53_routes_decode_coalesced_workspace_bytes(int64_t R, int64_t E, int64_t H, int64_t I);

/* glm53_routes_decode with expert coalescing: the slots are sorted by expert
 * on the device (glm53_route_plan, descriptors of up to 4 slots) and each
 * descriptor streams its expert's weights once for all of its slots (the
 * batched decode's kernels), writing each slot's BF16 down row at its own
 * position: the same bits as glm53_routes_decode.  Slots whose id is >= E
 * (the empty mark 0xFFFFFFFF among them) are skipped and their rows left
 * untouched.  R <= 4096, H and I multiples of 128, 16-byte aligned tensors.
 * The expert owner's half of batched expert-parallel decode (config 4 at
 * B = 16 / 64 per rank): the reference's cross-request batching with expert
 * coalescing (glm-5.3-flash-m3-ultra-runtime-architecture-2026-08-27.md:
 * 183-188), over the packed bank of glm53_flash_mlx/packed.py:747-876. */
int glm53_routes_decode_coalesced(const void* x_rows, int64_t R, int64_t H, const uint32_t* expert_ids,
                                  const uint8_t* gate_up_w, const float* gate_up_s, const uint8_t* down_w,
                                  const float* down_s, int64_t E, int64_t I, float limit, void* out_rows,
                                  void* workspace, size_t workspace_bytes, uint32_t* status, uint32_t flags,
                                  void* stream);

/* Direct-module combine of a small decode batch: out[t] = the BF16 sum, in
 * ascending expert id of token t's top_k routes, of BF16(f32(rows[t*top_k+j])
 * * scores[t*top_k+j]) (each add rounded to BF16), then + shared[t] (BF16 add;
 * shared may be NULL).  rows BF16 [T*top_k, H] (e.g. from glm53_routes_decode),
 * expert_ids / scores [T*top_k], out BF16 [T, H]; H % 8 == 0, 16-byte aligned
 * rows.  Replaces the expert-bucket scatter-add of DirectFP8MoE.__call__,
 * glm53_flash_mlx/fp8.py:384-399. */
int glm53_direct_combine(const void* rows, const uint32_t* expert_ids, const float* scores, int64_t T,
                         int top_k, int64_t H, const void* shared, void* out, void* stream);

/* Workspace bytes of glm53_batched_decode_moe. */
size_t glm53_batched_decode_workspace_bytes(int64_t T, int top_k, int64_t E, int64_t H, int64_t I);

/* A small decode batch (T tokens, T * top_k <= 4096 routes) through the packed
 * bank with the Direct module's multi-row semantics: the routes are sorted by
 * expert on the device (glm53_route_plan, descriptors of up to 8 routes), each
 * descriptor streams its expert's weights once for all its routes (per-route
 * values identical to glm53_routes_decode), and glm53_direct_combine's BF16
 * scatter-add in ascending expert id adds them per token, then `shared`
 * (BF16 [T, H], the shared expert's output, or NULL).  Route ids >= E are
 * skipped and raise GLM53_STATUS_BAD_EXPERT.  H, I multiples of 128.
 * Replaces DirectFP8MoE.__call__'s expert loop for more than one row,
 * glm53_flash_mlx/fp8.py:384-399. */
int glm53_batched_decode_moe(const void* x, int64_t T, int64_t H, const uint32_t* expert_ids,
                             const float* scores, int top_k, const uint8_t* gate_up_w,
                             const float* gate_up_s, const uint8_t* down_w, const float* down_s,
                             int64_t E, int64_t I, float limit, const void* shared, void* out,
                             void* workspace, size_t workspace_bytes, uint32_t* status,
                             uint32_t flags, void* stream);

/* Workspace bytes of glm53_batched_decode_moe_shared. */
size_t glm53_batched_decode_shared_workspace_bytes(int64_t T, int top_k, int64_t E, int64_t H, int64_t I);

/* glm53_batched_decode_moe with the shared expert computed in the same
 * coalesced kernels instead of passed in as BF16 rows: every token gets one
 * more route, to the shared expert (gate [I, H], up [I, H], down [H, I] E4M3
 * with their 128x128 block scales; its intermediate size equals the routed
 * experts' I) with weight 1.0.  Its weighted BF16 row is the shared expert's
 * BF16 output exactly, and the ascending-id combine adds it last, after the
 * routed experts, as DirectFP8MoE.__call__ adds the shared output
 * (glm53_flash_mlx/fp8.py:384-397).  The shared expert's weights stream once
 * per 4 tokens (L2 hits after the first).  Same limits as
 * glm53_batched_decode_moe with top_k < 32. */
int glm53_batched_decode_moe_shared(const void* x, int64_t T, int64_t H, const uint32_t* expert_ids,
                                    const float* scores, int top_k, const uint8_t* gate_up_w,
                                    const float* gate_up_s, const uint8_t* down_w, const float* down_s,
                                    int64_t E, int64_t I, const uint8_t* shared_gate_w,
                                    const float* shared_gate_s, const uint8_t* shared_up_w,
                                    const float* shared_up_s, const uint8_t* shared_down_w,
                                    const float* shared_down_s, float limit, void* out, void* workspace,
                                    size_t workspace_bytes, uint32_t* status, uint32_t flags, void* stream);

/* Expert-parallel dispatch packing on the tokens' home rank.  Experts are
 * split into `world` contiguous ranges of E / world; route (t, j) with expert
 * e goes to rank d = e / (E / world), into the next free of `capacity` slots
 * of destination d (slots in route order t * top_k + j):
 *   send_x [world * capacity, H] BF16 = the token's row,
 *   send_expert [world * capacity] = e - d * (E / world) or 0xFFFFFFFF (empty),
 *   slot_scores [world * capacity] = the route's score (kept home),
 *   route_pos [T * top_k] = d * capacity + slot (0xFFFFFFFF when dropped).
 * capacity >= T * top_k never drops; a drop raises GLM53_STATUS_BAD_GEOMETRY.
 * The exchange is an all-to-all of equal `capacity`-slot chunks (NCCL on the
 * host).  No counterpart in the reference (single device); it implements the
 * expert-parallel dispatch its MoE layer is to run with across GPUs. */
int glm53_ep_dispatch_pack(const void* x, int64_t T, int64_t H, const uint32_t* expert_ids,
                           const float* scores, int top_k, int64_t E, int world,
                           int64_t capacity, void* send_x, uint32_t* send_expert,
                           float* slot_scores, uint32_t* route_pos, uint32_t* status,
                           void* stream);

/* Expert-parallel combine on the home rank: out[t] = BF16(sum_j
 * f32(rows[route_pos[t,j]]) * slot_scores[route_pos[t,j]]) in slot order,
 * then + shared[t] (BF16 add) when shared is not NULL — the reduce of
 * glm53_flash_mlx/packed.py:168-179 and the shared add of packed.py:915-922,
 * applied to rows returned by their owners. */
int glm53_ep_combine(const void* rows, const uint32_t* route_pos, const float* slot_scores,
                     int64_t T, int top_k, int64_t H, const void* shared, void* out,
                     void* stream);

/* Expert-parallel decode over peer memory (NVLink) — the transport that
 * replaces the two all-to-alls.  No counterpart in the reference (single
 * device).  Every rank allocates one buffer of glm53_ep_shared_bytes(world,
 * capacity, H) bytes (glm53_ep_buffer_alloc, once per layer plan: zeroed,
 * with its CUDA IPC handle, 64 bytes) and maps every peer's
 * (glm53_ep_ipc_open); `peer_base` is a device array of the world buffer
 * addresses as seen by this rank (its own at index rank).  Per step, on one
 * stream: glm53_ep_dispatch_p2p (stores each route's token row and local
 * expert id into its owner's buffer and counts the arrival there),
 * glm53_ep_owner_decode_p2p (waits for every rank's slots of this step,
 * decodes them, stores each BF16 row into its home rank's buffer; the home
 * tokens' shared expert, shared_x [T_shared, H] -> shared_out BF16 rows, runs
 * in the same launches and streams while the slots are in flight),
 * glm53_ep_combine_p2p (waits for the rows, slot-ordered reduce + shared add,
 * advances the step counter).  Every rank must run the same steps; each wait
 * gives up after about two seconds with GLM53_STATUS_WAIT_TIMEOUT.
 * slot_route [world * capacity] is scratch; slot_scores and route_pos are as
 * in glm53_ep_dispatch_pack. */
size_t glm53_ep_shared_bytes(int world, int64_t capacity, int64_t H);
int glm53_ep_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle);
int glm53_ep_buffer_free(void* ptr);
int glm53_ep_ipc_open(const void* ipc_handle, void** ptr);
int glm53_ep_ipc_close(void* ptr);
int glm53_ep_dispatch_p2p(const void* x, int64_t T, int64_t H, const uint32_t* expert_ids,
                          const float* scores, int top_k, int64_t E, int world, int rank,
                          int64_t capacity, const unsigned long long* peer_base,
                          uint32_t* slot_route, float* slot_scores, uint32_t* route_pos,
                          uint32_t* status, void* stream);
int glm53_ep_owner_decode_p2p(void* buffer, int64_t H, int world, int64_t capacity, int rank,
                              const uint8_t* gate_up_w, const float* gate_up_s,
                              const uint8_t* down_w, const float* down_s, int64_t E, int64_t I,
                              const void* shared_x, int64_t T_shared,
                              const uint8_t* shared_gate_w, const float* shared_gate_s,
                              const uint8_t* shared_up_w, const float* shared_up_s,
                              const uint8_t* shared_down_w, const float* shared_down_s,
                              int64_t I_shared, void* shared_out, float limit,
                              const unsigned long long* peer_base, void* workspace,
                              size_t workspace_bytes, uint32_t* status, uint32_t flags,
                              void* stream);
int glm53_ep_combine_p2p(void* buffer, const uint32_t* route_pos, const float* slot_scores,
                         int64_t T, int top_k, int64_t H, int world, int64_t capacity,
                         const void* shared, void* out, uint32_t* status, void* stream);

/* Diagnostic: only the first stage of glm53_packed_decode_moe (fused
 * gate/up/SwiGLU of the selected experts and the shared expert); the BF16
 * hidden rows [top_k*I + I_shared] are left at the start of `workspace`.
 * Same arguments as glm53_packed_decode_moe minus `out`.  Counterpart of the
 * reference's stage-dumping diagnostic kernel
 * native_execution/native_indexer_plan.metal:231-321. */
int glm53_packed_decode_gate_up(const void* x, int64_t H, const uint32_t* expert_ids,
                                int top_k, const uint8_t* gate_up_w,
                                const float* gate_up_s, int64_t E, int64_t I,
                                const uint8_t* shared_gate_w, const float* shared_gate_s,
                                const uint8_t* shared_up_w, const float* shared_up_s,
                                int64_t I_shared, float limit, void* workspace,
                                size_t workspace_bytes, uint32_t* status, uint32_t flags,
                                void* stream);

/* Stable expert-sorted route plan and tile descriptors on the device.
 *   order[p] = route index at sorted position p; inverse[r] = its position;
 *   sorted_experts / sorted_scores (scores may be NULL) follow the order;
 *   route_offsets[E+1]; tile_offsets[E+1];
 *   descriptors (capacity ceil(R/tile_rows)+E): (expert, start, length),
 *   sentinel (0, R, 0) for unused slots; descriptor_count[0] = valid count;
 *   invalid_count[0] = routes whose id >= E (placed after all valid routes).
 * Replaces build_route_plan / build_grouped_tile_plan,
 * glm53_flash_mlx/grouped_fp8.py:157-203, and the native route plan
 * native_execution/native_prefill_moe_route_plan.h:16-82. */
int glm53_route_plan(const uint32_t* expert_ids, int64_t R, int64_t E,
                     int64_t tile_rows, const float* scores, uint32_t* order,
                     uint32_t* inverse, uint32_t* sorted_experts,
                     float* sorted_scores, uint32_t* route_offsets,
                     uint32_t* tile_experts, uint32_t* tile_starts,
                     uint32_t* tile_lengths, uint32_t* tile_offsets,
                     uint32_t* descriptor_count, uint32_t* invalid_count,
                     void* stream);

/* sorted_x[p,:] = x[order[p] / top_k, :] (the gathered rows of build_route_plan,
 * glm53_flash_mlx/grouped_fp8.py:164-166). */
int glm53_gather_rows(const void* x, int64_t H, const uint32_t* order,
                      int64_t R, int top_k, void* sorted_x, void* stream);

/* Grouped projection of sorted route rows: for every descriptor d,
 * out[start+i, :] = x[start+i, :] @ dequant(w[expert])^T (i < length).
 * x [R,K] BF16, w [E,N,K] E4M3, scale_inv [E, ceil(N/128), ceil(K/128)],
 * out [R,N] BF16; tile lengths must be <= 128.  The mma.sync tile path: the
 * weights enter the BF16 MMA as BF16(lut(c) * s), one rounding of the scaled
 * weight (relative 2^-9), so results carry that rounding on top of the
 * summation order; glm53_grouped_fp8_linear_ws (tcgen05, exact weights) is
 * the path the Python grouped_fp8_linear takes.
 * Replaces grouped_fp8_linear, glm53_flash_mlx/grouped_fp8.py:206-262
 * (kernel K12, grouped_fp8.py:30-154). */
int glm53_grouped_fp8_linear(const void* x, int64_t R, int64_t K,
                             const uint32_t* tile_experts,
                             const uint32_t* tile_starts,
                             const uint32_t* tile_lengths,
                             int64_t descriptor_capacity, const uint8_t* w,
                             int64_t E, int64_t N, const float* scale_inv,
                             void* out, uint32_t flags, void* stream);

/* hidden[R,I] = silu(min(gate, L)) * clip(up, -L, L) with BF16 per-op
 * rounding, gate_up [R,2I].
 * Replaces activate_gate_up, glm53_flash_mlx/grouped_fp8.py:265-270. */
/* Workspace bytes of glm53_grouped_fp8_linear_ws for R route rows of width K. */
size_t glm53_grouped_fp8_linear_workspace_bytes(int64_t R, int64_t K);

/* glm53_grouped_fp8_linear on the tcgen05 grouped GEMM: the weights decoded
 * exactly to FP16 (lut(c) * 2^8), the activations converted once to FP16 x
 * 2^-e rows in the workspace, FP32 accumulation in TMEM with the block scale
 * applied per 128-K block; results differ from the reference's FP32 sums
 * (grouped_fp8.py:30-154) only in summation order.  tile_rows = the longest
 * descriptor the plan may hold (build_grouped_tile_plan's tile_rows); a longer
 * one sets GLM53_STATUS_BAD_GEOMETRY in `status`, an expert id >= E sets
 * GLM53_STATUS_BAD_EXPERT (that descriptor is skipped).  K and N multiples of
 * 128, 16-byte aligned x, w and workspace.  Replaces grouped_fp8_linear,
 * glm53_flash_mlx/grouped_fp8.py:206-262. */
int glm53_grouped_fp8_linear_ws(const void* x, int64_t R, int64_t K, const uint32_t* tile_experts,
                                const uint32_t* tile_starts, const uint32_t* tile_lengths,
                                int64_t descriptor_capacity, int64_t tile_rows, const uint8_t* w, int64_t E,
                                int64_t N, const float* scale_inv, void* out, void* workspace,
                                size_t workspace_bytes, uint32_t* status, uint32_t flags, void* stream);

int glm53_activate_gate_up(const void* gate_up, int64_t R, int64_t I,
                           float limit, void* hidden, void* stream);

/* out[T,H] = BF16(sum_j f32(sorted_out[inverse[t*k+j]]) *
 * sorted_scores[inverse[t*k+j]]), then + shared[T,H] (BF16 add) if shared is
 * not NULL.
 * Replaces restore_and_reduce, glm53_flash_mlx/grouped_fp8.py:273-276, and the
 * `result + shared` of grouped_fp8.py:319-320. */
int glm53_restore_and_reduce(const void* sorted_out, const float* sorted_scores,
                             const uint32_t* inverse, int64_t T, int top_k,
                             int64_t H, const void* shared, void* out,
                             void* stream);

/* Workspace bytes needed by glm53_grouped_moe. */
size_t glm53_grouped_moe_workspace_bytes(int64_t T, int top_k, int64_t E,
                                         int64_t H, int64_t I, int64_t I_shared);

/* Byte offsets, inside glm53_grouped_moe's workspace (tensor-core path), of
 * the intermediates a call leaves there: offsets[0..7] = route order (u32
 * [R], sorted position -> route t * top_k + j), inverse (u32 [R]), sorted
 * expert ids (u32 [R]), sorted scores (f32 [R]), hidden rows (FP16 [R, I],
 * sorted order), down rows (BF16 [R, H], sorted order), the shared expert's
 * hidden rows (FP16 [T, I_shared]) and output rows (BF16 [T, H]); R = T *
 * top_k.  For inspection (the parity tests); no reference counterpart. */
int glm53_grouped_moe_workspace_layout(int64_t T, int top_k, int64_t E, int64_t H, int64_t I,
                                       int64_t I_shared, size_t* offsets);

/* Byte offsets of the E4M3 activation terms a GLM53_FLAG_F8_MMA call of
 * glm53_grouped_moe leaves in its workspace: offsets[0..5] = routed input
 * terms (u8 [R][hi H | lo H], sorted order), their scales (f32 [R]), the
 * routed hidden rows' scales (f32 [R]; the hidden terms [R][hi I | lo I]
 * replace the hidden rows in place), the shared expert's input terms (u8
 * [T][hi H | lo H]), their scales (f32 [T]) and its hidden rows' scales
 * (f32 [T]; terms in place of its hidden rows).  A row's activation is
 * (hi + lo) * scale.  For inspection (the parity tests). */
int glm53_grouped_moe_term_layout(int64_t T, int top_k, int64_t E, int64_t H, int64_t I,
                                  int64_t I_shared, size_t* offsets);

/* The activation split of the FP8 tensor-core path (GLM53_FLAG_F8_MMA):
 * each BF16 row x[r] ([rows, K], K % 8 == 0, K <= 4096) becomes E4M3 terms
 * terms[r] = [hi K | lo K] of x[r] * 2^-e (e = exponent of the row maximum
 * minus 8, at least -126; 0 for a zero row), hi = E4M3(x 2^-e),
 * lo = E4M3(x 2^-e - hi), both round-to-nearest-even and saturating, and
 * scale[r] = 2^e (NaN for a row with an infinite element).  terms may alias
 * x (16-byte aligned).  No reference counterpart: the reference multiplies
 * BF16 activations; this is the representation its FP8 tensor-core option
 * multiplies instead. */
int glm53_e4m3_split_rows(const void* x, int64_t rows, int64_t K, void* terms, float* scale, void* stream);

/* Whole grouped prefill MoE layer given routes: route plan, grouped gate/up
 * with fused SwiGLU, grouped down, slot-ordered FP32 combine, shared expert
 * and BF16 add.  Bank and shared layouts as in glm53_packed_decode_moe.
 * Replaces SortedGroupedFP8MoE.grouped_from_routes,
 * glm53_flash_mlx/grouped_fp8.py:294-321. */
int glm53_grouped_moe(const void* x, int64_t T, int64_t H,
                      const uint32_t* indices, const float* scores, int top_k,
                      const uint8_t* gate_up_w, const float* gate_up_s,
                      const uint8_t* down_w, const float* down_s, int64_t E,
                      int64_t I, const uint8_t* shared_gate_w,
                      const float* shared_gate_s, const uint8_t* shared_up_w,
                      const float* shared_up_s, const uint8_t* shared_down_w,
                      const float* shared_down_s, int64_t I_shared, float limit,
                      void* out, void* workspace, size_t workspace_bytes,
                      uint32_t* status, uint32_t flags, void* stream);

/* Diagnostic: the BF16 sigmoid stage of the SwiGLU epilogue over n BF16
 * gate values (the reference's formula sweep,
 * native_execution/native_indexer_plan.metal:323-366). */
int glm53_sigmoid_bf16(const void* gate, int64_t n, void* out, void* stream);

/* ---- FFN boundary around the MoE (mHC collapse + RMSNorm, hc expand) ---- */

/* Workspace bytes of glm53_hc_collapse_norm for T tokens (0 if H is not
 * supported). */
size_t glm53_hc_collapse_workspace_bytes(int64_t T, int64_t H);

/* mHC collapse of the 4-branch residual state and the post-attention RMSNorm
 * that feeds the router, for T tokens:
 *   state BF16 [T, 4, H]; hc_fn BF16 [24, 4H]; hc_scale FP32 [3];
 *   hc_base FP32 [24]; norm_weight BF16 [H] (or NULL: no RMSNorm);
 *   collapsed BF16 [T, H] (may be NULL); normalized BF16 [T, H] (NULL iff
 *   norm_weight is); post FP32 [T, 4]; comb FP32 [T, 4, 4] ([source][branch]).
 * m = (x . fn^T) / sqrt(mean(x^2) + hc_norm_eps) over x = state[t] (4H);
 * pre = sigmoid(m[0:4] scale[0] + base[0:4]) + hc_eps;
 * post = 2 sigmoid(m[4:8] scale[1] + base[4:8]);
 * comb = Sinkhorn(softmax(m[8:24] scale[2] + base[8:24]) + hc_eps,
 *                 sinkhorn_iters, hc_eps);
 * collapsed = BF16(sum_b pre[b] state[t][b]);
 * normalized = BF16(w * BF16(collapsed / sqrt(mean(collapsed^2) + rms_eps))).
 * branches must be 4 and H a multiple of 8 up to 8192; pointers 16-byte
 * aligned.  Replaces layer.ffn_hc (mlx-vlm deepseek_v4 hyper connection, not
 * in the reference) followed by layer.post_attention_layernorm, the sequence
 * of scripts/profile_native_prefill_ffn_entry_seam.py:79-81. */
int glm53_hc_collapse_norm(const void* state, int64_t T, int64_t H, int branches,
                           const void* hc_fn, const float* hc_scale,
                           const float* hc_base, int sinkhorn_iters, float hc_eps,
                           float hc_norm_eps, const void* norm_weight,
                           float rms_eps, void* collapsed, void* normalized,
                           float* post, float* comb, void* workspace,
                           size_t workspace_bytes, void* stream);

/* RMSNorm of T BF16 rows of H: out = BF16(w * BF16(x / sqrt(mean(x^2) + eps))).
 * Replaces MLX's fast rms_norm as layer.post_attention_layernorm
 * (scripts/profile_native_prefill_ffn_entry_seam.py:80). */
int glm53_rms_norm(const void* x, int64_t T, int64_t H, const void* weight,
                   float eps, void* out, void* stream);

/* hc expand of the MoE output into the 4-branch state:
 * out[t][b][d] = BF16(post[t][b] * moe[t][d] + mixed), mixed the FMA chain
 * over source s = 0..3 of comb[t][s][b] * residual[t][s][d].
 * moe BF16 [T, H]; residual, out BF16 [T, 4, H]; post FP32 [T, 4];
 * comb FP32 [T, 4, 4].  Replaces glm53_native_prefill_post_attention_hc_expand
 * (native_execution/native_indexer_plan.metal:2362-2389) as run by
 * NativePrefillMoEPlan::finish_hc (native_prefill_moe_plan.cpp:136-161). */
int glm53_hc_expand(const void* moe, const void* residual, const float* post,
                    const float* comb, int64_t T, int64_t H, int branches,
                    void* out, void* stream);

/* Sparse-attention output layout: head_major BF16 [heads, rows, dim] ->
 * row_major BF16 [rows, heads * dim] (a pure copy; dim a multiple of 8,
 * 16-byte aligned tensors), the o_proj input.  Replaces
 * glm53_native_prefill_dsa_head_to_row_bfloat16
 * (native_execution/native_indexer_plan.metal:2290-2304) of
 * NativePrefillDSAOutputPlan::execute (native_prefill_dsa_output_plan.cpp:68-106). */
int glm53_head_major_to_rows(const void* head_major, int64_t heads, int64_t rows,
                             int64_t dim, void* row_major, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GLM53_B200_H_ */
