// Internal (non-ABI) declarations shared between the kernel translation units.
#pragma once

#include "common.cuh"

namespace glm53 {

// glm53_fp8_linear routes M <= kGemvMaxRows to the bandwidth GEMV and larger
// M to the tensor-core GEMM.
constexpr int64_t kGemvMaxRows = 16;

int fp8_linear_small_m(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w, int64_t N,
                       const float* s, uint16_t* y, uint32_t flags, cudaStream_t stream);

// Tensor-core grouped GEMM (grouped.cu).
//   A rows: x[a_index ? a_index[start+i] / a_div : start+i, :]  (BF16 [*, K])
//   B: expert e rows of w_gate (and w_up for the fused SwiGLU mode).
struct GroupedGemmArgs {
  const uint16_t* x;          // activations, row stride K
  const uint32_t* a_index;    // optional row indirection (sorted route order)
  int a_div;                  // divisor applied to a_index (top_k)
  int64_t R;                  // rows addressed by descriptors (routes)
  int64_t K;
  const uint32_t* tile_experts;
  const uint32_t* tile_starts;
  const uint32_t* tile_lengths;
  int64_t capacity;           // descriptor slots (dense mode: ceil(R / 128))
  bool dense;                 // descriptors implicit: (0, 128 d, min(128, R - 128 d))
  const uint8_t* w_gate;      // [E, N_out, K] (plain) or gate rows (SwiGLU)
  const uint8_t* w_up;        // up rows (SwiGLU) or nullptr
  int64_t w_expert_stride;    // bytes between experts
  const float* s_gate;
  const float* s_up;
  int64_t s_expert_stride;    // floats between experts
  int64_t E;
  int64_t N;                  // output columns (plain: N; SwiGLU: I)
  bool swiglu;
  float limit;
  uint16_t* out;              // [R, N] BF16
  uint32_t* status;
};

int grouped_gemm(const GroupedGemmArgs& a, cudaStream_t stream);

bool dense_gemm_supported(int64_t K, int64_t N, const void* w);
int dense_fp8_gemm(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w, int64_t N,
                   const float* s, uint16_t* y, cudaStream_t stream);

// Route plan (route_plan.cu), usable inside composite entry points.
int route_plan(const uint32_t* ids, int64_t R, int64_t E, int64_t tile_rows, const float* scores,
               uint32_t* order, uint32_t* inverse, uint32_t* sorted_experts, float* sorted_scores,
               uint32_t* route_offsets, uint32_t* tile_experts, uint32_t* tile_starts,
               uint32_t* tile_lengths, uint32_t* tile_offsets, uint32_t* descriptor_count,
               uint32_t* invalid_count, cudaStream_t stream);
// route_plan for long route lists, on several blocks (the same outputs):
// scratch of route_plan_scratch_bytes(R, E); at most 4,096 routes, or without
// scratch, it runs route_plan.
size_t route_plan_scratch_bytes(int64_t R, int64_t E);
int route_plan_chunked(const uint32_t* ids, int64_t R, int64_t E, int64_t tile_rows, const float* scores,
                       uint32_t* order, uint32_t* inverse, uint32_t* sorted_experts, float* sorted_scores,
                       uint32_t* route_offsets, uint32_t* tile_experts, uint32_t* tile_starts, uint32_t* tile_lengths,
                       uint32_t* tile_offsets, uint32_t* descriptor_count, uint32_t* invalid_count, uint32_t* scratch,
                       cudaStream_t stream);

// tcgen05 grouped GEMM (grouped_tc.cu).  Rows of x16 (FP16, row multiplier
// xscale) are routes; descriptors as for GroupedGemmArgs, each at most
// max_rows routes.  Plain: out [R, N] BF16 = x . W^T.  SwiGLU: out [R, I] FP16
// = the reference's BF16 SwiGLU of the gate tile (w rows [u_off.. of w_up for
// the up tile), stored as FP16.
struct TcGemm {
  const __half* x16;
  const float* xscale;
  int64_t R, K;
  const uint32_t* tile_experts;
  const uint32_t* tile_starts;
  const uint32_t* tile_lengths;
  int64_t capacity;
  int64_t max_rows;       // longest descriptor (ignored when dense)
  bool dense;             // descriptors implicit: (0, 128 d, min(128, R - 128 d))
  const uint8_t* w;       // gate (or plain) weights, w_rows rows per expert
  const uint8_t* w_up;    // up weights (SwiGLU), u_rows rows per expert
  int64_t w_rows, u_rows, u_off;
  const float* s_gate;    // scale table of w: [E][w_rows/128][K/128] (row offset included)
  const float* s_up;
  int64_t s_expert;       // floats between experts in the scale tables
  int64_t E;
  int64_t N;              // plain output columns
  int64_t I;              // SwiGLU hidden columns
  bool swiglu;            // gate/up form: out holds [R][gate I | up I] BF16 rows (the reference's
                          // gate and up values; swiglu_rows / swiglu_split apply the activation)
  float limit;
  bool finite;            // no 0x7F/0xFF codes: hardware E4M3 conversion
  uint16_t* out;
  uint32_t* status;
  // split-K (plain dense GEMMs only): each tile's k-blocks are cut into
  // `splits` contiguous ranges computed by different CTAs, whose FP32 partial
  // sums go to `partial` [splits][R][N] and are added in range order by a
  // second kernel (grouped_tc_splitk_bytes gives the size)
  int splits;
  float* partial;
  // kind::f8f6f4 kernel (finite banks): x8 holds the activation rows as
  // [R][hi K | lo K] E4M3 terms (rows_to_e4m3_split), xscale their 2^e; the
  // SwiGLU form writes BF16 hidden rows
  bool f8;
  const uint8_t* x8;
};

// Split count for a plain dense GEMM of `tiles` output tiles over nkb 128-K
// blocks: enough CTAs to cover the SMs, at least four k-blocks per range.
int grouped_tc_splits(int64_t tiles, int64_t nkb);
size_t grouped_tc_splitk_bytes(int64_t R, int64_t N, int splits);

bool grouped_tc_supported(int64_t K, int64_t N, float limit, bool swiglu);
bool grouped_f8_supported(int64_t K, int64_t N, bool swiglu);
// FP32 router logits on the tensor cores: partial[z][t][e] (FP64) of x BF16
// [T, H] against the weights' three BF16 planes [3][E][H], K split into
// `splits` ranges; abort_out is set when a bounded wait gave up.
bool router_tc_supported(int64_t T, int64_t H, int64_t E);
int router_tc_splits(int64_t T, int64_t E);
int router_logits_tc(const uint16_t* x, int64_t T, int64_t H, const uint16_t* planes, int64_t E, double* partial,
                     int splits, uint32_t* abort_out, cudaStream_t st);
// y[r] = [hi K | lo K] E4M3 terms of x[order ? order[r] / div : r] * 2^-e_r
// (K <= 4096; y may alias x when order is null), scale[r] = 2^e_r.
int rows_to_e4m3_split(const uint16_t* x, int64_t K, const uint32_t* order, int div, int64_t rows, uint8_t* y,
                       float* scale, cudaStream_t st);
// The reference's BF16 SwiGLU of [R][gate I | up I] BF16 rows (a SwiGLU-form
// grouped_tc output): FP16 hidden rows [R, I], or the E4M3 terms
// [R][hi I | lo I] of the BF16 hidden rows and their scales (I <= 4096).
int swiglu_rows(const uint16_t* gu, int64_t R, int64_t I, float limit, __half* hidden, cudaStream_t st);
int swiglu_split(const uint16_t* gu, int64_t R, int64_t I, float limit, uint8_t* terms, float* scale,
                 cudaStream_t st);
int grouped_tc(const TcGemm& g, cudaStream_t stream);
// y[r] = FP16(x[order ? order[r] / div : r] * 2^-e_r), scale[r] = 2^e_r.
int rows_to_f16(const uint16_t* x, int64_t H, const uint32_t* order, int div, int64_t rows, __half* y, float* scale,
                cudaStream_t stream);

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// glm53_router_topk; with pdl the small-T kernel is launched as a
// programmatic dependent of the previous kernel on the stream (router.cu).
int router_topk(const void* x, int64_t T, int64_t H, const float* w, int64_t E, const float* bias, int top_k,
                int n_group, int topk_group, int norm_topk_prob, float routed_scaling_factor, uint32_t* indices,
                float* scores, float* logits, void* workspace, size_t workspace_bytes, cudaStream_t st, bool pdl);

// Device address of a pinned (device-mapped) host buffer, or nullptr for
// pageable memory (capi.cu).
void* mapped_host(const void* p);
// Small host <-> device copy: a kernel over the pinned buffer's mapping when
// both addresses and the size are 16-byte multiples (*by_kernel = true), else
// cudaMemcpyAsync (capi.cu).  When the copy runs as a kernel and `status` and
// `status_mirror` (pinned host) are given, the kernel also copies the device
// status word into the host word.  pdl: the kernel is launched as a
// programmatic dependent of the previous kernel (it copies at once and reads
// the status word after that kernel has finished); only for a destination
// the previous kernel does not touch.
cudaError_t small_copy(void* dst, const void* src, size_t bytes, bool to_device, cudaStream_t st, bool* by_kernel,
                       const uint32_t* status = nullptr, uint32_t* status_mirror = nullptr, bool pdl = false);
// One-thread kernel copying the device status word into a pinned host word
// (GLM53_ERR_INVALID when host_word is not device-mapped).
int mirror_status(const uint32_t* status, uint32_t* host_word, cudaStream_t st, const char* fn);

// Peer-memory expert parallelism: every rank allocates one buffer of this
// layout and maps every peer's (CUDA IPC).  Slot (src, s) of recv_x/recv_e is
// written by rank src; slot (owner, s) of back by rank owner; the counters
// only grow (one per arriving CTA), the epoch counts this rank's steps.
struct EpLayout {
  size_t recv_x, recv_e, back, cnt_dispatch, cnt_back, epoch, done, expected, bytes;
};

inline EpLayout ep_layout(int world, int cap, int64_t H) {
  EpLayout l;
  const size_t slots = (size_t)world * cap;
  l.recv_x = 0;
  l.recv_e = align_up(slots * H * 2, 256);
  l.back = l.recv_e + align_up(slots * 4, 256);
  l.cnt_dispatch = l.back + align_up(slots * H * 2, 256);
  l.cnt_back = l.cnt_dispatch + 256;
  l.epoch = l.cnt_back + 256;
  l.done = l.epoch + 256;
  l.expected = l.done + 256;  // back-buffer arrivals expected up to the last finished step
  l.bytes = l.expected + 256;
  return l;
}

// Longest wait of the expert-parallel peer handshakes, in ns (default two
// seconds; glm53_set_wait_limit_ns changes it for later launches).
unsigned long long ep_wait_limit_ns();

// Bounded wait of one thread until *counter >= target (system-scope acquire);
// false (and GLM53_STATUS_WAIT_TIMEOUT) after limit_ns of globaltimer time.
__device__ __forceinline__ bool wait_counter_geq(const unsigned long long* counter, unsigned long long target,
                                                 uint32_t* status, unsigned long long limit_ns) {
  unsigned long long t0 = 0;
  for (uint32_t it = 0;; ++it) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(counter) : "memory");
    if (v >= target) return true;
    if ((it & 255u) == 255u) {
      unsigned long long now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > limit_ns) {
        atomicOr(status, kStatusWaitTimeout);
        return false;
      }
    }
  }
}

}  // namespace glm53
