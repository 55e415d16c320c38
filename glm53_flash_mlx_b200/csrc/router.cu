// FP32 router (G0): logits, sigmoid, bias, optional group mask, top-k,
// normalisation and scaling.
//
// Replaces Float32Gate.__call__ (glm53_flash_mlx/patch.py:131-142) and the
// mlx-vlm group_expert_select it calls (mlx-vlm 0.6.17 @ e82d557, not vendored
// in the reference; restated from its published algorithm):
//   s = sigmoid(logits); choice = s + e_score_correction_bias;
//   if n_group > 1: group score = sum of the top-2 choices in each group, the
//     n_group - topk_group lowest groups have their choices set to 0.0;
//   idx = top_k of choice; scores = s[idx]; if top_k > 1 and norm_topk_prob:
//     scores /= sum(scores); scores *= routed_scaling_factor.
// The reference's argpartition leaves slot order unspecified; here slots are
// in descending choice, ties to the lower expert id.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace glm53 {

constexpr int kRouterSmallT = 32;  // tokens handled by the fused GEMV+top-k launch (decode batches)
constexpr int kRouterMaxE = 1024;  // 32 lanes x 32 values per lane
constexpr int kRouterMaxK = 32;

struct TopkParams {
  int E, top_k, n_group, topk_group, norm;
  float scale;
};

// Order-preserving map of a float onto uint32 (larger float -> larger key);
// key 0 is below every non-NaN value and marks an empty position.
__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Inverse of order_key.
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// sigmoid(logit) and its selection key sigmoid + bias (the reference's
// `choice`), shared by both router paths.
__device__ __forceinline__ void route_key(float logit, float bias, float& sig, uint32_t& key) {
  sig = 1.0f / (1.0f + expf(-logit));
  key = order_key(sig + bias);
}

// One warp selects the top-k of one token from its keys and sigmoids
// (value i of lane l is expert e = l + 32 i; key 0 marks e >= E).  Shared
// scratch `choice_smem` holds E floats for the group mask.
template <int PER>
__device__ void warp_topk_core(uint32_t (&key)[PER], const float (&sig)[PER], const TopkParams& p,
                               uint32_t* idx_out, float* score_out, float* choice_smem) {
  const int lane = threadIdx.x & 31;
  if (p.n_group > 1) {
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      int e = lane + 32 * i;
      if (e < p.E) choice_smem[e] = key_value(key[i]);
    }
    __syncwarp();
    const int per_group = p.E / p.n_group;
    // lane g computes the top-2 sum of group g (n_group <= 32)
    float gscore = -INFINITY;
    if (lane < p.n_group) {
      float b1 = -INFINITY, b2 = -INFINITY;
      for (int e = lane * per_group; e < (lane + 1) * per_group; ++e) {
        float v = choice_smem[e];
        if (v > b1) { b2 = b1; b1 = v; } else if (v > b2) { b2 = v; }
      }
      gscore = b1 + b2;
    }
    // drop the n_group - topk_group lowest groups (ties: the higher index first)
    uint32_t dropped = 0;
    for (int d = 0; d < p.n_group - p.topk_group; ++d) {
      float v = (lane < p.n_group && !((dropped >> lane) & 1u)) ? gscore : INFINITY;
      int g = lane;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, v, o);
        int og = __shfl_xor_sync(0xffffffffu, g, o);
        if (ov < v || (ov == v && og > g)) { v = ov; g = og; }
      }
      dropped |= 1u << g;
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      int e = lane + 32 * i;
      if (e < p.E && ((dropped >> (e / per_group)) & 1u)) key[i] = order_key(0.0f);
    }
    __syncwarp();
  }
  // k rounds of a warp arg-max on the keys: the largest choice wins, ties go
  // to the lower expert id (the lowest i of a lane, then the lowest lane).
  // Slot j's pick stays in lane j.
  uint32_t taken = 0;  // bit i: value i of this lane selected
  uint32_t my_idx = 0;
  float my_sig = 0.f;
  for (int j = 0; j < p.top_k; ++j) {
    uint32_t bk = 0u;
    int bi = -1;
    float bs = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      if (!((taken >> i) & 1u) && key[i] > bk) {
        bk = key[i];
        bi = i;
        bs = sig[i];
      }
    }
    const uint32_t wmax = __reduce_max_sync(0xffffffffu, bk);
    const uint32_t cand = (bi >= 0 && bk == wmax) ? (uint32_t)(32 * bi + lane) : 0xffffffffu;
    const uint32_t best = __reduce_min_sync(0xffffffffu, cand);
    const float ps = __shfl_sync(0xffffffffu, bs, best & 31);
    if ((best & 31) == (uint32_t)lane) taken |= 1u << (best >> 5);
    if (lane == j) {
      my_idx = best;
      my_sig = ps;
    }
  }
  // normaliser summed in slot order
  float total = 0.f;
  for (int j = 0; j < p.top_k; ++j) total = total + __shfl_sync(0xffffffffu, my_sig, j);
  if (lane < p.top_k) {
    float v = my_sig;
    if (p.top_k > 1 && p.norm) v = v / total;
    idx_out[lane] = my_idx;
    score_out[lane] = v * p.scale;
  }
}

// Top-k from logits (the tiled path's separate top-k kernel).
template <int PER>
__device__ void warp_topk(const float* logits, const float* __restrict__ bias, const TopkParams& p,
                          uint32_t* idx_out, float* score_out, float* choice_smem) {
  const int lane = threadIdx.x & 31;
  uint32_t key[PER];
  float sig[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    key[i] = 0u;
    sig[i] = 0.f;
    if (e < p.E) route_key(__ldcg(logits + e), bias[e], sig[i], key[i]);
  }
  warp_topk_core<PER>(key, sig, p, idx_out, score_out, choice_smem);
}

// Top-k from keys and sigmoids already computed per expert (the fused path:
// every block computed its own expert's, so the last block only loads them).
template <int PER>
__device__ void warp_topk_keys(const uint32_t* keys, const float* sigs, const TopkParams& p, uint32_t* idx_out,
                               float* score_out, float* choice_smem) {
  const int lane = threadIdx.x & 31;
  uint32_t key[PER];
  float sig[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    key[i] = e < p.E ? __ldcg(keys + e) : 0u;
    sig[i] = e < p.E ? __ldcg(sigs + e) : 0.f;
  }
  warp_topk_core<PER>(key, sig, p, idx_out, score_out, choice_smem);
}

// FP32 GEMV for T <= kRouterSmallT tokens: one block per expert row, each
// thread sums float4 slices k = 4*tid + 1024*i in K order, then an ordered
// warp / block reduction, and one rounding to FP32.  The sums are FP64: every
// product of a BF16 activation and an FP32 weight is exact in FP64 (32
// significant bits) and 4096 FP64 additions leave an error near 2^-41 of the
// terms' magnitude, so each logit is the exact dot product rounded once to
// FP32 (the FP32 router of patch.py:131-142 evaluated to full FP32 accuracy:
// a logit near zero keeps its relative accuracy).  The last block to finish
// runs the top-k.  The
// group-mask scratch (8 warps x E floats) is dynamic shared memory, present
// only when n_group > 1, so that the router's blocks leave room on the SMs
// for a decode stage launched as their programmatic dependent.
template <int TG, int T_MAX, int PER>
__global__ void __launch_bounds__(256) router_small_kernel(
    const uint16_t* __restrict__ x, int T, int H, const float* __restrict__ w,
    const float* __restrict__ bias, TopkParams p, float* logits, float* sig_buf, uint32_t* key_buf,
    uint32_t* counter, uint32_t* __restrict__ idx, float* __restrict__ scores) {
  __shared__ double part[8][T_MAX];
  __shared__ bool is_last;
  extern __shared__ float choice_dyn[];  // [8][E] when n_group > 1
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x;
  const float* wr = w + (size_t)e * H;
  // The weights and the bias never depend on the previous kernel: the first
  // kRouterPre float4 of this thread's slice of the row (all of it for
  // H <= 4096) are in flight before the wait below.
  constexpr int kRouterPre = 4;
  float4 pre[kRouterPre];
#pragma unroll
  for (int i = 0; i < kRouterPre; ++i) {
    const int k = 4 * threadIdx.x + 1024 * i;
    pre[i] = k < H ? __ldcs(reinterpret_cast<const float4*>(wr + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const float be = threadIdx.x < T ? __ldg(bias + e) : 0.f;
  // launched as a programmatic dependent of the kernel that writes x: wait
  // for it (a no-op otherwise) before reading x or writing any result.  Then
  // a dependent launched with programmatic serialisation may start; it waits
  // (griddepcontrol.wait) before it reads this kernel's results, and may read
  // x right away.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // Tokens in groups of TG (the unrolled body stays TG tokens wide): every
  // token's products are summed in the same K order by the same thread,
  // whatever T and the group, so a token's logit does not depend on the
  // batch it rides in.
  const int t_end = T_MAX == TG ? 1 : T;  // one group (a fixed trip count) when T_MAX == TG
  for (int t0 = 0; t0 < t_end; t0 += TG) {
    double acc[TG];
#pragma unroll
    for (int t = 0; t < TG; ++t) acc[t] = 0.0;
    // the products in K order: the prefetched float4 first, then the rest of
    // the row (H > 4096)
    auto accumulate = [&](int k, const float4 wv) {
#pragma unroll
      for (int t = 0; t < TG; ++t) {
        if (t0 + t < T) {
          const uint2 raw = __ldg(reinterpret_cast<const uint2*>(x + (size_t)(t0 + t) * H + k));
          acc[t] = fma((double)__uint_as_float(raw.x << 16), (double)wv.x, acc[t]);
          acc[t] = fma((double)__uint_as_float(raw.x & 0xFFFF0000u), (double)wv.y, acc[t]);
          acc[t] = fma((double)__uint_as_float(raw.y << 16), (double)wv.z, acc[t]);
          acc[t] = fma((double)__uint_as_float(raw.y & 0xFFFF0000u), (double)wv.w, acc[t]);
        }
      }
    };
#pragma unroll
    for (int i = 0; i < kRouterPre; ++i) {
      const int k = 4 * threadIdx.x + 1024 * i;
      if (k < H) accumulate(k, pre[i]);
    }
#pragma unroll 4
    for (int k = 4 * threadIdx.x + 1024 * kRouterPre; k < H; k += 1024)
      accumulate(k, __ldcs(reinterpret_cast<const float4*>(wr + k)));
#pragma unroll
    for (int t = 0; t < TG; ++t) {
      double v = acc[t];
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && t0 + t < T_MAX) part[warp][t0 + t] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x < T_MAX && threadIdx.x < T) {
    double d = 0.0;
#pragma unroll
    for (int ww = 0; ww < 8; ++ww) d += part[ww][threadIdx.x];
    const float v = (float)d;
    const size_t o = (size_t)threadIdx.x * p.E + e;
    logits[o] = v;
    route_key(v, be, sig_buf[o], key_buf[o]);
    __threadfence();  // the writers publish before the block signals completion
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned prev = atomicAdd(counter, 1u);
    is_last = (prev == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int t = warp; t < T; t += 8) {  // one warp per token
    warp_topk_keys<PER>(key_buf + (size_t)t * p.E, sig_buf + (size_t)t * p.E, p, idx + (size_t)t * p.top_k,
                        scores + (size_t)t * p.top_k, choice_dyn + (size_t)warp * p.E);
  }
  if (threadIdx.x == 0) *counter = 0u;  // leave the workspace reusable
}

// Tiled GEMM for larger T: logits[T,E] = x[T,H] @ w[E,H]^T.  64x64 output
// tile per block, 256 threads, 4x4 outputs each.  Each 16-wide K slice is
// summed in FP32 and the slice sums are accumulated in FP64, so the error
// stays near that of a 16-term FP32 sum however long H is.
__global__ void __launch_bounds__(256) router_gemm_kernel(const uint16_t* __restrict__ x, int T, int H,
                                                          const float* __restrict__ w, int E,
                                                          float* __restrict__ logits) {
  constexpr int BM = 64, BN = 64, BK = 16;
  __shared__ float xs[BK][BM + 4];
  __shared__ float ws[BK][BN + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int t0 = blockIdx.x * BM, e0 = blockIdx.y * BN;
  double acc[4][4] = {};
  for (int k0 = 0; k0 < H; k0 += BK) {
    for (int i = threadIdx.x; i < BM * BK; i += 256) {
      int r = i / BK, k = i % BK;
      int t = t0 + r, e = e0 + r;
      xs[k][r] = (t < T && k0 + k < H) ? bf16_bits_to_f32(x[(size_t)t * H + k0 + k]) : 0.f;
      ws[k][r] = (e < E && k0 + k < H) ? w[(size_t)e * H + k0 + k] : 0.f;
    }
    __syncthreads();
    float part[4][4] = {};
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = xs[k][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = ws[k][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) part[i][j] = fmaf(a[i], b[j], part[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] += (double)part[i][j];
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int t = t0 + ty * 4 + i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int e = e0 + tx * 4 + j;
      if (e < E) logits[(size_t)t * E + e] = (float)acc[i][j];
    }
  }
}

// Tensor-core FP32 router logits for T > 8 tokens.  x is BF16, hence exact
// as a BF16 MMA operand; every FP32 weight splits exactly into three BF16
// numbers w = hi + mid + lo (8 + 8 + 8 significant bits).  For each 16-wide
// K slice three m16n8k16 BF16 MMAs with a zero accumulator give the slice's
// exact products summed in FP32, and their sum is added into a double-FP32
// accumulator (sum s plus error term c, Knuth's TwoSum: s + c carries about
// 48 significant bits, so the accumulation adds no error an FP64 one would
// not) -- the slice-then-FP64 scheme of router_gemm_kernel on the tensor
// cores without FP64 arithmetic, which is slow on this part.  Block tile 64 tokens x 64 experts, 4 warps of 32 x 32.
// With `partial`, blockIdx.z takes K range [z k_len, (z+1) k_len) and
// stores its FP64 sums to partial[z][t][e] (router_logits_reduce adds the
// ranges in z order); otherwise one CTA covers all of K and stores FP32.
constexpr int kRmBT = 64, kRmBE = 64, kRmBK = 32;

__device__ __forceinline__ void mma_16816_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two FP32 values -> their exact three-part BF16 split, packed in pairs.
__device__ __forceinline__ void split3_bf16x2(float a, float b, uint32_t& hi, uint32_t& mid, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const float ra = a - __low2float(h), rb = b - __high2float(h);
  const __nv_bfloat162 m = __floats2bfloat162_rn(ra, rb);
  const __nv_bfloat162 l = __floats2bfloat162_rn(ra - __low2float(m), rb - __high2float(m));
  hi = *reinterpret_cast<const uint32_t*>(&h);
  mid = *reinterpret_cast<const uint32_t*>(&m);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

__global__ void __launch_bounds__(128) router_mma_kernel(const uint16_t* __restrict__ x, int T, int H,
                                                         const float* __restrict__ w, int E,
                                                         float* __restrict__ logits, int k_len,
                                                         double* __restrict__ partial) {
  __shared__ __align__(16) uint16_t xs[kRmBT][kRmBK + 8];
  __shared__ __align__(16) float ws[kRmBE][kRmBK + 4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const int t0 = blockIdx.x * kRmBT, e0 = blockIdx.y * kRmBE;
  const int wt = (warp >> 1) * 32, we = (warp & 1) * 32;
  float acc[2][4][4], err[2][4][4];
#pragma unroll
  for (int m = 0; m < 2; ++m)
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[m][n][c] = err[m][n][c] = 0.f;
  const int k_begin = blockIdx.z * k_len, k_end = min(H, k_begin + k_len);
  for (int k0 = k_begin; k0 < k_end; k0 += kRmBK) {
    for (int i = threadIdx.x; i < kRmBT * (kRmBK / 8); i += blockDim.x) {
      const int r = i / (kRmBK / 8), c = i - r * (kRmBK / 8);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (t0 + r < T) v = *reinterpret_cast<const uint4*>(x + (size_t)(t0 + r) * H + k0 + 8 * c);
      *reinterpret_cast<uint4*>(&xs[r][8 * c]) = v;
    }
    for (int i = threadIdx.x; i < kRmBE * (kRmBK / 4); i += blockDim.x) {
      const int r = i / (kRmBK / 4), c = i - r * (kRmBK / 4);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e0 + r < E) v = *reinterpret_cast<const float4*>(w + (size_t)(e0 + r) * H + k0 + 4 * c);
      *reinterpret_cast<float4*>(&ws[r][4 * c]) = v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kRmBK; kk += 16) {
      uint32_t a[2][4];
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const int row = wt + 16 * m + g;
        a[m][0] = *reinterpret_cast<const uint32_t*>(&xs[row][kk + 2 * q]);
        a[m][1] = *reinterpret_cast<const uint32_t*>(&xs[row + 8][kk + 2 * q]);
        a[m][2] = *reinterpret_cast<const uint32_t*>(&xs[row][kk + 2 * q + 8]);
        a[m][3] = *reinterpret_cast<const uint32_t*>(&xs[row + 8][kk + 2 * q + 8]);
      }
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const float* wr = &ws[we + 8 * n + g][kk];
        const float2 w0 = *reinterpret_cast<const float2*>(wr + 2 * q);
        const float2 w1 = *reinterpret_cast<const float2*>(wr + 2 * q + 8);
        uint32_t bh0, bm0, bl0, bh1, bm1, bl1;
        split3_bf16x2(w0.x, w0.y, bh0, bm0, bl0);
        split3_bf16x2(w1.x, w1.y, bh1, bm1, bl1);
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          float dh[4] = {0.f, 0.f, 0.f, 0.f}, dm[4] = {0.f, 0.f, 0.f, 0.f}, dl[4] = {0.f, 0.f, 0.f, 0.f};
          mma_16816_bf16(dh, a[m], bh0, bh1);
          mma_16816_bf16(dm, a[m], bm0, bm1);
          mma_16816_bf16(dl, a[m], bl0, bl1);
#pragma unroll
          for (int c = 0; c < 4; ++c) {  // TwoSum(acc, v): acc + v = t + (error, added to err)
            const float v = __fadd_rn(dh[c], __fadd_rn(dm[c], dl[c]));
            const float t = __fadd_rn(acc[m][n][c], v);
            const float bp = __fsub_rn(t, acc[m][n][c]);
            const float e = __fadd_rn(__fsub_rn(acc[m][n][c], __fsub_rn(t, bp)), __fsub_rn(v, bp));
            err[m][n][c] = __fadd_rn(err[m][n][c], e);
            acc[m][n][c] = t;
          }
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int m = 0; m < 2; ++m)
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int t = t0 + wt + 16 * m + g + (c >= 2 ? 8 : 0);
        const int e = e0 + we + 8 * n + 2 * q + (c & 1);
        if (t >= T || e >= E) continue;
        const double v = (double)acc[m][n][c] + (double)err[m][n][c];
        if (partial)
          partial[((size_t)blockIdx.z * T + t) * E + e] = v;
        else
          logits[(size_t)t * E + e] = (float)v;
      }
}

// logits[t][e] = FP32 of the K ranges' FP64 sums added in range order.
__global__ void __launch_bounds__(256) router_logits_reduce(const double* __restrict__ partial, int splits,
                                                            int64_t n, float* __restrict__ logits) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    double v = partial[i];
    for (int z = 1; z < splits; ++z) v += partial[(size_t)z * n + i];
    logits[i] = (float)v;
  }
}

// K ranges of the tensor-core router for T tokens and E experts: enough
// CTAs (about 1280, over eight per SM) to hide the tile loads, at most 8.
static int router_splits(int64_t T, int64_t E) {
  const int64_t base = ((T + kRmBT - 1) / kRmBT) * ((E + kRmBE - 1) / kRmBE);
  int s = 1;
  while (s < 8 && base * s * 2 <= 1280) s *= 2;
  return s;
}

// With `aborted` set (the tensor-core logits kernel gave up on a bounded
// wait), every slot gets the expert id E, which the MoE kernels reject.
template <int PER>
__global__ void __launch_bounds__(256) router_topk_kernel(const float* logits, int T,
                                                          const float* __restrict__ bias, TopkParams p,
                                                          uint32_t* __restrict__ idx,
                                                          float* __restrict__ scores,
                                                          const uint32_t* __restrict__ aborted) {
  __shared__ float choice_smem[8][kRouterMaxE];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  if (aborted && *aborted) {
    for (int j = lane; j < p.top_k; j += 32) {
      idx[(size_t)t * p.top_k + j] = (uint32_t)p.E;
      scores[(size_t)t * p.top_k + j] = 0.f;
    }
    return;
  }
  warp_topk<PER>(logits + (size_t)t * p.E, bias, p, idx + (size_t)t * p.top_k,
                 scores + (size_t)t * p.top_k, choice_smem[warp]);
}

// ---------------------------------------------------------------------------
// FP32 router logits on the FP64 tensor cores, for 9 <= T <= 64 tokens.
//
// D[e][t] = sum_k W[e][k] * X[t][k] with mma.sync m8n8k4 .f64: every product
// of a BF16 activation and an FP32 weight is exact in FP64 and the sums are
// FP64, so each logit is the dot product to within ~2^-40 of its terms'
// magnitude before its one rounding to FP32 (the accuracy of the one-token
// kernel above; the two may differ in the last FP32 bit, as any two FP64
// summation orders may).  One 8-expert x 8-token tile per warp and MMA.
// Beyond 8 tokens this beats the per-expert CTAs, whose register-held token
// groups run one after another and whose last CTA selects every token's
// top-k in turn (here one warp per token, in parallel).  Both kernels run few
// warps per SM and are bound by latency rather than by an FP64 pipe (ncu at
// T = 16: the DMMA subpipe busy 29% of active cycles).
// Grid (E/8 expert tiles, H/1024 K ranges), 8 warps per CTA, 128 K per warp:
// lane (g, q) holds the A element W[e0+g][k] and the B element X[8n+g][k]
// of k = kb + 4q + j in MMA j (j = 0..3) of each 16-wide K chunk kb, so its
// loads are one float4 of weights and one 8-byte activation vector per chunk.
// The 8 warps' tiles are added in warp order, the CTA's sums stored as FP64
// partials [K range][T][E]; router_partial_topk_kernel adds the K ranges in
// order, rounds to FP32 and selects the top-k.
// ---------------------------------------------------------------------------
constexpr int kRdK = 1024;   // K per CTA (8 warps x 128)
constexpr int kRdMaxT = 64;  // tokens per launch (8 token tiles)

__device__ __forceinline__ void dmma_884(double (&d)[2], double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};\n"
               : "+d"(d[0]), "+d"(d[1])
               : "d"(a), "d"(b));
}

template <int NT>
__global__ void __launch_bounds__(256) router_dmma_kernel(const uint16_t* __restrict__ x, int T, int H,
                                                          const float* __restrict__ w, int E,
                                                          double* __restrict__ partial) {
  __shared__ double red[8][8][8 * NT];  // [warp][expert of the tile][token]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const int e0 = blockIdx.x * 8, s = blockIdx.y;
  const int kb0 = s * kRdK + warp * 128;
  const bool erow = e0 + g < E;
  const float* wp = w + (size_t)(erow ? e0 + g : 0) * H + kb0 + 4 * q;
  // this warp's weights (never written by the previous kernel) are in flight
  // before the wait for the activations
  float4 wv[8];
#pragma unroll
  for (int c = 0; c < 8; ++c)
    wv[c] = erow ? __ldcs(reinterpret_cast<const float4*>(wp + 16 * c)) : make_float4(0.f, 0.f, 0.f, 0.f);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  double acc[NT][2];
#pragma unroll
  for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = 0.0;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int k = kb0 + 16 * c + 4 * q;
    const double a0 = wv[c].x, a1 = wv[c].y, a2 = wv[c].z, a3 = wv[c].w;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int t = 8 * n + g;
      const uint2 raw = t < T ? __ldg(reinterpret_cast<const uint2*>(x + (size_t)t * H + k)) : make_uint2(0u, 0u);
      dmma_884(acc[n], a0, (double)__uint_as_float(raw.x << 16));
      dmma_884(acc[n], a1, (double)__uint_as_float(raw.x & 0xFFFF0000u));
      dmma_884(acc[n], a2, (double)__uint_as_float(raw.y << 16));
      dmma_884(acc[n], a3, (double)__uint_as_float(raw.y & 0xFFFF0000u));
    }
  }
  // lane (g, q) holds D[e0 + g][8n + 2q + {0, 1}]
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    red[warp][g][8 * n + 2 * q] = acc[n][0];
    red[warp][g][8 * n + 2 * q + 1] = acc[n][1];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 8 * T; i += 256) {
    const int t = i >> 3, ge = i & 7;
    if (e0 + ge < E) {
      double v = red[0][ge][t];
#pragma unroll
      for (int ww = 1; ww < 8; ++ww) v += red[ww][ge][t];
      partial[((size_t)s * T + t) * E + e0 + ge] = v;
    }
  }
}

// One warp per token: the logit of expert e is the FP32 rounding of the K
// ranges' FP64 partials added in range order; then the top-k of
// router_topk_kernel.  Launched as a programmatic dependent of
// router_dmma_kernel.
template <int PER>
__global__ void __launch_bounds__(256) router_partial_topk_kernel(const double* __restrict__ partial, int splits,
                                                                  int T, const float* __restrict__ bias,
                                                                  TopkParams p, float* __restrict__ logits,
                                                                  uint32_t* __restrict__ idx,
                                                                  float* __restrict__ scores) {
  __shared__ float choice_smem[8][kRouterMaxE];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (t >= T) return;
  uint32_t key[PER];
  float sig[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    key[i] = 0u;
    sig[i] = 0.f;
    if (e < p.E) {
      double v = __ldcg(partial + (size_t)t * p.E + e);
      for (int z = 1; z < splits; ++z) v += __ldcg(partial + ((size_t)z * T + t) * p.E + e);
      const float l = (float)v;
      if (logits) logits[(size_t)t * p.E + e] = l;
      route_key(l, __ldg(bias + e), sig[i], key[i]);
    }
  }
  warp_topk_core<PER>(key, sig, p, idx + (size_t)t * p.top_k, scores + (size_t)t * p.top_k, choice_smem[warp]);
}

// 9..64 tokens (up to 8 the one-CTA-per-expert kernel, its token group sized
// to T, measured faster: 9.4 against 13.6 us at T = 8 / 9).
static bool router_dmma_supported(int64_t T, int64_t H) {
  return T > 8 && T <= kRdMaxT && H % kRdK == 0 && H <= 8 * kRdK;
}

template <int NT>
static void launch_dmma_t(const uint16_t* x, int T, int H, const float* w, int E, double* partial, cudaStream_t st,
                          bool pdl) {
  const dim3 grid((unsigned)((E + 7) / 8), (unsigned)(H / kRdK));
  if (pdl)
    launch_programmatic(router_dmma_kernel<NT>, grid, dim3(256), 0, st, x, T, H, w, E, partial);
  else
    router_dmma_kernel<NT><<<grid, 256, 0, st>>>(x, T, H, w, E, partial);
}

template <int PER>
static int launch_dmma(const uint16_t* x, int T, int H, const float* w, const float* bias, TopkParams p,
                       double* partial, float* logits, uint32_t* idx, float* scores, cudaStream_t st, bool pdl) {
  // token tiles sized to T: every tile's MMAs run whether its tokens exist or not
  if (T <= 16)
    launch_dmma_t<2>(x, T, H, w, p.E, partial, st, pdl);
  else if (T <= 24)
    launch_dmma_t<3>(x, T, H, w, p.E, partial, st, pdl);
  else if (T <= 32)
    launch_dmma_t<4>(x, T, H, w, p.E, partial, st, pdl);
  else if (T <= 48)
    launch_dmma_t<6>(x, T, H, w, p.E, partial, st, pdl);
  else
    launch_dmma_t<8>(x, T, H, w, p.E, partial, st, pdl);
  int rc = check_launch("router_dmma_kernel");
  if (rc) return rc;
  launch_programmatic(router_partial_topk_kernel<PER>, dim3((unsigned)((T + 7) / 8)), dim3(256), 0, st,
                      (const double*)partial, H / kRdK, T, bias, p, logits, idx, scores);
  return check_launch("router_partial_topk_kernel");
}

template <int PER>
static int launch_topk(const float* logits, int T, const float* bias, TopkParams p, uint32_t* idx,
                       float* scores, cudaStream_t st, const uint32_t* aborted = nullptr) {
  router_topk_kernel<PER><<<(T + 7) / 8, 256, 0, st>>>(logits, T, bias, p, idx, scores, aborted);
  return check_launch("router_topk_kernel");
}

// The weights' exact three-way BF16 split w = hi + mid + lo, as three planes
// [3][E][H] for the tensor-core logits kernel.
__global__ void __launch_bounds__(256) router_split_kernel(const float* __restrict__ w, int64_t n4,
                                                           uint16_t* __restrict__ planes, int64_t plane) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(w)[i];
    uint32_t h0, m0, l0, h1, m1, l1;
    split3_bf16x2(v.x, v.y, h0, m0, l0);
    split3_bf16x2(v.z, v.w, h1, m1, l1);
    reinterpret_cast<uint2*>(planes)[i] = make_uint2(h0, h1);
    reinterpret_cast<uint2*>(planes + plane)[i] = make_uint2(m0, m1);
    reinterpret_cast<uint2*>(planes + 2 * plane)[i] = make_uint2(l0, l1);
  }
}

struct RouterScratch {
  float* logits;
  float* sig;
  uint32_t* key;
  uint32_t* counter;
};

template <int TG, int T_MAX, int PER>
static void launch_small_t(const uint16_t* x, int T, int H, const float* w, const float* bias, TopkParams p,
                           const RouterScratch& r, uint32_t* idx, float* scores, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.E);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = p.n_group > 1 ? (size_t)8 * p.E * sizeof(float) : 0;  // <= 32 KB (E <= 1024)
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, router_small_kernel<TG, T_MAX, PER>, x, T, H, w, bias, p, r.logits, r.sig, r.key,
                     r.counter, idx, scores);
}

template <int PER>
static int launch_small(const uint16_t* x, int T, int H, const float* w, const float* bias, TopkParams p,
                        const RouterScratch& r, uint32_t* idx, float* scores, cudaStream_t st, bool pdl) {
  // the token group is sized to T up to 8 tokens (T = 2: 5.7 us with a
  // 2-token group, 8.1 us with the 8-token one, whose absent tokens' work is
  // issued predicated off)
  if (T <= 1)
    launch_small_t<1, 1, PER>(x, T, H, w, bias, p, r, idx, scores, st, pdl);
  else if (T <= 2)
    launch_small_t<2, 2, PER>(x, T, H, w, bias, p, r, idx, scores, st, pdl);
  else if (T <= 4)
    launch_small_t<4, 4, PER>(x, T, H, w, bias, p, r, idx, scores, st, pdl);
  else if (T <= 8)
    launch_small_t<8, 8, PER>(x, T, H, w, bias, p, r, idx, scores, st, pdl);
  else
    launch_small_t<8, kRouterSmallT, PER>(x, T, H, w, bias, p, r, idx, scores, st, pdl);
  return check_launch("router_small_kernel");
}

}  // namespace glm53

using namespace glm53;

// Workspace: logits | sigmoids | keys (T x E each) | completion counter |
// FP64 partial logits of the K ranges (tensor-core path, T > 32).
// For T > 32 also: the tensor-core path's FP64 range partials (or the
// mma.sync path's, whichever is larger), the weights' three BF16 planes (for
// H <= 8192) and its abort word.
static size_t router_partial_bytes(int64_t T, int64_t E) {
  size_t b = 0;
  if (T > 8 && T <= kRdMaxT) b = (size_t)8 * T * E * sizeof(double);  // up to 8 K ranges (H <= 8192)
  if (T > kRouterSmallT) {
    const int s = std::max(router_splits(T, E), router_tc_splits(T, E));
    b = std::max(b, (size_t)s * (size_t)T * (size_t)E * sizeof(double));
  }
  return align_up(b, 256);
}

static size_t router_planes_bytes(int64_t T, int64_t E) {
  return T > kRouterSmallT ? align_up((size_t)3 * E * 8192 * 2, 256) + 256 : 0;
}

extern "C" size_t glm53_router_workspace_bytes(int64_t T, int64_t E) {
  const size_t base = 3 * align_up((size_t)std::max<int64_t>(T, 1) * (size_t)E * sizeof(float), 256) + 256;
  return base + router_partial_bytes(T, E) + router_planes_bytes(T, E);
}

namespace glm53 {

// glm53_router_topk; with pdl the small-T kernel is launched as a
// programmatic dependent of the previous kernel on the stream (which writes x).
int router_topk(const void* x, int64_t T, int64_t H, const float* w, int64_t E, const float* bias, int top_k,
                int n_group, int topk_group, int norm_topk_prob, float routed_scaling_factor, uint32_t* indices,
                float* scores, float* logits, void* workspace, size_t workspace_bytes, cudaStream_t st, bool pdl) {
  if (T < 0 || H <= 0 || E <= 0 || E > kRouterMaxE || top_k <= 0 || top_k > kRouterMaxK || top_k > E) {
    set_last_error("glm53_router_topk: unsupported geometry T=%lld H=%lld E=%lld top_k=%d",
                   (long long)T, (long long)H, (long long)E, top_k);
    return GLM53_ERR_INVALID;
  }
  if (n_group > 1 && (n_group > 32 || E % n_group != 0 || topk_group < 1 || topk_group > n_group)) {
    set_last_error("glm53_router_topk: invalid grouping n_group=%d topk_group=%d", n_group, topk_group);
    return GLM53_ERR_INVALID;
  }
  if (T == 0) return GLM53_OK;
  if (!x || !w || !bias || !indices || !scores || !workspace ||
      workspace_bytes < glm53_router_workspace_bytes(T, E)) {
    set_last_error("glm53_router_topk: missing pointer or workspace too small");
    return GLM53_ERR_INVALID;
  }
  char* ws = (char*)workspace;
  const size_t plane = align_up((size_t)T * E * sizeof(float), 256);
  float* lbuf = logits ? logits : (float*)ws;
  const RouterScratch rs{lbuf, (float*)(ws + plane), (uint32_t*)(ws + 2 * plane), (uint32_t*)(ws + 3 * plane)};
  TopkParams p{(int)E, top_k, n_group < 1 ? 1 : n_group, topk_group, norm_topk_prob, routed_scaling_factor};
  const bool vec = (H % 4 == 0) && (((uintptr_t)w & 15) == 0) && (((uintptr_t)x & 7) == 0);
  const int per = (int)((E + 31) / 32);
  if (router_dmma_supported(T, H) && vec) {
    double* partial = (double*)(ws + 3 * plane + 256);
    if (per <= 4)
      return launch_dmma<4>((const uint16_t*)x, (int)T, (int)H, w, bias, p, partial, logits, indices, scores, st, pdl);
    if (per <= 10)
      return launch_dmma<10>((const uint16_t*)x, (int)T, (int)H, w, bias, p, partial, logits, indices, scores, st,
                             pdl);
    return launch_dmma<32>((const uint16_t*)x, (int)T, (int)H, w, bias, p, partial, logits, indices, scores, st, pdl);
  }
  if (T <= kRouterSmallT && vec) {
    if (per <= 4)
      return launch_small<4>((const uint16_t*)x, (int)T, (int)H, w, bias, p, rs, indices, scores, st, pdl);
    if (per <= 10)
      return launch_small<10>((const uint16_t*)x, (int)T, (int)H, w, bias, p, rs, indices, scores, st, pdl);
    return launch_small<32>((const uint16_t*)x, (int)T, (int)H, w, bias, p, rs, indices, scores, st, pdl);
  }
  dim3 grid((unsigned)((T + 63) / 64), (unsigned)((E + 63) / 64));
  int rc;
  double* partial_buf = (double*)(ws + 3 * plane + 256);
  if (router_tc_supported(T, H, E) && (((uintptr_t)x | (uintptr_t)w) & 15) == 0) {
    // tensor cores: the weights' BF16 planes, the logits' K-range partials,
    // their sum in range order, the top-k
    uint16_t* planes = (uint16_t*)((char*)partial_buf + router_partial_bytes(T, E));
    uint32_t* aborted = (uint32_t*)((char*)planes + router_planes_bytes(T, E) - 256);
    const int64_t n4 = E * H / 4;
    if (cudaMemsetAsync(aborted, 0, sizeof(uint32_t), st) != cudaSuccess) {
      set_last_error("glm53_router_topk: memset failed");
      return GLM53_ERR_CUDA;
    }
    router_split_kernel<<<(unsigned)std::min<int64_t>((n4 + 255) / 256, 1184), 256, 0, st>>>(w, n4, planes, E * H);
    rc = check_launch("router_split_kernel");
    if (rc) return rc;
    // at most one K range per 128-wide K block (small H with few tiles)
    const int splits = std::min(router_tc_splits(T, E), (int)(H / 128));
    rc = router_logits_tc((const uint16_t*)x, T, H, planes, E, partial_buf, splits, aborted, st);
    if (rc) return rc;
    const int64_t n = T * E;
    router_logits_reduce<<<(unsigned)std::min<int64_t>((n + 255) / 256, 1184), 256, 0, st>>>(partial_buf, splits, n,
                                                                                             lbuf);
    rc = check_launch("router_logits_reduce");
    if (rc) return rc;
    if (per <= 4) return launch_topk<4>(lbuf, (int)T, bias, p, indices, scores, st, aborted);
    if (per <= 10) return launch_topk<10>(lbuf, (int)T, bias, p, indices, scores, st, aborted);
    return launch_topk<32>(lbuf, (int)T, bias, p, indices, scores, st, aborted);
  }
  if (H % kRmBK == 0 && (((uintptr_t)x | (uintptr_t)w) & 15) == 0) {
    int splits = router_splits(T, E);
    while (splits > 1 && (H / kRmBK) % splits != 0) splits /= 2;
    double* partial = splits > 1 ? partial_buf : nullptr;
    grid.z = (unsigned)splits;
    router_mma_kernel<<<grid, 128, 0, st>>>((const uint16_t*)x, (int)T, (int)H, w, (int)E, lbuf,
                                            (int)(H / splits), partial);
    rc = check_launch("router_mma_kernel");
    if (!rc && partial) {
      const int64_t n = T * E;
      router_logits_reduce<<<(unsigned)std::min<int64_t>((n + 255) / 256, 1184), 256, 0, st>>>(partial, splits, n,
                                                                                               lbuf);
      rc = check_launch("router_logits_reduce");
    }
  } else {
    router_gemm_kernel<<<grid, 256, 0, st>>>((const uint16_t*)x, (int)T, (int)H, w, (int)E, lbuf);
    rc = check_launch("router_gemm_kernel");
  }
  if (rc) return rc;
  if (per <= 4) return launch_topk<4>(lbuf, (int)T, bias, p, indices, scores, st);
  if (per <= 10) return launch_topk<10>(lbuf, (int)T, bias, p, indices, scores, st);
  return launch_topk<32>(lbuf, (int)T, bias, p, indices, scores, st);
}

}  // namespace glm53

extern "C" int glm53_router_topk(const void* x, int64_t T, int64_t H, const float* w, int64_t E,
                                 const float* bias, int top_k, int n_group, int topk_group,
                                 int norm_topk_prob, float routed_scaling_factor, uint32_t* indices,
                                 float* scores, float* logits, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  // the small-T kernel is always a programmatic dependent of the previous
  // kernel: it writes nothing and reads only its weights before
  // griddepcontrol.wait, and a previous kernel that never lets dependents
  // launch early simply delays it to that kernel's end
  return router_topk(x, T, H, w, E, bias, top_k, n_group, topk_group, norm_topk_prob, routed_scaling_factor,
                     indices, scores, logits, workspace, workspace_bytes, (cudaStream_t)stream, true);
}
