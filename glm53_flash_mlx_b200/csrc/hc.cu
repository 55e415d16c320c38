// FFN boundary of a GLM-5.3 layer around the MoE: the mHC collapse of the
// 4-branch residual state with the post-attention RMSNorm that feeds the
// router, and the hc expand of the MoE output back into the 4-branch state.
//
// Reference flow (scripts/trace_grouped_fp8_route_amplification.py:178-214,
// scripts/profile_native_prefill_ffn_entry_seam.py:79-87):
//   collapsed, post, comb = layer.ffn_hc(state)      # mlx-vlm deepseek_v4
//   normalized = layer.post_attention_layernorm(collapsed)
//   moe = layer.mlp(normalized)
//   state = hc_expand(moe, state, post, comb)       # native_indexer_plan.metal:2362-2389
//
// Collapse (two launches):
//   hc_mix_kernel      the mixing projection m = x . fn^T over K = 4H per
//                      token (24 outputs) and the token's sum of squares,
//                      split over K: BF16 mma.sync m16n8k16 with FP32
//                      accumulation, 16 tokens x 24 outputs per CTA, each
//                      lane streaming 16-byte runs of the state and of fn
//                      (through a per-warp cp.async ring for one tile);
//                      partial sums to caller workspace [T][ksplit][25].
//   hc_finish_*        sums the partials in a fixed order, r = 1/sqrt(mean(x^2)
//                      + eps), pre/post by sigmoid, comb by softmax + Sinkhorn
//                      on 16 lanes of a warp (row sums by lane shuffles within
//                      a row group, column sums across groups), collapsed =
//                      BF16(sum_b pre[b] x[b]) in registers, then the RMSNorm
//                      of the collapsed row.  One CTA per token for small T
//                      (a ninth warp runs the Sinkhorn beside the collapse);
//                      eight tokens per CTA (one Sinkhorn per warp) for large T.
// Expand (one launch): one thread per 8 hidden columns of a token writes all
//   4 branches, so each residual run is read once and used 4 times.
#include "common.cuh"
#include "gemv_tile.cuh"

namespace glm53 {
namespace {

constexpr int kHcBranches = 4;
constexpr int kHcMix = (2 + kHcBranches) * kHcBranches;  // 24 mixing outputs
constexpr int kHcPart = kHcMix + 1;                      // + sum of squares
constexpr int kHcTileTokens = 16;
constexpr int kHcMixThreads = 128;
constexpr int kHcFinishThreads = 256;
constexpr int kHcTokenThreads = kHcFinishThreads + 32;  // + the coefficient warp
constexpr int kHcMaxChunks = 4;  // 8-column chunks per finish thread: H <= 8192
constexpr int kHcMaxSplit = 64;
constexpr int kHcStages = 4;  // cp.async ring depth of a mix warp, in 32-column K blocks
constexpr int kHcPieces = 5;  // 16-byte pieces per lane per K block: 2 state rows + 3 fn rows

__device__ __forceinline__ void mma_bf16_16816(float c[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float sq_sum8(uint4 v) {
  float s = 0.0f;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float lo = __uint_as_float(w[i] << 16), hi = __uint_as_float(w[i] & 0xffff0000u);
    s = fmaf(lo, lo, s);
    s = fmaf(hi, hi, s);
  }
  return s;
}

// One token tile (T <= 16, decode): the mixing projection through a per-warp
// cp.async ring.  Grid (1, ksplit), 4 warps.  Warp w of split y takes a
// contiguous run of 32-column K blocks (the (4y + w)-th of 4*ksplit equal
// runs), so consecutive copies stay in one DRAM page of each row.  Lane (g = lane/4,
// q = lane%4) copies 8 consecutive K values of token rows g and g+8 and of fn
// rows g, g+8, g+16 per block into its own slots of a per-warp cp.async ring
// kHcStages blocks deep (bytes in flight cost no registers) and reads back
// exactly what it copied, so the ring needs no barrier.  Two k16 MMA steps
// use values 0-3 and 4-7 of each run: the MMA sums over its 16 K positions in
// any pairing of A and B that agrees, and both operands use the same one
// (logical k = 2q+e <- 8q+e and 2q+8+e <- 8q+2+e in the first step, +4 in the
// second).
__global__ void __launch_bounds__(kHcMixThreads) hc_mix_ring_kernel(const uint16_t* __restrict__ state,
                                                                const uint16_t* __restrict__ fn, int64_t T,
                                                                int64_t K, int ksplit, float* __restrict__ part) {
  __shared__ uint4 ring[kHcMixThreads / 32][kHcStages][32][kHcPieces];
  __shared__ float red[kHcMixThreads / 32][kHcTileTokens][kHcPart];
  // The finish kernel is this grid's programmatic dependent: it may start
  // (and load the state) now; it reads the partial sums after griddepcontrol.wait.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int64_t t0 = (int64_t)blockIdx.x * kHcTileTokens;
  const bool ok0 = t0 + g < T, ok1 = t0 + g + 8 < T;
  const uint16_t* src[kHcPieces] = {state + (ok0 ? (t0 + g) * K : 0) + q * 8,
                                    state + (ok1 ? (t0 + g + 8) * K : 0) + q * 8, fn + (int64_t)g * K + q * 8,
                                    fn + (int64_t)(g + 8) * K + q * 8, fn + (int64_t)(g + 16) * K + q * 8};
  const bool valid[kHcPieces] = {ok0, ok1, true, true, true};
  const int64_t nkb = K / 32;
  const int64_t warps = (int64_t)ksplit * (kHcMixThreads / 32);
  const int64_t per = (nkb + warps - 1) / warps;
  const int64_t kb_begin = ((int64_t)blockIdx.y * (kHcMixThreads / 32) + warp) * per;
  const int64_t kb_end = kb_begin + per < nkb ? kb_begin + per : nkb;
  const int64_t n = kb_end > kb_begin ? kb_end - kb_begin : 0;
  uint4 (*slots)[32][kHcPieces] = ring[warp];
  // Copy K block kb_begin + i into slot i % kHcStages (zeros past the run).
  auto issue = [&](int64_t i) {
    const bool in = i < n;
    const int64_t k = in ? (kb_begin + i) * 32 : 0;
#pragma unroll
    for (int p = 0; p < kHcPieces; ++p)
      cp_async_16(&slots[i % kHcStages][lane][p], src[p] + k, in && valid[p]);
    cp_async_commit_group();
  };
  float acc[3][4];
#pragma unroll
  for (int j = 0; j < 3; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
  float sq0 = 0.0f, sq1 = 0.0f;
#pragma unroll
  for (int i = 0; i < kHcStages - 1; ++i) issue(i);
  for (int64_t i = 0; i < n; ++i) {
    issue(i + kHcStages - 1);
    cp_async_wait_group<kHcStages - 1>();
    const uint4* r = slots[i % kHcStages][lane];
    const uint4 a0 = r[0], a1 = r[1], b0 = r[2], b1 = r[3], b2 = r[4];
    sq0 += sq_sum8(a0);
    sq1 += sq_sum8(a1);
    mma_bf16_16816(acc[0], a0.x, a1.x, a0.y, a1.y, b0.x, b0.y);
    mma_bf16_16816(acc[0], a0.z, a1.z, a0.w, a1.w, b0.z, b0.w);
    mma_bf16_16816(acc[1], a0.x, a1.x, a0.y, a1.y, b1.x, b1.y);
    mma_bf16_16816(acc[1], a0.z, a1.z, a0.w, a1.w, b1.z, b1.w);
    mma_bf16_16816(acc[2], a0.x, a1.x, a0.y, a1.y, b2.x, b2.y);
    mma_bf16_16816(acc[2], a0.z, a1.z, a0.w, a1.w, b2.z, b2.w);
  }
  cp_async_wait_group<0>();
  sq0 += __shfl_xor_sync(0xffffffffu, sq0, 1);
  sq0 += __shfl_xor_sync(0xffffffffu, sq0, 2);
  sq1 += __shfl_xor_sync(0xffffffffu, sq1, 1);
  sq1 += __shfl_xor_sync(0xffffffffu, sq1, 2);
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    red[warp][g][8 * j + 2 * q] = acc[j][0];
    red[warp][g][8 * j + 2 * q + 1] = acc[j][1];
    red[warp][g + 8][8 * j + 2 * q] = acc[j][2];
    red[warp][g + 8][8 * j + 2 * q + 1] = acc[j][3];
  }
  if (q == 0) {
    red[warp][g][kHcMix] = sq0;
    red[warp][g + 8][kHcMix] = sq1;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kHcTileTokens * kHcPart; i += kHcMixThreads) {
    const int r = i / kHcPart, c = i % kHcPart;
    if (t0 + r >= T) continue;
    const float v = ((red[0][r][c] + red[1][r][c]) + red[2][r][c]) + red[3][r][c];
    part[((t0 + r) * ksplit + blockIdx.y) * kHcPart + c] = v;
  }
}

// More than one token tile: the same work with each lane loading its 16-byte
// runs into registers (measured faster than the ring at T = 256 and 2048).
// Grid (ceil(T/16), ksplit), 4 warps.  Warp w of split y takes a contiguous
// run of 32-column K blocks (the (4y + w)-th of 4*ksplit equal runs), so
// consecutive loads of a lane stay in one DRAM page of each row.  Lane (g = lane/4, q = lane%4)
// loads 8 consecutive K values of token rows g and g+8 and of fn rows g,
// g+8, g+16; two k16 MMA steps use values 0-3 and 4-7 of each run.  The MMA
// sums over its 16 K positions in any pairing of A and B that agrees, and
// both operands use the same one: logical k = 2q+e <- 8q+e and 2q+8+e <-
// 8q+2+e in the first step (+4 in the second).
__global__ void __launch_bounds__(kHcMixThreads) hc_mix_kernel(const uint16_t* __restrict__ state,
                                                                const uint16_t* __restrict__ fn, int64_t T,
                                                                int64_t K, int ksplit, float* __restrict__ part) {
  __shared__ float red[kHcMixThreads / 32][kHcTileTokens][kHcPart];
  // The finish kernel is this grid's programmatic dependent: it may start
  // (and load the state) now; it reads the partial sums after griddepcontrol.wait.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int64_t t0 = (int64_t)blockIdx.x * kHcTileTokens;
  const bool ok0 = t0 + g < T, ok1 = t0 + g + 8 < T;
  const uint16_t* a0p = state + (ok0 ? (t0 + g) * K : 0) + q * 8;
  const uint16_t* a1p = state + (ok1 ? (t0 + g + 8) * K : 0) + q * 8;
  const uint16_t* bp = fn + (int64_t)g * K + q * 8;
  const int64_t nkb = K / 32;
  const int64_t warps = (int64_t)ksplit * (kHcMixThreads / 32);
  const int64_t per = (nkb + warps - 1) / warps;
  const int64_t kb_begin = ((int64_t)blockIdx.y * (kHcMixThreads / 32) + warp) * per;
  const int64_t kb_end = kb_begin + per < nkb ? kb_begin + per : nkb;
  float acc[3][4];
#pragma unroll
  for (int j = 0; j < 3; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
  float sq0 = 0.0f, sq1 = 0.0f;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  constexpr int U = 4;
  for (int64_t kb = kb_begin; kb < kb_end; kb += U) {
    uint4 a0[U], a1[U], b[U][3];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t k = (kb + u) * 32;
      const bool in = kb + u < kb_end;
      a0[u] = (in && ok0) ? ldg_stream(reinterpret_cast<const uint4*>(a0p + k)) : zero;
      a1[u] = (in && ok1) ? ldg_stream(reinterpret_cast<const uint4*>(a1p + k)) : zero;
#pragma unroll
      for (int j = 0; j < 3; ++j)
        b[u][j] = in ? __ldg(reinterpret_cast<const uint4*>(bp + (int64_t)j * 8 * K + k)) : zero;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      sq0 += sq_sum8(a0[u]);
      sq1 += sq_sum8(a1[u]);
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        mma_bf16_16816(acc[j], a0[u].x, a1[u].x, a0[u].y, a1[u].y, b[u][j].x, b[u][j].y);
        mma_bf16_16816(acc[j], a0[u].z, a1[u].z, a0[u].w, a1[u].w, b[u][j].z, b[u][j].w);
      }
    }
  }
  sq0 += __shfl_xor_sync(0xffffffffu, sq0, 1);
  sq0 += __shfl_xor_sync(0xffffffffu, sq0, 2);
  sq1 += __shfl_xor_sync(0xffffffffu, sq1, 1);
  sq1 += __shfl_xor_sync(0xffffffffu, sq1, 2);
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    red[warp][g][8 * j + 2 * q] = acc[j][0];
    red[warp][g][8 * j + 2 * q + 1] = acc[j][1];
    red[warp][g + 8][8 * j + 2 * q] = acc[j][2];
    red[warp][g + 8][8 * j + 2 * q + 1] = acc[j][3];
  }
  if (q == 0) {
    red[warp][g][kHcMix] = sq0;
    red[warp][g + 8][kHcMix] = sq1;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kHcTileTokens * kHcPart; i += kHcMixThreads) {
    const int r = i / kHcPart, c = i % kHcPart;
    if (t0 + r >= T) continue;
    const float v = ((red[0][r][c] + red[1][r][c]) + red[2][r][c]) + red[3][r][c];
    part[((t0 + r) * ksplit + blockIdx.y) * kHcPart + c] = v;
  }
}

__device__ __forceinline__ float sigmoid_f32(float z) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-z)));
}

// Pairwise sum (v0 + v1) + (v2 + v3) of the four lanes {l, l^m, l^2m, l^3m}
// (m = 1 for a comb row, 4 for a column); every lane of the group gets it.
__device__ __forceinline__ float group4_sum(float v, int m) {
  const float pair = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
  return __fadd_rn(pair, __shfl_xor_sync(0xffffffffu, pair, 2 * m));
}

__device__ __forceinline__ float block_sum_256(float v, float* scratch) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) scratch[warp] = v;
  __syncthreads();
  float s = 0.0f;
#pragma unroll
  for (int w = 0; w < kHcFinishThreads / 32; ++w) s += scratch[w];
  return s;
}

struct HcFinishArgs {
  const uint16_t* state;  // [T, 4, H]
  const float* part;      // [T][ksplit][25]
  int ksplit;
  int64_t T, H;
  const float* scale;
  const float* base;
  int iters;
  float eps, norm_eps;
  const uint16_t* norm_w;  // nullptr: no RMSNorm
  float rms_eps;
  uint16_t* collapsed;   // may be nullptr
  uint16_t* normalized;  // nullptr iff norm_w is nullptr
  float* post;
  float* comb;
};

// One warp, token t, from its 25 reduced sums mix[] (shared memory, visible
// to the warp): lanes 0-3 write pre[b] to pre_out and post[b] to global memory.
__device__ __forceinline__ void hc_pre_post(const HcFinishArgs& a, int64_t t, const float* mix, float* pre_out) {
  const int l = threadIdx.x & 31;
  if (l >= kHcBranches) return;
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(mix[kHcMix], (float)(kHcBranches * a.H)),
                                                    a.norm_eps)));
  const float zp = __fadd_rn(__fmul_rn(__fmul_rn(mix[l], r), a.scale[0]), a.base[l]);
  pre_out[l] = __fadd_rn(sigmoid_f32(zp), a.eps);
  const float zq = __fadd_rn(__fmul_rn(__fmul_rn(mix[kHcBranches + l], r), a.scale[1]), a.base[kHcBranches + l]);
  a.post[t * kHcBranches + l] = __fmul_rn(2.0f, sigmoid_f32(zq));
}

// One whole warp, token t: comb by softmax + Sinkhorn.  Lane l < 16 holds
// comb[i = l/4][j = l%4]; lanes 16-31 mirror the arithmetic on a copy so every
// shuffle has all 32 lanes.
__device__ __forceinline__ void hc_comb(const HcFinishArgs& a, int64_t t, const float* mix) {
  const int l = threadIdx.x & 31;
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(mix[kHcMix], (float)(kHcBranches * a.H)),
                                                    a.norm_eps)));
  const int li = l & 15;
  const float z = __fadd_rn(__fmul_rn(__fmul_rn(mix[2 * kHcBranches + li], r), a.scale[2]),
                            a.base[2 * kHcBranches + li]);
  float mx = fmaxf(z, __shfl_xor_sync(0xffffffffu, z, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  const float e = expf(__fadd_rn(z, -mx));
  float c = __fadd_rn(__fdiv_rn(e, group4_sum(e, 1)), a.eps);
  for (int it = 0; it < a.iters; ++it) {
    if (it > 0) c = __fdiv_rn(c, __fadd_rn(group4_sum(c, 1), a.eps));
    c = __fdiv_rn(c, __fadd_rn(group4_sum(c, 4), a.eps));
  }
  if (l < 16) a.comb[t * 16 + l] = c;
}

__device__ __forceinline__ void hc_coefficients(const HcFinishArgs& a, int64_t t, const float* mix,
                                                float* pre_out) {
  hc_pre_post(a, t, mix, pre_out);
  hc_comb(a, t, mix);
}

// The four branch runs of 8 columns at chunk c of token t.
__device__ __forceinline__ void load_branches(const HcFinishArgs& a, int64_t t, int c, uint4 x[kHcBranches]) {
  const uint16_t* xs = a.state + t * kHcBranches * a.H + (int64_t)c * 8;
#pragma unroll
  for (int b = 0; b < kHcBranches; ++b) x[b] = ldg_stream(reinterpret_cast<const uint4*>(xs + b * a.H));
}

// collapsed = BF16(((p0 x0 + p1 x1) + p2 x2) + p3 x3) for 8 columns, products
// and sums rounded one by one.
__device__ __forceinline__ uint4 collapse8(const uint4 x[kHcBranches], const float* pre) {
  const float p0 = pre[0], p1 = pre[1], p2 = pre[2], p3 = pre[3];
  const uint16_t* h0 = reinterpret_cast<const uint16_t*>(&x[0]);
  const uint16_t* h1 = reinterpret_cast<const uint16_t*>(&x[1]);
  const uint16_t* h2 = reinterpret_cast<const uint16_t*>(&x[2]);
  const uint16_t* h3 = reinterpret_cast<const uint16_t*>(&x[3]);
  uint16_t o[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    float y = __fmul_rn(p0, bf16_bits_to_f32(h0[e]));
    y = __fadd_rn(y, __fmul_rn(p1, bf16_bits_to_f32(h1[e])));
    y = __fadd_rn(y, __fmul_rn(p2, bf16_bits_to_f32(h2[e])));
    y = __fadd_rn(y, __fmul_rn(p3, bf16_bits_to_f32(h3[e])));
    o[e] = f32_to_bf16_bits(y);
  }
  return *reinterpret_cast<const uint4*>(o);
}

// out = BF16(w * BF16(x * inv)) for 8 columns (MLX fast rms_norm rounding).
__device__ __forceinline__ uint4 norm8(uint4 xv, uint4 wv, float inv) {
  const uint16_t* w = reinterpret_cast<const uint16_t*>(&wv);
  const uint16_t* x = reinterpret_cast<const uint16_t*>(&xv);
  uint16_t o[8];
#pragma unroll
  for (int e = 0; e < 8; ++e)
    o[e] = f32_to_bf16_bits(__fmul_rn(bf16_bits_to_f32(w[e]), bf16_round(__fmul_rn(bf16_bits_to_f32(x[e]), inv))));
  return *reinterpret_cast<const uint4*>(o);
}

__device__ __forceinline__ float rms_inv(float sumsq, int64_t H, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sumsq, (float)H), eps)));
}

// Sum over the 256 collapse threads of a token CTA (warps 0-7), on named
// barrier 1 so that the coefficient warp (warp 8) is not waited for.
__device__ __forceinline__ float collapse_warps_sum(float v, float* scratch) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
  asm volatile("bar.sync 1, %0;" ::"n"(kHcFinishThreads) : "memory");
  float s = 0.0f;
#pragma unroll
  for (int w = 0; w < kHcFinishThreads / 32; ++w) s += scratch[w];
  return s;
}

// Small T: one CTA per token, 8 collapse warps + 1 coefficient warp.  The
// collapse threads issue the loads of their state chunks first; the 25 sums
// are reduced (8 groups of splits g, g+8, ... in parallel, then the groups in
// order); the coefficient warp computes pre and post, then runs the Sinkhorn
// iterations for comb while warps 0-7 collapse and normalise the row (which
// need only pre).  Barrier 0 is last used before that split.
template <int MAXC>
__global__ void __launch_bounds__(kHcTokenThreads) hc_finish_token_kernel(HcFinishArgs a) {
  __shared__ float s_red[8][kHcPart];
  __shared__ float s_mix[kHcPart];
  __shared__ float s_pre[kHcBranches];
  __shared__ float s_sum[kHcFinishThreads / 32];
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  const bool coef_warp = tid >= kHcFinishThreads;
  const int nchunks = (int)(a.H / 8);
  uint4 xv[MAXC][kHcBranches];
  if (!coef_warp) {
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = tid + i * kHcFinishThreads;
      if (c < nchunks) load_branches(a, t, c, xv[i]);
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the mix kernel's partial sums
  if (tid < 8 * kHcPart) {
    const int g = tid / kHcPart, col = tid % kHcPart;
    const float* p = a.part + t * a.ksplit * kHcPart + col;
    float v[kHcMaxSplit / 8];
#pragma unroll
    for (int j = 0; j < kHcMaxSplit / 8; ++j) {
      const int s = g + 8 * j;
      v[j] = s < a.ksplit ? p[(int64_t)s * kHcPart] : 0.0f;
    }
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < kHcMaxSplit / 8; ++j) acc = __fadd_rn(acc, v[j]);
    s_red[g][col] = acc;
  }
  __syncthreads();
  if (tid < kHcPart) {
    float acc = 0.0f;
#pragma unroll
    for (int g = 0; g < 8; ++g) acc = __fadd_rn(acc, s_red[g][tid]);
    s_mix[tid] = acc;
  }
  __syncthreads();
  if (coef_warp) hc_pre_post(a, t, s_mix, s_pre);
  __syncthreads();
  if (coef_warp) {
    hc_comb(a, t, s_mix);
    return;
  }
  uint4 cv[MAXC];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + i * kHcFinishThreads;
    if (c >= nchunks) break;
    cv[i] = collapse8(xv[i], s_pre);
    if (a.collapsed) *reinterpret_cast<uint4*>(a.collapsed + t * a.H + c * 8) = cv[i];
    ss += sq_sum8(cv[i]);
  }
  if (a.norm_w == nullptr) return;
  const float inv = rms_inv(collapse_warps_sum(ss, s_sum), a.H, a.rms_eps);
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + i * kHcFinishThreads;
    if (c >= nchunks) break;
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(a.norm_w + c * 8));
    *reinterpret_cast<uint4*>(a.normalized + t * a.H + c * 8) = norm8(cv[i], wv, inv);
  }
}

// Large T (ksplit <= 8, H <= 4096): eight tokens per CTA.  Warp w reduces the
// sums of token t0 + w (lane = column, its ksplit loads in flight together)
// and runs that token's Sinkhorn, so eight run at once per CTA; then all
// threads collapse and normalise the eight rows in turn, the next row's state
// loads issued before the current row's norm reduction.
__global__ void __launch_bounds__(kHcFinishThreads) hc_finish_group_kernel(HcFinishArgs a) {
  constexpr int TPC = 8, MAXC = 2;
  __shared__ float s_mix[TPC][kHcPart];
  __shared__ float s_pre[TPC][kHcBranches];
  __shared__ float s_sum[2][kHcFinishThreads / 32];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t t0 = (int64_t)blockIdx.x * TPC;
  const int ntok = (int)(a.T - t0 < TPC ? a.T - t0 : TPC);
  const int nchunks = (int)(a.H / 8);
  uint4 xv[MAXC][kHcBranches];
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + i * kHcFinishThreads;
    if (c < nchunks) load_branches(a, t0, c, xv[i]);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the mix kernel's partial sums
  if (warp < ntok) {
    const int64_t t = t0 + warp;
    if (lane < kHcPart) {
      const float* p = a.part + t * a.ksplit * kHcPart + lane;
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = j < a.ksplit ? p[(int64_t)j * kHcPart] : 0.0f;
      float acc = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) acc = __fadd_rn(acc, v[j]);
      s_mix[warp][lane] = acc;
    }
    __syncwarp();
    hc_coefficients(a, t, s_mix[warp], s_pre[warp]);
  }
  __syncthreads();
  for (int k = 0; k < ntok; ++k) {
    const int64_t t = t0 + k;
    uint4 cv[MAXC];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = tid + i * kHcFinishThreads;
      if (c >= nchunks) break;
      cv[i] = collapse8(xv[i], s_pre[k]);
      if (a.collapsed) *reinterpret_cast<uint4*>(a.collapsed + t * a.H + c * 8) = cv[i];
      ss += sq_sum8(cv[i]);
    }
    if (k + 1 < ntok) {
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = tid + i * kHcFinishThreads;
        if (c < nchunks) load_branches(a, t + 1, c, xv[i]);
      }
    }
    if (a.norm_w == nullptr) continue;
    // Alternate scratch rows: a row is rewritten only two tokens later, after
    // every thread has passed the intervening token's barrier.
    const float inv = rms_inv(block_sum_256(ss, s_sum[k & 1]), a.H, a.rms_eps);
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = tid + i * kHcFinishThreads;
      if (c >= nchunks) break;
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(a.norm_w + c * 8));
      *reinterpret_cast<uint4*>(a.normalized + t * a.H + c * 8) = norm8(cv[i], wv, inv);
    }
  }
}

// RMSNorm of BF16 rows alone: one CTA per row.
template <int MAXC>
__global__ void __launch_bounds__(kHcFinishThreads) rms_norm_kernel(const uint16_t* __restrict__ x, int64_t H,
                                                                    const uint16_t* __restrict__ w, float eps,
                                                                    uint16_t* __restrict__ out) {
  __shared__ float s_sum[kHcFinishThreads / 32];
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  const int nchunks = (int)(H / 8);
  uint4 xv[MAXC];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + i * kHcFinishThreads;
    if (c >= nchunks) break;
    xv[i] = __ldg(reinterpret_cast<const uint4*>(x + t * H + c * 8));
    ss += sq_sum8(xv[i]);
  }
  const float inv = rms_inv(block_sum_256(ss, s_sum), H, eps);
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + i * kHcFinishThreads;
    if (c >= nchunks) break;
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + c * 8));
    *reinterpret_cast<uint4*>(out + t * H + c * 8) = norm8(xv[i], wv, inv);
  }
}

// out[t][b][d] = BF16(post[t][b] * moe[t][d] + sum_s fma-chain comb[t][s][b] *
// residual[t][s][d]), the order of native_indexer_plan.metal:2377-2388.
__global__ void __launch_bounds__(256) hc_expand_kernel(const uint16_t* __restrict__ moe,
                                                         const uint16_t* __restrict__ residual,
                                                         const float* __restrict__ post,
                                                         const float* __restrict__ comb, int64_t T, int64_t H,
                                                         uint16_t* __restrict__ out) {
  const int64_t chunks = H / 8;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= T * chunks) return;
  const int64_t t = idx / chunks, d = (idx % chunks) * 8;
  const uint4 mv = ldg_stream(reinterpret_cast<const uint4*>(moe + t * H + d));
  uint4 rv[kHcBranches];
#pragma unroll
  for (int s = 0; s < kHcBranches; ++s)
    rv[s] = ldg_stream(reinterpret_cast<const uint4*>(residual + (t * kHcBranches + s) * H + d));
  const float4 pv = __ldg(reinterpret_cast<const float4*>(post + t * kHcBranches));
  float cm[16];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 c4 = __ldg(reinterpret_cast<const float4*>(comb + t * 16) + i);
    cm[4 * i] = c4.x;
    cm[4 * i + 1] = c4.y;
    cm[4 * i + 2] = c4.z;
    cm[4 * i + 3] = c4.w;
  }
  const float pb[4] = {pv.x, pv.y, pv.z, pv.w};
  const uint16_t* m = reinterpret_cast<const uint16_t*>(&mv);
#pragma unroll
  for (int b = 0; b < kHcBranches; ++b) {
    uint16_t o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float mixed = 0.0f;
#pragma unroll
      for (int s = 0; s < kHcBranches; ++s)
        mixed = __fmaf_rn(cm[s * 4 + b], bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(&rv[s])[e]), mixed);
      o[e] = f32_to_bf16_bits(__fadd_rn(__fmul_rn(pb[b], bf16_bits_to_f32(m[e])), mixed));
    }
    *reinterpret_cast<uint4*>(out + (t * kHcBranches + b) * H + d) = *reinterpret_cast<const uint4*>(o);
  }
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// K split of the mixing projection: about four CTAs per SM in total, at
// least one 32-column K block per warp, a power of two up to 64.
int hc_split(int64_t T, int64_t H) {
  const int64_t tiles = (T + kHcTileTokens - 1) / kHcTileTokens;
  const int64_t nkb = kHcBranches * H / 32;
  int s = 1;
  while (s < kHcMaxSplit && tiles * s < 4 * kNumSMs && (int64_t)(2 * s) * (kHcMixThreads / 32) <= nkb) s *= 2;
  return s;
}

bool hc_geometry_ok(int64_t H) { return H > 0 && H % 8 == 0 && H / 8 <= kHcMaxChunks * kHcFinishThreads; }

}  // namespace
}  // namespace glm53

using namespace glm53;

extern "C" size_t glm53_hc_collapse_workspace_bytes(int64_t T, int64_t H) {
  if (T <= 0 || !hc_geometry_ok(H)) return 0;
  return (size_t)T * hc_split(T, H) * kHcPart * sizeof(float);
}

extern "C" int glm53_hc_collapse_norm(const void* state, int64_t T, int64_t H, int branches, const void* hc_fn,
                                      const float* hc_scale, const float* hc_base, int sinkhorn_iters,
                                      float hc_eps, float hc_norm_eps, const void* norm_weight, float rms_eps,
                                      void* collapsed, void* normalized, float* post, float* comb,
                                      void* workspace, size_t workspace_bytes, void* stream) {
  if (branches != kHcBranches) {
    set_last_error("glm53_hc_collapse_norm: %d branches; the kernels are built for 4", branches);
    return GLM53_ERR_INVALID;
  }
  if (T < 0 || !hc_geometry_ok(H)) {
    set_last_error("glm53_hc_collapse_norm: hidden size %lld must be a positive multiple of 8 up to %d",
                   (long long)H, kHcMaxChunks * kHcFinishThreads * 8);
    return GLM53_ERR_INVALID;
  }
  if (sinkhorn_iters < 1 || sinkhorn_iters > 1000) {
    set_last_error("glm53_hc_collapse_norm: sinkhorn_iters %d outside [1, 1000]", sinkhorn_iters);
    return GLM53_ERR_INVALID;
  }
  if ((norm_weight == nullptr) != (normalized == nullptr)) {
    set_last_error("glm53_hc_collapse_norm: norm_weight and normalized must both be given or both be NULL");
    return GLM53_ERR_INVALID;
  }
  if (T == 0) return GLM53_OK;
  if (!state || !hc_fn || !hc_scale || !hc_base || !post || !comb || !workspace) {
    set_last_error("glm53_hc_collapse_norm: NULL argument");
    return GLM53_ERR_INVALID;
  }
  if (!aligned16(state) || !aligned16(hc_fn) || !aligned16(post) || !aligned16(comb) || !aligned16(workspace) ||
      (collapsed && !aligned16(collapsed)) || (normalized && !aligned16(normalized)) ||
      (norm_weight && !aligned16(norm_weight))) {
    set_last_error("glm53_hc_collapse_norm: state, fn, norm weight, outputs and workspace must be 16-byte aligned");
    return GLM53_ERR_INVALID;
  }
  const size_t need = glm53_hc_collapse_workspace_bytes(T, H);
  if (workspace_bytes < need) {
    set_last_error("glm53_hc_collapse_norm: workspace %zu bytes < %zu", workspace_bytes, need);
    return GLM53_ERR_INVALID;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const int ksplit = hc_split(T, H);
  const int64_t K = kHcBranches * H;
  float* part = static_cast<float*>(workspace);
  dim3 grid((unsigned)((T + kHcTileTokens - 1) / kHcTileTokens), (unsigned)ksplit);
  if (T <= kHcTileTokens)
    hc_mix_ring_kernel<<<grid, kHcMixThreads, 0, st>>>((const uint16_t*)state, (const uint16_t*)hc_fn, T, K, ksplit,
                                                       part);
  else
    hc_mix_kernel<<<grid, kHcMixThreads, 0, st>>>((const uint16_t*)state, (const uint16_t*)hc_fn, T, K, ksplit, part);
  int rc = check_launch("hc_mix_kernel");
  if (rc) return rc;
  HcFinishArgs a{(const uint16_t*)state, part, ksplit, T, H, hc_scale, hc_base, sinkhorn_iters, hc_eps,
                 hc_norm_eps, (const uint16_t*)norm_weight, rms_eps, (uint16_t*)collapsed, (uint16_t*)normalized,
                 post, comb};
  // Launched as the mix kernel's programmatic dependent (the state loads of
  // its first row overlap the mix kernel; griddepcontrol.wait orders the rest).
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kHcFinishThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (ksplit <= 8 && H <= 2 * 8 * kHcFinishThreads && T >= 512) {
    cfg.gridDim = dim3((unsigned)((T + 7) / 8));
    cudaLaunchKernelEx(&cfg, hc_finish_group_kernel, a);
  } else if (H <= 2 * 8 * kHcFinishThreads) {
    cfg.gridDim = dim3((unsigned)T);
    cfg.blockDim = dim3(kHcTokenThreads);
    cudaLaunchKernelEx(&cfg, hc_finish_token_kernel<2>, a);
  } else {
    cfg.gridDim = dim3((unsigned)T);
    cfg.blockDim = dim3(kHcTokenThreads);
    cudaLaunchKernelEx(&cfg, hc_finish_token_kernel<kHcMaxChunks>, a);
  }
  return check_launch("hc_finish_kernel");
}

extern "C" int glm53_rms_norm(const void* x, int64_t T, int64_t H, const void* weight, float eps, void* out,
                              void* stream) {
  if (T < 0 || !hc_geometry_ok(H)) {
    set_last_error("glm53_rms_norm: hidden size %lld must be a positive multiple of 8 up to %d", (long long)H,
                   kHcMaxChunks * kHcFinishThreads * 8);
    return GLM53_ERR_INVALID;
  }
  if (T == 0) return GLM53_OK;
  if (!x || !weight || !out || !aligned16(x) || !aligned16(weight) || !aligned16(out)) {
    set_last_error("glm53_rms_norm: x, weight and out must be non-NULL and 16-byte aligned");
    return GLM53_ERR_INVALID;
  }
  cudaStream_t st = (cudaStream_t)stream;
  if (H <= 2 * 8 * kHcFinishThreads)
    rms_norm_kernel<2><<<(unsigned)T, kHcFinishThreads, 0, st>>>((const uint16_t*)x, H, (const uint16_t*)weight, eps,
                                                                 (uint16_t*)out);
  else
    rms_norm_kernel<kHcMaxChunks><<<(unsigned)T, kHcFinishThreads, 0, st>>>((const uint16_t*)x, H,
                                                                            (const uint16_t*)weight, eps,
                                                                            (uint16_t*)out);
  return check_launch("rms_norm_kernel");
}

extern "C" int glm53_hc_expand(const void* moe, const void* residual, const float* post, const float* comb,
                               int64_t T, int64_t H, int branches, void* out, void* stream) {
  if (branches != kHcBranches) {
    set_last_error("glm53_hc_expand: %d branches; the kernel is built for 4", branches);
    return GLM53_ERR_INVALID;
  }
  if (T < 0 || H <= 0 || H % 8 != 0) {
    set_last_error("glm53_hc_expand: hidden size %lld must be a positive multiple of 8", (long long)H);
    return GLM53_ERR_INVALID;
  }
  if (T == 0) return GLM53_OK;
  if (!moe || !residual || !post || !comb || !out) {
    set_last_error("glm53_hc_expand: NULL argument");
    return GLM53_ERR_INVALID;
  }
  if (!aligned16(moe) || !aligned16(residual) || !aligned16(post) || !aligned16(comb) || !aligned16(out)) {
    set_last_error("glm53_hc_expand: tensors must be 16-byte aligned");
    return GLM53_ERR_INVALID;
  }
  const int64_t threads = T * (H / 8);
  hc_expand_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint16_t*)moe, (const uint16_t*)residual, post, comb, T, H, (uint16_t*)out);
  return check_launch("hc_expand_kernel");
}
