// Block-128 E4M3 linear (G1): y[M,N] = x[M,K] @ dequant(w[N,K], s)^T.
//
// Replaces block_fp8_linear (glm53_flash_mlx/fp8.py:254-299) and its Metal
// kernels K1/K2 (fp8.py:41-116).  Small M is HBM-bound: every weight byte is
// read once with 16-byte streaming loads and decoded in registers into
// tensor-core fragments (gemv_tile.cuh).  Large M goes to the tcgen05 GEMM
// (grouped_tc.cu, one dense "expert") when the caller passes a workspace
// (glm53_fp8_linear_ws), else to the mma.sync GEMM (grouped.cu).
#include <algorithm>

#include "common.cuh"
#include "gemv_tile.cuh"
#include "kernels.cuh"

namespace glm53 {

// Tensor-core GEMV: persistent blocks over 16-row tiles for one chunk of up
// to 8 activation rows (blockIdx.y); K split across ksplit_for(K) warps, each
// streaming its K range through a cp.async ring; ordered cross-warp sum.
// Requires K % 128 == 0 and 16-byte aligned x / w rows.
// Ring depth P (64-wide K slices in flight per warp): 8, or 5 when that is
// what lets every 16-row tile run in one wave (three blocks per SM instead of
// two): config 1 (6144 x 4096, 384 tiles) measured 8.30 -> 6.86 us per call,
// while shapes that fit one wave at depth 8 are fastest there (4096 x 12288:
// 12.7 us at 8, 17.0 at 5).
// TG groups of KS warps per block stream TG tiles at once over one staged copy
// of the activation rows (group g takes the block's tiles g, g + TG, ...): with
// eight rows staged (64 KB at K = 4096) only one block fits an SM, and two
// groups keep as many bytes in flight as the one-row launch's blocks do.
// Every output is the same ordered sum of the same per-warp K ranges whatever
// TG, P and the grid.
template <int KS, int TG, bool FINITE, int P>
__global__ void __launch_bounds__(32 * KS * TG) gemv_stream_kernel(const uint16_t* __restrict__ x, int M, int K,
                                                                   const uint8_t* __restrict__ w, int N,
                                                                   const float* __restrict__ s,
                                                                   uint16_t* __restrict__ y, int chunk) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const int grp = warp / KS, kwarp = warp - grp * KS;
  const int m0 = blockIdx.y * chunk;
  const int ncols = min(chunk, M - m0);
  const int stride = (xs_stride(K) + 7) & ~7;
  uint4* ring = reinterpret_cast<uint4*>(smem) + (size_t)warp * P * 64;
  __half* xs = reinterpret_cast<__half*>(reinterpret_cast<uint4*>(smem) + (size_t)KS * TG * P * 64);
  float* red = reinterpret_cast<float*>(xs + (size_t)chunk * stride);  // [TG][2][KS][128]
  float* scratch = red + TG * 2 * KS * 128;
  const int ntiles = (N + 15) >> 4;
  const int cta_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int my_tiles = cta_tiles > grp ? (cta_tiles - 1 - grp) / TG + 1 : 0;
  auto row_of = [&](int it) { return (blockIdx.x + (grp + it * TG) * gridDim.x) << 4; };
  const int kper = K / KS;
  const int nslice = kper >> 6;
  const int kw = kwarp * kper + 16 * q;
  const int scols = K >> 7;
  // issue cursor (tile, slice) runs P - 1 slices ahead of the consume cursor
  int i_it = 0, i_sl = 0;
  auto issue = [&]() {
    if (i_it < my_tiles) {
      const int row0 = row_of(i_it);
      const int k = kw + 64 * i_sl;
      uint4* dst = ring + ((i_it * nslice + i_sl) % P) * 64 + lane;
      const bool v0 = row0 + g < N, v8 = row0 + g + 8 < N;
      cp_async_16_l2_256(dst, v0 ? (const void*)(w + (size_t)(row0 + g) * K + k) : (const void*)w, v0);
      cp_async_16_l2_256(dst + 32, v8 ? (const void*)(w + (size_t)(row0 + g + 8) * K + k) : (const void*)w, v8);
      if (++i_sl == nslice) {
        i_sl = 0;
        ++i_it;
      }
    }
    cp_async_commit_group();
  };
#pragma unroll 1
  for (int p = 0; p < P - 1; ++p) issue();
  // Launched as a programmatic dependent of the previous kernel on the stream:
  // the weight slices above never depend on it, so they stream while it
  // finishes; x is read and y written only after it has completed.  The next
  // kernel may launch now (its CTAs take SMs as this grid's CTAs exit).
  pdl_trigger();
  pdl_wait();
  const float smul = decode_unscale<FINITE>() * stage_f16(xs, stride, x + (size_t)m0 * K, K, ncols, K, scratch);
  float part[4] = {0.f, 0.f, 0.f, 0.f}, tot[4] = {0.f, 0.f, 0.f, 0.f};
  // this warp's block scales of the current tile, the next tile's prefetched
  const int nb = kper >> 7;
  auto srow_of = [&](int it) { return s + (size_t)(row_of(it) >> 7) * scols + ((kwarp * kper) >> 7); };
  WarpScales cur, nxt;
  cur.load(srow_of(0), nb, my_tiles > 0);
  int u = 0;
  for (int it = 0; it < my_tiles; ++it) {
    const int row0 = row_of(it);
    nxt.load(srow_of(it + 1), nb, it + 1 < my_tiles);
    for (int sl = 0; sl < nslice; ++sl, ++u) {
      issue();
      cp_async_wait_group<P - 1>();
      const uint4* src = ring + (u % P) * 64 + lane;
      const uint4 f0 = src[0], f1 = src[32];
      uint32_t xw[8];
      load_x_frag(xw, xs + (g < ncols ? g : 0) * stride + kw + 64 * sl, g < ncols);
      mma_slice<FINITE>(part, f0, f1, xw);
      if (sl & 1) promote(tot, part, cur.at(sl >> 1) * smul);
    }
    cur = nxt;
    float* r = red + ((grp * 2 + (it & 1)) * KS + kwarp) * 128;
    r[g * 8 + 2 * q] = tot[0];
    r[g * 8 + 2 * q + 1] = tot[1];
    r[(g + 8) * 8 + 2 * q] = tot[2];
    r[(g + 8) * 8 + 2 * q + 1] = tot[3];
#pragma unroll
    for (int c = 0; c < 4; ++c) tot[c] = 0.f;
    // the group's KS warps only (barrier 1 + group; stage_f16 used barrier 0)
    asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(32 * KS) : "memory");
    const float* rb = red + (grp * 2 + (it & 1)) * KS * 128;
    for (int i = threadIdx.x - grp * 32 * KS; i < 128; i += 32 * KS) {
      const int rr = i >> 3, c = i & 7;
      if (c < ncols && row0 + rr < N) {
        float v = 0.f;
#pragma unroll
        for (int ww = 0; ww < KS; ++ww) v = v + rb[ww * 128 + i];
        y[(size_t)(m0 + c) * N + row0 + rr] = f32_to_bf16_bits(v);
      }
    }
  }
  cp_async_wait_group<0>();
}

// Generic path for any K / alignment: one warp per (row m, output n).
__global__ void __launch_bounds__(256) fp8_linear_scalar_kernel(const uint16_t* __restrict__ x, int64_t M,
                                                                int64_t K, const uint8_t* __restrict__ w,
                                                                int64_t N, const float* __restrict__ s,
                                                                uint16_t* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (warp >= M * N) return;
  const int64_t m = warp / N, n = warp % N;
  const int64_t scale_cols = (K + kBlock - 1) / kBlock;
  const uint8_t* wr = w + n * K;
  const uint16_t* xr = x + m * K;
  const float* srow = s + (n / kBlock) * scale_cols;
  float acc = 0.f;
  for (int64_t k = lane; k < K; k += 32)
    acc = fmaf(bf16_bits_to_f32(xr[k]) * e4m3_to_f32_scaled(wr[k]), srow[k / kBlock] * 256.0f, acc);
  acc = warp_sum(acc);
  if (lane == 0) y[m * N + n] = f32_to_bf16_bits(acc);
}

static size_t gemv_smem(int KS, int P, int chunk, int64_t K, int TG = 1) {
  return (size_t)KS * TG * P * 64 * 16 + (size_t)chunk * ((xs_stride(K) + 7) & ~7) * 2 +
         (size_t)(TG * 2 * KS * 128 + 32) * sizeof(float);
}

// Blocks per SM the launch counts on: up to three (one 16-row tile per block
// for N up to 444 * 16 rows, so no block streams two tiles while others idle).
static int gemv_per_sm(size_t smem) { return std::max(1, std::min(3, (int)((220 * 1024) / smem))); }

template <int KS, int TG, bool FINITE, int P>
static int launch_gemv_ring(const uint16_t* x, int M, int K, const uint8_t* w, int N, const float* s, uint16_t* y,
                            int chunk, cudaStream_t stream) {
  const size_t smem = gemv_smem(KS, P, chunk, K, TG);
  int rc_attr = ensure_max_smem((const void*)gemv_stream_kernel<KS, TG, FINITE, P>, smem);
  if (rc_attr) return rc_attr;
  const int ntiles = (N + 15) / 16;
  const int chunks = (M + chunk - 1) / chunk;
  const int per_sm = gemv_per_sm(smem);
  const int bx = std::max(1, std::min((ntiles + TG - 1) / TG, (sm_count() * per_sm + chunks - 1) / chunks));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)bx, (unsigned)chunks);
  cfg.blockDim = dim3(32 * KS * TG);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, gemv_stream_kernel<KS, TG, FINITE, P>, x, M, K, w, N, s, y, chunk);
  return check_launch("gemv_stream_kernel");
}

template <int KS, bool FINITE>
static int launch_gemv_stream(const uint16_t* x, int M, int K, const uint8_t* w, int N, const float* s,
                              uint16_t* y, cudaStream_t stream) {
  int chunk = std::min(8, M);
  while (chunk > 1 && gemv_smem(KS, 8, chunk, K) > 200 * 1024) chunk = (chunk + 1) / 2;
  // two tile groups per block when the staged rows leave room for only one
  // single-group block per SM and two groups' rings fit beside them
  if (KS * 2 <= 16 && gemv_per_sm(gemv_smem(KS, 8, chunk, K)) == 1 &&
      gemv_smem(KS, 8, chunk, K, 2) <= 220 * 1024)
    return launch_gemv_ring<KS, 2, FINITE, 8>(x, M, K, w, N, s, y, chunk, stream);
  const int64_t units = (int64_t)((N + 15) / 16) * ((M + chunk - 1) / chunk);
  const int64_t wave8 = (int64_t)sm_count() * gemv_per_sm(gemv_smem(KS, 8, chunk, K));
  const int64_t wave5 = (int64_t)sm_count() * gemv_per_sm(gemv_smem(KS, 5, chunk, K));
  if (units > wave8 && units <= wave5)
    return launch_gemv_ring<KS, 1, FINITE, 5>(x, M, K, w, N, s, y, chunk, stream);
  return launch_gemv_ring<KS, 1, FINITE, 8>(x, M, K, w, N, s, y, chunk, stream);
}

template <bool FINITE>
static int dispatch_gemv(const uint16_t* x, int M, int K, const uint8_t* w, int N, const float* s, uint16_t* y,
                         cudaStream_t stream) {
  switch (ksplit_for(K)) {
    case 8: return launch_gemv_stream<8, FINITE>(x, M, K, w, N, s, y, stream);
    case 6: return launch_gemv_stream<6, FINITE>(x, M, K, w, N, s, y, stream);
    case 4: return launch_gemv_stream<4, FINITE>(x, M, K, w, N, s, y, stream);
    case 3: return launch_gemv_stream<3, FINITE>(x, M, K, w, N, s, y, stream);
    case 2: return launch_gemv_stream<2, FINITE>(x, M, K, w, N, s, y, stream);
    default: return launch_gemv_stream<1, FINITE>(x, M, K, w, N, s, y, stream);
  }
}

int fp8_linear_small_m(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w, int64_t N,
                       const float* s, uint16_t* y, uint32_t flags, cudaStream_t stream) {
  const bool tc = (K % 128 == 0) && (((uintptr_t)w & 15) == 0) && (((uintptr_t)x & 15) == 0) &&
                  gemv_smem(ksplit_for(K), 8, 1, K) <= 200 * 1024 && N <= INT32_MAX - 16;
  if (!tc) {
    int64_t warps = M * N;
    int64_t blocks = (warps + 7) / 8;
    fp8_linear_scalar_kernel<<<(unsigned)blocks, 256, 0, stream>>>(x, M, K, w, N, s, y);
    return check_launch("fp8_linear_scalar_kernel");
  }
  if (flags & GLM53_FLAG_E4M3_FINITE) return dispatch_gemv<true>(x, (int)M, (int)K, w, (int)N, s, y, stream);
  return dispatch_gemv<false>(x, (int)M, (int)K, w, (int)N, s, y, stream);
}

}  // namespace glm53

using namespace glm53;

// Workspace of glm53_fp8_linear_ws: FP16 activation rows and their power-of-two
// multipliers for the tcgen05 path.
static size_t linear_ws_bytes(int64_t M, int64_t K) {
  return align_up((size_t)M * K * sizeof(__half), 256) + align_up((size_t)M * sizeof(float), 256);
}

extern "C" size_t glm53_fp8_linear_workspace_bytes(int64_t M, int64_t K) {
  return M > 0 && K > 0 ? linear_ws_bytes(M, K) : 0;
}

// K-range count of the tcgen05 GEMM for M rows x N outputs (1: no split).
static int linear_splits(int64_t M, int64_t K, int64_t N) {
  if (M <= kGemvMaxRows || K % 128 != 0) return 1;
  return grouped_tc_splits(((M + 127) / 128) * ((N + 127) / 128), K / 128);
}

extern "C" size_t glm53_fp8_linear_splitk_workspace_bytes(int64_t M, int64_t K, int64_t N) {
  if (M <= 0 || K <= 0 || N <= 0) return 0;
  return linear_ws_bytes(M, K) + grouped_tc_splitk_bytes(M, N, linear_splits(M, K, N));
}

extern "C" int glm53_fp8_linear_ws(const void* x, int64_t M, int64_t K, const uint8_t* w, int64_t N,
                                   const float* scale_inv, void* y, void* workspace, size_t workspace_bytes,
                                   uint32_t* status, uint32_t flags, void* stream) {
  if (M < 0 || K <= 0 || N <= 0 || (M > 0 && (!x || !w || !scale_inv || !y))) {
    set_last_error("glm53_fp8_linear_ws: invalid arguments M=%lld K=%lld N=%lld", (long long)M, (long long)K,
                   (long long)N);
    return GLM53_ERR_INVALID;
  }
  if (M == 0) return GLM53_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const bool aligned = ((((uintptr_t)x | (uintptr_t)w | (uintptr_t)workspace) & 15) == 0) && K % 8 == 0;
  if (M > kGemvMaxRows && workspace && status && workspace_bytes >= linear_ws_bytes(M, K) && aligned &&
      grouped_tc_supported(K, N, 0.0f, false) && M <= INT32_MAX / 2) {
    __half* x16 = (__half*)workspace;
    float* xscale = (float*)((char*)workspace + align_up((size_t)M * K * sizeof(__half), 256));
    int rc = rows_to_f16((const uint16_t*)x, K, nullptr, 1, M, x16, xscale, st);
    if (rc) return rc;
    TcGemm g{};
    g.x16 = x16;
    g.xscale = xscale;
    g.R = M;
    g.K = K;
    g.capacity = (M + 127) / 128;
    g.max_rows = 128;
    g.dense = true;
    g.w = w;
    g.w_rows = N;
    g.s_gate = scale_inv;
    g.E = 1;
    g.N = N;
    g.swiglu = false;
    g.finite = (flags & GLM53_FLAG_E4M3_FINITE) != 0;
    g.out = (uint16_t*)y;
    g.status = status;
    // fewer output tiles than SMs: split K when the caller's workspace holds
    // the partial sums (glm53_fp8_linear_splitk_workspace_bytes)
    const int splits = linear_splits(M, K, N);
    if (splits > 1 && workspace_bytes >= linear_ws_bytes(M, K) + grouped_tc_splitk_bytes(M, N, splits)) {
      g.splits = splits;
      g.partial = (float*)((char*)workspace + linear_ws_bytes(M, K));
    }
    return grouped_tc(g, st);
  }
  return glm53_fp8_linear(x, M, K, w, N, scale_inv, y, flags, stream);
}

extern "C" int glm53_fp8_linear(const void* x, int64_t M, int64_t K, const uint8_t* w, int64_t N,
                                const float* scale_inv, void* y, uint32_t flags, void* stream) {
  if (M < 0 || K <= 0 || N <= 0 || (M > 0 && (!x || !w || !scale_inv || !y))) {
    set_last_error("glm53_fp8_linear: invalid arguments M=%lld K=%lld N=%lld", (long long)M,
                   (long long)K, (long long)N);
    return GLM53_ERR_INVALID;
  }
  if (M == 0) return GLM53_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (M > kGemvMaxRows && dense_gemm_supported(K, N, w))
    return dense_fp8_gemm((const uint16_t*)x, M, K, w, N, scale_inv, (uint16_t*)y, st);
  return fp8_linear_small_m((const uint16_t*)x, M, K, w, N, scale_inv, (uint16_t*)y, flags, st);
}
