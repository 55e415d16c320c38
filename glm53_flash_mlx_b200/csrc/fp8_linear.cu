// Block-128 E4M3 linear (G1): y[M,N] = x[M,K] @ dequant(w[N,K], s)^T.
//
// Replaces block_fp8_linear (glm53_flash_mlx/fp8.py:254-299) and its Metal
// kernels K1/K2 (fp8.py:41-116).  Small M is HBM-bound: every weight byte is
// read once with 16-byte streaming loads, decoded in registers and multiplied
// against FP32 activations held in shared memory.  Large M goes to the
// tensor-core grouped GEMM with a single expert (grouped.cu).
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace glm53 {

// Activations are stored in shared memory as FP32 with the float4 index of
// (chunk c, quarter q) at 4c + (q ^ ((c >> 1) & 3)): the 8 lanes of one
// LDS.128 phase read chunks c..c+7 and land in 8 distinct bank groups.
__device__ __forceinline__ int xs_swizzle(int c, int q) { return 4 * c + (q ^ ((c >> 1) & 3)); }

// Dot product of the 16 codes of chunk c with the swizzled activations.
__device__ __forceinline__ float dot16_swz(uint4 w, const float4* xs4, int c) {
  float f[4];
  float acc = 0.f;
  uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    e4m3x4_to_f32(words[q], f);
    float4 xv = xs4[xs_swizzle(c, q)];
    acc = fmaf(xv.x, f[0], acc);
    acc = fmaf(xv.y, f[1], acc);
    acc = fmaf(xv.z, f[2], acc);
    acc = fmaf(xv.w, f[3], acc);
  }
  return acc;
}

__device__ __forceinline__ void load_x_swizzled(float* xs, const uint16_t* x, int K, int tid, int nthreads) {
  const int nchunks = K >> 4;
  for (int i = tid; i < (K >> 2); i += nthreads) {
    int c = i >> 2, q = i & 3;
    const uint2 raw = *reinterpret_cast<const uint2*>(x + 4 * i);
    float4 v;
    v.x = __uint_as_float(raw.x << 16);
    v.y = __uint_as_float(raw.x & 0xFFFF0000u);
    v.z = __uint_as_float(raw.y << 16);
    v.w = __uint_as_float(raw.y & 0xFFFF0000u);
    reinterpret_cast<float4*>(xs)[xs_swizzle(c, q)] = v;
  }
  (void)nchunks;
}

// One warp per output row; MR activation rows share each weight load.
// Requires K % 16 == 0 and 16-byte aligned rows.
template <int MR, int U>
__global__ void __launch_bounds__(256) fp8_gemv_kernel(const uint16_t* __restrict__ x, int M, int K,
                                                       const uint8_t* __restrict__ w, int N,
                                                       const float* __restrict__ s,
                                                       uint16_t* __restrict__ y) {
  extern __shared__ float4 smem_x4[];
  float* xs = reinterpret_cast<float*>(smem_x4);
  const int m0 = blockIdx.y * MR;
  const int mr = min(MR, M - m0);
  for (int m = 0; m < mr; ++m)
    load_x_swizzled(xs + (size_t)m * K, x + (size_t)(m0 + m) * K, K, threadIdx.x, blockDim.x);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int nchunks = K >> 4;
  const int scale_cols = (K + kBlock - 1) / kBlock;
  for (int n = blockIdx.x * warps + (threadIdx.x >> 5); n < N; n += gridDim.x * warps) {
    const uint4* wr = reinterpret_cast<const uint4*>(w + (size_t)n * K);
    const float* srow = s + (size_t)(n / kBlock) * scale_cols;
    float acc[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[m] = 0.f;
    for (int c0 = 0; c0 < nchunks; c0 += 32 * U) {
      uint4 wv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        int c = c0 + u * 32 + lane;
        if (c < nchunks) wv[u] = ldg_stream(wr + c);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        int c = c0 + u * 32 + lane;
        if (c < nchunks) {
          float sc = __ldg(srow + (c >> 3)) * 256.0f;
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            if (m < mr) acc[m] = fmaf(sc, dot16_swz(wv[u], smem_x4 + (size_t)m * (K >> 2), c), acc[m]);
          }
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      float v = warp_sum(acc[m]);
      if (lane == 0 && m < mr) y[(size_t)(m0 + m) * N + n] = f32_to_bf16_bits(v);
    }
  }
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

template <int MR>
static int launch_gemv(const uint16_t* x, int M, int K, const uint8_t* w, int N, const float* s,
                       uint16_t* y, cudaStream_t stream) {
  constexpr int U = 4;
  const size_t smem = (size_t)MR * K * sizeof(float);
  if (smem > 48 * 1024) {
    int rc_attr = ensure_max_smem((const void*)fp8_gemv_kernel<MR, U>, smem);
    if (rc_attr) return rc_attr;
  }
  const int warps = 8;
  int sms = sm_count();
  int per_sm = std::max(1, std::min(8, (int)((200 * 1024) / std::max<size_t>(smem, 1))));
  int blocks = std::min((N + warps - 1) / warps, sms * per_sm);
  dim3 grid(blocks, (M + MR - 1) / MR);
  fp8_gemv_kernel<MR, U><<<grid, warps * 32, smem, stream>>>(x, M, K, w, N, s, y);
  return check_launch("fp8_gemv_kernel");
}

int fp8_linear_small_m(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w, int64_t N,
                       const float* s, uint16_t* y, cudaStream_t stream) {
  const bool vec = (K % 16 == 0) && (((uintptr_t)w & 15) == 0) && (((uintptr_t)x & 7) == 0) &&
                   K <= 24576;
  if (!vec) {
    int64_t warps = M * N;
    int64_t blocks = (warps + 7) / 8;
    fp8_linear_scalar_kernel<<<(unsigned)blocks, 256, 0, stream>>>(x, M, K, w, N, s, y);
    return check_launch("fp8_linear_scalar_kernel");
  }
  const size_t per_row = (size_t)K * sizeof(float);
  if (M >= 4 && 4 * per_row <= 96 * 1024) return launch_gemv<4>(x, (int)M, (int)K, w, (int)N, s, y, stream);
  if (M >= 2 && 2 * per_row <= 96 * 1024) return launch_gemv<2>(x, (int)M, (int)K, w, (int)N, s, y, stream);
  return launch_gemv<1>(x, (int)M, (int)K, w, (int)N, s, y, stream);
}

}  // namespace glm53

using namespace glm53;

extern "C" int glm53_fp8_linear(const void* x, int64_t M, int64_t K, const uint8_t* w, int64_t N,
                                const float* scale_inv, void* y, void* stream) {
  if (M < 0 || K <= 0 || N <= 0 || (M > 0 && (!x || !w || !scale_inv || !y))) {
    set_last_error("glm53_fp8_linear: invalid arguments M=%lld K=%lld N=%lld", (long long)M,
                   (long long)K, (long long)N);
    return GLM53_ERR_INVALID;
  }
  if (M == 0) return GLM53_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (M > kGemvMaxRows && dense_gemm_supported(K, N, w))
    return dense_fp8_gemm((const uint16_t*)x, M, K, w, N, scale_inv, (uint16_t*)y, st);
  return fp8_linear_small_m((const uint16_t*)x, M, K, w, N, scale_inv, (uint16_t*)y, st);
}
