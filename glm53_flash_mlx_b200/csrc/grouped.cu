// Grouped block-FP8 GEMM over expert-sorted routes (G5) and the prefill MoE
// composition around it.
//
// Replaces grouped_fp8_linear / activate_gate_up / restore_and_reduce /
// SortedGroupedFP8MoE.grouped_from_routes (glm53_flash_mlx/grouped_fp8.py:
// 206-321; Metal kernel K12 at grouped_fp8.py:30-154).
//
// Tile: 128 routes x 128 weight rows x 64 K, 8 warps (4 along M x 2 along N).
// A (BF16 activations) is gathered row by row with cp.async, optionally through
// the sorted route order, so the sorted copy of x is never materialised.
// B (E4M3 codes) is staged raw and decoded in shared memory to BF16 with the
// 128x128 block scale folded in (BF16(lut(c) * s): exact E4M3 -> BF16, one
// rounding of the scaled weight), then multiplied with BF16 MMA and FP32
// accumulation.  The SwiGLU mode pairs gate rows and up rows of the same
// hidden column inside one warp so the epilogue applies the reference's BF16
// SwiGLU (glm53_flash_mlx/packed.py:146-163) before anything is stored.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace glm53 {

constexpr int BM = 128, BN = 128, BK = 64;
constexpr int kGemmThreads = 256;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::); }

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                            uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// [rows][64] BF16 tile, 16-byte chunks XOR-swizzled by row: conflict-free
// cp.async stores and ldmatrix reads.
__device__ __forceinline__ int tile_off(int row, int chunk) { return row * BK + ((chunk ^ (row & 7)) << 3); }

struct __align__(16) GemmSmem {
  uint16_t a[2][BM * BK];     // 2 x 16 KB
  uint8_t braw[2][BN * BK];   // 2 x 8 KB
  uint16_t b[BN * BK];        // 16 KB decoded
};

template <bool SWIGLU>
__global__ void __launch_bounds__(kGemmThreads) grouped_mma_kernel(GroupedGemmArgs g) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  GemmSmem& sm = *reinterpret_cast<GemmSmem*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int d = blockIdx.x;
  int64_t start;
  int len;
  uint32_t e;
  if (g.dense) {
    start = (int64_t)d * BM;
    if (start >= g.R) return;
    len = (int)((g.R - start) < BM ? (g.R - start) : BM);
    e = 0;
  } else {
    start = g.tile_starts[d];
    if (start >= g.R) return;
    { const uint32_t tl = g.tile_lengths[d]; len = (int)(tl < (uint32_t)BM ? tl : (uint32_t)BM); }
    e = g.tile_experts[d];
    if (e >= (uint32_t)g.E) {
      if (tid == 0) atomicOr(g.status, kStatusBadExpert);
      return;
    }
  }
  if (len <= 0) return;
  const int64_t K = g.K;
  const int ktiles = (int)(K / BK);
  const int scols = (int)((K + kBlock - 1) / kBlock);
  // B tile row -> weight row.  Plain: n0 + j.  SwiGLU: hidden column
  // h0 + 32*(j/64) + (j%32), gate for (j/32) even, up for odd.
  const int64_t n_tile = blockIdx.y;
  const uint8_t* wg = g.w_gate + (size_t)e * g.w_expert_stride;
  const uint8_t* wu = SWIGLU ? g.w_up + (size_t)e * g.w_expert_stride : nullptr;
  const float* sg = g.s_gate + (size_t)e * g.s_expert_stride;
  const float* su = SWIGLU ? g.s_up + (size_t)e * g.s_expert_stride : nullptr;
  const int64_t col0 = SWIGLU ? n_tile * 64 : n_tile * BN;

  // per-thread load assignments
  // A: 128 rows x 8 chunks = 1024 chunks, 4 per thread
  const uint16_t* a_src[4];
  int a_dst[4];
  bool a_ok[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = tid + i * kGemmThreads;
    const int row = idx >> 3, chunk = idx & 7;
    a_ok[i] = row < len;
    int64_t src_row = 0;
    if (a_ok[i]) {
      const int64_t p = start + row;
      src_row = g.a_index ? (int64_t)(g.a_index[p] / (uint32_t)g.a_div) : p;
    }
    a_src[i] = g.x + src_row * K + chunk * 8;
    a_dst[i] = tile_off(row, chunk);
  }
  // B: 128 rows x 4 chunks of 16 codes = 512 chunks, 2 per thread
  const uint8_t* b_src[2];
  int b_dst[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int idx = tid + i * kGemmThreads;
    const int row = idx >> 2, chunk = idx & 3;
    int64_t wrow;
    const uint8_t* base;
    if (SWIGLU) {
      wrow = col0 + 32 * (row >> 6) + (row & 31);
      base = ((row >> 5) & 1) ? wu : wg;
    } else {
      wrow = col0 + row;
      base = wg;
    }
    b_src[i] = base + wrow * K + chunk * 16;
    b_dst[i] = row * BK + chunk * 16;
  }
  // decode assignment: thread handles row dr, 32 codes starting at 32*dh
  const int dr = tid >> 1, dh = tid & 1;
  const float* srow;
  {
    int64_t wrow;
    const float* sb;
    if (SWIGLU) {
      wrow = col0 + 32 * (dr >> 6) + (dr & 31);
      sb = ((dr >> 5) & 1) ? su : sg;
    } else {
      wrow = col0 + dr;
      sb = sg;
    }
    srow = sb + (wrow / kBlock) * scols;
  }

  auto issue = [&](int kt, int stage) {
    const int64_t k0 = (int64_t)kt * BK;
    const uint32_t abase = smem_u32(sm.a[stage]);
#pragma unroll
    for (int i = 0; i < 4; ++i) cp_async16(abase + a_dst[i] * 2, a_src[i] + k0, a_ok[i]);
    const uint32_t bbase = smem_u32(sm.braw[stage]);
#pragma unroll
    for (int i = 0; i < 2; ++i) cp_async16(bbase + b_dst[i], b_src[i] + k0, true);
    cp_async_commit();
  };

  float acc[2][8][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[i][j][q] = 0.f;

  const int wm = warp & 3, wn = warp >> 2;
  issue(0, 0);
  for (int kt = 0; kt < ktiles; ++kt) {
    const int stage = kt & 1;
    cp_async_wait_all();
    __syncthreads();
    // decode raw E4M3 -> scaled BF16
    {
      const float sc = __ldg(srow + (kt * BK) / kBlock) * 256.0f;
      const uint4* src = reinterpret_cast<const uint4*>(sm.braw[stage] + dr * BK + dh * 32);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint4 w = src[h];
        const uint32_t words[4] = {w.x, w.y, w.z, w.w};
        uint32_t packed[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float f[4];
          e4m3x4_to_f32(words[q], f);
          __nv_bfloat162 p0 = __floats2bfloat162_rn(f[0] * sc, f[1] * sc);
          __nv_bfloat162 p1 = __floats2bfloat162_rn(f[2] * sc, f[3] * sc);
          packed[2 * q] = *reinterpret_cast<uint32_t*>(&p0);
          packed[2 * q + 1] = *reinterpret_cast<uint32_t*>(&p1);
        }
        const int chunk = dh * 4 + h * 2;
        *reinterpret_cast<uint4*>(sm.b + tile_off(dr, chunk)) =
            make_uint4(packed[0], packed[1], packed[2], packed[3]);
        *reinterpret_cast<uint4*>(sm.b + tile_off(dr, chunk + 1)) =
            make_uint4(packed[4], packed[5], packed[6], packed[7]);
      }
    }
    __syncthreads();
    if (kt + 1 < ktiles) issue(kt + 1, stage ^ 1);
    const uint32_t abase = smem_u32(sm.a[stage]);
    const uint32_t bbase = smem_u32(sm.b);
#pragma unroll
    for (int kk = 0; kk < BK / 16; ++kk) {
      uint32_t af[2][4];
#pragma unroll
      for (int mi = 0; mi < 2; ++mi) {
        const int row = wm * 32 + mi * 16 + (lane & 15);
        const int chunk = kk * 2 + (lane >> 4);
        ldmatrix_x4(abase + tile_off(row, chunk) * 2, af[mi][0], af[mi][1], af[mi][2], af[mi][3]);
      }
      uint32_t bf[8][2];
#pragma unroll
      for (int nj = 0; nj < 4; ++nj) {
        const int row = wn * 64 + nj * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int chunk = kk * 2 + ((lane >> 3) & 1);
        ldmatrix_x4(bbase + tile_off(row, chunk) * 2, bf[2 * nj][0], bf[2 * nj][1], bf[2 * nj + 1][0],
                    bf[2 * nj + 1][1]);
      }
#pragma unroll
      for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int ni = 0; ni < 8; ++ni) mma_bf16(acc[mi][ni], af[mi], bf[ni]);
    }
  }

  // epilogue
  const int r_in = lane >> 2, c_in = (lane & 3) * 2;
#pragma unroll
  for (int mi = 0; mi < 2; ++mi) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int row = wm * 32 + mi * 16 + r_in + half * 8;
      if (row >= len) continue;
      const int64_t orow = start + row;
      if (SWIGLU) {
#pragma unroll
        for (int ni = 0; ni < 4; ++ni) {
          const int64_t hcol = col0 + wn * 32 + ni * 8 + c_in;
          const uint16_t h0 = swiglu_bf16(acc[mi][ni][half * 2], acc[mi][ni + 4][half * 2], g.limit);
          const uint16_t h1 = swiglu_bf16(acc[mi][ni][half * 2 + 1], acc[mi][ni + 4][half * 2 + 1], g.limit);
          *reinterpret_cast<uint32_t*>(g.out + orow * g.N + hcol) = (uint32_t)h0 | ((uint32_t)h1 << 16);
        }
      } else {
#pragma unroll
        for (int ni = 0; ni < 8; ++ni) {
          const int64_t col = col0 + wn * 64 + ni * 8 + c_in;
          const uint16_t v0 = f32_to_bf16_bits(acc[mi][ni][half * 2]);
          const uint16_t v1 = f32_to_bf16_bits(acc[mi][ni][half * 2 + 1]);
          *reinterpret_cast<uint32_t*>(g.out + orow * g.N + col) = (uint32_t)v0 | ((uint32_t)v1 << 16);
        }
      }
    }
  }
}

int grouped_gemm(const GroupedGemmArgs& a, cudaStream_t stream) {
  if (a.K % BK != 0 || (a.swiglu ? a.N % 64 != 0 : a.N % BN != 0) || a.R < 0) {
    set_last_error("grouped_gemm: unsupported geometry K=%lld N=%lld", (long long)a.K, (long long)a.N);
    return GLM53_ERR_INVALID;
  }
  if (a.R == 0 || a.capacity == 0) return GLM53_OK;
  const size_t smem = sizeof(GemmSmem);
  const int n_tiles = (int)(a.swiglu ? a.N / 64 : a.N / BN);
  dim3 grid((unsigned)a.capacity, (unsigned)n_tiles);
  const void* fn = a.swiglu ? (const void*)grouped_mma_kernel<true> : (const void*)grouped_mma_kernel<false>;
  int rc_attr = ensure_max_smem(fn, smem);
  if (rc_attr) return rc_attr;
  if (a.swiglu)
    grouped_mma_kernel<true><<<grid, kGemmThreads, smem, stream>>>(a);
  else
    grouped_mma_kernel<false><<<grid, kGemmThreads, smem, stream>>>(a);
  return check_launch("grouped_mma_kernel");
}

bool dense_gemm_supported(int64_t K, int64_t N, const void* w) {
  return K % BK == 0 && N % BN == 0 && (((uintptr_t)w) & 15) == 0;
}

int dense_fp8_gemm(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w, int64_t N, const float* s,
                   uint16_t* y, cudaStream_t stream) {
  GroupedGemmArgs a{};
  a.x = x;
  a.a_index = nullptr;
  a.a_div = 1;
  a.R = M;
  a.K = K;
  a.capacity = (M + BM - 1) / BM;
  a.dense = true;
  a.w_gate = w;
  a.s_gate = s;
  a.E = 1;
  a.N = N;
  a.swiglu = false;
  a.out = y;
  a.status = nullptr;
  return grouped_gemm(a, stream);
}

// ---------------------------------------------------------------------------
// Elementwise pieces
// ---------------------------------------------------------------------------

__global__ void gather_rows_kernel(const uint16_t* __restrict__ x, int64_t H, const uint32_t* __restrict__ order,
                                   int64_t R, int top_k, uint16_t* __restrict__ out) {
  const int64_t chunks = H / 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= R * chunks) return;
  const int64_t p = i / chunks, c = i % chunks;
  const int64_t t = order[p] / (uint32_t)top_k;
  reinterpret_cast<uint4*>(out + p * H)[c] = reinterpret_cast<const uint4*>(x + t * H)[c];
}

__global__ void gather_rows_scalar_kernel(const uint16_t* __restrict__ x, int64_t H,
                                          const uint32_t* __restrict__ order, int64_t R, int top_k,
                                          uint16_t* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= R * H) return;
  const int64_t p = i / H, c = i % H;
  out[i] = x[(int64_t)(order[p] / (uint32_t)top_k) * H + c];
}

__global__ void activate_kernel(const uint16_t* __restrict__ gu, int64_t R, int64_t I, float limit,
                                uint16_t* __restrict__ hidden) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= R * I) return;
  const int64_t r = i / I, c = i % I;
  hidden[i] = swiglu_bf16(bf16_bits_to_f32(gu[r * 2 * I + c]), bf16_bits_to_f32(gu[r * 2 * I + I + c]), limit);
}

// out[t,h] = BF16(sum_j f32(rows[inv[t*k+j], h]) * score[inv]) (+ shared).
// Vector path: 8 columns per thread.
__global__ void combine_kernel(const uint16_t* __restrict__ rows, const float* __restrict__ sorted_scores,
                               const uint32_t* __restrict__ inverse, const uint32_t* __restrict__ sorted_experts,
                               int64_t E, int64_t T, int top_k, int64_t H, const uint16_t* __restrict__ shared,
                               uint16_t* __restrict__ out, uint32_t* status) {
  const int64_t chunks = H / 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * chunks) return;
  const int64_t t = i / chunks, c = i % chunks;
  float total[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) total[q] = 0.f;
  for (int j = 0; j < top_k; ++j) {
    const uint32_t pos = inverse[t * top_k + j];
    if (sorted_experts && sorted_experts[pos] >= (uint32_t)E) {
      if (status) atomicOr(status, kStatusBadExpert);
      continue;
    }
    const float sc = sorted_scores[pos];
    const uint4 v = reinterpret_cast<const uint4*>(rows + (int64_t)pos * H)[c];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      total[2 * q] = total[2 * q] + __fmul_rn(__uint_as_float(w[q] << 16), sc);
      total[2 * q + 1] = total[2 * q + 1] + __fmul_rn(__uint_as_float(w[q] & 0xFFFF0000u), sc);
    }
  }
  uint32_t o[4];
  uint4 sh = make_uint4(0, 0, 0, 0);
  if (shared) sh = reinterpret_cast<const uint4*>(shared + t * H)[c];
  const uint32_t sw[4] = {sh.x, sh.y, sh.z, sh.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float lo = bf16_round(total[2 * q]);
    float hi = bf16_round(total[2 * q + 1]);
    if (shared) {
      lo = lo + __uint_as_float(sw[q] << 16);
      hi = hi + __uint_as_float(sw[q] & 0xFFFF0000u);
    }
    o[q] = (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
  }
  reinterpret_cast<uint4*>(out + t * H)[c] = make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void combine_scalar_kernel(const uint16_t* __restrict__ rows, const float* __restrict__ sorted_scores,
                                      const uint32_t* __restrict__ inverse, int64_t T, int top_k, int64_t H,
                                      const uint16_t* __restrict__ shared, uint16_t* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * H) return;
  const int64_t t = i / H, h = i % H;
  float total = 0.f;
  for (int j = 0; j < top_k; ++j) {
    const uint32_t pos = inverse[t * top_k + j];
    total = total + __fmul_rn(bf16_bits_to_f32(rows[(int64_t)pos * H + h]), sorted_scores[pos]);
  }
  float r = bf16_round(total);
  if (shared) r = r + bf16_bits_to_f32(shared[i]);
  out[i] = f32_to_bf16_bits(r);
}

static int combine(const uint16_t* rows, const float* sorted_scores, const uint32_t* inverse,
                   const uint32_t* sorted_experts, int64_t E, int64_t T, int top_k, int64_t H,
                   const uint16_t* shared, uint16_t* out, uint32_t* status, cudaStream_t st) {
  const bool vec = H % 8 == 0 && (((uintptr_t)rows | (uintptr_t)out | (uintptr_t)shared) & 15) == 0;
  if (vec) {
    const int64_t n = T * (H / 8);
    combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(rows, sorted_scores, inverse, sorted_experts, E, T,
                                                                 top_k, H, shared, out, status);
    return check_launch("combine_kernel");
  }
  const int64_t n = T * H;
  combine_scalar_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(rows, sorted_scores, inverse, T, top_k, H,
                                                                      shared, out);
  return check_launch("combine_scalar_kernel");
}

}  // namespace glm53

using namespace glm53;

extern "C" int glm53_gather_rows(const void* x, int64_t H, const uint32_t* order, int64_t R, int top_k,
                                 void* sorted_x, void* stream) {
  if (H <= 0 || R < 0 || top_k <= 0 || (R > 0 && (!x || !order || !sorted_x))) {
    set_last_error("glm53_gather_rows: invalid arguments");
    return GLM53_ERR_INVALID;
  }
  if (R == 0) return GLM53_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (H % 8 == 0 && (((uintptr_t)x | (uintptr_t)sorted_x) & 15) == 0) {
    const int64_t n = R * (H / 8);
    gather_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>((const uint16_t*)x, H, order, R, top_k,
                                                                     (uint16_t*)sorted_x);
  } else {
    const int64_t n = R * H;
    gather_rows_scalar_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>((const uint16_t*)x, H, order, R, top_k,
                                                                            (uint16_t*)sorted_x);
  }
  return check_launch("gather_rows");
}

extern "C" int glm53_grouped_fp8_linear(const void* x, int64_t R, int64_t K, const uint32_t* tile_experts,
                                        const uint32_t* tile_starts, const uint32_t* tile_lengths,
                                        int64_t descriptor_capacity, const uint8_t* w, int64_t E, int64_t N,
                                        const float* scale_inv, void* out, uint32_t flags, void* stream) {
  (void)flags;  // the BF16 tile path decodes exactly for every code
  if (R < 0 || K <= 0 || N <= 0 || E <= 0 || descriptor_capacity < 0 ||
      (R > 0 && (!x || !tile_experts || !tile_starts || !tile_lengths || !w || !scale_inv || !out))) {
    set_last_error("glm53_grouped_fp8_linear: invalid arguments");
    return GLM53_ERR_INVALID;
  }
  if (K % 128 != 0 || N % 128 != 0 || (((uintptr_t)w | (uintptr_t)x) & 15) != 0) {
    set_last_error("glm53_grouped_fp8_linear: block-aligned dimensions required (K=%lld N=%lld)", (long long)K,
                   (long long)N);
    return GLM53_ERR_INVALID;
  }
  GroupedGemmArgs a{};
  a.x = (const uint16_t*)x;
  a.a_div = 1;
  a.R = R;
  a.K = K;
  a.tile_experts = tile_experts;
  a.tile_starts = tile_starts;
  a.tile_lengths = tile_lengths;
  a.capacity = descriptor_capacity;
  a.w_gate = w;
  a.w_expert_stride = N * K;
  a.s_gate = scale_inv;
  a.s_expert_stride = (N / 128) * (K / 128);
  a.E = E;
  a.N = N;
  a.out = (uint16_t*)out;
  a.status = nullptr;
  return grouped_gemm(a, (cudaStream_t)stream);
}

extern "C" size_t glm53_grouped_fp8_linear_workspace_bytes(int64_t R, int64_t K) {
  if (R <= 0 || K <= 0) return 0;
  return align_up((size_t)R * K * sizeof(__half), 256) + align_up((size_t)R * sizeof(float), 256);
}

extern "C" int glm53_grouped_fp8_linear_ws(const void* x, int64_t R, int64_t K, const uint32_t* tile_experts,
                                           const uint32_t* tile_starts, const uint32_t* tile_lengths,
                                           int64_t descriptor_capacity, int64_t tile_rows, const uint8_t* w,
                                           int64_t E, int64_t N, const float* scale_inv, void* out,
                                           void* workspace, size_t workspace_bytes, uint32_t* status,
                                           uint32_t flags, void* stream) {
  const char* fn = "glm53_grouped_fp8_linear_ws";
  if (R < 0 || K <= 0 || N <= 0 || E <= 0 || descriptor_capacity < 0 || tile_rows <= 0 ||
      (R > 0 && (!x || !tile_experts || !tile_starts || !tile_lengths || !w || !scale_inv || !out || !status))) {
    set_last_error("%s: invalid arguments", fn);
    return GLM53_ERR_INVALID;
  }
  if (K % 128 != 0 || N % 128 != 0 || (((uintptr_t)w | (uintptr_t)x) & 15) != 0) {
    set_last_error("%s: block-aligned dimensions required (K=%lld N=%lld)", fn, (long long)K, (long long)N);
    return GLM53_ERR_INVALID;
  }
  if (R == 0 || descriptor_capacity == 0) return GLM53_OK;
  if (!workspace || workspace_bytes < glm53_grouped_fp8_linear_workspace_bytes(R, K) ||
      (((uintptr_t)workspace) & 15) != 0 || R > INT32_MAX / 2 || !grouped_tc_supported(K, N, 0.0f, false)) {
    set_last_error("%s: workspace missing or too small, or geometry outside the tensor-core path", fn);
    return GLM53_ERR_INVALID;
  }
  cudaStream_t st = (cudaStream_t)stream;
  __half* x16 = (__half*)workspace;
  float* xscale = (float*)((char*)workspace + align_up((size_t)R * K * sizeof(__half), 256));
  int rc = rows_to_f16((const uint16_t*)x, K, nullptr, 1, R, x16, xscale, st);
  if (rc) return rc;
  TcGemm g{};
  g.x16 = x16;
  g.xscale = xscale;
  g.R = R;
  g.K = K;
  g.tile_experts = tile_experts;
  g.tile_starts = tile_starts;
  g.tile_lengths = tile_lengths;
  g.capacity = descriptor_capacity;
  g.max_rows = tile_rows;
  g.dense = false;
  g.w = w;
  g.w_rows = N;
  g.s_gate = scale_inv;
  g.s_expert = (N / 128) * (K / 128);
  g.E = E;
  g.N = N;
  g.swiglu = false;
  g.finite = (flags & GLM53_FLAG_E4M3_FINITE) != 0;
  g.out = (uint16_t*)out;
  g.status = status;
  return grouped_tc(g, st);
}

extern "C" int glm53_activate_gate_up(const void* gate_up, int64_t R, int64_t I, float limit, void* hidden,
                                      void* stream) {
  if (R < 0 || I <= 0 || (R > 0 && (!gate_up || !hidden))) {
    set_last_error("glm53_activate_gate_up: invalid arguments");
    return GLM53_ERR_INVALID;
  }
  if (R == 0) return GLM53_OK;
  const int64_t n = R * I;
  activate_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>((const uint16_t*)gate_up, R, I,
                                                                                   limit, (uint16_t*)hidden);
  return check_launch("activate_kernel");
}

extern "C" int glm53_restore_and_reduce(const void* sorted_out, const float* sorted_scores, const uint32_t* inverse,
                                        int64_t T, int top_k, int64_t H, const void* shared, void* out,
                                        void* stream) {
  if (T < 0 || H <= 0 || top_k <= 0 || (T > 0 && (!sorted_out || !sorted_scores || !inverse || !out))) {
    set_last_error("glm53_restore_and_reduce: invalid arguments");
    return GLM53_ERR_INVALID;
  }
  if (T == 0) return GLM53_OK;
  return combine((const uint16_t*)sorted_out, sorted_scores, inverse, nullptr, 0, T, top_k, H,
                 (const uint16_t*)shared, (uint16_t*)out, nullptr, (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// Whole grouped prefill layer
// ---------------------------------------------------------------------------

namespace {
// Routes per descriptor of the tensor-core (tcgen05) path; the fallback path
// uses BM-route descriptors, and the capacity covers both.
constexpr int kTcTileRows = 128;

struct MoeWorkspace {
  uint32_t *order, *inverse, *sorted_experts, *route_offsets, *tile_offsets, *tile_experts, *tile_starts,
      *tile_lengths, *counts, *plan_scratch;
  float *sorted_scores, *xscale, *shared_xscale, *shared_partial, *hscale, *shared_hscale;
  int shared_splits;
  uint16_t *hidden, *down, *shared_hidden, *shared_out;
  __half *x16, *shared_x16;
  int64_t capacity;
  size_t bytes;
};

MoeWorkspace carve(void* base, int64_t T, int top_k, int64_t E, int64_t H, int64_t I, int64_t Is) {
  MoeWorkspace w{};
  const int64_t R = T * top_k;
  w.capacity = (R + kTcTileRows - 1) / kTcTileRows + E;
  size_t off = 0;
  char* b = (char*)base;
  auto take = [&](size_t n) {
    void* p = b ? (void*)(b + off) : nullptr;
    off = align_up(off + n, 256);
    return p;
  };
  w.order = (uint32_t*)take(R * 4);
  w.inverse = (uint32_t*)take(R * 4);
  w.sorted_experts = (uint32_t*)take(R * 4);
  w.sorted_scores = (float*)take(R * 4);
  w.route_offsets = (uint32_t*)take((E + 1) * 4);
  w.tile_offsets = (uint32_t*)take((E + 1) * 4);
  w.tile_experts = (uint32_t*)take(w.capacity * 4);
  w.tile_starts = (uint32_t*)take(w.capacity * 4);
  w.tile_lengths = (uint32_t*)take(w.capacity * 4);
  w.counts = (uint32_t*)take(2 * 4);
  w.hidden = (uint16_t*)take((size_t)R * I * 2);
  // down rows [R, H]; before the down projection the same bytes hold the
  // gate/up rows [R][gate I | up I] (likewise for the shared expert)
  w.down = (uint16_t*)take((size_t)R * std::max(H, 2 * I) * 2);
  w.shared_hidden = (uint16_t*)take((size_t)T * (Is > 0 ? Is : 1) * 2);
  w.shared_out = (uint16_t*)take((size_t)T * std::max(H, 2 * Is) * 2);
  w.x16 = (__half*)take((size_t)R * H * 2);
  w.xscale = (float*)take((size_t)R * 4);
  w.shared_x16 = (__half*)take((size_t)T * H * 2);
  w.shared_xscale = (float*)take((size_t)T * 4);
  // split-K partials of the shared expert's down projection (few output
  // tiles at small T)
  w.shared_splits = Is > 0 && Is % 128 == 0 ? grouped_tc_splits(((T + 127) / 128) * ((H + 127) / 128), Is / 128) : 1;
  w.shared_partial = w.shared_splits > 1 ? (float*)take(grouped_tc_splitk_bytes(T, H, w.shared_splits)) : nullptr;
  // range multipliers of the hidden rows' E4M3 terms (kind::f8f6f4 path)
  w.hscale = (float*)take((size_t)R * 4);
  w.shared_hscale = (float*)take((size_t)T * 4);
  w.plan_scratch = (uint32_t*)take(route_plan_scratch_bytes(R, E));
  w.bytes = off;
  return w;
}
}  // namespace

// Tensor-core composition: route plan (128-route descriptors), sorted FP16
// activations, tcgen05 gate/up with the SwiGLU epilogue (FP16 hidden rows),
// tcgen05 down, the dense shared expert on the same kernels, combine.
static int grouped_moe_tc(const MoeWorkspace& w, const void* x, int64_t T, int64_t H, const uint32_t* indices,
                          const float* scores, int top_k, const uint8_t* gate_up_w, const float* gate_up_s,
                          const uint8_t* down_w, const float* down_s, int64_t E, int64_t I,
                          const uint8_t* shared_gate_w, const float* shared_gate_s, const uint8_t* shared_up_w,
                          const float* shared_up_s, const uint8_t* shared_down_w, const float* shared_down_s,
                          int64_t Is, float limit, uint16_t* out, uint32_t* status, bool finite, bool f8,
                          cudaStream_t st) {
  const int64_t R = T * top_k;
  // kind::f8f6f4 for a gate/up + down pair: finite banks whose shapes fit the
  // kernel; the shared pair also needs an unsplit down projection
  const bool routed_f8 = f8 && finite && grouped_f8_supported(H, I, true) && grouped_f8_supported(I, H, false);
  const bool shared_f8 = f8 && finite && Is > 0 && grouped_f8_supported(H, Is, true) &&
                         grouped_f8_supported(Is, H, false) && w.shared_splits == 1;
  int rc = route_plan_chunked(indices, R, E, kTcTileRows, scores, w.order, w.inverse, w.sorted_experts,
                              w.sorted_scores, w.route_offsets, w.tile_experts, w.tile_starts, w.tile_lengths,
                              w.tile_offsets, w.counts, w.counts + 1, w.plan_scratch, st);
  if (rc) return rc;
  if (routed_f8)
    rc = rows_to_e4m3_split((const uint16_t*)x, H, w.order, top_k, R, reinterpret_cast<uint8_t*>(w.x16), w.xscale,
                            st);
  else
    rc = rows_to_f16((const uint16_t*)x, H, w.order, top_k, R, w.x16, w.xscale, st);
  if (rc) return rc;
  const int64_t hcols = H / 128, icols = I / 128;
  TcGemm gu{};
  gu.x16 = w.x16;
  gu.xscale = w.xscale;
  gu.f8 = routed_f8;
  gu.x8 = reinterpret_cast<const uint8_t*>(w.x16);
  gu.R = R;
  gu.K = H;
  gu.tile_experts = w.tile_experts;
  gu.tile_starts = w.tile_starts;
  gu.tile_lengths = w.tile_lengths;
  gu.capacity = (R + kTcTileRows - 1) / kTcTileRows + E;
  gu.max_rows = kTcTileRows;
  gu.w = gate_up_w;
  gu.w_up = gate_up_w;
  gu.w_rows = 2 * I;
  gu.u_rows = 2 * I;
  gu.u_off = I;
  gu.s_gate = gate_up_s;
  gu.s_up = gate_up_s + icols * hcols;
  gu.s_expert = 2 * icols * hcols;
  gu.E = E;
  gu.I = I;
  gu.swiglu = true;
  gu.limit = limit;
  gu.finite = finite;
  gu.out = w.down;  // [R][gate I | up I]
  gu.status = status;
  rc = grouped_tc(gu, st);
  if (rc) return rc;
  TcGemm dn = gu;
  dn.x16 = reinterpret_cast<const __half*>(w.hidden);
  dn.xscale = nullptr;
  if (routed_f8) {
    // SwiGLU -> the E4M3 terms of the BF16 hidden rows
    rc = swiglu_split(w.down, R, I, limit, reinterpret_cast<uint8_t*>(w.hidden), w.hscale, st);
    if (rc) return rc;
    dn.x8 = reinterpret_cast<const uint8_t*>(w.hidden);
    dn.xscale = w.hscale;
  } else {
    rc = swiglu_rows(w.down, R, I, limit, reinterpret_cast<__half*>(w.hidden), st);
    if (rc) return rc;
  }
  dn.K = I;
  dn.w = down_w;
  dn.w_up = nullptr;
  dn.w_rows = H;
  dn.u_rows = 0;
  dn.u_off = 0;
  dn.s_gate = down_s;
  dn.s_up = nullptr;
  dn.s_expert = hcols * icols;
  dn.N = H;
  dn.I = 0;
  dn.swiglu = false;
  dn.out = w.down;
  rc = grouped_tc(dn, st);
  if (rc) return rc;
  const uint16_t* shared_ptr = nullptr;
  if (Is > 0) {
    if (shared_f8)
      rc = rows_to_e4m3_split((const uint16_t*)x, H, nullptr, 1, T, reinterpret_cast<uint8_t*>(w.shared_x16),
                              w.shared_xscale, st);
    else
      rc = rows_to_f16((const uint16_t*)x, H, nullptr, 1, T, w.shared_x16, w.shared_xscale, st);
    if (rc) return rc;
    TcGemm sg{};
    sg.x16 = w.shared_x16;
    sg.xscale = w.shared_xscale;
    sg.f8 = shared_f8;
    sg.x8 = reinterpret_cast<const uint8_t*>(w.shared_x16);
    sg.R = T;
    sg.K = H;
    sg.capacity = (T + kTcTileRows - 1) / kTcTileRows;
    sg.max_rows = kTcTileRows;
    sg.dense = true;
    sg.w = shared_gate_w;
    sg.w_up = shared_up_w;
    sg.w_rows = Is;
    sg.u_rows = Is;
    sg.u_off = 0;
    sg.s_gate = shared_gate_s;
    sg.s_up = shared_up_s;
    sg.s_expert = 0;
    sg.E = 1;
    sg.I = Is;
    sg.swiglu = true;
    sg.limit = limit;
    sg.finite = finite;
    sg.out = w.shared_out;  // [T][gate Is | up Is]
    sg.status = status;
    rc = grouped_tc(sg, st);
    if (rc) return rc;
    TcGemm sd = sg;
    sd.x16 = reinterpret_cast<const __half*>(w.shared_hidden);
    sd.xscale = nullptr;
    if (shared_f8) {
      rc = swiglu_split(w.shared_out, T, Is, limit, reinterpret_cast<uint8_t*>(w.shared_hidden), w.shared_hscale,
                        st);
      if (rc) return rc;
      sd.x8 = reinterpret_cast<const uint8_t*>(w.shared_hidden);
      sd.xscale = w.shared_hscale;
    } else {
      rc = swiglu_rows(w.shared_out, T, Is, limit, reinterpret_cast<__half*>(w.shared_hidden), st);
      if (rc) return rc;
    }
    sd.K = Is;
    sd.w = shared_down_w;
    sd.w_up = nullptr;
    sd.w_rows = H;
    sd.u_rows = 0;
    sd.s_gate = shared_down_s;
    sd.s_up = nullptr;
    sd.N = H;
    sd.I = 0;
    sd.swiglu = false;
    sd.out = w.shared_out;
    sd.splits = w.shared_splits;
    sd.partial = w.shared_partial;
    rc = grouped_tc(sd, st);
    if (rc) return rc;
    shared_ptr = w.shared_out;
  }
  return combine(w.down, w.sorted_scores, w.inverse, w.sorted_experts, E, T, top_k, H, shared_ptr, out, status, st);
}

extern "C" size_t glm53_grouped_moe_workspace_bytes(int64_t T, int top_k, int64_t E, int64_t H, int64_t I,
                                                    int64_t I_shared) {
  return carve(nullptr, T, top_k, E, H, I, I_shared).bytes;
}

extern "C" int glm53_grouped_moe_workspace_layout(int64_t T, int top_k, int64_t E, int64_t H, int64_t I,
                                                  int64_t I_shared, size_t* offsets) {
  if (!offsets || T < 0 || top_k <= 0 || E <= 0 || H <= 0 || I <= 0 || I_shared < 0) {
    set_last_error("glm53_grouped_moe_workspace_layout: invalid arguments");
    return GLM53_ERR_INVALID;
  }
  // offsets from a base of 256 (any aligned base gives the same offsets)
  char* const base = reinterpret_cast<char*>(256);
  const MoeWorkspace w = carve(base, T, top_k, E, H, I, I_shared);
  const void* parts[8] = {w.order, w.inverse, w.sorted_experts, w.sorted_scores,
                          w.hidden, w.down, w.shared_hidden, w.shared_out};
  for (int i = 0; i < 8; ++i) offsets[i] = (size_t)(reinterpret_cast<const char*>(parts[i]) - base);
  return GLM53_OK;
}

extern "C" int glm53_grouped_moe_term_layout(int64_t T, int top_k, int64_t E, int64_t H, int64_t I,
                                             int64_t I_shared, size_t* offsets) {
  if (!offsets || T < 0 || top_k <= 0 || E <= 0 || H <= 0 || I <= 0 || I_shared < 0) {
    set_last_error("glm53_grouped_moe_term_layout: invalid arguments");
    return GLM53_ERR_INVALID;
  }
  char* const base = reinterpret_cast<char*>(256);
  const MoeWorkspace w = carve(base, T, top_k, E, H, I, I_shared);
  const void* parts[6] = {w.x16, w.xscale, w.hscale, w.shared_x16, w.shared_xscale, w.shared_hscale};
  for (int i = 0; i < 6; ++i) offsets[i] = (size_t)(reinterpret_cast<const char*>(parts[i]) - base);
  return GLM53_OK;
}

extern "C" int glm53_e4m3_split_rows(const void* x, int64_t rows, int64_t K, void* terms, float* scale,
                                     void* stream) {
  if (rows < 0 || K <= 0 || (rows > 0 && (!x || !terms || !scale))) {
    set_last_error("glm53_e4m3_split_rows: invalid arguments");
    return GLM53_ERR_INVALID;
  }
  return rows_to_e4m3_split((const uint16_t*)x, K, nullptr, 1, rows, (uint8_t*)terms, scale, (cudaStream_t)stream);
}

extern "C" int glm53_grouped_moe(const void* x, int64_t T, int64_t H, const uint32_t* indices, const float* scores,
                                 int top_k, const uint8_t* gate_up_w, const float* gate_up_s, const uint8_t* down_w,
                                 const float* down_s, int64_t E, int64_t I, const uint8_t* shared_gate_w,
                                 const float* shared_gate_s, const uint8_t* shared_up_w, const float* shared_up_s,
                                 const uint8_t* shared_down_w, const float* shared_down_s, int64_t I_shared,
                                 float limit, void* out, void* workspace, size_t workspace_bytes, uint32_t* status,
                                 uint32_t flags, void* stream) {
  if (T < 0 || H <= 0 || I <= 0 || E <= 0 || top_k <= 0 || I_shared < 0) {
    set_last_error("glm53_grouped_moe: invalid geometry");
    return GLM53_ERR_INVALID;
  }
  if (H % 128 != 0 || I % 128 != 0 || I_shared % 128 != 0) {
    set_last_error("glm53_grouped_moe: block-aligned dimensions required (H=%lld I=%lld I_shared=%lld)",
                   (long long)H, (long long)I, (long long)I_shared);
    return GLM53_ERR_INVALID;
  }
  if (T == 0) return GLM53_OK;
  const bool has_shared = I_shared > 0;
  if (!x || !indices || !scores || !gate_up_w || !gate_up_s || !down_w || !down_s || !out || !status ||
      !workspace || workspace_bytes < glm53_grouped_moe_workspace_bytes(T, top_k, E, H, I, I_shared) ||
      (has_shared && (!shared_gate_w || !shared_gate_s || !shared_up_w || !shared_up_s || !shared_down_w ||
                      !shared_down_s))) {
    set_last_error("glm53_grouped_moe: missing pointer or workspace too small");
    return GLM53_ERR_INVALID;
  }
  cudaStream_t st = (cudaStream_t)stream;
  MoeWorkspace w = carve(workspace, T, top_k, E, H, I, I_shared);
  const int64_t R = T * top_k;
  if (grouped_tc_supported(H, I, limit, true) && grouped_tc_supported(I, H, limit, false) &&
      (!has_shared || (I_shared % 128 == 0 && grouped_tc_supported(I_shared, H, limit, false))) &&
      ((((uintptr_t)x | (uintptr_t)gate_up_w | (uintptr_t)down_w) & 15) == 0) &&
      (!has_shared || ((((uintptr_t)shared_gate_w | (uintptr_t)shared_up_w | (uintptr_t)shared_down_w) & 15) == 0)))
    return grouped_moe_tc(w, x, T, H, indices, scores, top_k, gate_up_w, gate_up_s, down_w, down_s, E, I,
                          shared_gate_w, shared_gate_s, shared_up_w, shared_up_s, shared_down_w, shared_down_s,
                          I_shared, limit, (uint16_t*)out, status, (flags & GLM53_FLAG_E4M3_FINITE) != 0,
                          (flags & GLM53_FLAG_F8_MMA) != 0, st);
  int rc = route_plan(indices, R, E, BM, scores, w.order, w.inverse, w.sorted_experts, w.sorted_scores,
                      w.route_offsets, w.tile_experts, w.tile_starts, w.tile_lengths, w.tile_offsets, w.counts,
                      w.counts + 1, st);
  if (rc) return rc;
  const int64_t half = I / 128, hcols = H / 128, icols = I / 128;
  GroupedGemmArgs gu{};
  gu.x = (const uint16_t*)x;
  gu.a_index = w.order;
  gu.a_div = top_k;
  gu.R = R;
  gu.K = H;
  gu.tile_experts = w.tile_experts;
  gu.tile_starts = w.tile_starts;
  gu.tile_lengths = w.tile_lengths;
  gu.capacity = w.capacity;
  gu.w_gate = gate_up_w;
  gu.w_up = gate_up_w + I * H;
  gu.w_expert_stride = 2 * I * H;
  gu.s_gate = gate_up_s;
  gu.s_up = gate_up_s + half * hcols;
  gu.s_expert_stride = 2 * half * hcols;
  gu.E = E;
  gu.N = I;
  gu.swiglu = true;
  gu.limit = limit;
  gu.out = w.hidden;
  gu.status = status;
  rc = grouped_gemm(gu, st);
  if (rc) return rc;
  GroupedGemmArgs dn{};
  dn.x = w.hidden;
  dn.a_div = 1;
  dn.R = R;
  dn.K = I;
  dn.tile_experts = w.tile_experts;
  dn.tile_starts = w.tile_starts;
  dn.tile_lengths = w.tile_lengths;
  dn.capacity = w.capacity;
  dn.w_gate = down_w;
  dn.w_expert_stride = H * I;
  dn.s_gate = down_s;
  dn.s_expert_stride = hcols * icols;
  dn.E = E;
  dn.N = H;
  dn.out = w.down;
  dn.status = status;
  rc = grouped_gemm(dn, st);
  if (rc) return rc;
  const uint16_t* shared_ptr = nullptr;
  if (has_shared) {
    const int64_t scols = I_shared / 128;
    GroupedGemmArgs sg{};
    sg.x = (const uint16_t*)x;
    sg.a_div = 1;
    sg.R = T;
    sg.K = H;
    sg.capacity = (T + BM - 1) / BM;
    sg.dense = true;
    sg.w_gate = shared_gate_w;
    sg.w_up = shared_up_w;
    sg.s_gate = shared_gate_s;
    sg.s_up = shared_up_s;
    sg.E = 1;
    sg.N = I_shared;
    sg.swiglu = true;
    sg.limit = limit;
    sg.out = w.shared_hidden;
    sg.status = status;
    rc = grouped_gemm(sg, st);
    if (rc) return rc;
    GroupedGemmArgs sd{};
    sd.x = w.shared_hidden;
    sd.a_div = 1;
    sd.R = T;
    sd.K = I_shared;
    sd.capacity = (T + BM - 1) / BM;
    sd.dense = true;
    sd.w_gate = shared_down_w;
    sd.s_gate = shared_down_s;
    sd.E = 1;
    sd.N = H;
    sd.out = w.shared_out;
    sd.status = status;
    (void)scols;
    rc = grouped_gemm(sd, st);
    if (rc) return rc;
    shared_ptr = w.shared_out;
  }
  return combine(w.down, w.sorted_scores, w.inverse, w.sorted_experts, E, T, top_k, H, shared_ptr, (uint16_t*)out,
                 status, st);
}
