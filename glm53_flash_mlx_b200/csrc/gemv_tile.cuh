// Tensor-core GEMV building blocks for the bandwidth-bound paths (decode MoE,
// small-M block linear).
//
// One warp computes 16 weight rows x up to 8 activation columns with
// mma.sync m16n8k16 (FP16 operands, FP32 accumulation):
//   * each lane loads 16 contiguous E4M3 codes of weight rows g and g+8
//     (g = lane / 4) at byte offset 16*(lane % 4) of a 64-wide K slice, and
//     decodes them exactly in registers (e4m3x4_to_h2: lut(c)/256 in FP16);
//   * inside MMA i (i = 0..3) of the slice, the K slot pair {2q, 2q+1} of lane
//     q = lane % 4 stands for k = 16q + 4i + {0, 1} and {8+2q, 9+2q} for
//     16q + 4i + {2, 3}; activations use the same mapping, so every lane's
//     weight and activation loads stay 16- and 32-byte vectors;
//   * the 128x128 block scale (times 256 and the activation's power-of-two
//     range scale) is applied in FP32 once per 128-K block ("promotion").
// Activations are staged in shared memory as FP16 multiplied by 2^-e, with e
// chosen from the largest |x| so FP16 cannot overflow (BF16 values in FP16
// range convert exactly).  Splitting K across warps depends only on K, so
// every caller of these functions produces the same FP32 sums for the same row.
#pragma once

#include "common.cuh"

namespace glm53 {

__device__ __forceinline__ void mma_16816_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Warps that split K = number of contiguous K ranges, each a multiple of 128.
__host__ __device__ __forceinline__ int ksplit_for(int64_t K) {
  if (K % (128 * 8) == 0) return 8;
  if (K % (128 * 6) == 0) return 6;
  if (K % (128 * 4) == 0) return 4;
  if (K % (128 * 3) == 0) return 3;
  if (K % (128 * 2) == 0) return 2;
  return 1;
}

// Row stride (halves) of a staged activation tile: +8 halves (16 bytes) keeps
// the LDS.128 phases of neighbouring columns on distinct banks.
__host__ __device__ __forceinline__ int xs_stride(int64_t K) { return (int)K + 8; }

// Stage `ncols` BF16 vectors of length K (row stride src_stride) into shared
// memory as FP16 * 2^-e; returns the multiplier 2^e (same in every block
// because every block stages the same values).  K % 8 == 0, 16-byte aligned
// source rows.  Uses `red` (>= 32 floats of shared memory) for the max.
__device__ __forceinline__ float stage_f16(__half* xs, int stride, const uint16_t* src, int64_t src_stride,
                                           int ncols, int K, float* red) {
  const int n8 = K >> 3;
  float m = 0.f;
  for (int i = threadIdx.x; i < ncols * n8; i += blockDim.x) {
    const int c = i / n8, j = i - c * n8;
    const uint4 v = *reinterpret_cast<const uint4*>(src + (int64_t)c * src_stride + 8 * j);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      m = fmaxf(m, fabsf(__uint_as_float(w[t] << 16)));
      m = fmaxf(m, fabsf(__uint_as_float(w[t] & 0xFFFF0000u)));
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float mx = red[0];
  int e = 0;
  if (mx >= 16384.0f) {  // keep |x| * 2^-e < 2^15 (FP16 max 65504)
    int ex;
    frexpf(mx, &ex);  // mx = f * 2^ex, f in [0.5, 1)
    e = ex - 14;
  }
  const float down = ldexpf(1.0f, -e);
  for (int i = threadIdx.x; i < ncols * n8; i += blockDim.x) {
    const int c = i / n8, j = i - c * n8;
    const uint4 v = *reinterpret_cast<const uint4*>(src + (int64_t)c * src_stride + 8 * j);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      __half2 h = __floats2half2_rn(__uint_as_float(w[t] << 16) * down, __uint_as_float(w[t] & 0xFFFF0000u) * down);
      o[t] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(xs + c * stride + 8 * j) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  __syncthreads();
  return ldexpf(1.0f, e);
}

// ---------------------------------------------------------------------------
// Streaming: every lane copies its own 16-byte weight fragments into a
// per-warp shared-memory ring with cp.async (L2 only) and later reads back
// exactly what it wrote, so the ring needs no barrier: cp.async.wait_group
// orders each lane's own copies.  The kernels feed one continuous stream of
// 64-wide K slices per warp across tiles, so the ring never drains between
// tiles.
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte global -> shared copy; `valid == false` writes zeros and reads
// nothing (src must still be a mapped address).
__device__ __forceinline__ void cp_async_16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_addr(dst)), "l"(src),
               "r"(valid ? 16 : 0));
}
// As cp_async_16, with the hint that L2 fetch the whole aligned 256-byte
// block around the source from DRAM.  The decode streams read each weight row
// 64 bytes per slice; the longer DRAM bursts measured about 1 us less per
// config-2 decode step on B200 (the 128-byte hint: no change).
__device__ __forceinline__ void cp_async_16_l2_256(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16, %2;\n" ::"r"(smem_addr(dst)), "l"(src),
               "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void cp_async_commit_group() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Four E4M3 codes -> two FP16x2 (codes 0,1 and 2,3).  FINITE: the hardware
// conversion, exact for every code except 0x7F/0xFF (NaN in E4M3FN), values
// lut(c); otherwise the exact bit re-bias of common.cuh, values lut(c)/256.
template <bool FINITE>
__device__ __forceinline__ void e4m3x4_frag(uint32_t w, uint32_t& lo, uint32_t& hi) {
  if (FINITE) {
    const uint16_t a = (uint16_t)(w & 0xFFFFu), b = (uint16_t)(w >> 16);
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(lo) : "h"(a));
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(hi) : "h"(b));
  } else {
    e4m3x4_to_h2(w, lo, hi);
  }
}

// Scale multiplier that undoes the decode's factor (lut/256 for the exact path).
template <bool FINITE>
__host__ __device__ __forceinline__ constexpr float decode_unscale() {
  return FINITE ? 1.0f : 256.0f;
}

// Four m16n8k16 MMAs of one 64-wide K slice of one 16-row weight tile:
// va/vb = this lane's 16 codes of tile rows g and g+8, xw = its activation words.
template <bool FINITE>
__device__ __forceinline__ void mma_slice(float (&part)[4], uint4 va, uint4 vb, const uint32_t (&xw)[8]) {
  const uint32_t wa[4] = {va.x, va.y, va.z, va.w};
  const uint32_t wb[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t a0, a1, a2, a3;
    e4m3x4_frag<FINITE>(wa[i], a0, a2);
    e4m3x4_frag<FINITE>(wb[i], a1, a3);
    mma_16816_f16(part, a0, a1, a2, a3, xw[2 * i], xw[2 * i + 1]);
  }
}

// This lane's activation words for one slice: 16 FP16 values at xp (column
// g = lane / 4, K offset 16 * (lane % 4)); zeros when the column is unused.
__device__ __forceinline__ void load_x_frag(uint32_t (&xw)[8], const __half* xp, bool xok) {
  uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
  if (xok) {
    xa = *reinterpret_cast<const uint4*>(xp);
    xb = *reinterpret_cast<const uint4*>(xp + 8);
  }
  xw[0] = xa.x;
  xw[1] = xa.y;
  xw[2] = xa.z;
  xw[3] = xa.w;
  xw[4] = xb.x;
  xw[5] = xb.y;
  xw[6] = xb.z;
  xw[7] = xb.w;
}

// Programmatic dependent launch.  pdl_wait: block until the grids this
// kernel depends on have completed and their writes are visible (returns at
// once when the kernel was launched without programmatic serialisation).
// pdl_trigger: let the next kernel, if launched with programmatic
// serialisation, start once every block of this grid has triggered or exited.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// One row of block scales spread over the warp (entry b in lane b % 32,
// register b / 32), loaded once up front so that a promotion never waits on
// memory.  Rows longer than 64 entries fall back to a load per promotion.
struct WarpScales {
  float r0, r1;
  const float* row;
  int n;
  __device__ __forceinline__ void load(const float* p, int count, bool ok) {
    const int lane = threadIdx.x & 31;
    row = p;
    n = count;
    r0 = (ok && lane < count) ? __ldg(p + lane) : 0.f;
    r1 = (ok && lane + 32 < count) ? __ldg(p + lane + 32) : 0.f;
  }
  // b is warp-uniform and every lane of the warp calls this.
  __device__ __forceinline__ float at(int b) const {
    if (n <= 64) return __shfl_sync(0xffffffffu, b < 32 ? r0 : r1, b & 31);
    return __ldg(row + b);
  }
};

// Promotion at the end of a 128-K block with one scale for rows g and g+8
// (tot[0..1]) and another for the other half of the tile (tot[2..3]).
__device__ __forceinline__ void promote2(float (&tot)[4], float (&part)[4], float s_lo, float s_hi) {
  tot[0] = fmaf(s_lo, part[0], tot[0]);
  tot[1] = fmaf(s_lo, part[1], tot[1]);
  tot[2] = fmaf(s_hi, part[2], tot[2]);
  tot[3] = fmaf(s_hi, part[3], tot[3]);
#pragma unroll
  for (int c = 0; c < 4; ++c) part[c] = 0.f;
}

// Promotion at the end of a 128-K block: tot += s * part; part = 0.
__device__ __forceinline__ void promote(float (&tot)[4], float (&part)[4], float s) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    tot[c] = fmaf(s, part[c], tot[c]);
    part[c] = 0.f;
  }
}

}  // namespace glm53
