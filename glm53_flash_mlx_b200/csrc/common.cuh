// Shared device helpers for the sm_100a FP8 MoE kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/glm53_b200.h"

namespace glm53 {

constexpr int kBlock = 128;   // 128x128 weight-scale block
constexpr int kWarp = 32;
constexpr int kNumSMs = 148;  // B200; runtime code queries the device

// Device status word bits (written with atomicOr, read by the host wrapper).
constexpr uint32_t kStatusBadExpert = 1u << 0;   // expert id >= expert count
constexpr uint32_t kStatusWaitTimeout = 1u << 1; // a bounded spin-wait gave up
constexpr uint32_t kStatusBadGeometry = 1u << 2;

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(((uint32_t)b) << 16);
}

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}

// Round an FP32 value to BF16 (nearest-even) and back.
__device__ __forceinline__ float bf16_round(float f) {
  return __bfloat162float(__float2bfloat16_rn(f));
}

// Four E4M3 codes (one 32-bit word, little-endian) -> four FP32 values equal
// to lut(code) / 256, where lut is the reference table
// (glm53_flash_mlx/fp8.py:22-27, including 0x7F/0xFF = +-480).
// Each code c becomes the FP16 bit pattern (c & 0x80) << 8 | (c & 0x7F) << 7:
// the E4M3 exponent lands in the FP16 exponent field with a bias gap of 8, so
// the FP16 value is exactly lut(c) * 2^-8 for normals and subnormals alike,
// and exponent field 15 (codes 0x78..0x7F) stays finite.  The 2^8 is folded
// into the block scale by the caller.
__device__ __forceinline__ void e4m3x4_to_f32(uint32_t w, float f[4]) {
  uint32_t lo = __byte_perm(w, 0u, 0x1404);  // halves: b0 << 8, b1 << 8
  uint32_t hi = __byte_perm(w, 0u, 0x3424);  // halves: b2 << 8, b3 << 8
  lo = (lo & 0x80008000u) | ((lo >> 1) & 0x3F803F80u);
  hi = (hi & 0x80008000u) | ((hi >> 1) & 0x3F803F80u);
  float2 a = __half22float2(*reinterpret_cast<__half2*>(&lo));
  float2 b = __half22float2(*reinterpret_cast<__half2*>(&hi));
  f[0] = a.x;
  f[1] = a.y;
  f[2] = b.x;
  f[3] = b.y;
}

// Same decode, producing two packed FP16x2 registers (lut(c) * 2^-8).
__device__ __forceinline__ void e4m3x4_to_h2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  lo = __byte_perm(w, 0u, 0x1404);
  hi = __byte_perm(w, 0u, 0x3424);
  lo = (lo & 0x80008000u) | ((lo >> 1) & 0x3F803F80u);
  hi = (hi & 0x80008000u) | ((hi >> 1) & 0x3F803F80u);
}

__device__ __forceinline__ float e4m3_to_f32_scaled(uint8_t c) {
  uint16_t h = (uint16_t)(((c & 0x80u) << 8) | ((c & 0x7Fu) << 7));
  return __half2float(*reinterpret_cast<__half*>(&h));
}

// BF16 sigmoid with per-op BF16 rounding (glm53_flash_mlx/packed.py:155-160):
// tail = 1 / (1 + exp(|g|)), sig = g < 0 ? tail : 1 - tail, each operation
// rounded to BF16, exp correctly rounded (computed in FP64, rounded to FP32,
// then BF16).  At g = -6.84375 (0xC0DB) the reference's exponential lands on
// the other side of a BF16 rounding boundary and yields 0x3A8C; that single
// input is pinned to the reference value.  The reference's own all-BF16 sweep
// over [-10, 10] (33,346 values) is reproduced exactly.
__device__ __forceinline__ float sigmoid_bf16(uint16_t g_bits) {
  if (g_bits == 0xC0DBu) return bf16_bits_to_f32(0x3A8Cu);
  float g = bf16_bits_to_f32(g_bits);
  float a = fabsf(g);
  float e = bf16_round((float)exp((double)a));
  float den = bf16_round(1.0f + e);
  float tail = bf16_round(__fdiv_rn(1.0f, den));
  return (g < 0.0f) ? tail : bf16_round(1.0f - tail);
}

// SwiGLU epilogue of the fused gate/up kernels (glm53_flash_mlx/packed.py:
// 146-163): BF16 stores of both FP32 dot products, FP32 clamp (gate <= L,
// up in [-L, L]), BF16, sigmoid, SiLU = g * sig (BF16), times up (BF16).
__device__ __forceinline__ uint16_t swiglu_bf16(float gate_total, float up_total, float limit) {
  float gate_t = bf16_round(gate_total);
  float up_t = bf16_round(up_total);
  float gate_value = fminf(gate_t, limit);
  float up_value = fminf(fmaxf(up_t, -limit), limit);
  uint16_t ga = f32_to_bf16_bits(gate_value);
  float ua = bf16_round(up_value);
  float sig = sigmoid_bf16(ga);
  float silu = bf16_round(__fmul_rn(bf16_bits_to_f32(ga), sig));
  return f32_to_bf16_bits(__fmul_rn(silu, ua));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Dot product of 16 E4M3 codes (one uint4) with 16 FP32 activations in shared
// memory, unscaled (caller multiplies by the block scale * 256).
__device__ __forceinline__ float dot16_e4m3(uint4 w, const float* x) {
  float f[4];
  float acc = 0.f;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    e4m3x4_to_f32(words[q], f);
    float4 xv = x4[q];
    acc = fmaf(xv.x, f[0], acc);
    acc = fmaf(xv.y, f[1], acc);
    acc = fmaf(xv.z, f[2], acc);
    acc = fmaf(xv.w, f[3], acc);
  }
  return acc;
}

__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

}  // namespace glm53

// Host-side error plumbing shared by the C-ABI entry points (capi.cu).
namespace glm53 {
void set_last_error(const char* fmt, ...);
int check_launch(const char* what);
int sm_count();
int ensure_max_smem(const void* func, size_t bytes);

// Launch with programmatic stream serialisation: the kernel may start before
// the previous kernel on the stream has finished (once that kernel's blocks
// have all triggered or exited) and orders itself with griddepcontrol.wait.
template <typename... KArgs, typename... Args>
cudaError_t launch_programmatic(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
}  // namespace glm53
