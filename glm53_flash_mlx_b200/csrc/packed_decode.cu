// Packed L=1 decode MoE (G3 + G4).
//
// Replaces PackedFP8MoE.__call__ decode (glm53_flash_mlx/packed.py:896-923):
//   K7  fused gate/up/SwiGLU over the selected experts  (packed.py:100-166)
//   K9  the same for the shared expert                  (packed.py:181-235)
//   K6  selected down projections                        (packed.py:66-98)
//   K8  FP32 slot-ordered weighted reduction             (packed.py:168-179)
//   shared down (K1) and the BF16 `result + shared` add  (packed.py:915-922)
// in two launches:
//   decode_gate_up_kernel: one warp per (slot, row) pair; the shared expert is
//     one more slot.  Each lane streams 16-byte chunks of the gate and up rows
//     and multiplies them against FP32 activations in shared memory.
//   decode_down_kernel: one warp per slot, a block owns RB output rows; the
//     per-slot dot products meet in shared memory and are reduced in slot
//     order with the reference's rounding points.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace glm53 {

__device__ __forceinline__ int xsw(int c, int q) { return 4 * c + (q ^ ((c >> 1) & 3)); }

__device__ __forceinline__ float dot16_x(uint4 w, const float4* xs4, int c) {
  float f[4];
  float acc = 0.f;
  uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    e4m3x4_to_f32(words[q], f);
    float4 xv = xs4[xsw(c, q)];
    acc = fmaf(xv.x, f[0], acc);
    acc = fmaf(xv.y, f[1], acc);
    acc = fmaf(xv.z, f[2], acc);
    acc = fmaf(xv.w, f[3], acc);
  }
  return acc;
}

// BF16 [n] -> swizzled FP32 in shared memory (n % 16 == 0).
__device__ __forceinline__ void stage_bf16_swizzled(float4* xs4, const uint16_t* src, int n) {
  for (int i = threadIdx.x; i < (n >> 2); i += blockDim.x) {
    const uint2 raw = *reinterpret_cast<const uint2*>(src + 4 * i);
    float4 v;
    v.x = __uint_as_float(raw.x << 16);
    v.y = __uint_as_float(raw.x & 0xFFFF0000u);
    v.z = __uint_as_float(raw.y << 16);
    v.w = __uint_as_float(raw.y & 0xFFFF0000u);
    xs4[xsw(i >> 2, i & 3)] = v;
  }
}

struct DecodeArgs {
  const uint16_t* x;
  int H, I, Is, E, top_k;
  const uint32_t* ids;
  const float* scores;
  const uint8_t* gu_w;
  const float* gu_s;
  const uint8_t* d_w;
  const float* d_s;
  const uint8_t* sg_w;
  const float* sg_s;
  const uint8_t* su_w;
  const float* su_s;
  const uint8_t* sd_w;
  const float* sd_s;
  float limit;
  uint16_t* hidden;  // [top_k*I + Is]
  uint16_t* out;     // [H]
  uint32_t* status;
};

// ---------------------------------------------------------------------------
// Gate/up/SwiGLU.  Vector path: H % 16 == 0, 16-byte aligned weights.
// ---------------------------------------------------------------------------
template <int CPL>  // 16-byte chunks per lane per row: ceil(H / 16 / 32)
__global__ void __launch_bounds__(256) decode_gate_up_kernel(DecodeArgs a) {
  extern __shared__ float4 xs4[];
  stage_bf16_swizzled(xs4, a.x, a.H);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  const int nchunks = a.H >> 4;
  const int cols = (a.H + kBlock - 1) / kBlock;
  const int half = (a.I + kBlock - 1) / kBlock;
  const int routed = a.top_k * a.I;
  const int items = routed + a.Is;
  for (int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); item < items; item += nwarps) {
    const uint8_t* gw;
    const uint8_t* uw;
    const float* gs;
    const float* us;
    if (item < routed) {
      const int slot = item / a.I, row = item - slot * a.I;
      const uint32_t e = a.ids[slot];
      if (e >= (uint32_t)a.E) {
        if (lane == 0) {
          atomicOr(a.status, kStatusBadExpert);
          a.hidden[item] = 0;
        }
        continue;
      }
      gw = a.gu_w + ((size_t)e * 2 * a.I + row) * a.H;
      uw = gw + (size_t)a.I * a.H;
      gs = a.gu_s + ((size_t)e * 2 * half + row / kBlock) * cols;
      us = gs + (size_t)half * cols;
    } else {
      const int row = item - routed;
      gw = a.sg_w + (size_t)row * a.H;
      uw = a.su_w + (size_t)row * a.H;
      gs = a.sg_s + (size_t)(row / kBlock) * cols;
      us = a.su_s + (size_t)(row / kBlock) * cols;
    }
    const uint4* g4 = reinterpret_cast<const uint4*>(gw);
    const uint4* u4 = reinterpret_cast<const uint4*>(uw);
    uint4 gv[CPL], uv[CPL];
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const int c = lane + 32 * j;
      if (c < nchunks) {
        gv[j] = ldg_stream(g4 + c);
        uv[j] = ldg_stream(u4 + c);
      }
    }
    float gacc = 0.f, uacc = 0.f;
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const int c = lane + 32 * j;
      if (c < nchunks) {
        const float gsc = __ldg(gs + (c >> 3)) * 256.0f;
        const float usc = __ldg(us + (c >> 3)) * 256.0f;
        gacc = fmaf(gsc, dot16_x(gv[j], xs4, c), gacc);
        uacc = fmaf(usc, dot16_x(uv[j], xs4, c), uacc);
      }
    }
    gacc = warp_sum(gacc);
    uacc = warp_sum(uacc);
    if (lane == 0) a.hidden[item] = swiglu_bf16(gacc, uacc, a.limit);
  }
}

// ---------------------------------------------------------------------------
// Down + weighted reduction + shared add.  Block = NS warps (one per slot,
// the shared expert last), RB output rows per block iteration.
// ---------------------------------------------------------------------------
constexpr int kDownRB = 4;
constexpr int kDownMaxSlots = 9;  // 8 routed + shared on the vector path

template <int CPL>  // chunks per lane per row: ceil(I / 16 / 32)
__global__ void __launch_bounds__(32 * kDownMaxSlots) decode_down_kernel(DecodeArgs a) {
  extern __shared__ float4 smem4[];
  const int ns = a.top_k + (a.Is > 0 ? 1 : 0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // per-slot activations: routed slots stride I, the shared slot stride Is
  float4* xs4 = smem4 + (size_t)warp * (max(a.I, a.Is) >> 2);
  float* dots = reinterpret_cast<float*>(smem4 + (size_t)ns * (max(a.I, a.Is) >> 2));  // [RB][ns]
  const bool shared_slot = (warp == a.top_k);
  const int kin = shared_slot ? a.Is : a.I;
  if (warp < ns) {
    const uint16_t* src = a.hidden + (shared_slot ? (size_t)a.top_k * a.I : (size_t)warp * a.I);
    for (int i = lane; i < (kin >> 2); i += 32) {
      const uint2 raw = *reinterpret_cast<const uint2*>(src + 4 * i);
      float4 v;
      v.x = __uint_as_float(raw.x << 16);
      v.y = __uint_as_float(raw.x & 0xFFFF0000u);
      v.z = __uint_as_float(raw.y << 16);
      v.w = __uint_as_float(raw.y & 0xFFFF0000u);
      xs4[xsw(i >> 2, i & 3)] = v;
    }
  }
  __syncthreads();
  uint32_t e = 0;
  bool valid = warp < ns;
  if (valid && !shared_slot) {
    e = a.ids[warp];
    if (e >= (uint32_t)a.E) {
      valid = false;
      if (lane == 0 && blockIdx.x == 0) atomicOr(a.status, kStatusBadExpert);
    }
  }
  const int nchunks = kin >> 4;
  const int cols = (kin + kBlock - 1) / kBlock;
  const int hrows = (a.H + kBlock - 1) / kBlock;
  const uint8_t* wbase = shared_slot ? a.sd_w : a.d_w + (size_t)e * a.H * a.I;
  const float* sbase = shared_slot ? a.sd_s : a.d_s + (size_t)e * hrows * cols;
  for (int h0 = blockIdx.x * kDownRB; h0 < a.H; h0 += gridDim.x * kDownRB) {
    if (warp < ns) {
      float acc[kDownRB];
      if (valid) {
        uint4 wv[kDownRB][CPL];
#pragma unroll
        for (int r = 0; r < kDownRB; ++r) {
          const uint4* w4 = reinterpret_cast<const uint4*>(wbase + (size_t)(h0 + r) * kin);
#pragma unroll
          for (int j = 0; j < CPL; ++j) {
            const int c = lane + 32 * j;
            if (c < nchunks && h0 + r < a.H) wv[r][j] = ldg_stream(w4 + c);
          }
        }
#pragma unroll
        for (int r = 0; r < kDownRB; ++r) {
          const float* srow = sbase + (size_t)((h0 + r) / kBlock) * cols;
          float v = 0.f;
#pragma unroll
          for (int j = 0; j < CPL; ++j) {
            const int c = lane + 32 * j;
            if (c < nchunks && h0 + r < a.H)
              v = fmaf(__ldg(srow + (c >> 3)) * 256.0f, dot16_x(wv[r][j], xs4, c), v);
          }
          acc[r] = warp_sum(v);
        }
      } else {
#pragma unroll
        for (int r = 0; r < kDownRB; ++r) acc[r] = 0.f;
      }
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < kDownRB; ++r) dots[r * ns + warp] = acc[r];
      }
    }
    __syncthreads();
    if (threadIdx.x < kDownRB && h0 + (int)threadIdx.x < a.H) {
      const int r = threadIdx.x;
      float total = 0.f;
      for (int j = 0; j < a.top_k; ++j) {
        // K6 stores BF16, K8 multiplies f32(down) by the FP32 route weight
        const float d = bf16_round(dots[r * ns + j]);
        total = total + __fmul_rn(d, a.scores[j]);
      }
      float res = bf16_round(total);
      if (a.Is > 0) res = res + bf16_round(dots[r * ns + a.top_k]);
      a.out[h0 + r] = f32_to_bf16_bits(res);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Generic (unaligned) path: one warp per dot product, scalar loads.
// ---------------------------------------------------------------------------
__global__ void decode_gate_up_scalar_kernel(DecodeArgs a) {
  const int lane = threadIdx.x & 31;
  const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int routed = a.top_k * a.I;
  if (item >= routed + a.Is) return;
  const int cols = (a.H + kBlock - 1) / kBlock;
  const int half = (a.I + kBlock - 1) / kBlock;
  const uint8_t *gw, *uw;
  const float *gs, *us;
  if (item < routed) {
    const int slot = item / a.I, row = item % a.I;
    const uint32_t e = a.ids[slot];
    if (e >= (uint32_t)a.E) {
      if (lane == 0) {
        atomicOr(a.status, kStatusBadExpert);
        a.hidden[item] = 0;
      }
      return;
    }
    gw = a.gu_w + ((size_t)e * 2 * a.I + row) * a.H;
    uw = gw + (size_t)a.I * a.H;
    gs = a.gu_s + ((size_t)e * 2 * half + row / kBlock) * cols;
    us = gs + (size_t)half * cols;
  } else {
    const int row = item - routed;
    gw = a.sg_w + (size_t)row * a.H;
    uw = a.su_w + (size_t)row * a.H;
    gs = a.sg_s + (size_t)(row / kBlock) * cols;
    us = a.su_s + (size_t)(row / kBlock) * cols;
  }
  float g = 0.f, u = 0.f;
  for (int k = lane; k < a.H; k += 32) {
    const float xv = bf16_bits_to_f32(a.x[k]);
    g = fmaf(xv * e4m3_to_f32_scaled(gw[k]), gs[k / kBlock] * 256.0f, g);
    u = fmaf(xv * e4m3_to_f32_scaled(uw[k]), us[k / kBlock] * 256.0f, u);
  }
  g = warp_sum(g);
  u = warp_sum(u);
  if (lane == 0) a.hidden[item] = swiglu_bf16(g, u, a.limit);
}

__global__ void decode_down_scalar_kernel(DecodeArgs a) {
  const int lane = threadIdx.x & 31;
  const int h = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (h >= a.H) return;
  float total = 0.f;
  for (int j = 0; j < a.top_k; ++j) {
    const uint32_t e = a.ids[j];
    float v = 0.f;
    if (e < (uint32_t)a.E) {
      const int cols = (a.I + kBlock - 1) / kBlock;
      const int hrows = (a.H + kBlock - 1) / kBlock;
      const uint8_t* wr = a.d_w + ((size_t)e * a.H + h) * a.I;
      const float* sr = a.d_s + ((size_t)e * hrows + h / kBlock) * cols;
      const uint16_t* xr = a.hidden + (size_t)j * a.I;
      for (int k = lane; k < a.I; k += 32)
        v = fmaf(bf16_bits_to_f32(xr[k]) * e4m3_to_f32_scaled(wr[k]), sr[k / kBlock] * 256.0f, v);
      v = warp_sum(v);
    }
    total = total + __fmul_rn(bf16_round(v), a.scores[j]);
  }
  float res = bf16_round(total);
  if (a.Is > 0) {
    const int cols = (a.Is + kBlock - 1) / kBlock;
    const uint8_t* wr = a.sd_w + (size_t)h * a.Is;
    const float* sr = a.sd_s + (size_t)(h / kBlock) * cols;
    const uint16_t* xr = a.hidden + (size_t)a.top_k * a.I;
    float v = 0.f;
    for (int k = lane; k < a.Is; k += 32)
      v = fmaf(bf16_bits_to_f32(xr[k]) * e4m3_to_f32_scaled(wr[k]), sr[k / kBlock] * 256.0f, v);
    v = warp_sum(v);
    res = res + bf16_round(v);
  }
  if (lane == 0) a.out[h] = f32_to_bf16_bits(res);
}

template <int CPL>
static int launch_gate_up(const DecodeArgs& a, cudaStream_t st) {
  const size_t smem = (size_t)a.H * sizeof(float);
  if (smem > 48 * 1024) {
    int rc_attr = ensure_max_smem((const void*)decode_gate_up_kernel<CPL>, smem);
    if (rc_attr) return rc_attr;
  }
  const int items = a.top_k * a.I + a.Is;
  const int blocks = std::min((items + 7) / 8, sm_count() * 4);
  decode_gate_up_kernel<CPL><<<blocks, 256, smem, st>>>(a);
  return check_launch("decode_gate_up_kernel");
}

template <int CPL>
static int launch_down(const DecodeArgs& a, cudaStream_t st) {
  const int ns = a.top_k + (a.Is > 0 ? 1 : 0);
  const size_t smem = (size_t)ns * std::max(a.I, a.Is) * sizeof(float) + (size_t)kDownRB * ns * sizeof(float);
  if (smem > 48 * 1024) {
    int rc_attr = ensure_max_smem((const void*)decode_down_kernel<CPL>, smem);
    if (rc_attr) return rc_attr;
  }
  const int row_blocks = (a.H + kDownRB - 1) / kDownRB;
  const int per_sm = std::max(1, std::min(4, (int)(200 * 1024 / smem)));
  const int blocks = std::min(row_blocks, sm_count() * per_sm);
  decode_down_kernel<CPL><<<blocks, 32 * ns, smem, st>>>(a);
  return check_launch("decode_down_kernel");
}

int packed_decode(const DecodeArgs& a, cudaStream_t st, bool gate_up_only) {
  const bool has_shared = a.Is > 0;
  const bool aligned =
      a.H % 16 == 0 && a.I % 16 == 0 && (!has_shared || a.Is % 16 == 0) &&
      ((uintptr_t)a.gu_w & 15) == 0 && ((uintptr_t)a.d_w & 15) == 0 && ((uintptr_t)a.x & 7) == 0 &&
      (!has_shared || ((((uintptr_t)a.sg_w | (uintptr_t)a.su_w | (uintptr_t)a.sd_w) & 15) == 0)) &&
      a.H <= 8192 && std::max(a.I, a.Is) <= 2048 && a.top_k + (has_shared ? 1 : 0) <= kDownMaxSlots;
  if (!aligned) {
    const int items = a.top_k * a.I + a.Is;
    decode_gate_up_scalar_kernel<<<(items + 7) / 8, 256, 0, st>>>(a);
    int rc = check_launch("decode_gate_up_scalar_kernel");
    if (rc || gate_up_only) return rc;
    decode_down_scalar_kernel<<<(a.H + 7) / 8, 256, 0, st>>>(a);
    return check_launch("decode_down_scalar_kernel");
  }
  const int cpl_h = (a.H / 16 + 31) / 32;
  int rc;
  if (cpl_h <= 4) rc = launch_gate_up<4>(a, st);
  else if (cpl_h <= 8) rc = launch_gate_up<8>(a, st);
  else rc = launch_gate_up<16>(a, st);
  if (rc || gate_up_only) return rc;
  const int cpl_i = (std::max(a.I, a.Is) / 16 + 31) / 32;
  if (cpl_i <= 1) return launch_down<1>(a, st);
  if (cpl_i <= 2) return launch_down<2>(a, st);
  if (cpl_i <= 3) return launch_down<3>(a, st);
  return launch_down<4>(a, st);
}

}  // namespace glm53

using namespace glm53;

extern "C" size_t glm53_packed_decode_workspace_bytes(int top_k, int64_t I, int64_t I_shared) {
  return align_up(((size_t)top_k * I + (size_t)I_shared) * sizeof(uint16_t), 256);
}

extern "C" int glm53_packed_decode_moe(const void* x, int64_t H, const uint32_t* expert_ids,
                                       const float* scores, int top_k, const uint8_t* gate_up_w,
                                       const float* gate_up_s, const uint8_t* down_w, const float* down_s,
                                       int64_t E, int64_t I, const uint8_t* shared_gate_w,
                                       const float* shared_gate_s, const uint8_t* shared_up_w,
                                       const float* shared_up_s, const uint8_t* shared_down_w,
                                       const float* shared_down_s, int64_t I_shared, float limit, void* out,
                                       void* workspace, size_t workspace_bytes, uint32_t* status,
                                       void* stream) {
  if (H <= 0 || I <= 0 || E <= 0 || top_k <= 0 || top_k > 16 || I_shared < 0 || H > INT32_MAX / 2 ||
      I > INT32_MAX / 64) {
    set_last_error("glm53_packed_decode_moe: invalid geometry H=%lld I=%lld E=%lld top_k=%d", (long long)H,
                   (long long)I, (long long)E, top_k);
    return GLM53_ERR_INVALID;
  }
  const bool has_shared = I_shared > 0;
  if (!x || !expert_ids || !scores || !gate_up_w || !gate_up_s || !down_w || !down_s || !out || !status ||
      !workspace || workspace_bytes < glm53_packed_decode_workspace_bytes(top_k, I, I_shared) ||
      (has_shared && (!shared_gate_w || !shared_gate_s || !shared_up_w || !shared_up_s || !shared_down_w ||
                      !shared_down_s))) {
    set_last_error("glm53_packed_decode_moe: missing pointer or workspace too small");
    return GLM53_ERR_INVALID;
  }
  DecodeArgs a;
  a.x = (const uint16_t*)x;
  a.H = (int)H;
  a.I = (int)I;
  a.Is = (int)I_shared;
  a.E = (int)std::min<int64_t>(E, INT32_MAX);
  a.top_k = top_k;
  a.ids = expert_ids;
  a.scores = scores;
  a.gu_w = gate_up_w;
  a.gu_s = gate_up_s;
  a.d_w = down_w;
  a.d_s = down_s;
  a.sg_w = shared_gate_w;
  a.sg_s = shared_gate_s;
  a.su_w = shared_up_w;
  a.su_s = shared_up_s;
  a.sd_w = shared_down_w;
  a.sd_s = shared_down_s;
  a.limit = limit;
  a.hidden = (uint16_t*)workspace;
  a.out = (uint16_t*)out;
  a.status = status;
  return packed_decode(a, (cudaStream_t)stream, false);
}

extern "C" int glm53_packed_decode_gate_up(const void* x, int64_t H, const uint32_t* expert_ids, int top_k,
                                           const uint8_t* gate_up_w, const float* gate_up_s, int64_t E, int64_t I,
                                           const uint8_t* shared_gate_w, const float* shared_gate_s,
                                           const uint8_t* shared_up_w, const float* shared_up_s, int64_t I_shared,
                                           float limit, void* workspace, size_t workspace_bytes, uint32_t* status,
                                           void* stream) {
  if (H <= 0 || I <= 0 || E <= 0 || top_k <= 0 || top_k > 16 || I_shared < 0 || H > INT32_MAX / 2 ||
      I > INT32_MAX / 64) {
    set_last_error("glm53_packed_decode_gate_up: invalid geometry");
    return GLM53_ERR_INVALID;
  }
  const bool has_shared = I_shared > 0;
  if (!x || !expert_ids || !gate_up_w || !gate_up_s || !status || !workspace ||
      workspace_bytes < glm53_packed_decode_workspace_bytes(top_k, I, I_shared) ||
      (has_shared && (!shared_gate_w || !shared_gate_s || !shared_up_w || !shared_up_s))) {
    set_last_error("glm53_packed_decode_gate_up: missing pointer or workspace too small");
    return GLM53_ERR_INVALID;
  }
  DecodeArgs a{};
  a.x = (const uint16_t*)x;
  a.H = (int)H;
  a.I = (int)I;
  a.Is = (int)I_shared;
  a.E = (int)std::min<int64_t>(E, INT32_MAX);
  a.top_k = top_k;
  a.ids = expert_ids;
  a.gu_w = gate_up_w;
  a.gu_s = gate_up_s;
  a.sg_w = shared_gate_w;
  a.sg_s = shared_gate_s;
  a.su_w = shared_up_w;
  a.su_s = shared_up_s;
  a.limit = limit;
  a.hidden = (uint16_t*)workspace;
  a.status = status;
  // the down-stage pointers are not used by this stage; keep the alignment
  // test of packed_decode() satisfied with the gate/up bank pointer
  a.d_w = gate_up_w;
  a.sd_w = has_shared ? shared_gate_w : nullptr;
  return packed_decode(a, (cudaStream_t)stream, true);
}
