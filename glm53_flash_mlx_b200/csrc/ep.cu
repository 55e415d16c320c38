// Expert-parallel decode: dispatch packing on the tokens' home rank.
//
// Experts are split into `world` contiguous ranges of E / world; a route
// (token t, slot j) with expert e goes to rank d = e / (E / world).  The send
// buffer has `capacity` slots per destination rank; within a destination the
// routes keep route order t * top_k + j (so the layout, and every result
// computed from it, is the same whatever the timing).  The exchange itself is
// an all-to-all over equal chunks of `capacity` slots (NCCL, host side); the
// owner runs glm53_routes_decode on the received slots and sends the BF16 rows
// back in the same slots; glm53_ep_combine reduces them in slot order.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace glm53 {

constexpr int kEpPlanThreads = 1024;
constexpr int kEpMaxWorld = 32;
constexpr uint32_t kEpEmpty = 0xFFFFFFFFu;

// One CTA: slot positions of all routes (stable per destination), the slot
// tables (local expert id or empty, score) and each route's position.
__global__ void __launch_bounds__(kEpPlanThreads) ep_plan_kernel(const uint32_t* __restrict__ ids,
                                                                 const float* __restrict__ scores, int R, int E,
                                                                 int world, int cap, uint32_t* __restrict__ send_expert,
                                                                 float* __restrict__ slot_scores,
                                                                 uint32_t* __restrict__ route_pos,
                                                                 uint32_t* __restrict__ status) {
  __shared__ uint32_t warp_counts[kEpPlanThreads / 32][kEpMaxWorld];
  __shared__ uint32_t base[kEpMaxWorld];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per_rank = E / world;
  for (int i = tid; i < world * cap; i += blockDim.x) {
    send_expert[i] = kEpEmpty;
    slot_scores[i] = 0.f;
  }
  if (tid < kEpMaxWorld) base[tid] = 0u;
  __syncthreads();
  for (int c0 = 0; c0 < R; c0 += blockDim.x) {
    const int r = c0 + tid;
    uint32_t e = r < R ? ids[r] : kEpEmpty;
    const bool bad = r < R && e >= (uint32_t)E;
    if (bad) atomicOr(status, kStatusBadExpert);
    const int d = (r < R && !bad) ? (int)(e / (uint32_t)per_rank) : -1;
    const uint32_t lt = (1u << lane) - 1u;
    uint32_t my_rank_in_warp = 0;
    for (int dd = 0; dd < world; ++dd) {
      const uint32_t m = __ballot_sync(0xffffffffu, d == dd);
      if (d == dd) my_rank_in_warp = __popc(m & lt);
      if (lane == 0) warp_counts[warp][dd] = __popc(m);
    }
    __syncthreads();
    // exclusive prefix over warps for this thread's destination
    uint32_t before = 0;
    if (d >= 0) {
      for (int w = 0; w < warp; ++w) before += warp_counts[w][d];
      const uint32_t slot = base[d] + before + my_rank_in_warp;
      if (slot < (uint32_t)cap) {
        const uint32_t pos = (uint32_t)d * cap + slot;
        send_expert[pos] = e - (uint32_t)(d * per_rank);
        slot_scores[pos] = scores[r];
        route_pos[r] = pos;
      } else {
        atomicOr(status, kStatusBadGeometry);  // capacity exceeded: the route is dropped
        route_pos[r] = kEpEmpty;
      }
    } else if (r < R) {
      route_pos[r] = kEpEmpty;
    }
    __syncthreads();
    if (tid < world) {
      uint32_t tot = 0;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += warp_counts[w][tid];
      base[tid] += tot;
    }
    __syncthreads();
  }
}

// send_x[pos] = x[token of the route]; one CTA per route.
__global__ void ep_pack_rows_kernel(const uint16_t* __restrict__ x, int H, int top_k,
                                    const uint32_t* __restrict__ route_pos, uint16_t* __restrict__ send_x) {
  const int r = blockIdx.x;
  const uint32_t pos = route_pos[r];
  if (pos == kEpEmpty) return;
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(r / top_k) * H);
  uint4* dst = reinterpret_cast<uint4*>(send_x + (size_t)pos * H);
  for (int i = threadIdx.x; i < (H >> 3); i += blockDim.x) dst[i] = src[i];
}

// out[t] = BF16(sum_j f32(rows[pos(t, j)]) * slot_scores[pos]) (+ shared[t],
// BF16 add): the decode's slot-ordered reduce (glm53_flash_mlx/packed.py:
// 168-179) over rows that came back from their owners; dropped routes
// (position kEpEmpty) contribute nothing.  8 columns per thread.
__global__ void ep_combine_kernel(const uint16_t* __restrict__ rows, const float* __restrict__ slot_scores,
                                  const uint32_t* __restrict__ route_pos, int64_t T, int top_k, int64_t H,
                                  const uint16_t* __restrict__ shared, uint16_t* __restrict__ out) {
  const int64_t chunks = H / 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * chunks) return;
  const int64_t t = i / chunks, c = i % chunks;
  float total[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) total[q] = 0.f;
  for (int j = 0; j < top_k; ++j) {
    const uint32_t pos = route_pos[t * top_k + j];
    if (pos == kEpEmpty) continue;
    const float sc = slot_scores[pos];
    const uint4 v = reinterpret_cast<const uint4*>(rows + (int64_t)pos * H)[c];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      total[2 * q] = total[2 * q] + __fmul_rn(__uint_as_float(w[q] << 16), sc);
      total[2 * q + 1] = total[2 * q + 1] + __fmul_rn(__uint_as_float(w[q] & 0xFFFF0000u), sc);
    }
  }
  uint4 sh = make_uint4(0, 0, 0, 0);
  if (shared) sh = reinterpret_cast<const uint4*>(shared + t * H)[c];
  const uint32_t sw[4] = {sh.x, sh.y, sh.z, sh.w};
  uint32_t o[4];
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

}  // namespace glm53

using namespace glm53;

extern "C" int glm53_ep_combine(const void* rows, const uint32_t* route_pos, const float* slot_scores, int64_t T,
                                int top_k, int64_t H, const void* shared, void* out, void* stream) {
  if (T < 0 || top_k <= 0 || H <= 0 || H % 8 != 0 ||
      (T > 0 && (!rows || !route_pos || !slot_scores || !out)) ||
      ((((uintptr_t)rows) | ((uintptr_t)out) | ((uintptr_t)shared)) & 15) != 0) {
    set_last_error("glm53_ep_combine: invalid arguments (H %% 8 == 0, 16-byte aligned rows required)");
    return GLM53_ERR_INVALID;
  }
  if (T == 0) return GLM53_OK;
  const int64_t n = T * (H / 8);
  ep_combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint16_t*)rows, slot_scores, route_pos, T, top_k, H, (const uint16_t*)shared, (uint16_t*)out);
  return check_launch("ep_combine_kernel");
}

extern "C" int glm53_ep_dispatch_pack(const void* x, int64_t T, int64_t H, const uint32_t* expert_ids,
                                      const float* scores, int top_k, int64_t E, int world, int64_t capacity,
                                      void* send_x, uint32_t* send_expert, float* slot_scores, uint32_t* route_pos,
                                      uint32_t* status, void* stream) {
  const char* fn = "glm53_ep_dispatch_pack";
  if (T < 0 || H <= 0 || top_k <= 0 || E <= 0 || world < 1 || world > kEpMaxWorld || E % world != 0 ||
      capacity <= 0 || H % 8 != 0 || T * top_k > INT32_MAX || world * capacity > INT32_MAX) {
    set_last_error("%s: invalid geometry (E must split evenly over 1..%d ranks, H %% 8 == 0)", fn, kEpMaxWorld);
    return GLM53_ERR_INVALID;
  }
  if (!x || !expert_ids || !scores || !send_x || !send_expert || !slot_scores || !route_pos || !status ||
      ((((uintptr_t)x) | ((uintptr_t)send_x)) & 15) != 0) {
    set_last_error("%s: missing pointer or unaligned rows", fn);
    return GLM53_ERR_INVALID;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const int R = (int)(T * top_k);
  ep_plan_kernel<<<1, kEpPlanThreads, 0, st>>>(expert_ids, scores, R, (int)E, world, (int)capacity, send_expert,
                                               slot_scores, route_pos, status);
  int rc = check_launch("ep_plan_kernel");
  if (rc || R == 0) return rc;
  ep_pack_rows_kernel<<<R, 256, 0, st>>>((const uint16_t*)x, (int)H, top_k, route_pos, (uint16_t*)send_x);
  return check_launch("ep_pack_rows_kernel");
}
