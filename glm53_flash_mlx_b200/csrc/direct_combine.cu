// Direct-module combine for a small batch of decode tokens.
//
// Replaces the scatter-add loop of DirectFP8MoE.__call__ for more than one
// row (glm53_flash_mlx/fp8.py:384-399): for every touched expert in ascending
// id, weighted = BF16(f32(expert_out) * f32(score)) is added into a BF16
// result row (BF16(f32(a) + f32(b)), the order index_add applies them), and
// the shared expert's BF16 output is added last.  The per-route expert
// outputs come from glm53_routes_decode; the CTAs of a token rank its slots
// by expert id (a token selects an expert at most once, ties keep slot order)
// and their threads sweep 8 columns each.
#include <algorithm>

#include "common.cuh"

namespace glm53 {

constexpr int kCombineMaxK = 32;

constexpr int kCombineThreads = 64;  // 8 columns each: 512 columns per CTA

// row_of_slot (optional) maps route slot -> row of `rows` (sorted order);
// slots whose expert id is >= E are skipped and flagged in *status.  Grid:
// (token, 512-column range).  The token's ids, scores and row indices are
// staged in shared memory in ascending expert order (a slot's rank = the
// slots with a smaller id, or the same id and a smaller slot index: a stable
// sort), then every thread issues its column chunk of eight rows at a time
// before adding them in that order.
__global__ void __launch_bounds__(kCombineThreads) direct_combine_kernel(
    const uint16_t* __restrict__ rows, const uint32_t* __restrict__ row_of_slot, const uint32_t* __restrict__ ids,
    const float* __restrict__ scores, int top_k, int H, uint32_t E, uint32_t* status,
    const uint16_t* __restrict__ shared, uint16_t* __restrict__ out) {
  __shared__ uint32_t sid[kCombineMaxK];
  __shared__ uint32_t srow[kCombineMaxK];  // in expert order; 0xFFFFFFFF = skipped slot
  __shared__ float ssc[kCombineMaxK];
  const int t = blockIdx.x, j = threadIdx.x;
  // launched as a programmatic dependent of the stage that writes `rows`
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (j < top_k) sid[j] = __ldg(ids + (size_t)t * top_k + j);
  __syncthreads();
  if (j < top_k) {
    const uint32_t key = sid[j];
    int rank = 0;
    for (int i = 0; i < top_k; ++i) {
      const uint32_t k2 = sid[i];
      rank += (k2 < key) || (k2 == key && i < j);
    }
    const size_t slot = (size_t)t * top_k + j;
    const bool ok = key < E;
    srow[rank] = ok ? (row_of_slot ? __ldg(row_of_slot + slot) : (uint32_t)slot) : 0xFFFFFFFFu;
    ssc[rank] = ok ? __ldg(scores + slot) : 0.f;
    if (!ok && status && blockIdx.y == 0) atomicOr(status, kStatusBadExpert);
  }
  __syncthreads();
  for (int c = 8 * (blockIdx.y * blockDim.x + threadIdx.x); c < H; c += 8 * blockDim.x * gridDim.y) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int j0 = 0; j0 < top_k; j0 += 8) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint32_t r = j0 + u < top_k ? srow[j0 + u] : 0xFFFFFFFFu;
        v[u] = r != 0xFFFFFFFFu ? *reinterpret_cast<const uint4*>(rows + (size_t)r * H + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (j0 + u >= top_k || srow[j0 + u] == 0xFFFFFFFFu) continue;
        const float sc = ssc[j0 + u];
        const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float lo = bf16_round(__fmul_rn(__uint_as_float(w[i] << 16), sc));
          const float hi = bf16_round(__fmul_rn(__uint_as_float(w[i] & 0xFFFF0000u), sc));
          acc[2 * i] = bf16_round(acc[2 * i] + lo);
          acc[2 * i + 1] = bf16_round(acc[2 * i + 1] + hi);
        }
      }
    }
    if (shared) {
      const uint4 v = *reinterpret_cast<const uint4*>(shared + (size_t)t * H + c);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] = bf16_round(acc[2 * i] + __uint_as_float(w[i] << 16));
        acc[2 * i + 1] = bf16_round(acc[2 * i + 1] + __uint_as_float(w[i] & 0xFFFF0000u));
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o[i] = (uint32_t)f32_to_bf16_bits(acc[2 * i]) | ((uint32_t)f32_to_bf16_bits(acc[2 * i + 1]) << 16);
    *reinterpret_cast<uint4*>(out + (size_t)t * H + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

static dim3 combine_grid(int64_t T, int64_t H) {
  const int64_t per = (H / 8 + kCombineThreads - 1) / kCombineThreads;
  return dim3((unsigned)T, (unsigned)std::min<int64_t>(per, 64));
}

int direct_combine_rows(const uint16_t* rows, const uint32_t* row_of_slot, const uint32_t* expert_ids,
                        const float* scores, int64_t T, int top_k, int64_t H, int64_t E, const uint16_t* shared,
                        uint16_t* out, uint32_t* status, cudaStream_t st) {
  launch_programmatic(direct_combine_kernel, combine_grid(T, H), dim3(kCombineThreads), 0, st, rows, row_of_slot,
                      expert_ids, scores, top_k, (int)H, (uint32_t)E, status, shared, out);
  return check_launch("direct_combine_kernel");
}

}  // namespace glm53

using namespace glm53;

extern "C" int glm53_direct_combine(const void* rows, const uint32_t* expert_ids, const float* scores, int64_t T,
                                    int top_k, int64_t H, const void* shared, void* out, void* stream) {
  if (T < 0 || top_k <= 0 || top_k > kCombineMaxK || H <= 0 || H % 8 != 0 || H > INT32_MAX / 2 ||
      (T > 0 && (!rows || !expert_ids || !scores || !out)) ||
      (((uintptr_t)rows | (uintptr_t)out | (uintptr_t)shared) & 15) != 0) {
    set_last_error("glm53_direct_combine: invalid arguments T=%lld top_k=%d H=%lld", (long long)T, top_k,
                   (long long)H);
    return GLM53_ERR_INVALID;
  }
  if (T == 0) return GLM53_OK;
  return direct_combine_rows((const uint16_t*)rows, nullptr, expert_ids, scores, T, top_k, H, 0xFFFFFFFFll,
                             (const uint16_t*)shared, (uint16_t*)out, nullptr, (cudaStream_t)stream);
}
