// Device route plan (G6): stable expert sort and tile descriptors.
//
// Replaces build_route_plan / build_grouped_tile_plan
// (glm53_flash_mlx/grouped_fp8.py:157-203) and the native route plan kernels
// (native_execution/native_indexer_plan.metal:1880-1982):
//   histogram (+ count of ids >= E), exclusive prefix, stable scatter by route
//   index, fixed-capacity descriptors with the (0, R, 0) sentinel.
// One 1024-thread block; routes are scattered 1024 at a time.  Within a chunk
// a route's rank among equal experts is (earlier warps' counts) + (earlier
// lanes in its warp, from __match_any_sync), so the order is stable.
#include "common.cuh"
#include "kernels.cuh"

namespace glm53 {

constexpr int kPlanThreads = 1024;
constexpr int kPlanWarps = kPlanThreads / 32;
constexpr int kPlanMaxE = 1024;

__global__ void __launch_bounds__(kPlanThreads) route_plan_kernel(
    const uint32_t* __restrict__ ids, int R, int E, int tile_rows, const float* __restrict__ scores,
    uint32_t* __restrict__ order, uint32_t* __restrict__ inverse, uint32_t* __restrict__ sorted_experts,
    float* __restrict__ sorted_scores, uint32_t* __restrict__ route_offsets,
    uint32_t* __restrict__ tile_experts, uint32_t* __restrict__ tile_starts,
    uint32_t* __restrict__ tile_lengths, uint32_t* __restrict__ tile_offsets,
    uint32_t* __restrict__ descriptor_count, uint32_t* __restrict__ invalid_count, int capacity) {
  extern __shared__ uint32_t sm[];
  uint32_t* cursor = sm;                      // [E+1]  (E = bucket of invalid ids)
  uint32_t* toff = cursor + (E + 1);          // [E+1]
  uint32_t* roff = toff + (E + 1);            // [E+1]
  uint32_t* wcount = roff + (E + 1);          // [kPlanWarps][E+1]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int B = E + 1;
  for (int i = tid; i < B; i += kPlanThreads) cursor[i] = 0;
  for (int i = tid; i < kPlanWarps * B; i += kPlanThreads) wcount[i] = 0;
  // launched as a programmatic dependent of the kernel that writes the ids:
  // nothing global is read or written before this
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __syncthreads();
  // 1. histogram (eight loads in flight per thread: the ids come from L2/HBM)
  for (int r0 = tid; r0 < R; r0 += 8 * kPlanThreads) {
    uint32_t ev[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int r = r0 + u * kPlanThreads;
      ev[u] = r < R ? __ldg(ids + r) : 0xffffffffu;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (r0 + u * kPlanThreads < R) atomicAdd(&cursor[ev[u] < (uint32_t)E ? ev[u] : (uint32_t)E], 1u);
  }
  __syncthreads();
  // 2. exclusive prefix of route counts and tile counts (warp 0)
  if (warp == 0) {
    uint32_t run_r = 0, run_t = 0;
    for (int base = 0; base < B; base += 32) {
      int e = base + lane;
      uint32_t c = (e < B) ? cursor[e] : 0u;
      uint32_t tc = (e < E) ? (c + tile_rows - 1) / tile_rows : 0u;
      uint32_t ic = c, it = tc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        uint32_t v = __shfl_up_sync(0xffffffffu, ic, o);
        uint32_t w = __shfl_up_sync(0xffffffffu, it, o);
        if (lane >= o) { ic += v; it += w; }
      }
      if (e < B) {
        roff[e] = run_r + ic - c;
        toff[e] = run_t + it - tc;
      }
      run_r += __shfl_sync(0xffffffffu, ic, 31);
      run_t += __shfl_sync(0xffffffffu, it, 31);
    }
    if (lane == 0) {
      // roff[E] = number of valid routes; toff[E] = number of valid tiles
      *invalid_count = cursor[E];
      *descriptor_count = toff[E];
    }
  }
  __syncthreads();
  for (int i = tid; i < B; i += kPlanThreads) {
    route_offsets[i] = roff[i];
    if (i <= E) tile_offsets[i] = toff[i];
    cursor[i] = roff[i];
  }
  __syncthreads();
  // 3. stable scatter, 1024 routes per step (the next step's id and score
  // are loaded while this one is placed)
  uint32_t next_e = tid < R ? __ldg(ids + tid) : 0u;
  float next_s = (tid < R && scores && sorted_scores) ? __ldg(scores + tid) : 0.f;
  for (int base = 0; base < R; base += kPlanThreads) {
    const int r = base + tid;
    const bool live = r < R;
    const uint32_t e_r = next_e;
    const float s_r = next_s;
    if (r + kPlanThreads < R) {
      next_e = __ldg(ids + r + kPlanThreads);
      if (scores && sorted_scores) next_s = __ldg(scores + r + kPlanThreads);
    }
    uint32_t key = 0xffffffffu;
    if (live) key = e_r < (uint32_t)E ? e_r : (uint32_t)E;
    const uint32_t peers = __match_any_sync(0xffffffffu, key);
    const uint32_t rank = __popc(peers & ((1u << lane) - 1u));
    if (live && rank == 0) wcount[warp * B + key] = __popc(peers);
    __syncthreads();
    if (live) {
      uint32_t before = 0;
      for (int w = 0; w < warp; ++w) before += wcount[w * B + key];
      const uint32_t pos = cursor[key] + before + rank;
      order[pos] = (uint32_t)r;
      inverse[r] = pos;
      sorted_experts[pos] = e_r;
      if (scores && sorted_scores) sorted_scores[pos] = s_r;
    }
    __syncthreads();
    for (int k = tid; k < B; k += kPlanThreads) {
      uint32_t add = 0;
      for (int w = 0; w < kPlanWarps; ++w) {
        add += wcount[w * B + k];
        wcount[w * B + k] = 0;
      }
      cursor[k] += add;
    }
    __syncthreads();
  }
  // 4. descriptors: owner = expert e with toff[e] <= d < toff[e+1]
  const uint32_t valid_tiles = toff[E];
  for (int d = tid; d < capacity; d += kPlanThreads) {
    if ((uint32_t)d < valid_tiles) {
      int lo = 0, hi = E - 1;  // largest e with toff[e] <= d
      while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (toff[mid] <= (uint32_t)d) lo = mid; else hi = mid - 1;
      }
      const uint32_t start = roff[lo] + ((uint32_t)d - toff[lo]) * (uint32_t)tile_rows;
      const uint32_t remaining = roff[lo + 1] - start;
      tile_experts[d] = (uint32_t)lo;
      tile_starts[d] = start;
      tile_lengths[d] = remaining < (uint32_t)tile_rows ? remaining : (uint32_t)tile_rows;
    } else {
      tile_experts[d] = 0u;
      tile_starts[d] = (uint32_t)R;
      tile_lengths[d] = 0u;
    }
  }
}

int route_plan(const uint32_t* ids, int64_t R, int64_t E, int64_t tile_rows, const float* scores,
               uint32_t* order, uint32_t* inverse, uint32_t* sorted_experts, float* sorted_scores,
               uint32_t* route_offsets, uint32_t* tile_experts, uint32_t* tile_starts,
               uint32_t* tile_lengths, uint32_t* tile_offsets, uint32_t* descriptor_count,
               uint32_t* invalid_count, cudaStream_t stream) {
  if (R < 0 || R > (1ll << 30) || E <= 0 || E > kPlanMaxE || tile_rows <= 0 || tile_rows > 4096) {
    set_last_error("route_plan: unsupported geometry R=%lld E=%lld tile_rows=%lld", (long long)R,
                   (long long)E, (long long)tile_rows);
    return GLM53_ERR_INVALID;
  }
  const int64_t capacity = (R + tile_rows - 1) / tile_rows + E;
  const size_t smem = (size_t)(3 + kPlanWarps) * (E + 1) * sizeof(uint32_t);
  if (smem > 48 * 1024) {
    int rc_attr = ensure_max_smem((const void*)route_plan_kernel, smem);
    if (rc_attr) return rc_attr;
  }
  launch_programmatic(route_plan_kernel, dim3(1), dim3(kPlanThreads), smem, stream, ids, (int)R, (int)E,
                      (int)tile_rows, scores, order, inverse, sorted_experts, sorted_scores, route_offsets,
                      tile_experts, tile_starts, tile_lengths, tile_offsets, descriptor_count, invalid_count,
                      (int)capacity);
  return check_launch("route_plan_kernel");
}

// ---------------------------------------------------------------------------
// Chunked plan for long route lists (the grouped prefill: 16,384 routes at
// T = 2048): the single block above scatters 1024 routes per step with three
// block barriers each, 16 steps at T = 2048 and 64 at T = 8192.  Here every
// chunk of kPlanChunk routes is counted and scattered by a block of its own:
//   plan_count_kernel    per-chunk expert histograms;
//   plan_offsets_kernel  (one block) exclusive prefixes over experts, each
//                        chunk's starting position per expert (earlier
//                        chunks first), and the descriptors;
//   plan_scatter_kernel  each chunk places its routes from its own starting
//                        positions, in route order within the chunk (the
//                        same rank rule as above).
// The order, inverse, sorted ids and scores and descriptors are identical to
// the single-block kernel's: a stable sort by expert, ties in route order.
// ---------------------------------------------------------------------------

constexpr int kPlanChunk = 2048;

__global__ void __launch_bounds__(kPlanThreads) plan_count_kernel(const uint32_t* __restrict__ ids, int R, int E,
                                                                  uint32_t* __restrict__ counts) {
  extern __shared__ uint32_t hist[];  // [E+1]
  const int B = E + 1, tid = threadIdx.x;
  for (int i = tid; i < B; i += kPlanThreads) hist[i] = 0;
  __syncthreads();
  const int r0 = blockIdx.x * kPlanChunk;
#pragma unroll
  for (int u = 0; u < kPlanChunk / kPlanThreads; ++u) {
    const int r = r0 + u * kPlanThreads + tid;
    if (r < R) {
      const uint32_t e = __ldg(ids + r);
      atomicAdd(&hist[e < (uint32_t)E ? e : (uint32_t)E], 1u);
    }
  }
  __syncthreads();
  for (int i = tid; i < B; i += kPlanThreads) counts[(size_t)blockIdx.x * B + i] = hist[i];
}

__global__ void __launch_bounds__(kPlanThreads) plan_offsets_kernel(
    const uint32_t* __restrict__ counts, int chunks, int R, int E, int tile_rows, uint32_t* __restrict__ chunk_start,
    uint32_t* __restrict__ route_offsets, uint32_t* __restrict__ tile_experts, uint32_t* __restrict__ tile_starts,
    uint32_t* __restrict__ tile_lengths, uint32_t* __restrict__ tile_offsets, uint32_t* __restrict__ descriptor_count,
    uint32_t* __restrict__ invalid_count, int capacity) {
  extern __shared__ uint32_t sm[];
  uint32_t* total = sm;           // [E+1]
  uint32_t* roff = total + E + 1;  // [E+1]
  uint32_t* toff = roff + E + 1;   // [E+1]
  const int B = E + 1, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < B; e += kPlanThreads) {
    uint32_t t = 0;
    for (int b = 0; b < chunks; ++b) t += counts[(size_t)b * B + e];
    total[e] = t;
  }
  __syncthreads();
  if (warp == 0) {
    uint32_t run_r = 0, run_t = 0;
    for (int base = 0; base < B; base += 32) {
      const int e = base + lane;
      const uint32_t c = (e < B) ? total[e] : 0u;
      const uint32_t tc = (e < E) ? (c + tile_rows - 1) / tile_rows : 0u;
      uint32_t ic = c, it = tc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, ic, o);
        const uint32_t w = __shfl_up_sync(0xffffffffu, it, o);
        if (lane >= o) {
          ic += v;
          it += w;
        }
      }
      if (e < B) {
        roff[e] = run_r + ic - c;
        toff[e] = run_t + it - tc;
      }
      run_r += __shfl_sync(0xffffffffu, ic, 31);
      run_t += __shfl_sync(0xffffffffu, it, 31);
    }
    if (lane == 0) {
      *invalid_count = total[E];
      *descriptor_count = toff[E];
    }
  }
  __syncthreads();
  for (int e = tid; e < B; e += kPlanThreads) {
    route_offsets[e] = roff[e];
    tile_offsets[e] = toff[e];
    uint32_t run = roff[e];
    for (int b = 0; b < chunks; ++b) {
      chunk_start[(size_t)b * B + e] = run;
      run += counts[(size_t)b * B + e];
    }
  }
  const uint32_t valid_tiles = toff[E];
  for (int d = tid; d < capacity; d += kPlanThreads) {
    if ((uint32_t)d < valid_tiles) {
      int lo = 0, hi = E - 1;  // largest e with toff[e] <= d
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (toff[mid] <= (uint32_t)d) lo = mid; else hi = mid - 1;
      }
      const uint32_t start = roff[lo] + ((uint32_t)d - toff[lo]) * (uint32_t)tile_rows;
      const uint32_t remaining = roff[lo + 1] - start;
      tile_experts[d] = (uint32_t)lo;
      tile_starts[d] = start;
      tile_lengths[d] = remaining < (uint32_t)tile_rows ? remaining : (uint32_t)tile_rows;
    } else {
      tile_experts[d] = 0u;
      tile_starts[d] = (uint32_t)R;
      tile_lengths[d] = 0u;
    }
  }
}

__global__ void __launch_bounds__(kPlanThreads) plan_scatter_kernel(
    const uint32_t* __restrict__ ids, int R, int E, const float* __restrict__ scores,
    const uint32_t* __restrict__ chunk_start, uint32_t* __restrict__ order, uint32_t* __restrict__ inverse,
    uint32_t* __restrict__ sorted_experts, float* __restrict__ sorted_scores) {
  extern __shared__ uint32_t sm[];
  const int B = E + 1, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t* cursor = sm;          // [E+1]
  uint32_t* wcount = cursor + B;  // [kPlanWarps][E+1]
  for (int i = tid; i < B; i += kPlanThreads) cursor[i] = chunk_start[(size_t)blockIdx.x * B + i];
  for (int i = tid; i < kPlanWarps * B; i += kPlanThreads) wcount[i] = 0;
  __syncthreads();
  const int r0 = blockIdx.x * kPlanChunk;
  for (int u = 0; u < kPlanChunk / kPlanThreads; ++u) {
    const int r = r0 + u * kPlanThreads + tid;
    const bool live = r < R;
    uint32_t e_r = 0, key = 0xffffffffu;
    float s_r = 0.f;
    if (live) {
      e_r = __ldg(ids + r);
      if (scores && sorted_scores) s_r = __ldg(scores + r);
      key = e_r < (uint32_t)E ? e_r : (uint32_t)E;
    }
    const uint32_t peers = __match_any_sync(0xffffffffu, key);
    const uint32_t rank = __popc(peers & ((1u << lane) - 1u));
    if (live && rank == 0) wcount[warp * B + key] = __popc(peers);
    __syncthreads();
    if (live) {
      uint32_t before = 0;
      for (int w = 0; w < warp; ++w) before += wcount[w * B + key];
      const uint32_t pos = cursor[key] + before + rank;
      order[pos] = (uint32_t)r;
      inverse[r] = pos;
      sorted_experts[pos] = e_r;
      if (scores && sorted_scores) sorted_scores[pos] = s_r;
    }
    __syncthreads();
    for (int k = tid; k < B; k += kPlanThreads) {
      uint32_t add = 0;
      for (int w = 0; w < kPlanWarps; ++w) {
        add += wcount[w * B + k];
        wcount[w * B + k] = 0;
      }
      cursor[k] += add;
    }
    __syncthreads();
  }
}

size_t route_plan_scratch_bytes(int64_t R, int64_t E) {
  const int64_t chunks = (R + kPlanChunk - 1) / kPlanChunk;
  return (size_t)2 * chunks * (E + 1) * sizeof(uint32_t);
}

int route_plan_chunked(const uint32_t* ids, int64_t R, int64_t E, int64_t tile_rows, const float* scores,
                       uint32_t* order, uint32_t* inverse, uint32_t* sorted_experts, float* sorted_scores,
                       uint32_t* route_offsets, uint32_t* tile_experts, uint32_t* tile_starts, uint32_t* tile_lengths,
                       uint32_t* tile_offsets, uint32_t* descriptor_count, uint32_t* invalid_count, uint32_t* scratch,
                       cudaStream_t stream) {
  if (!scratch || R <= 2 * kPlanChunk)
    return route_plan(ids, R, E, tile_rows, scores, order, inverse, sorted_experts, sorted_scores, route_offsets,
                      tile_experts, tile_starts, tile_lengths, tile_offsets, descriptor_count, invalid_count, stream);
  if (R > (1ll << 30) || E <= 0 || E > kPlanMaxE || tile_rows <= 0 || tile_rows > 4096) {
    set_last_error("route_plan: unsupported geometry R=%lld E=%lld tile_rows=%lld", (long long)R,
                   (long long)E, (long long)tile_rows);
    return GLM53_ERR_INVALID;
  }
  const int chunks = (int)((R + kPlanChunk - 1) / kPlanChunk);
  const int64_t capacity = (R + tile_rows - 1) / tile_rows + E;
  uint32_t* counts = scratch;
  uint32_t* chunk_start = scratch + (size_t)chunks * (E + 1);
  const size_t smem_count = (size_t)(E + 1) * sizeof(uint32_t);
  const size_t smem_off = 3 * smem_count;
  const size_t smem_scatter = (size_t)(1 + kPlanWarps) * smem_count;
  if (smem_scatter > 48 * 1024) {
    const int rc_attr = ensure_max_smem((const void*)plan_scatter_kernel, smem_scatter);
    if (rc_attr) return rc_attr;
  }
  plan_count_kernel<<<chunks, kPlanThreads, smem_count, stream>>>(ids, (int)R, (int)E, counts);
  int rc = check_launch("plan_count_kernel");
  if (rc) return rc;
  plan_offsets_kernel<<<1, kPlanThreads, smem_off, stream>>>(counts, chunks, (int)R, (int)E, (int)tile_rows,
                                                             chunk_start, route_offsets, tile_experts, tile_starts,
                                                             tile_lengths, tile_offsets, descriptor_count,
                                                             invalid_count, (int)capacity);
  rc = check_launch("plan_offsets_kernel");
  if (rc) return rc;
  plan_scatter_kernel<<<chunks, kPlanThreads, smem_scatter, stream>>>(ids, (int)R, (int)E, scores, chunk_start, order,
                                                                      inverse, sorted_experts, sorted_scores);
  return check_launch("plan_scatter_kernel");
}

}  // namespace glm53

using namespace glm53;

extern "C" int glm53_route_plan(const uint32_t* expert_ids, int64_t R, int64_t E, int64_t tile_rows,
                                const float* scores, uint32_t* order, uint32_t* inverse,
                                uint32_t* sorted_experts, float* sorted_scores, uint32_t* route_offsets,
                                uint32_t* tile_experts, uint32_t* tile_starts, uint32_t* tile_lengths,
                                uint32_t* tile_offsets, uint32_t* descriptor_count, uint32_t* invalid_count,
                                void* stream) {
  if ((R > 0 && (!expert_ids || !order || !inverse || !sorted_experts)) || !route_offsets || !tile_experts ||
      !tile_starts || !tile_lengths || !tile_offsets || !descriptor_count || !invalid_count) {
    set_last_error("glm53_route_plan: missing pointer");
    return GLM53_ERR_INVALID;
  }
  return route_plan(expert_ids, R, E, tile_rows, scores, order, inverse, sorted_experts, sorted_scores,
                    route_offsets, tile_experts, tile_starts, tile_lengths, tile_offsets, descriptor_count,
                    invalid_count, (cudaStream_t)stream);
}
