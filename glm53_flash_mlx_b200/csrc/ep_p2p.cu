// Expert-parallel decode over peer memory (NVLink): the transport that
// replaces the two all-to-alls with stores into the peers' buffers.
//
// Every rank allocates one buffer of layout ep_layout(world, capacity, H)
// (glm53_ep_buffer_alloc) and maps every peer's through CUDA IPC
// (glm53_ep_ipc_open); a device array of the world buffer bases is passed to
// the kernels.  One decode step:
//   glm53_ep_dispatch_p2p  plan the slots (route order per destination), then
//                          one CTA per destination slot stores the token row
//                          and the local expert id into the owner's recv_x /
//                          recv_e at slot (rank, s) and counts one arrival on
//                          the owner (system-scope fence, then atomic add);
//   glm53_ep_owner_decode_p2p  gate/up waits until all world * capacity
//                          arrivals of this step are in, then the per-route
//                          decode; down stores each BF16 row into the home
//                          rank's back buffer and counts one arrival per CTA
//                          of a routed row (empty slots count nothing);
//   glm53_ep_combine_p2p   waits until the rows of every route it sent are
//                          in, reduces in slot order, adds the shared rows,
//                          and advances the step counter.
// Buffers are single: a rank only writes step n + 1 into a peer after its own
// combine of step n, which waited for that peer's down stage of step n, which
// ran after the peer's gate/up finished reading its slots.  Every wait is
// bounded (two seconds unless glm53_set_wait_limit_ns says otherwise) and
// reports GLM53_STATUS_WAIT_TIMEOUT.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "kernels.cuh"

namespace glm53 {

constexpr uint32_t kP2pEmpty = 0xFFFFFFFFu;
constexpr int kP2pMaxWorld = 32;

// One CTA per destination slot k = (d, s).  Warp 0 finds the slot's route:
// the s-th route, in route order, whose expert lives on rank d.  The CTA
// stores the token row and the local expert id (or the empty mark) into rank
// d's buffer at slot (rank, s), records the slot's score, and counts one
// arrival on rank d.  CTA 0 also writes every route's slot position (or the
// empty mark when its destination is full or its expert id is out of range).
__global__ void p2p_dispatch_kernel(const uint16_t* __restrict__ x, int H, int top_k,
                                    const uint32_t* __restrict__ ids, const float* __restrict__ scores, int R, int E,
                                    int world, int rank, int cap, const unsigned long long* __restrict__ peer_base,
                                    EpLayout lay, float* __restrict__ slot_scores, uint32_t* __restrict__ route_pos,
                                    uint32_t* __restrict__ status) {
  __shared__ uint32_t s_route;
  const int k = blockIdx.x, d = k / cap, s = k - d * cap;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int per_rank = E / world;
  char* base = reinterpret_cast<char*>(peer_base[d]);
  const size_t slot = (size_t)rank * cap + s;
  // One token (T = 1): every slot carries row 0 whatever the routes, so it
  // is stored before the routes are known, while the router still runs (an
  // empty slot's row is never read).  x is final here: this grid launches
  // only once the router has passed its own wait for the kernel that wrote
  // x; and the owner finished reading this slot in the previous step, which
  // this rank's previous combine waited for.
  const bool row_first = R == top_k;
  if (row_first) {
    const uint4* src = reinterpret_cast<const uint4*>(x);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(base + lay.recv_x) + slot * H);
    for (int i = threadIdx.x; i < (H >> 3); i += blockDim.x) dst[i] = src[i];
  }
  // launched as a programmatic dependent of the router: the owner decode may
  // launch at once (its routed CTAs wait for the arrivals, its shared-expert
  // CTAs for this grid), and the routes are read after the router finished
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (warp == 0) {
    uint32_t found = kP2pEmpty, seen = 0;
    for (int c0 = 0; c0 < R && found == kP2pEmpty; c0 += 32) {
      const int r = c0 + lane;
      const uint32_t e = r < R ? ids[r] : kP2pEmpty;
      const bool mine = r < R && e < (uint32_t)E && (int)(e / (uint32_t)per_rank) == d;
      const uint32_t m = __ballot_sync(0xffffffffu, mine);
      if ((uint32_t)s < seen + __popc(m)) {
        const uint32_t pre = __popc(m & ((1u << lane) - 1u));
        const uint32_t hit = __ballot_sync(0xffffffffu, mine && pre == (uint32_t)s - seen);
        found = (uint32_t)(c0 + __ffs(hit) - 1);
      }
      seen += __popc(m);
    }
    if (lane == 0) s_route = found;
  }
  if (k == 0) {
    for (int r = threadIdx.x; r < R; r += blockDim.x) {
      const uint32_t e = ids[r];
      uint32_t pos = kP2pEmpty;
      if (e >= (uint32_t)E) {
        atomicOr(status, kStatusBadExpert);
      } else {
        const int dd = (int)(e / (uint32_t)per_rank);
        uint32_t rank_in_d = 0;
        for (int r2 = 0; r2 < r; ++r2) {
          const uint32_t e2 = ids[r2];
          rank_in_d += (e2 < (uint32_t)E && (int)(e2 / (uint32_t)per_rank) == dd) ? 1u : 0u;
        }
        if (rank_in_d < (uint32_t)cap) {
          pos = (uint32_t)dd * cap + rank_in_d;
        } else {
          atomicOr(status, kStatusBadGeometry);  // capacity exceeded: the route is dropped
        }
      }
      route_pos[r] = pos;
    }
  }
  __syncthreads();
  const uint32_t r = s_route;
  if (threadIdx.x == 0) {
    slot_scores[k] = r == kP2pEmpty ? 0.f : scores[r];
    reinterpret_cast<uint32_t*>(base + lay.recv_e)[slot] = r == kP2pEmpty ? kP2pEmpty : ids[r] - (uint32_t)(d * per_rank);
  }
  if (r != kP2pEmpty && !row_first) {
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(r / top_k) * H);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(base + lay.recv_x) + slot * H);
    for (int i = threadIdx.x; i < (H >> 3); i += blockDim.x) dst[i] = src[i];
  }
  // release: the block barrier orders every thread's stores before thread 0's
  // system-scope fence (cumulative), which orders them before the arrival
  // (one fence per CTA; a fence in every thread cost more)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    atomicAdd(reinterpret_cast<unsigned long long*>(base + lay.cnt_dispatch), 1ull);
  }
}

// Combine after waiting for every owner's rows of this step: each routed
// slot this rank sent comes back as cta_per_row arrivals (the owners' down
// CTAs of that row), so this step expects cta_per_row x (sent routes) more
// than the running total kept in the buffer.
__global__ void p2p_combine_kernel(const char* __restrict__ buf, EpLayout lay, const float* __restrict__ slot_scores,
                                   const uint32_t* __restrict__ route_pos, int64_t T, int top_k, int64_t H,
                                   const uint16_t* __restrict__ shared, uint16_t* __restrict__ out,
                                   unsigned long long cta_per_row, uint32_t* status,
                                   unsigned long long wait_ns) {
  __shared__ unsigned long long s_step;
  // launched as a programmatic dependent of the owner's down stage: the home
  // tokens' shared rows come from that grid
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) {
    unsigned long long sent = 0;
    for (int64_t r = 0; r < T * top_k; ++r) sent += route_pos[r] != kP2pEmpty ? 1ull : 0ull;
    s_step = sent * cta_per_row;
    const unsigned long long before = *reinterpret_cast<const unsigned long long*>(buf + lay.expected);
    wait_counter_geq(reinterpret_cast<const unsigned long long*>(buf + lay.cnt_back), before + s_step, status,
                     wait_ns);
  }
  __syncthreads();
  const uint16_t* rows = reinterpret_cast<const uint16_t*>(buf + lay.back);
  const int64_t chunks = H / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < T * chunks; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / chunks, c = i % chunks;
    float total[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) total[q] = 0.f;
    for (int j = 0; j < top_k; ++j) {
      const uint32_t pos = route_pos[t * top_k + j];
      if (pos == kP2pEmpty) continue;
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
  // the last CTA to finish advances the step counter (every CTA has read it)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    char* b = const_cast<char*>(buf);
    unsigned int* done = reinterpret_cast<unsigned int*>(b + lay.done);
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *reinterpret_cast<unsigned long long*>(b + lay.expected) += s_step;
      *reinterpret_cast<unsigned long long*>(b + lay.epoch) += 1ull;
      *done = 0u;
      __threadfence();
    }
  }
}

// 256-thread launch with programmatic stream serialisation: the kernel may
// start before the previous kernel on the stream has finished and orders
// itself with griddepcontrol.wait.
template <typename... KArgs, typename... Args>
static void launch_pdl(void (*kernel)(KArgs...), dim3 grid, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

static bool p2p_geometry(int world, int rank, int64_t cap, int64_t H) {
  return world >= 1 && world <= kP2pMaxWorld && rank >= 0 && rank < world && cap > 0 && H > 0 && H % 64 == 0 &&
         (int64_t)world * cap <= (1 << 20);
}

}  // namespace glm53

using namespace glm53;

extern "C" size_t glm53_ep_shared_bytes(int world, int64_t capacity, int64_t H) {
  if (!p2p_geometry(world, 0, capacity, H)) return 0;
  return ep_layout(world, (int)capacity, H).bytes;
}

extern "C" int glm53_ep_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes == 0) {
    set_last_error("glm53_ep_buffer_alloc: invalid arguments");
    return GLM53_ERR_INVALID;
  }
  void* p = nullptr;
  cudaError_t err = cudaMalloc(&p, bytes);
  if (err == cudaSuccess) err = cudaMemset(p, 0, bytes);
  if (err == cudaSuccess) err = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
  if (err != cudaSuccess) {
    if (p) cudaFree(p);
    set_last_error("glm53_ep_buffer_alloc: %s", cudaGetErrorString(err));
    return GLM53_ERR_CUDA;
  }
  *ptr = p;
  return GLM53_OK;
}

extern "C" int glm53_ep_buffer_free(void* ptr) {
  const cudaError_t err = cudaFree(ptr);
  if (err != cudaSuccess) {
    set_last_error("glm53_ep_buffer_free: %s", cudaGetErrorString(err));
    return GLM53_ERR_CUDA;
  }
  return GLM53_OK;
}

extern "C" int glm53_ep_ipc_open(const void* ipc_handle, void** ptr) {
  if (!ipc_handle || !ptr) {
    set_last_error("glm53_ep_ipc_open: invalid arguments");
    return GLM53_ERR_INVALID;
  }
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  const cudaError_t err = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) {
    set_last_error("glm53_ep_ipc_open: %s", cudaGetErrorString(err));
    return GLM53_ERR_CUDA;
  }
  return GLM53_OK;
}

extern "C" int glm53_ep_ipc_close(void* ptr) {
  const cudaError_t err = cudaIpcCloseMemHandle(ptr);
  if (err != cudaSuccess) {
    set_last_error("glm53_ep_ipc_close: %s", cudaGetErrorString(err));
    return GLM53_ERR_CUDA;
  }
  return GLM53_OK;
}

extern "C" int glm53_ep_dispatch_p2p(const void* x, int64_t T, int64_t H, const uint32_t* expert_ids,
                                     const float* scores, int top_k, int64_t E, int world, int rank,
                                     int64_t capacity, const unsigned long long* peer_base, uint32_t* slot_route,
                                     float* slot_scores, uint32_t* route_pos, uint32_t* status, void* stream) {
  const char* fn = "glm53_ep_dispatch_p2p";
  if (!p2p_geometry(world, rank, capacity, H) || T < 0 || top_k <= 0 || E <= 0 || E % world != 0 ||
      T * top_k > INT32_MAX) {
    set_last_error("%s: invalid geometry", fn);
    return GLM53_ERR_INVALID;
  }
  if (!x || !expert_ids || !scores || !peer_base || !slot_route || !slot_scores || !route_pos || !status ||
      (((uintptr_t)x) & 15) != 0) {
    set_last_error("%s: missing pointer or unaligned rows", fn);
    return GLM53_ERR_INVALID;
  }
  (void)slot_route;
  cudaStream_t st = (cudaStream_t)stream;
  const EpLayout lay = ep_layout(world, (int)capacity, H);
  launch_pdl(p2p_dispatch_kernel, dim3((unsigned)(world * capacity)), st, (const uint16_t*)x, (int)H, top_k,
             expert_ids, scores, (int)(T * top_k), (int)E, world, rank, (int)capacity, peer_base, lay, slot_scores,
             route_pos, status);
  return check_launch("p2p_dispatch_kernel");
}

extern "C" int glm53_ep_combine_p2p(void* buffer, const uint32_t* route_pos, const float* slot_scores, int64_t T,
                                    int top_k, int64_t H, int world, int64_t capacity, const void* shared, void* out,
                                    uint32_t* status, void* stream) {
  const char* fn = "glm53_ep_combine_p2p";
  if (!p2p_geometry(world, 0, capacity, H) || T < 0 || top_k <= 0 || !buffer || !route_pos || !slot_scores ||
      !out || !status || ((((uintptr_t)out) | ((uintptr_t)shared)) & 15) != 0) {
    set_last_error("%s: invalid arguments", fn);
    return GLM53_ERR_INVALID;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const EpLayout lay = ep_layout(world, (int)capacity, H);
  // an owner's down stage counts one arrival per CTA of a routed row: H / 64
  const unsigned long long cta_per_row = (unsigned long long)(H / 64);
  const int64_t n = std::max<int64_t>(T * (H / 8), 1);
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 1024);
  launch_pdl(p2p_combine_kernel, dim3((unsigned)blocks), st, (const char*)buffer, lay, slot_scores, route_pos, T,
             top_k, H, (const uint16_t*)shared, (uint16_t*)out, cta_per_row, status, ep_wait_limit_ns());
  return check_launch("p2p_combine_kernel");
}
