// Coalesced decode of a small batch: every touched expert streams its
// weights once for all of the batch's routes to it.
//
// The expert side of the Direct module's multi-row path
// (glm53_flash_mlx/fp8.py:384-399: per touched expert, gate/up, SwiGLU and
// down over the rows routed to it), for up to a few hundred routes.  The
// routes are sorted by expert (route_plan, descriptors of up to kBdCols = 8
// routes, every N column of the MMA); a descriptor's routes ride in the N
// columns of the m16n8k16 GEMV tiles of gemv_tile.cuh (the single-token decode
// uses column 0 only), so each weight tile is loaded once per descriptor
// instead of once per route.  Every output column of an MMA is its own dot
// product, so a route's values are those of the per-route decode
// (glm53_routes_decode).
//   batched_gate_up_kernel: work item = (descriptor, 8 x WARPS hidden rows);
//     each warp 8 gate + 8 up rows over the whole K; BF16 SwiGLU per column;
//     hidden rows in sorted route order.
//   batched_down_kernel: work item = (descriptor, 16 x WARPS output rows);
//     each warp 16 rows over the whole K = I; BF16 down rows in sorted route
//     order.
// Both are persistent over the device-side descriptor count (no host sync),
// one 16-warp CTA per SM where the staged rows fit: the descriptor's route
// rows are staged once per SM and the warps run through the items of one
// descriptor without a barrier (only a new descriptor's staging waits for
// every warp).
#include <algorithm>

#include "common.cuh"
#include "gemv_tile.cuh"
#include "kernels.cuh"

namespace glm53 {

constexpr int kBdCols = 8;        // routes per descriptor (the MMA's N columns)
constexpr int kBdRing = 8;        // gate/up: K slices in flight per warp
constexpr int kBdRingDown = 12;   // down: its K streams are short
constexpr int kBdMaxRoutes = 4096;
constexpr size_t kBdSmemCta = 232448;  // opt-in shared memory of one CTA (sm_100)
constexpr size_t kBdSmemSm = 233472;   // shared memory of one SM

__host__ __device__ __forceinline__ int bd_align16(int v) { return (v + 15) & ~15; }

struct BatchedArgs {
  const uint16_t* x;  // [T, H] BF16 tokens
  int H, I, E, top_k;
  const uint32_t* order;  // sorted position -> route t * top_k + j
  const uint32_t* tile_experts;
  const uint32_t* tile_starts;
  const uint32_t* tile_lengths;
  const uint32_t* descriptor_count;
  const uint8_t* gu_w;
  const float* gu_s;
  const uint8_t* d_w;
  const float* d_s;
  // shared expert as expert id E (routes of weight 1.0), or null
  const uint8_t* sg_w;
  const float* sg_s;
  const uint8_t* su_w;
  const float* su_s;
  const uint8_t* sd_w;
  const float* sd_s;
  float limit;
  uint16_t* hidden;  // [R, I] sorted route order
  uint16_t* rows;    // [R, H] sorted route order, or route order through `scatter`
  const uint32_t* scatter;  // sorted position -> output row (null: sorted order)
  uint32_t* status;
};

// Stage `ncols` token rows (route order[c] reads token order[c] / top_k) into
// shared memory as FP16 * 2^-e; returns 2^e (stage_f16's rule, gathered).
__device__ __forceinline__ float stage_routes_f16(__half* xs, int stride, const uint16_t* x, const uint32_t* order,
                                                  int top_k, int ncols, int K, float* red) {
  const int n8 = K >> 3;
  float m = 0.f;
  for (int i = threadIdx.x; i < ncols * n8; i += blockDim.x) {
    const int c = i / n8, j = i - c * n8;
    const uint16_t* src = x + (size_t)(__ldg(order + c) / (uint32_t)top_k) * K + 8 * j;
    const uint4 v = *reinterpret_cast<const uint4*>(src);
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
  if (mx >= 16384.0f) {
    int ex;
    frexpf(mx, &ex);
    e = ex - 14;
  }
  const float down = ldexpf(1.0f, -e);
  for (int i = threadIdx.x; i < ncols * n8; i += blockDim.x) {
    const int c = i / n8, j = i - c * n8;
    const uint16_t* src = x + (size_t)(__ldg(order + c) / (uint32_t)top_k) * K + 8 * j;
    const uint4 v = *reinterpret_cast<const uint4*>(src);
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

template <int WARPS, bool FINITE>
__global__ void __launch_bounds__(32 * WARPS, 1) batched_gate_up_kernel(BatchedArgs a) {
  constexpr int P = kBdRing;
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  uint4* ring = reinterpret_cast<uint4*>(smem) + (size_t)warp * P * 64;
  __half* xs = reinterpret_cast<__half*>(reinterpret_cast<uint4*>(smem) + (size_t)WARPS * P * 64);
  const int stride = bd_align16(a.H + 8);
  float* red = reinterpret_cast<float*>(xs + (size_t)kBdCols * stride);
  const int groups = a.I / (8 * WARPS);
  // launched as a programmatic dependent of the route plan: wait for it, then
  // let the down stage launch (it reads only the plan before its own wait)
  pdl_wait();
  pdl_trigger();
  const int nwork = (int)__ldg(a.descriptor_count) * groups;
  const int cols = a.H >> 7, half = a.I >> 7;
  const int nslice = a.H >> 6;
  // a contiguous run of work items per CTA (consecutive items share their
  // descriptor, whose route rows are staged once), the runs balanced to
  // within one item
  const int w_begin = (int)((int64_t)blockIdx.x * nwork / gridDim.x);
  const int w_end = (int)((int64_t)(blockIdx.x + 1) * nwork / gridDim.x);
  int staged = -1;
  float staged_mul = 0.f;
  for (int w = w_begin; w < w_end; ++w) {
    const int d = w / groups, grp = w - d * groups;
    const uint32_t e = __ldg(a.tile_experts + d), start = __ldg(a.tile_starts + d);
    const int len = (int)min(__ldg(a.tile_lengths + d), (uint32_t)kBdCols);
    const bool shared = a.sg_w && e == (uint32_t)a.E;
    const bool valid = e < (uint32_t)a.E || shared;
    const uint32_t es = e < (uint32_t)a.E ? e : 0u;
    const int r0 = grp * 8 * WARPS + warp * 8;
    const uint8_t* gw = shared ? a.sg_w + (size_t)r0 * a.H : a.gu_w + ((size_t)es * 2 * a.I + r0) * a.H;
    const uint8_t* uw = shared ? a.su_w + (size_t)r0 * a.H : gw + (size_t)a.I * a.H;
    const float* gs = shared ? a.sg_s + (size_t)(r0 >> 7) * cols : a.gu_s + ((size_t)es * 2 * half + (r0 >> 7)) * cols;
    const float* us = shared ? a.su_s + (size_t)(r0 >> 7) * cols : gs + (size_t)half * cols;
    const uint8_t* pg = gw + (size_t)g * a.H + 16 * q;
    const uint8_t* pu = uw + (size_t)g * a.H + 16 * q;
    auto issue = [&](int sl) {
      uint4* dst = ring + (sl % P) * 64 + lane;
      cp_async_16_l2_256(dst, valid ? (const void*)(pg + 64 * sl) : (const void*)a.x, valid);
      cp_async_16_l2_256(dst + 32, valid ? (const void*)(pu + 64 * sl) : (const void*)a.x, valid);
    };
#pragma unroll
    for (int s = 0; s < P - 1; ++s) {
      if (s < nslice) issue(s);
      cp_async_commit_group();
    }
    WarpScales ssg, ssu;
    ssg.load(gs, cols, valid);
    ssu.load(us, cols, valid);
    if (d != staged) {
      if (staged >= 0) __syncthreads();  // every warp is done with the previous descriptor's rows
      staged_mul = stage_routes_f16(xs, stride, a.x, a.order + start, a.top_k, len, a.H, red);
      staged = d;
    }
    const float smul = decode_unscale<FINITE>() * staged_mul;
    float part[4] = {0.f, 0.f, 0.f, 0.f}, tot[4] = {0.f, 0.f, 0.f, 0.f};
    for (int sl = 0; sl < nslice; ++sl) {
      if (sl + P - 1 < nslice) issue(sl + P - 1);
      cp_async_commit_group();
      cp_async_wait_group<P - 1>();
      const uint4* src = ring + (sl % P) * 64 + lane;
      const uint4 fg = src[0], fu = src[32];
      uint32_t xw[8];
      load_x_frag(xw, xs + g * stride + 64 * sl + 16 * q, g < len);
      mma_slice<FINITE>(part, fg, fu, xw);
      if (sl & 1) promote2(tot, part, ssg.at(sl >> 1) * smul, ssu.at(sl >> 1) * smul);
    }
    cp_async_wait_group<0>();
    // lane (g, q) holds gate / up of hidden row r0 + g for columns 2q and 2q + 1
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int c = 2 * q + cc;
      if (c < len) a.hidden[(size_t)(start + c) * a.I + r0 + g] = valid ? swiglu_bf16(tot[cc], tot[2 + cc], a.limit)
                                                                         : (uint16_t)0;
    }
    if (!valid && threadIdx.x == 0) atomicOr(a.status, kStatusBadExpert);
  }
}

template <int WARPS, bool FINITE>
__global__ void __launch_bounds__(32 * WARPS) batched_down_kernel(BatchedArgs a) {
  constexpr int P = kBdRingDown;
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const int K = a.I;
  uint4* ring = reinterpret_cast<uint4*>(smem) + (size_t)warp * P * 64;
  __half* hs = reinterpret_cast<__half*>(reinterpret_cast<uint4*>(smem) + (size_t)WARPS * P * 64);
  const int stride = bd_align16(K + 8);
  float* red = reinterpret_cast<float*>(hs + (size_t)kBdCols * stride);
  const int groups = a.H / (16 * WARPS);
  // Launched as a programmatic dependent of the gate/up stage, which starts
  // it only after the route plan completed: the plan and the weights are read
  // before griddepcontrol.wait, the hidden rows after it.
  const int nwork = (int)__ldg(a.descriptor_count) * groups;
  const int cols = K >> 7;
  const int nslice = K >> 6;
  const int w_begin = (int)((int64_t)blockIdx.x * nwork / gridDim.x);  // balanced runs, as in gate/up
  const int w_end = (int)((int64_t)(blockIdx.x + 1) * nwork / gridDim.x);
  int staged = -1;
  float staged_mul = 0.f;
  for (int w = w_begin; w < w_end; ++w) {
    const int d = w / groups, grp = w - d * groups;
    const uint32_t e = __ldg(a.tile_experts + d), start = __ldg(a.tile_starts + d);
    const int len = (int)min(__ldg(a.tile_lengths + d), (uint32_t)kBdCols);
    const bool shared = a.sd_w && e == (uint32_t)a.E;
    const bool valid = e < (uint32_t)a.E || shared;
    const uint32_t es = e < (uint32_t)a.E ? e : 0u;
    const int row0 = grp * 16 * WARPS + warp * 16;
    const uint8_t* w0 = shared ? a.sd_w + (size_t)row0 * K : a.d_w + ((size_t)es * a.H + row0) * K;
    const float* srow = shared ? a.sd_s + (size_t)(row0 >> 7) * cols
                               : a.d_s + ((size_t)es * (a.H >> 7) + (row0 >> 7)) * cols;
    const uint8_t* p0 = w0 + (size_t)g * K + 16 * q;
    const uint8_t* p8 = p0 + (size_t)8 * K;
    auto issue = [&](int sl) {
      uint4* dst = ring + (sl % P) * 64 + lane;
      cp_async_16_l2_256(dst, valid ? (const void*)(p0 + 64 * sl) : (const void*)a.x, valid);
      cp_async_16_l2_256(dst + 32, valid ? (const void*)(p8 + 64 * sl) : (const void*)a.x, valid);
    };
#pragma unroll
    for (int s = 0; s < P - 1; ++s) {
      if (s < nslice) issue(s);
      cp_async_commit_group();
    }
    WarpScales sd;
    sd.load(srow, cols, valid);
    if (d != staged) {
      if (staged >= 0) {
        __syncthreads();  // every warp is done with the previous descriptor's rows
      } else {
        pdl_wait();  // the gate/up stage's hidden rows
        pdl_trigger();
      }
      staged_mul = stage_f16(hs, stride, a.hidden + (size_t)start * K, K, len, K, red);
      staged = d;
    }
    const float hmul = decode_unscale<FINITE>() * staged_mul;
    float part[4] = {0.f, 0.f, 0.f, 0.f}, tot[4] = {0.f, 0.f, 0.f, 0.f};
    for (int sl = 0; sl < nslice; ++sl) {
      if (sl + P - 1 < nslice) issue(sl + P - 1);
      cp_async_commit_group();
      cp_async_wait_group<P - 1>();
      const uint4* src = ring + (sl % P) * 64 + lane;
      const uint4 f0 = src[0], f8 = src[32];
      uint32_t xw[8];
      load_x_frag(xw, hs + g * stride + 64 * sl + 16 * q, g < len);
      mma_slice<FINITE>(part, f0, f8, xw);
      if (sl & 1) promote(tot, part, sd.at(sl >> 1) * hmul);
    }
    cp_async_wait_group<0>();
    // lane (g, q): rows row0 + g (tot[0..1]) and row0 + g + 8 (tot[2..3]), columns 2q, 2q + 1
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int c = 2 * q + cc;
      if (c < len) {
        const size_t out_row = a.scatter ? (size_t)__ldg(a.scatter + start + c) : (size_t)(start + c);
        uint16_t* dst = a.rows + out_row * a.H + row0;
        dst[g] = valid ? f32_to_bf16_bits(tot[cc]) : (uint16_t)0;
        dst[g + 8] = valid ? f32_to_bf16_bits(tot[2 + cc]) : (uint16_t)0;
      }
    }
    if (!valid && threadIdx.x == 0) atomicOr(a.status, kStatusBadExpert);
  }
}

// Workspace: route plan (order, inverse, sorted experts / scores, offsets,
// descriptors, counts) | hidden [R, I] | rows [R, H].
struct BatchedWorkspace {
  size_t order, inverse, sorted_experts, sorted_scores, route_offsets, tile_offsets, tile_experts, tile_starts,
      tile_lengths, counts, hidden, rows, bytes;
};

static BatchedWorkspace batched_workspace(int64_t R, int64_t E, int64_t H, int64_t I) {
  BatchedWorkspace w;
  const int64_t cap = (R + kBdCols - 1) / kBdCols + E;
  size_t off = 0;
  auto take = [&](size_t n) {
    const size_t o = off;
    off = align_up(off + n, 256);
    return o;
  };
  w.order = take(R * 4);
  w.inverse = take(R * 4);
  w.sorted_experts = take(R * 4);
  w.sorted_scores = take(R * 4);
  w.route_offsets = take((E + 1) * 4);
  w.tile_offsets = take((E + 1) * 4);
  w.tile_experts = take(cap * 4);
  w.tile_starts = take(cap * 4);
  w.tile_lengths = take(cap * 4);
  w.counts = take(2 * 4);
  w.hidden = take((size_t)R * I * 2);
  w.rows = take((size_t)R * H * 2);
  w.bytes = off;
  return w;
}

static size_t bd_smem(int warps, int ring, int K) {
  return (size_t)warps * ring * 64 * 16 + (size_t)kBdCols * bd_align16(K + 8) * 2 + 32 * sizeof(float);
}

// Warps per CTA: 16 where the rings and the staged rows fit one CTA and the
// rows split evenly (rows_per_warp x 16 divides `rows`), else 8, else 4;
// 0 when even 4 do not fit.
static int bd_warps(int ring, int K, int rows_per_warp, int rows) {
  for (int w : {16, 8, 4})
    if (bd_smem(w, ring, K) <= kBdSmemCta && rows % (rows_per_warp * w) == 0) return w;
  return 0;
}

template <int WARPS, bool FINITE>
static int launch_gate_up(const BatchedArgs& a, int64_t capacity, cudaStream_t st) {
  const size_t smem = bd_smem(WARPS, kBdRing, a.H);
  int rc = ensure_max_smem((const void*)batched_gate_up_kernel<WARPS, FINITE>, smem);
  if (rc) return rc;
  const int per_sm = std::max(1, std::min(64 / WARPS, (int)(kBdSmemSm / (smem + 1024))));
  const int64_t items = capacity * (a.I / (8 * WARPS));
  launch_programmatic(batched_gate_up_kernel<WARPS, FINITE>,
                      dim3((unsigned)std::min<int64_t>(items, (int64_t)per_sm * sm_count())), dim3(32 * WARPS), smem,
                      st, a);
  return check_launch("batched_gate_up_kernel");
}

template <int WARPS, bool FINITE>
static int launch_down(const BatchedArgs& a, int64_t capacity, cudaStream_t st) {
  const size_t smem = bd_smem(WARPS, kBdRingDown, a.I);
  int rc = ensure_max_smem((const void*)batched_down_kernel<WARPS, FINITE>, smem);
  if (rc) return rc;
  const int per_sm = std::max(1, std::min(64 / WARPS, (int)(kBdSmemSm / (smem + 1024))));
  const int64_t items = capacity * (a.H / (16 * WARPS));
  launch_programmatic(batched_down_kernel<WARPS, FINITE>,
                      dim3((unsigned)std::min<int64_t>(items, (int64_t)per_sm * sm_count())), dim3(32 * WARPS), smem,
                      st, a);
  return check_launch("batched_down_kernel");
}

template <bool FINITE>
static int launch_batched(const BatchedArgs& a, int64_t capacity, cudaStream_t st) {
  const int wg = bd_warps(kBdRing, a.H, 8, a.I), wd = bd_warps(kBdRingDown, a.I, 16, a.H);
  if (!wg || !wd) {
    set_last_error("batched decode: H=%d / I=%d rows do not fit one CTA's shared memory", a.H, a.I);
    return GLM53_ERR_INVALID;
  }
  int rc = wg == 16 ? launch_gate_up<16, FINITE>(a, capacity, st)
           : wg == 8 ? launch_gate_up<8, FINITE>(a, capacity, st)
                     : launch_gate_up<4, FINITE>(a, capacity, st);
  if (rc) return rc;
  return wd == 16 ? launch_down<16, FINITE>(a, capacity, st)
         : wd == 8 ? launch_down<8, FINITE>(a, capacity, st)
                   : launch_down<4, FINITE>(a, capacity, st);
}

// Every token's routes plus one route to the shared expert (id E, weight
// 1.0, last in the token's slots); ids >= E become 0xFFFFFFFF (still bad).
__global__ void extend_routes_kernel(const uint32_t* __restrict__ ids, const float* __restrict__ scores, int64_t T,
                                     int top_k, uint32_t E, uint32_t* __restrict__ ids2, float* __restrict__ scores2) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the router's ids and scores
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * (top_k + 1)) return;
  const int64_t t = i / (top_k + 1);
  const int j = (int)(i - t * (top_k + 1));
  if (j == top_k) {
    ids2[i] = E;
    scores2[i] = 1.0f;
  } else {
    const uint32_t e = ids[t * top_k + j];
    ids2[i] = e < E ? e : 0xFFFFFFFFu;
    scores2[i] = scores[t * top_k + j];
  }
}

// Combine through the sorted-order rows (direct_combine.cu).
int direct_combine_rows(const uint16_t* rows, const uint32_t* row_of_slot, const uint32_t* expert_ids,
                        const float* scores, int64_t T, int top_k, int64_t H, int64_t E, const uint16_t* shared,
                        uint16_t* out, uint32_t* status, cudaStream_t st);

}  // namespace glm53

using namespace glm53;

extern "C" size_t glm53_batched_decode_workspace_bytes(int64_t T, int top_k, int64_t E, int64_t H, int64_t I) {
  return batched_workspace(T * top_k, E, H, I).bytes;
}

// The plan of T * (top_k + 1) routes over E + 1 experts, then the extended
// ids and scores.
extern "C" size_t glm53_batched_decode_shared_workspace_bytes(int64_t T, int top_k, int64_t E, int64_t H, int64_t I) {
  const int64_t R = T * (top_k + 1);
  return batched_workspace(R, E + 1, H, I).bytes + 2 * align_up((size_t)R * 4, 256);
}

// Shared expert weights of glm53_batched_decode_moe_shared (all null: none).
struct SharedWeights {
  const uint8_t* g_w;
  const float* g_s;
  const uint8_t* u_w;
  const float* u_s;
  const uint8_t* d_w;
  const float* d_s;
};

// top_k / E here count the shared-expert route and expert when sw.g_w is set
// (the caller extended the routes).
static int batched_decode(const char* fn, const void* x, int64_t T, int64_t H, const uint32_t* expert_ids,
                          const float* scores, int top_k, const uint8_t* gate_up_w, const float* gate_up_s,
                          const uint8_t* down_w, const float* down_s, int64_t E, int64_t I, float limit,
                          const void* shared, const SharedWeights& sw, void* out, void* workspace,
                          size_t workspace_bytes, uint32_t* status, uint32_t flags, cudaStream_t st) {
  const int64_t R = T * top_k;
  if (T < 0 || top_k <= 0 || top_k > 32 || H <= 0 || I <= 0 || E <= 0 || H % 128 != 0 || I % 128 != 0 ||
      H > 32768 || I > 32768 || R > kBdMaxRoutes) {
    set_last_error("%s: unsupported geometry T=%lld top_k=%d H=%lld I=%lld", fn, (long long)T, top_k, (long long)H,
                   (long long)I);
    return GLM53_ERR_INVALID;
  }
  if (T == 0) return GLM53_OK;
  const BatchedWorkspace wl = batched_workspace(R, E, H, I);
  if (!x || !expert_ids || !scores || !gate_up_w || !gate_up_s || !down_w || !down_s || !out || !workspace ||
      !status || workspace_bytes < wl.bytes ||
      (((uintptr_t)x | (uintptr_t)gate_up_w | (uintptr_t)down_w | (uintptr_t)out | (uintptr_t)shared) & 15) != 0) {
    set_last_error("%s: missing pointer, misaligned tensor or workspace too small", fn);
    return GLM53_ERR_INVALID;
  }
  char* ws = (char*)workspace;
  BatchedArgs a{};
  a.x = (const uint16_t*)x;
  a.H = (int)H;
  a.I = (int)I;
  a.E = (int)E;
  a.top_k = top_k;
  a.order = (const uint32_t*)(ws + wl.order);
  a.tile_experts = (const uint32_t*)(ws + wl.tile_experts);
  a.tile_starts = (const uint32_t*)(ws + wl.tile_starts);
  a.tile_lengths = (const uint32_t*)(ws + wl.tile_lengths);
  a.descriptor_count = (const uint32_t*)(ws + wl.counts);
  a.gu_w = gate_up_w;
  a.gu_s = gate_up_s;
  a.d_w = down_w;
  a.d_s = down_s;
  a.sg_w = sw.g_w;
  a.sg_s = sw.g_s;
  a.su_w = sw.u_w;
  a.su_s = sw.u_s;
  a.sd_w = sw.d_w;
  a.sd_s = sw.d_s;
  if (sw.g_w) a.E = (int)(E - 1);  // the shared expert is id E - 1 of the extended routes
  a.limit = limit;
  a.hidden = (uint16_t*)(ws + wl.hidden);
  a.rows = (uint16_t*)(ws + wl.rows);
  a.status = status;
  int rc = route_plan(expert_ids, R, E, kBdCols, scores, (uint32_t*)(ws + wl.order), (uint32_t*)(ws + wl.inverse),
                      (uint32_t*)(ws + wl.sorted_experts), (float*)(ws + wl.sorted_scores),
                      (uint32_t*)(ws + wl.route_offsets), (uint32_t*)(ws + wl.tile_experts),
                      (uint32_t*)(ws + wl.tile_starts), (uint32_t*)(ws + wl.tile_lengths),
                      (uint32_t*)(ws + wl.tile_offsets), (uint32_t*)(ws + wl.counts),
                      (uint32_t*)(ws + wl.counts) + 1, st);
  if (rc) return rc;
  const int64_t capacity = (R + kBdCols - 1) / kBdCols + E;
  rc = (flags & GLM53_FLAG_E4M3_FINITE) ? launch_batched<true>(a, capacity, st) : launch_batched<false>(a, capacity, st);
  if (rc) return rc;
  return direct_combine_rows(a.rows, (const uint32_t*)(ws + wl.inverse), expert_ids, scores, T, top_k, H, E,
                             (const uint16_t*)shared, (uint16_t*)out, status, st);
}

extern "C" size_t glm53_routes_decode_coalesced_workspace_bytes(int64_t R, int64_t E, int64_t H, int64_t I) {
  return R > 0 && E > 0 ? batched_workspace(R, E, H, I).bytes : 0;
}

extern "C" int glm53_routes_decode_coalesced(const void* x_rows, int64_t R, int64_t H, const uint32_t* expert_ids,
                                             const uint8_t* gate_up_w, const float* gate_up_s,
                                             const uint8_t* down_w, const float* down_s, int64_t E, int64_t I,
                                             float limit, void* out_rows, void* workspace, size_t workspace_bytes,
                                             uint32_t* status, uint32_t flags, void* stream) {
  const char* fn = "glm53_routes_decode_coalesced";
  if (R < 0 || H <= 0 || I <= 0 || E <= 0 || H % 128 != 0 || I % 128 != 0 || H > 32768 || I > 32768 ||
      R > kBdMaxRoutes || E >= 0x7FFFFFFF) {
    set_last_error("%s: unsupported geometry R=%lld H=%lld I=%lld E=%lld", fn, (long long)R, (long long)H,
                   (long long)I, (long long)E);
    return GLM53_ERR_INVALID;
  }
  if (R == 0) return GLM53_OK;
  const BatchedWorkspace wl = batched_workspace(R, E, H, I);
  if (!x_rows || !expert_ids || !gate_up_w || !gate_up_s || !down_w || !down_s || !out_rows || !workspace ||
      !status || workspace_bytes < wl.bytes ||
      (((uintptr_t)x_rows | (uintptr_t)gate_up_w | (uintptr_t)down_w | (uintptr_t)out_rows |
        (uintptr_t)workspace) & 15) != 0) {
    set_last_error("%s: missing pointer, misaligned tensor or workspace too small", fn);
    return GLM53_ERR_INVALID;
  }
  cudaStream_t st = (cudaStream_t)stream;
  char* ws = (char*)workspace;
  BatchedArgs a{};
  a.x = (const uint16_t*)x_rows;
  a.H = (int)H;
  a.I = (int)I;
  a.E = (int)E;
  a.top_k = 1;  // route r reads row r
  a.order = (const uint32_t*)(ws + wl.order);
  a.tile_experts = (const uint32_t*)(ws + wl.tile_experts);
  a.tile_starts = (const uint32_t*)(ws + wl.tile_starts);
  a.tile_lengths = (const uint32_t*)(ws + wl.tile_lengths);
  a.descriptor_count = (const uint32_t*)(ws + wl.counts);
  a.gu_w = gate_up_w;
  a.gu_s = gate_up_s;
  a.d_w = down_w;
  a.d_s = down_s;
  a.limit = limit;
  a.hidden = (uint16_t*)(ws + wl.hidden);
  a.rows = (uint16_t*)out_rows;
  a.scatter = (const uint32_t*)(ws + wl.order);
  a.status = status;
  // ids >= E (the empty-slot mark among them) fall into the plan's invalid
  // bucket: no descriptor, so their rows are left untouched
  int rc = route_plan(expert_ids, R, E, kBdCols, nullptr, (uint32_t*)(ws + wl.order), (uint32_t*)(ws + wl.inverse),
                      (uint32_t*)(ws + wl.sorted_experts), nullptr, (uint32_t*)(ws + wl.route_offsets),
                      (uint32_t*)(ws + wl.tile_experts), (uint32_t*)(ws + wl.tile_starts),
                      (uint32_t*)(ws + wl.tile_lengths), (uint32_t*)(ws + wl.tile_offsets),
                      (uint32_t*)(ws + wl.counts), (uint32_t*)(ws + wl.counts) + 1, st);
  if (rc) return rc;
  const int64_t capacity = (R + kBdCols - 1) / kBdCols + E;
  return (flags & GLM53_FLAG_E4M3_FINITE) ? launch_batched<true>(a, capacity, st) : launch_batched<false>(a, capacity, st);
}

extern "C" int glm53_batched_decode_moe(const void* x, int64_t T, int64_t H, const uint32_t* expert_ids,
                                        const float* scores, int top_k, const uint8_t* gate_up_w,
                                        const float* gate_up_s, const uint8_t* down_w, const float* down_s,
                                        int64_t E, int64_t I, float limit, const void* shared, void* out,
                                        void* workspace, size_t workspace_bytes, uint32_t* status, uint32_t flags,
                                        void* stream) {
  return batched_decode("glm53_batched_decode_moe", x, T, H, expert_ids, scores, top_k, gate_up_w, gate_up_s, down_w,
                        down_s, E, I, limit, shared, SharedWeights{}, out, workspace, workspace_bytes, status, flags,
                        (cudaStream_t)stream);
}

extern "C" int glm53_batched_decode_moe_shared(const void* x, int64_t T, int64_t H, const uint32_t* expert_ids,
                                               const float* scores, int top_k, const uint8_t* gate_up_w,
                                               const float* gate_up_s, const uint8_t* down_w, const float* down_s,
                                               int64_t E, int64_t I, const uint8_t* shared_gate_w,
                                               const float* shared_gate_s, const uint8_t* shared_up_w,
                                               const float* shared_up_s, const uint8_t* shared_down_w,
                                               const float* shared_down_s, float limit, void* out, void* workspace,
                                               size_t workspace_bytes, uint32_t* status, uint32_t flags,
                                               void* stream) {
  const char* fn = "glm53_batched_decode_moe_shared";
  if (T < 0 || top_k <= 0 || top_k >= 32 || E <= 0 || E >= 0x7FFFFFFF || !expert_ids || !scores || !workspace ||
      !shared_gate_w || !shared_gate_s || !shared_up_w || !shared_up_s || !shared_down_w || !shared_down_s ||
      (((uintptr_t)shared_gate_w | (uintptr_t)shared_up_w | (uintptr_t)shared_down_w) & 15) != 0 ||
      workspace_bytes < glm53_batched_decode_shared_workspace_bytes(T, top_k, E, H, I)) {
    set_last_error("%s: invalid arguments or workspace too small", fn);
    return GLM53_ERR_INVALID;
  }
  if (T == 0) return GLM53_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t R = T * (top_k + 1);
  const size_t plan = batched_workspace(R, E + 1, H, I).bytes;
  uint32_t* ids2 = (uint32_t*)((char*)workspace + plan);
  float* scores2 = (float*)((char*)workspace + plan + align_up((size_t)R * 4, 256));
  launch_programmatic(extend_routes_kernel, dim3((unsigned)((R + 255) / 256)), dim3(256), 0, st, expert_ids, scores,
                      T, top_k, (uint32_t)E, ids2, scores2);
  int rc = check_launch("extend_routes_kernel");
  if (rc) return rc;
  const SharedWeights sw{shared_gate_w, shared_gate_s, shared_up_w, shared_up_s, shared_down_w, shared_down_s};
  return batched_decode(fn, x, T, H, ids2, scores2, top_k + 1, gate_up_w, gate_up_s, down_w, down_s, E + 1, I, limit,
                        nullptr, sw, out, workspace, plan, status, flags, st);
}
