// One-token decode MoE (G3 + G4) on tensor-core GEMV tiles.
//
// Replaces PackedFP8MoE.__call__ decode (glm53_flash_mlx/packed.py:896-923):
//   K7  fused gate/up/SwiGLU over the selected experts  (packed.py:100-166)
//   K9  the same for the shared expert                  (packed.py:181-235)
//   K6  selected down projections                        (packed.py:66-98)
//   K8  FP32 slot-ordered weighted reduction             (packed.py:168-179)
//   shared down (K1) and the BF16 `result + shared` add  (packed.py:915-922)
// and the Direct module's selected-expert decode over separately allocated
// experts (glm53_flash_mlx/fp8.py:372-383, kernels K3/K4 at fp8.py:142-251),
// in two launches:
//   decode_gate_up_v4: one warp per (slot, 8 hidden rows).  Its m16 MMA tile
//     is the 8 gate rows (tile rows 0-7) and the 8 up rows (rows 8-15) of
//     those hidden rows, over the whole K; lane 4g ends up holding gate and
//     up of hidden row g and applies the BF16 SwiGLU itself.
//   decode_down_v4: one warp per (slot, 16 output rows) over the whole K;
//     per-slot dot products go to workspace and the last warp of each 16-row
//     block (completion counter) reduces them in slot order with the
//     reference's rounding points and adds the shared expert.
// Weight fragments stream through per-warp cp.async rings (gemv_tile.cuh);
// weight copies are issued before the activations are staged.
// Shapes the tiles do not cover take a scalar path, one warp per dot product.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "gemv_tile.cuh"
#include "kernels.cuh"

namespace glm53 {

constexpr int kMaxSlots = 16;

struct DecodeArgs {
  const uint16_t* x;
  int H, I, Is, E, top_k;
  const uint32_t* ids;  // bank mode: device expert ids
  const float* scores;
  // bank mode (PackedFP8ExpertBank layout)
  const uint8_t* gu_w;
  const float* gu_s;
  const uint8_t* d_w;
  const float* d_s;
  // table mode: per routed slot, the expert's own tensors (Direct experts)
  bool table;
  const uint8_t* tg_w[kMaxSlots];
  const float* tg_s[kMaxSlots];
  const uint8_t* tu_w[kMaxSlots];
  const float* tu_s[kMaxSlots];
  const uint8_t* td_w[kMaxSlots];
  const float* td_s[kMaxSlots];
  // shared expert (Is == 0 when absent)
  const uint8_t* sg_w;
  const float* sg_s;
  const uint8_t* su_w;
  const float* su_s;
  const uint8_t* sd_w;
  const float* sd_s;
  float limit;
  // mHC post-expand fused into the final reduce (glm53_packed_decode_moe_hc):
  // instead of out[h], write hc_out[b][h] = BF16(post[b] * moe[h] + FMA chain
  // over the 4 sources comb[s][b] * residual[s][h]) for the 4 branches b
  const uint16_t* hc_residual;  // [4, H] BF16
  const float* hc_post;         // [4]
  const float* hc_comb;         // [4][4], comb[source][branch]
  uint16_t* hc_out;             // [4, H] BF16
  uint16_t* hidden;    // [top_k*I + Is]
  float* partial;      // [(top_k + 1) * H] per-slot down dot products
  uint32_t* counters;  // [H / 16] completion counters (zero between calls)
  uint16_t* out;       // [H]
  uint32_t* status;
  // per-route mode (expert-parallel owners): slot j reads x + j * x_stride and
  // writes its BF16 down row to route_out[j]; no reduction, no shared expert;
  // slots whose expert id is kEmptySlot are skipped
  int64_t x_stride;
  uint16_t* route_out;
  // peer-memory expert parallelism (per-route mode): the slots arrive from
  // other GPUs; gate/up waits until *arrivals >= (*epoch + 1) * arrivals_per_step
  // before reading them, and down writes slot j = (home, s) to the home rank's
  // back buffer at slot (rank, s), then counts one arrival there per CTA
  const unsigned long long* arrivals;
  const unsigned long long* epoch;
  unsigned long long arrivals_per_step;
  unsigned long long wait_ns;  // bound of the arrival wait
  const unsigned long long* peer_base;  // [world] buffer bases (device pointers)
  int64_t back_off, back_cnt_off;
  int rank, cap;
  // per-route mode: n_shared shared-expert slots after the routed ones, slot
  // top_k + t reading shared_x + t * H and writing shared_out + t * H
  int n_shared;
  const uint16_t* shared_x;
  uint16_t* shared_out;
  // split execution (GLM53_FLAG_SHARED_ONLY / GLM53_FLAG_SKIP_SHARED): the
  // unit ranges each launch covers (end 0 = all), and the number of slot
  // partials the last-arriver reduce waits for (0 = every slot)
  int gu_begin, gu_end, dn_begin, dn_end, dn_expect;
  bool dn_no_reduce;
  // the shared-expert slots (which wait for nothing) take the first CTAs of
  // both grids instead of the last.  Peer-memory owners then run the routed
  // slots in slot-position-major order, (src 0, s 0), (src 1, s 0), ...:
  // routes fill each source's slots from s = 0, so the occupied slots come
  // first and the empty ones (which only wait and exit) last
  bool shared_first;
  // GLM53_FLAG_AFTER_ROUTER: gate/up is a programmatic dependent of the
  // router; its routed CTAs wait for the router (griddepcontrol.wait) before
  // they read the expert ids and only then let the down grid launch
  bool after_router;
  // peer-memory owners: gate/up is launched as a programmatic dependent of
  // the dispatch (its CTAs are resident and wait for the dispatch grid, then
  // the routed ones for their arrivals), and the down stage lets the combine
  // launch early
  bool pdl_owner;
  // host decode steps: the down stage lets the next step's input copy launch
  // once the gate/up grid has finished (no kernel of this step reads the
  // input row after that), so its host read overlaps the down stage
  bool trigger_after_wait;
};

// Physical routed slot p of a peer-memory owner grid -> slot (src, s) = src * cap + s.
__host__ __device__ __forceinline__ int owner_slot(const DecodeArgs& a, int p) {
  const int world = a.top_k / a.cap;
  return (p % world) * a.cap + p / world;
}

constexpr uint32_t kEmptySlot = 0xFFFFFFFFu;

// Shared-expert slots: one (sharing x) in the packed decode, n_shared in the
// per-route modes.
__host__ __device__ __forceinline__ int shared_slots(const DecodeArgs& a) {
  return a.Is > 0 ? (a.n_shared > 0 ? a.n_shared : 1) : 0;
}

__host__ __device__ __forceinline__ int align16i(int v) { return (v + 15) & ~15; }

constexpr int kWarpsPerBlock = 4;
constexpr int kRing = 8;       // gate/up: 64-wide K slices in flight per warp (1 KB each)
constexpr int kRingDown = 12;  // down: its per-warp streams are short (I/64 slices), so deeper
// Gate/up launched as a programmatic dependent of the router: the block
// scheduler fills the SMs one after another for such a grid, so 4-warp CTAs
// would crowd about 60% of the SMs.  One 12-warp CTA per SM instead (its
// shared memory is at least half an SM's), which still leaves room for two
// down CTAs to prefetch beside it; 16-warp CTAs with a 7-deep ring where the
// slot's I/8 units divide by 16 but not by 12 (I = 2048).  Shapes that fit
// neither launch the 4-warp CTAs after the router completes.
constexpr int kWideWarps = 12;
constexpr int kWideRing = 9;
constexpr int kWide16Warps = 16;
constexpr int kWide16Ring = 7;

// ---------------------------------------------------------------------------
// Gate / up / SwiGLU
// ---------------------------------------------------------------------------

struct GateUpRows {
  const uint8_t* g;  // gate row r0
  const uint8_t* u;  // up row r0
  const float* sg;   // block-scale row of the gate rows
  const float* su;
  int hoff;          // hidden index of row r0
  bool valid;
};

__device__ __forceinline__ GateUpRows gate_up_rows(const DecodeArgs& a, int unit) {
  GateUpRows r;
  const int per = a.I >> 3;
  const int routed = a.top_k * per;
  const int cols = a.H >> 7;
  if (unit < routed) {
    const int slot = unit / per, r0 = (unit - slot * per) << 3;
    r.hoff = slot * a.I + r0;
    if (a.table) {
      r.valid = true;
      r.g = a.tg_w[slot] + (size_t)r0 * a.H;
      r.u = a.tu_w[slot] + (size_t)r0 * a.H;
      r.sg = a.tg_s[slot] + (size_t)(r0 >> 7) * cols;
      r.su = a.tu_s[slot] + (size_t)(r0 >> 7) * cols;
    } else {
      const int half = a.I >> 7;
      const uint32_t e = a.ids[slot];
      r.valid = e < (uint32_t)a.E;
      const uint32_t es = r.valid ? e : 0u;
      r.g = a.gu_w + ((size_t)es * 2 * a.I + r0) * a.H;
      r.u = r.g + (size_t)a.I * a.H;
      r.sg = a.gu_s + ((size_t)es * 2 * half + (r0 >> 7)) * cols;
      r.su = r.sg + (size_t)half * cols;
    }
  } else {
    const int per_s = a.Is >> 3;
    const int u2 = unit - routed, t = u2 / per_s;
    const int r0 = (u2 - t * per_s) << 3;
    r.valid = true;
    r.hoff = a.top_k * a.I + t * a.Is + r0;
    r.g = a.sg_w + (size_t)r0 * a.H;
    r.u = a.su_w + (size_t)r0 * a.H;
    r.sg = a.sg_s + (size_t)(r0 >> 7) * cols;
    r.su = a.su_s + (size_t)(r0 >> 7) * cols;
  }
  return r;
}

// W warps per CTA, one unit (8 gate + 8 up rows) per warp, P slices in flight per warp.
template <bool FINITE, int W, int P>
__global__ void __launch_bounds__(32 * W) decode_gate_up_v4(DecodeArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  uint4* ring = reinterpret_cast<uint4*>(smem) + (size_t)warp * P * 64;
  __half* xs = reinterpret_cast<__half*>(reinterpret_cast<uint4*>(smem) + (size_t)W * P * 64);
  float* scratch = reinterpret_cast<float*>(xs + align16i(a.H + 8));
  const int routed_units = a.top_k * (a.I >> 3);
  const int nunits = a.gu_end ? a.gu_end : routed_units + shared_slots(a) * (a.Is >> 3);
  int unit = a.gu_begin + blockIdx.x * W + warp;
  // every unit of a block belongs to one slot (I/8 and I_shared/8 are
  // multiples of W here)
  int unit0 = a.gu_begin + blockIdx.x * W;
  if (a.shared_first) {  // physical order: shared units, then routed units (owners: by slot position)
    const int S = nunits - routed_units, per = a.I >> 3;
    auto logical = [&](int u) {
      if (u < S) return routed_units + u;
      u -= S;
      if (!a.arrivals) return u;
      const int p = u / per;
      return owner_slot(a, p) * per + (u - p * per);
    };
    unit = logical(unit);
    unit0 = logical(unit0);
  }
  const bool active = unit < nunits;
  const int jb = unit0 < routed_units ? unit0 / (a.I >> 3) : a.top_k + (unit0 - routed_units) / (a.Is >> 3);
  const uint16_t* xb = jb < a.top_k ? a.x + (size_t)jb * a.x_stride
                                    : (a.shared_x ? a.shared_x + (size_t)(jb - a.top_k) * a.H : a.x);
  const bool wait_router = a.after_router && jb < a.top_k;  // CTA-uniform
  // after the dispatch grid (the home rows; and so that this grid's
  // completion implies the dispatch's, which the combine relies on)
  if (a.pdl_owner) pdl_wait();
  float xmul = 0.f;
  if (wait_router) {
    // the activation row does not depend on routing: stage it while the router runs
    xmul = stage_f16(xs, a.H + 8, xb, 0, 1, a.H, scratch);
    pdl_wait();  // the router's results
  }
  if (a.arrivals && jb < a.top_k) {  // peer-memory dispatch: wait for every rank's slots
    if (threadIdx.x == 0) wait_counter_geq(a.arrivals, (*a.epoch + 1ull) * a.arrivals_per_step, a.status, a.wait_ns);
    __syncthreads();
  }
  // the down stage may launch now: its prologue only streams weights.  After
  // the router, the routed CTAs let it launch once their own weight streams
  // are issued (measured 1.1 us faster per step than at once).
  if (!wait_router) pdl_trigger();
  if (a.route_out && jb < a.top_k && a.ids[jb] == kEmptySlot) return;
  GateUpRows rw{};
  if (active) rw = gate_up_rows(a, unit);
  const bool ld = active && rw.valid;
  const uint8_t* pg = ld ? rw.g + (size_t)g * a.H + 16 * q : nullptr;
  const uint8_t* pu = ld ? rw.u + (size_t)g * a.H + 16 * q : nullptr;
  const int nslice = a.H >> 6;
  auto issue = [&](int sl) {
    uint4* d = ring + (sl % P) * 64 + lane;
    cp_async_16_l2_256(d, ld ? (const void*)(pg + 64 * sl) : (const void*)a.x, ld);
    cp_async_16_l2_256(d + 32, ld ? (const void*)(pu + 64 * sl) : (const void*)a.x, ld);
  };
#pragma unroll
  for (int s = 0; s < P - 1; ++s) {
    if (s < nslice) issue(s);
    cp_async_commit_group();
  }
  if (wait_router) pdl_trigger();  // the down prologue reads expert ids this CTA has seen final
  WarpScales ssg, ssu;
  ssg.load(rw.sg, a.H >> 7, ld);
  ssu.load(rw.su, a.H >> 7, ld);
  const float smul =
      decode_unscale<FINITE>() * (wait_router ? xmul : stage_f16(xs, a.H + 8, xb, 0, 1, a.H, scratch));
  float part[4] = {0.f, 0.f, 0.f, 0.f}, tot[4] = {0.f, 0.f, 0.f, 0.f};
  for (int sl = 0; sl < nslice; ++sl) {
    if (sl + P - 1 < nslice) issue(sl + P - 1);
    cp_async_commit_group();
    cp_async_wait_group<P - 1>();
    const uint4* src = ring + (sl % P) * 64 + lane;
    const uint4 fg = src[0], fu = src[32];
    uint32_t xw[8];
    load_x_frag(xw, xs + 64 * sl + 16 * q, g == 0);
    mma_slice<FINITE>(part, fg, fu, xw);
    if ((sl & 1) && ld) promote2(tot, part, ssg.at(sl >> 1) * smul, ssu.at(sl >> 1) * smul);
  }
  cp_async_wait_group<0>();
  if (active && q == 0) a.hidden[rw.hoff + g] = rw.valid ? swiglu_bf16(tot[0], tot[2], a.limit) : (uint16_t)0;
  if (active && !rw.valid && lane == 0) atomicOr(a.status, kStatusBadExpert);
}

// ---------------------------------------------------------------------------
// Down + slot-ordered reduce + shared add
// ---------------------------------------------------------------------------

// Down stage of one CTA in peer-memory mode (all four warps on slot jb).  A
// routed slot arrived from rank jb / cap: its expert id is read after an
// acquire of the arrival counter (which gate/up already saw complete), the
// weights start streaming, and only then does the CTA wait for the gate/up
// grid; the BF16 rows go straight into the home rank's back buffer and one
// arrival per CTA is counted there.  Empty slots and shared-expert slots
// (jb >= top_k, rows written locally) count nothing.
template <bool FINITE>
__device__ __forceinline__ void decode_down_peer(const DecodeArgs& a, int jb, int unit0) {
  constexpr int P = kRingDown;
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const int K = a.I;
  uint4* ring = reinterpret_cast<uint4*>(smem) + (size_t)warp * P * 64;
  __half* xs = reinterpret_cast<__half*>(reinterpret_cast<uint4*>(smem) + (size_t)kWarpsPerBlock * P * 64);
  float* scratch = reinterpret_cast<float*>(xs + align16i(K + 8));
  const int rtiles = a.H >> 4;
  const int tile = unit0 + warp - jb * rtiles;
  const int row0 = tile << 4;
  const int cols = K >> 7;
  const bool routed = jb < a.top_k;
  const int home = routed ? jb / a.cap : 0, s = routed ? jb - home * a.cap : 0;
  char* hb = reinterpret_cast<char*>(routed ? a.peer_base[home] : 0ull);
  uint32_t e = 0;
  if (routed) {
    if (threadIdx.x == 0) wait_counter_geq(a.arrivals, (*a.epoch + 1ull) * a.arrivals_per_step, a.status, a.wait_ns);
    __syncthreads();
    e = a.ids[jb];
  }
  if (e != kEmptySlot) {  // uniform over the CTA
    const bool valid = !routed || e < (uint32_t)a.E;
    const uint32_t es = valid ? e : 0u;
    const uint8_t* w0 = routed ? a.d_w + ((size_t)es * a.H + row0) * K : a.sd_w + (size_t)row0 * K;
    const float* srow = routed ? a.d_s + ((size_t)es * (a.H >> 7) + (row0 >> 7)) * cols
                               : a.sd_s + (size_t)(row0 >> 7) * cols;
    const uint8_t* p0 = w0 + (size_t)g * K + 16 * q;
    const uint8_t* p8 = w0 + (size_t)(g + 8) * K + 16 * q;
    const int nslice = K >> 6;
    auto issue = [&](int sl) {
      uint4* d = ring + (sl % P) * 64 + lane;
      cp_async_16_l2_256(d, valid ? (const void*)(p0 + 64 * sl) : (const void*)a.x, valid);
      cp_async_16_l2_256(d + 32, valid ? (const void*)(p8 + 64 * sl) : (const void*)a.x, valid);
    };
#pragma unroll
    for (int k = 0; k < P - 1; ++k) {
      if (k < nslice) issue(k);
      cp_async_commit_group();
    }
    WarpScales sd;
    sd.load(srow, cols, valid);
    if (a.pdl_owner) pdl_trigger();  // the combine may launch; it waits for this grid
    pdl_wait();  // the hidden rows come from the gate/up grid
    const float smul =
        decode_unscale<FINITE>() * stage_f16(xs, K + 8, a.hidden + (size_t)jb * a.I, 0, 1, K, scratch);
    float part[4] = {0.f, 0.f, 0.f, 0.f}, tot[4] = {0.f, 0.f, 0.f, 0.f};
    for (int sl = 0; sl < nslice; ++sl) {
      if (sl + P - 1 < nslice) issue(sl + P - 1);
      cp_async_commit_group();
      cp_async_wait_group<P - 1>();
      const uint4* src = ring + (sl % P) * 64 + lane;
      const uint4 f0 = src[0], f8 = src[32];
      uint32_t xw[8];
      load_x_frag(xw, xs + 64 * sl + 16 * q, g == 0);
      mma_slice<FINITE>(part, f0, f8, xw);
      if ((sl & 1) && valid) promote(tot, part, sd.at(sl >> 1) * smul);
    }
    cp_async_wait_group<0>();
    if (q == 0) {
      uint16_t* dst = routed ? reinterpret_cast<uint16_t*>(hb + a.back_off) + ((size_t)a.rank * a.cap + s) * a.H
                             : a.shared_out + (size_t)(jb - a.top_k) * a.H;
      dst[row0 + g] = valid ? f32_to_bf16_bits(tot[0]) : (uint16_t)0;
      dst[row0 + g + 8] = valid ? f32_to_bf16_bits(tot[2]) : (uint16_t)0;
    }
    if (!valid && lane == 0) atomicOr(a.status, kStatusBadExpert);
  }
  if (routed && e != kEmptySlot) {  // empty slots send nothing home and count nothing
    // release: the block barrier, then one cumulative system-scope fence
    // before the arrival
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      atomicAdd(reinterpret_cast<unsigned long long*>(hb + a.back_cnt_off), 1ull);
    }
  }
}

template <bool FINITE>
__global__ void __launch_bounds__(32 * kWarpsPerBlock) decode_down_v4(DecodeArgs a) {
  constexpr int P = kRingDown;
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const int ns = a.top_k + shared_slots(a);
  const int K = a.I;  // I_shared == I on this path
  uint4* ring = reinterpret_cast<uint4*>(smem) + (size_t)warp * P * 64;
  __half* xs = reinterpret_cast<__half*>(reinterpret_cast<uint4*>(smem) + (size_t)kWarpsPerBlock * P * 64);
  float* scratch = reinterpret_cast<float*>(xs + align16i(K + 8));
  const int rtiles = a.H >> 4;
  const int nunits = a.dn_end ? a.dn_end : ns * rtiles;
  const int unit = a.dn_begin + blockIdx.x * kWarpsPerBlock + warp;
  const bool active = unit < nunits;
  const int j = active ? unit / rtiles : 0;
  const int tile = unit - j * rtiles;
  const int row0 = tile << 4;
  const int cols = K >> 7;
  // every unit of a block belongs to one slot (H/16 is a multiple of 4 here)
  const int jb = min((int)(a.dn_begin + blockIdx.x * kWarpsPerBlock) / rtiles, ns - 1);
  if (a.peer_base) {
    int u0 = a.dn_begin + blockIdx.x * kWarpsPerBlock;
    if (a.shared_first) {  // physical order: shared slots' tiles, then routed by slot position
      const int S = (ns - a.top_k) * rtiles;
      if (u0 < S) {
        u0 = a.top_k * rtiles + u0;
      } else {
        u0 -= S;
        const int p = u0 / rtiles;
        u0 = owner_slot(a, p) * rtiles + (u0 - p * rtiles);
      }
    }
    decode_down_peer<FINITE>(a, u0 / rtiles, u0);
    return;
  }
  if (a.route_out && jb < a.top_k && a.ids[jb] == kEmptySlot) return;
  bool valid = active;
  const uint8_t* w0 = nullptr;
  const float* srow = nullptr;
  if (active) {
    if (j >= a.top_k) {
      w0 = a.sd_w + (size_t)row0 * K;
      srow = a.sd_s + (size_t)(row0 >> 7) * cols;
    } else if (a.table) {
      w0 = a.td_w[j] + (size_t)row0 * K;
      srow = a.td_s[j] + (size_t)(row0 >> 7) * cols;
    } else {
      const uint32_t e = __ldcg(a.ids + j);  // from L2: the router wrote it while this grid's producer ran
      valid = e < (uint32_t)a.E;
      const uint32_t es = valid ? e : 0u;
      w0 = a.d_w + ((size_t)es * a.H + row0) * K;
      srow = a.d_s + ((size_t)es * (a.H >> 7) + (row0 >> 7)) * cols;
    }
  }
  const bool ld = active && valid;
  const uint8_t* p0 = ld ? w0 + (size_t)g * K + 16 * q : nullptr;
  const uint8_t* p8 = ld ? w0 + (size_t)(g + 8) * K + 16 * q : nullptr;
  const int nslice = K >> 6;
  auto issue = [&](int sl) {
    uint4* d = ring + (sl % P) * 64 + lane;
    cp_async_16_l2_256(d, ld ? (const void*)(p0 + 64 * sl) : (const void*)a.x, ld);
    cp_async_16_l2_256(d + 32, ld ? (const void*)(p8 + 64 * sl) : (const void*)a.x, ld);
  };
#pragma unroll
  for (int s = 0; s < P - 1; ++s) {
    if (s < nslice) issue(s);
    cp_async_commit_group();
  }
  WarpScales sd;
  sd.load(srow, cols, ld);
  // weights are streaming; the hidden rows come from the gate/up stage
  pdl_wait();
  if (a.trigger_after_wait) pdl_trigger();
  const float smul =
      decode_unscale<FINITE>() * stage_f16(xs, K + 8, a.hidden + (size_t)jb * a.I, 0, 1, K, scratch);
  float part[4] = {0.f, 0.f, 0.f, 0.f}, tot[4] = {0.f, 0.f, 0.f, 0.f};
  for (int sl = 0; sl < nslice; ++sl) {
    if (sl + P - 1 < nslice) issue(sl + P - 1);
    cp_async_commit_group();
    cp_async_wait_group<P - 1>();
    const uint4* src = ring + (sl % P) * 64 + lane;
    const uint4 f0 = src[0], f8 = src[32];
    uint32_t xw[8];
    load_x_frag(xw, xs + 64 * sl + 16 * q, g == 0);
    mma_slice<FINITE>(part, f0, f8, xw);
    if ((sl & 1) && ld) promote(tot, part, sd.at(sl >> 1) * smul);
  }
  cp_async_wait_group<0>();
  if (!active) return;
  if (a.route_out) {  // per-route mode: this slot's BF16 down rows, as K6 stores them
    uint16_t* dst = j < a.top_k ? a.route_out + (size_t)j * a.H : a.shared_out + (size_t)(j - a.top_k) * a.H;
    if (q == 0) {
      dst[row0 + g] = valid ? f32_to_bf16_bits(tot[0]) : (uint16_t)0;
      dst[row0 + g + 8] = valid ? f32_to_bf16_bits(tot[2]) : (uint16_t)0;
    }
    if (!valid && lane == 0) atomicOr(a.status, kStatusBadExpert);
    return;
  }
  if (q == 0) {
    a.partial[(size_t)j * a.H + row0 + g] = valid ? tot[0] : 0.f;
    a.partial[(size_t)j * a.H + row0 + g + 8] = valid ? tot[2] : 0.f;
  }
  if (!valid && lane == 0) atomicOr(a.status, kStatusBadExpert);
  if (a.dn_no_reduce) return;  // shared-only pass: the partial waits in the workspace
  __syncwarp();
  __threadfence();
  unsigned last = 0;
  const int expect = a.dn_expect ? a.dn_expect : ns;
  if (lane == 0) last = atomicAdd(&a.counters[tile], 1u) == (unsigned)(expect - 1);
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return;
  __threadfence();
  if (lane < 16) {
    const int h = row0 + lane;
    float total = 0.f;
    for (int s2 = 0; s2 < a.top_k; ++s2) {
      // K6 stores each slot's dot product as BF16; K8 weights it in FP32
      const float d = bf16_round(__ldcg(a.partial + (size_t)s2 * a.H + h));
      total = total + __fmul_rn(d, a.scores[s2]);
    }
    float res = bf16_round(total);
    if (a.Is > 0) res = res + bf16_round(__ldcg(a.partial + (size_t)a.top_k * a.H + h));
    if (a.hc_out) {
      // hc expand with the arithmetic order of glm53_hc_expand
      // (native_indexer_plan.metal:2377-2388)
      const float moe = bf16_bits_to_f32(f32_to_bf16_bits(res));
      float rv[4];
#pragma unroll
      for (int src = 0; src < 4; ++src) rv[src] = bf16_bits_to_f32(a.hc_residual[(size_t)src * a.H + h]);
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        float mixed = 0.0f;
#pragma unroll
        for (int src = 0; src < 4; ++src) mixed = __fmaf_rn(__ldg(a.hc_comb + src * 4 + b), rv[src], mixed);
        a.hc_out[(size_t)b * a.H + h] = f32_to_bf16_bits(__fadd_rn(__fmul_rn(__ldg(a.hc_post + b), moe), mixed));
      }
    } else if ((((uintptr_t)a.out) & 15) == 0) {
      // two 16-byte stores per 16-row tile (the output may be host memory
      // mapped over PCIe, where small writes cost)
      const uint32_t v = f32_to_bf16_bits(res);
      const uint32_t w = v | (__shfl_down_sync(0x0000FFFFu, v, 1) << 16);  // even lanes: rows h, h + 1
      const uint32_t w1 = __shfl_down_sync(0x0000FFFFu, w, 2);
      const uint32_t w2 = __shfl_down_sync(0x0000FFFFu, w, 4);
      const uint32_t w3 = __shfl_down_sync(0x0000FFFFu, w, 6);
      if ((lane & 7) == 0) *reinterpret_cast<uint4*>(a.out + h) = make_uint4(w, w1, w2, w3);
    } else {
      a.out[h] = f32_to_bf16_bits(res);
    }
  }
  if (lane == 0) a.counters[tile] = 0u;  // leave the workspace reusable
}

// ---------------------------------------------------------------------------
// Generic (unaligned) path: one warp per dot product, scalar loads.
// ---------------------------------------------------------------------------

__device__ __forceinline__ void scalar_rows(const DecodeArgs& a, int item, const uint8_t*& gw, const uint8_t*& uw,
                                            const float*& gs, const float*& us, bool& valid) {
  const int routed = a.top_k * a.I;
  const int cols = (a.H + kBlock - 1) / kBlock;
  const int half = (a.I + kBlock - 1) / kBlock;
  valid = true;
  if (item < routed) {
    const int slot = item / a.I, row = item % a.I;
    if (a.table) {
      gw = a.tg_w[slot] + (size_t)row * a.H;
      uw = a.tu_w[slot] + (size_t)row * a.H;
      gs = a.tg_s[slot] + (size_t)(row / kBlock) * cols;
      us = a.tu_s[slot] + (size_t)(row / kBlock) * cols;
      return;
    }
    const uint32_t e = a.ids[slot];
    if (e >= (uint32_t)a.E) {
      valid = false;
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
}

__global__ void decode_gate_up_scalar_kernel(DecodeArgs a) {
  const int lane = threadIdx.x & 31;
  const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item >= a.top_k * a.I + a.Is) return;
  const uint8_t *gw = nullptr, *uw = nullptr;
  const float *gs = nullptr, *us = nullptr;
  bool valid;
  scalar_rows(a, item, gw, uw, gs, us, valid);
  if (!valid) {
    if (lane == 0) {
      atomicOr(a.status, kStatusBadExpert);
      a.hidden[item] = 0;
    }
    return;
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
  const int cols = (a.I + kBlock - 1) / kBlock;
  const int hrows = (a.H + kBlock - 1) / kBlock;
  float total = 0.f;
  for (int j = 0; j < a.top_k; ++j) {
    const uint8_t* wr;
    const float* sr;
    if (a.table) {
      wr = a.td_w[j] + (size_t)h * a.I;
      sr = a.td_s[j] + (size_t)(h / kBlock) * cols;
    } else {
      const uint32_t e = a.ids[j];
      if (e >= (uint32_t)a.E) {
        if (lane == 0) atomicOr(a.status, kStatusBadExpert);
        continue;
      }
      wr = a.d_w + ((size_t)e * a.H + h) * a.I;
      sr = a.d_s + ((size_t)e * hrows + h / kBlock) * cols;
    }
    const uint16_t* xr = a.hidden + (size_t)j * a.I;
    float v = 0.f;
    for (int k = lane; k < a.I; k += 32)
      v = fmaf(bf16_bits_to_f32(xr[k]) * e4m3_to_f32_scaled(wr[k]), sr[k / kBlock] * 256.0f, v);
    v = warp_sum(v);
    total = total + __fmul_rn(bf16_round(v), a.scores[j]);
  }
  float res = bf16_round(total);
  if (a.Is > 0) {
    const int scols = (a.Is + kBlock - 1) / kBlock;
    const uint8_t* wr = a.sd_w + (size_t)h * a.Is;
    const float* sr = a.sd_s + (size_t)(h / kBlock) * scols;
    const uint16_t* xr = a.hidden + (size_t)a.top_k * a.I;
    float v = 0.f;
    for (int k = lane; k < a.Is; k += 32)
      v = fmaf(bf16_bits_to_f32(xr[k]) * e4m3_to_f32_scaled(wr[k]), sr[k / kBlock] * 256.0f, v);
    v = warp_sum(v);
    res = res + bf16_round(v);
  }
  if (lane == 0) a.out[h] = f32_to_bf16_bits(res);
}

// ---------------------------------------------------------------------------
// Launch
// ---------------------------------------------------------------------------

static bool tensor_core_shape(const DecodeArgs& a) {
  const bool has_shared = a.Is > 0;
  bool aligned = (((uintptr_t)a.x | (uintptr_t)a.hidden) & 15) == 0;
  if (a.table) {
    for (int j = 0; j < a.top_k; ++j)
      aligned = aligned && ((((uintptr_t)a.tg_w[j] | (uintptr_t)a.tu_w[j] | (uintptr_t)a.td_w[j]) & 15) == 0);
  } else {
    aligned = aligned && ((((uintptr_t)a.gu_w | (uintptr_t)a.d_w) & 15) == 0);
  }
  if (has_shared) aligned = aligned && ((((uintptr_t)a.sg_w | (uintptr_t)a.su_w | (uintptr_t)a.sd_w) & 15) == 0);
  // H % 64 keeps every 4-warp block of the down kernel inside one slot
  return aligned && a.H % 128 == 0 && a.I % 128 == 0 && (!has_shared || a.Is == a.I) && a.H <= 32768 &&
         a.I <= 32768;
}

// Launch with or without programmatic stream serialisation (the kernel may
// start before the previous kernel on the stream has finished; it orders
// itself with pdl_wait).
static cudaError_t launch_decode(void (*kernel)(DecodeArgs), int blocks, size_t smem, cudaStream_t st, bool pdl,
                                 const DecodeArgs& a, int warps = kWarpsPerBlock) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(32 * warps);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, a);
}

// Shared memory of one SM and the per-CTA reservation on the current device
// (queried once per device).
static void sm_smem(size_t& per_sm, size_t& reserved) {
  constexpr int kMaxDevices = 64;
  static std::atomic<int> cache[kMaxDevices][2];  // zero-initialised: not yet queried
  int dev = 0;
  cudaGetDevice(&dev);
  int v = dev < kMaxDevices ? cache[dev][0].load(std::memory_order_acquire) : 0;
  int r = dev < kMaxDevices ? cache[dev][1].load(std::memory_order_relaxed) : 0;
  if (v == 0) {
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&r, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    if (dev < kMaxDevices) {
      cache[dev][1].store(r, std::memory_order_relaxed);
      cache[dev][0].store(v, std::memory_order_release);
    }
  }
  per_sm = (size_t)v;
  reserved = (size_t)r;
}

template <bool FINITE, int W, int P>
static int launch_gate_up(const DecodeArgs& a, cudaStream_t st, bool pdl, size_t min_smem) {
  const size_t smem = std::max(min_smem, (size_t)W * P * 64 * 16 + (size_t)align16i(a.H + 8) * 2 + 32 * sizeof(float));
  if (smem > 48 * 1024) {
    int rc = ensure_max_smem((const void*)decode_gate_up_v4<FINITE, W, P>, smem);
    if (rc) return rc;
  }
  const int units = (a.gu_end ? a.gu_end : a.top_k * (a.I >> 3) + shared_slots(a) * (a.Is >> 3)) - a.gu_begin;
  launch_decode(decode_gate_up_v4<FINITE, W, P>, (units + W - 1) / W, smem, st, pdl, a, W);
  return check_launch("decode_gate_up_v4");
}

template <bool FINITE>
static int launch_v4(const DecodeArgs& a, cudaStream_t st, bool gate_up_only) {
  {
    int rc;
    auto fits = [&](int w) { return (a.I >> 3) % w == 0 && (a.Is >> 3) % w == 0; };
    if (a.after_router && (fits(kWideWarps) || fits(kWide16Warps))) {
      size_t per_sm = 0, reserved = 0;
      sm_smem(per_sm, reserved);
      const size_t half_sm = per_sm / 2 + 16 - std::min(reserved, per_sm / 2);  // one CTA per SM
      rc = fits(kWideWarps) ? launch_gate_up<FINITE, kWideWarps, kWideRing>(a, st, true, half_sm)
                            : launch_gate_up<FINITE, kWide16Warps, kWide16Ring>(a, st, true, half_sm);
    } else {
      // not as a dependent of the router: griddepcontrol.wait then returns at once
      rc = launch_gate_up<FINITE, kWarpsPerBlock, kRing>(a, st, a.pdl_owner, 0);
    }
    if (rc || gate_up_only) return rc;
  }
  const size_t smem = (size_t)kWarpsPerBlock * kRingDown * 64 * 16 + (size_t)align16i(a.I + 8) * 2 + 32 * sizeof(float);
  if (smem > 48 * 1024) {
    int rc = ensure_max_smem((const void*)decode_down_v4<FINITE>, smem);
    if (rc) return rc;
  }
  const int ns = a.top_k + shared_slots(a);
  const int units = (a.dn_end ? a.dn_end : ns * (a.H >> 4)) - a.dn_begin;
  // the previous kernel is always this call's gate/up stage
  launch_decode(decode_down_v4<FINITE>, (units + kWarpsPerBlock - 1) / kWarpsPerBlock, smem, st, true, a);
  return check_launch("decode_down_v4");
}

int packed_decode(const DecodeArgs& a_in, cudaStream_t st, bool gate_up_only, uint32_t flags) {
  DecodeArgs a = a_in;
  const bool shared_only = (flags & GLM53_FLAG_SHARED_ONLY) != 0, skip_shared = (flags & GLM53_FLAG_SKIP_SHARED) != 0;
  if (shared_only || skip_shared) {
    if ((shared_only && skip_shared) || a.Is <= 0 || a.route_out || a.table || !tensor_core_shape(a)) {
      set_last_error("split decode: needs a shared expert, the tensor-core shapes, and one of the two flags");
      return GLM53_ERR_INVALID;
    }
    const int routed_units = a.top_k * (a.I >> 3), rtiles = a.H >> 4;
    if (shared_only) {  // the shared expert's gate/up and its down partial
      a.gu_begin = routed_units;
      a.gu_end = routed_units + (a.Is >> 3);
      a.dn_begin = a.top_k * rtiles;
      a.dn_end = (a.top_k + 1) * rtiles;
      a.dn_no_reduce = true;
    } else {  // the routed slots; the reduce adds the shared partial already in the workspace
      a.gu_end = routed_units;
      a.dn_end = a.top_k * rtiles;
      a.dn_expect = a.top_k;
    }
  }
  if (shared_only || skip_shared) a.after_router = false;
  a.shared_first = a.shared_first || a.after_router;
  if (!tensor_core_shape(a)) {
    const int items = a.top_k * a.I + a.Is;
    decode_gate_up_scalar_kernel<<<(items + 7) / 8, 256, 0, st>>>(a);
    int rc = check_launch("decode_gate_up_scalar_kernel");
    if (rc || gate_up_only) return rc;
    decode_down_scalar_kernel<<<(a.H + 7) / 8, 256, 0, st>>>(a);
    return check_launch("decode_down_scalar_kernel");
  }
  if (flags & GLM53_FLAG_E4M3_FINITE) return launch_v4<true>(a, st, gate_up_only);
  return launch_v4<false>(a, st, gate_up_only);
}

// Workspace: BF16 hidden rows | FP32 per-slot down dot products | counters.
struct DecodeWorkspace {
  size_t hidden, partial, counters, bytes;
};

static DecodeWorkspace decode_workspace(int top_k, int64_t H, int64_t I, int64_t I_shared) {
  DecodeWorkspace w;
  w.hidden = 0;
  w.partial = align_up(((size_t)top_k * I + (size_t)I_shared) * sizeof(uint16_t), 256);
  w.counters = w.partial + align_up((size_t)(top_k + 1) * H * sizeof(float), 256);
  w.bytes = w.counters + align_up((size_t)((H + 15) / 16) * sizeof(uint32_t), 256);
  return w;
}

static int check_geometry(const char* fn, int64_t H, int64_t I, int top_k, int64_t I_shared) {
  if (H <= 0 || I <= 0 || top_k <= 0 || top_k > kMaxSlots || I_shared < 0 || H > INT32_MAX / 2 ||
      I > INT32_MAX / 64 || I_shared > INT32_MAX / 64) {
    set_last_error("%s: invalid geometry H=%lld I=%lld top_k=%d I_shared=%lld", fn, (long long)H, (long long)I,
                   top_k, (long long)I_shared);
    return GLM53_ERR_INVALID;
  }
  return GLM53_OK;
}

static void fill_common(DecodeArgs& a, const void* x, int64_t H, const float* scores, int top_k, int64_t I,
                        const uint8_t* sg_w, const float* sg_s, const uint8_t* su_w, const float* su_s,
                        const uint8_t* sd_w, const float* sd_s, int64_t Is, float limit, void* out, void* workspace,
                        uint32_t* status) {
  a.x = (const uint16_t*)x;
  a.H = (int)H;
  a.I = (int)I;
  a.Is = (int)Is;
  a.top_k = top_k;
  a.scores = scores;
  a.sg_w = sg_w;
  a.sg_s = sg_s;
  a.su_w = su_w;
  a.su_s = su_s;
  a.sd_w = sd_w;
  a.sd_s = sd_s;
  a.limit = limit;
  const DecodeWorkspace wl = decode_workspace(top_k, H, I, Is);
  a.hidden = (uint16_t*)((char*)workspace + wl.hidden);
  a.partial = (float*)((char*)workspace + wl.partial);
  a.counters = (uint32_t*)((char*)workspace + wl.counters);
  a.out = (uint16_t*)out;
  a.status = status;
}

}  // namespace glm53

using namespace glm53;

extern "C" size_t glm53_packed_decode_workspace_bytes(int top_k, int64_t H, int64_t I, int64_t I_shared) {
  return decode_workspace(top_k, H, I, I_shared).bytes;
}

extern "C" int glm53_packed_decode_workspace_layout(int top_k, int64_t H, int64_t I, int64_t I_shared,
                                                    size_t* offsets) {
  if (!offsets || top_k <= 0 || H <= 0 || I <= 0 || I_shared < 0) {
    set_last_error("glm53_packed_decode_workspace_layout: invalid arguments");
    return GLM53_ERR_INVALID;
  }
  const DecodeWorkspace w = decode_workspace(top_k, H, I, I_shared);
  offsets[0] = w.hidden;
  offsets[1] = w.partial;
  return GLM53_OK;
}

static int packed_decode_moe_impl(const void* x, int64_t H, const uint32_t* expert_ids, const float* scores,
                                  int top_k, const uint8_t* gate_up_w, const float* gate_up_s, const uint8_t* down_w,
                                  const float* down_s, int64_t E, int64_t I, const uint8_t* shared_gate_w,
                                  const float* shared_gate_s, const uint8_t* shared_up_w, const float* shared_up_s,
                                  const uint8_t* shared_down_w, const float* shared_down_s, int64_t I_shared,
                                  float limit, void* out, void* workspace, size_t workspace_bytes, uint32_t* status,
                                  uint32_t flags, void* stream, bool trigger_after_wait);

extern "C" int glm53_packed_decode_moe(const void* x, int64_t H, const uint32_t* expert_ids, const float* scores,
                                       int top_k, const uint8_t* gate_up_w, const float* gate_up_s,
                                       const uint8_t* down_w, const float* down_s, int64_t E, int64_t I,
                                       const uint8_t* shared_gate_w, const float* shared_gate_s,
                                       const uint8_t* shared_up_w, const float* shared_up_s,
                                       const uint8_t* shared_down_w, const float* shared_down_s, int64_t I_shared,
                                       float limit, void* out, void* workspace, size_t workspace_bytes,
                                       uint32_t* status, uint32_t flags, void* stream) {
  return packed_decode_moe_impl(x, H, expert_ids, scores, top_k, gate_up_w, gate_up_s, down_w, down_s, E, I,
                                shared_gate_w, shared_gate_s, shared_up_w, shared_up_s, shared_down_w, shared_down_s,
                                I_shared, limit, out, workspace, workspace_bytes, status, flags, stream, false);
}

static int packed_decode_moe_impl(const void* x, int64_t H, const uint32_t* expert_ids, const float* scores,
                                  int top_k, const uint8_t* gate_up_w, const float* gate_up_s, const uint8_t* down_w,
                                  const float* down_s, int64_t E, int64_t I, const uint8_t* shared_gate_w,
                                  const float* shared_gate_s, const uint8_t* shared_up_w, const float* shared_up_s,
                                  const uint8_t* shared_down_w, const float* shared_down_s, int64_t I_shared,
                                  float limit, void* out, void* workspace, size_t workspace_bytes, uint32_t* status,
                                  uint32_t flags, void* stream, bool trigger_after_wait) {
  int rc = check_geometry("glm53_packed_decode_moe", H, I, top_k, I_shared);
  if (rc) return rc;
  const bool has_shared = I_shared > 0;
  if (E <= 0 || !x || !expert_ids || !scores || !gate_up_w || !gate_up_s || !down_w || !down_s || !out || !status ||
      !workspace || workspace_bytes < glm53_packed_decode_workspace_bytes(top_k, H, I, I_shared) ||
      (has_shared && (!shared_gate_w || !shared_gate_s || !shared_up_w || !shared_up_s || !shared_down_w ||
                      !shared_down_s))) {
    set_last_error("glm53_packed_decode_moe: missing pointer, E <= 0 or workspace too small");
    return GLM53_ERR_INVALID;
  }
  DecodeArgs a{};
  fill_common(a, x, H, scores, top_k, I, shared_gate_w, shared_gate_s, shared_up_w, shared_up_s, shared_down_w,
              shared_down_s, I_shared, limit, out, workspace, status);
  a.E = (int)std::min<int64_t>(E, INT32_MAX);
  a.ids = expert_ids;
  a.gu_w = gate_up_w;
  a.gu_s = gate_up_s;
  a.d_w = down_w;
  a.d_s = down_s;
  a.after_router = (flags & GLM53_FLAG_AFTER_ROUTER) != 0;
  a.trigger_after_wait = trigger_after_wait;
  return packed_decode(a, (cudaStream_t)stream, false, flags);
}

extern "C" int glm53_packed_decode_moe_hc(const void* x, int64_t H, const uint32_t* expert_ids, const float* scores,
                                          int top_k, const uint8_t* gate_up_w, const float* gate_up_s,
                                          const uint8_t* down_w, const float* down_s, int64_t E, int64_t I,
                                          const uint8_t* shared_gate_w, const float* shared_gate_s,
                                          const uint8_t* shared_up_w, const float* shared_up_s,
                                          const uint8_t* shared_down_w, const float* shared_down_s,
                                          int64_t I_shared, float limit, const void* residual, const float* post,
                                          const float* comb, void* out_state, void* workspace,
                                          size_t workspace_bytes, uint32_t* status, uint32_t flags, void* stream) {
  const char* fn = "glm53_packed_decode_moe_hc";
  int rc = check_geometry(fn, H, I, top_k, I_shared);
  if (rc) return rc;
  const bool has_shared = I_shared > 0;
  if (E <= 0 || !x || !expert_ids || !scores || !gate_up_w || !gate_up_s || !down_w || !down_s || !residual ||
      !post || !comb || !out_state || !status || !workspace ||
      workspace_bytes < glm53_packed_decode_workspace_bytes(top_k, H, I, I_shared) ||
      (has_shared && (!shared_gate_w || !shared_gate_s || !shared_up_w || !shared_up_s || !shared_down_w ||
                      !shared_down_s))) {
    set_last_error("%s: missing pointer, E <= 0 or workspace too small", fn);
    return GLM53_ERR_INVALID;
  }
  if (flags & GLM53_FLAG_SHARED_ONLY) {
    set_last_error("%s: GLM53_FLAG_SHARED_ONLY computes no output to expand", fn);
    return GLM53_ERR_INVALID;
  }
  DecodeArgs a{};
  fill_common(a, x, H, scores, top_k, I, shared_gate_w, shared_gate_s, shared_up_w, shared_up_s, shared_down_w,
              shared_down_s, I_shared, limit, nullptr, workspace, status);
  a.E = (int)std::min<int64_t>(E, INT32_MAX);
  a.ids = expert_ids;
  a.gu_w = gate_up_w;
  a.gu_s = gate_up_s;
  a.d_w = down_w;
  a.d_s = down_s;
  a.after_router = (flags & GLM53_FLAG_AFTER_ROUTER) != 0;
  a.hc_residual = (const uint16_t*)residual;
  a.hc_post = post;
  a.hc_comb = comb;
  a.hc_out = (uint16_t*)out_state;
  if (!tensor_core_shape(a)) {
    set_last_error("%s: H, I and I_shared must be multiples of 128 with 16-byte aligned tensors", fn);
    return GLM53_ERR_INVALID;
  }
  return packed_decode(a, (cudaStream_t)stream, false, flags);
}

extern "C" int glm53_selected_decode_moe(const void* x, int64_t H, const float* scores, int top_k,
                                         const uint8_t* const* gate_w, const float* const* gate_s,
                                         const uint8_t* const* up_w, const float* const* up_s,
                                         const uint8_t* const* down_w, const float* const* down_s, int64_t I,
                                         const uint8_t* shared_gate_w, const float* shared_gate_s,
                                         const uint8_t* shared_up_w, const float* shared_up_s,
                                         const uint8_t* shared_down_w, const float* shared_down_s,
                                         int64_t I_shared, float limit, void* out, void* workspace,
                                         size_t workspace_bytes, uint32_t* status, uint32_t flags, void* stream) {
  int rc = check_geometry("glm53_selected_decode_moe", H, I, top_k, I_shared);
  if (rc) return rc;
  const bool has_shared = I_shared > 0;
  if (!x || !scores || !gate_w || !gate_s || !up_w || !up_s || !down_w || !down_s || !out || !status ||
      !workspace || workspace_bytes < glm53_packed_decode_workspace_bytes(top_k, H, I, I_shared) ||
      (has_shared && (!shared_gate_w || !shared_gate_s || !shared_up_w || !shared_up_s || !shared_down_w ||
                      !shared_down_s))) {
    set_last_error("glm53_selected_decode_moe: missing pointer or workspace too small");
    return GLM53_ERR_INVALID;
  }
  DecodeArgs a{};
  fill_common(a, x, H, scores, top_k, I, shared_gate_w, shared_gate_s, shared_up_w, shared_up_s, shared_down_w,
              shared_down_s, I_shared, limit, out, workspace, status);
  a.E = top_k;
  a.table = true;
  for (int j = 0; j < top_k; ++j) {
    if (!gate_w[j] || !gate_s[j] || !up_w[j] || !up_s[j] || !down_w[j] || !down_s[j]) {
      set_last_error("glm53_selected_decode_moe: missing expert pointer for slot %d", j);
      return GLM53_ERR_INVALID;
    }
    a.tg_w[j] = gate_w[j];
    a.tg_s[j] = gate_s[j];
    a.tu_w[j] = up_w[j];
    a.tu_s[j] = up_s[j];
    a.td_w[j] = down_w[j];
    a.td_s[j] = down_s[j];
  }
  return packed_decode(a, (cudaStream_t)stream, false, flags);
}

extern "C" int glm53_decode_step_host(const glm53_decode_step_desc* d, const void* x_host, void* out_host,
                                      void* stream) {
  const char* fn = "glm53_decode_step_host";
  if (!d || !d->x || !d->out || d->top_k != 8 || d->H <= 0 || d->H % 128 != 0 || d->I <= 0 || d->I % 128 != 0 ||
      d->I_shared % 128 != 0 || (((uintptr_t)d->x | (uintptr_t)d->out) & 15) != 0) {
    set_last_error("%s: invalid descriptor (top_k 8, H and I multiples of 128, 16-byte aligned x and out)", fn);
    return GLM53_ERR_INVALID;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const size_t row = (size_t)d->H * 2;
  bool copy_kernel = false;
  if (x_host) {
    // a programmatic dependent of the previous step's down stage, which lets
    // it launch once no kernel of that step reads d->x any more
    cudaError_t e = small_copy(d->x, x_host, row, true, st, &copy_kernel, d->status, d->status_host, true);
    if (e != cudaSuccess) {
      set_last_error("%s: input copy: %s", fn, cudaGetErrorString(e));
      return GLM53_ERR_CUDA;
    }
  }
  if (d->status_host && !copy_kernel) {
    // the copy kernel did not mirror the status word: a one-thread kernel does
    const int mrc = mirror_status(d->status, d->status_host, st, fn);
    if (mrc) return mrc;
  }
  int rc = router_topk(d->x, 1, d->H, d->router_w, d->E, d->router_bias, d->top_k, d->n_group, d->topk_group,
                       d->norm_topk_prob, d->routed_scaling_factor, d->expert_ids, d->scores, nullptr,
                       d->router_workspace, d->router_workspace_bytes, st, copy_kernel);
  if (rc) return rc;
  void* mapped_out = out_host && (((uintptr_t)out_host) & 15) == 0 ? mapped_host(out_host) : nullptr;
  rc = packed_decode_moe_impl(d->x, d->H, d->expert_ids, d->scores, d->top_k, d->gate_up_w, d->gate_up_s, d->down_w,
                              d->down_s, d->E, d->I, d->shared_gate_w, d->shared_gate_s, d->shared_up_w,
                              d->shared_up_s, d->shared_down_w, d->shared_down_s, d->I_shared, d->limit,
                              mapped_out ? mapped_out : d->out, d->decode_workspace, d->decode_workspace_bytes,
                              d->status, d->flags | GLM53_FLAG_AFTER_ROUTER, stream, true);
  if (rc || !out_host || mapped_out) return rc;
  const cudaError_t e = cudaMemcpyAsync(out_host, d->out, row, cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) {
    set_last_error("%s: output copy: %s", fn, cudaGetErrorString(e));
    return GLM53_ERR_CUDA;
  }
  return GLM53_OK;
}

extern "C" int glm53_packed_decode_gate_up(const void* x, int64_t H, const uint32_t* expert_ids, int top_k,
                                           const uint8_t* gate_up_w, const float* gate_up_s, int64_t E, int64_t I,
                                           const uint8_t* shared_gate_w, const float* shared_gate_s,
                                           const uint8_t* shared_up_w, const float* shared_up_s, int64_t I_shared,
                                           float limit, void* workspace, size_t workspace_bytes, uint32_t* status,
                                           uint32_t flags, void* stream) {
  int rc = check_geometry("glm53_packed_decode_gate_up", H, I, top_k, I_shared);
  if (rc) return rc;
  const bool has_shared = I_shared > 0;
  if (E <= 0 || !x || !expert_ids || !gate_up_w || !gate_up_s || !status || !workspace ||
      workspace_bytes < glm53_packed_decode_workspace_bytes(top_k, H, I, I_shared) ||
      (has_shared && (!shared_gate_w || !shared_gate_s || !shared_up_w || !shared_up_s))) {
    set_last_error("glm53_packed_decode_gate_up: missing pointer, E <= 0 or workspace too small");
    return GLM53_ERR_INVALID;
  }
  DecodeArgs a{};
  // the down stage's pointers are unused by this stage; the shape check sees
  // the gate/up pointers in their place
  fill_common(a, x, H, nullptr, top_k, I, shared_gate_w, shared_gate_s, shared_up_w, shared_up_s,
              has_shared ? shared_gate_w : nullptr, shared_gate_s, I_shared, limit, nullptr, workspace, status);
  a.E = (int)std::min<int64_t>(E, INT32_MAX);
  a.ids = expert_ids;
  a.gu_w = gate_up_w;
  a.gu_s = gate_up_s;
  a.d_w = gate_up_w;
  return packed_decode(a, (cudaStream_t)stream, true, flags);
}

// ---------------------------------------------------------------------------
// Per-route decode (expert-parallel owners)
// ---------------------------------------------------------------------------

extern "C" size_t glm53_routes_decode_workspace_bytes(int64_t R, int64_t H, int64_t I) {
  return align_up((size_t)std::max<int64_t>(R, 1) * (size_t)I * sizeof(uint16_t), 256);
}

extern "C" int glm53_routes_decode(const void* x_rows, int64_t R, int64_t H, const uint32_t* expert_ids,
                                   const uint8_t* gate_up_w, const float* gate_up_s, const uint8_t* down_w,
                                   const float* down_s, int64_t E, int64_t I, float limit, void* out_rows,
                                   void* workspace, size_t workspace_bytes, uint32_t* status, uint32_t flags,
                                   void* stream) {
  const char* fn = "glm53_routes_decode";
  if (R < 0 || H <= 0 || I <= 0 || E <= 0 || H > INT32_MAX / 2 || I > INT32_MAX / 64 || R > INT32_MAX / I) {
    set_last_error("%s: invalid geometry R=%lld H=%lld I=%lld E=%lld", fn, (long long)R, (long long)H, (long long)I,
                   (long long)E);
    return GLM53_ERR_INVALID;
  }
  if (R == 0) return GLM53_OK;
  if (!x_rows || !expert_ids || !gate_up_w || !gate_up_s || !down_w || !down_s || !out_rows || !status ||
      !workspace || workspace_bytes < glm53_routes_decode_workspace_bytes(R, H, I)) {
    set_last_error("%s: missing pointer or workspace too small", fn);
    return GLM53_ERR_INVALID;
  }
  DecodeArgs a{};
  a.x = (const uint16_t*)x_rows;
  a.H = (int)H;
  a.I = (int)I;
  a.Is = 0;
  a.top_k = (int)R;
  a.E = (int)std::min<int64_t>(E, INT32_MAX);
  a.ids = expert_ids;
  a.gu_w = gate_up_w;
  a.gu_s = gate_up_s;
  a.d_w = down_w;
  a.d_s = down_s;
  a.limit = limit;
  a.hidden = (uint16_t*)workspace;
  a.status = status;
  a.x_stride = H;
  a.route_out = (uint16_t*)out_rows;
  if (!tensor_core_shape(a) || (((uintptr_t)out_rows) & 15) != 0) {
    set_last_error("%s: H and I must be multiples of 128 with 16-byte aligned tensors", fn);
    return GLM53_ERR_INVALID;
  }
  return packed_decode(a, (cudaStream_t)stream, false, flags);
}

extern "C" int glm53_ep_owner_decode_p2p(void* buffer, int64_t H, int world, int64_t capacity, int rank,
                                         const uint8_t* gate_up_w, const float* gate_up_s, const uint8_t* down_w,
                                         const float* down_s, int64_t E, int64_t I, const void* shared_x,
                                         int64_t T_shared, const uint8_t* shared_gate_w, const float* shared_gate_s,
                                         const uint8_t* shared_up_w, const float* shared_up_s,
                                         const uint8_t* shared_down_w, const float* shared_down_s, int64_t I_shared,
                                         void* shared_out, float limit, const unsigned long long* peer_base,
                                         void* workspace, size_t workspace_bytes, uint32_t* status, uint32_t flags,
                                         void* stream) {
  const char* fn = "glm53_ep_owner_decode_p2p";
  const bool has_shared = I_shared > 0 && T_shared > 0;
  if (world < 1 || world > 32 || rank < 0 || rank >= world || capacity <= 0 || H <= 0 || H % 64 != 0 || I <= 0 ||
      E <= 0 || (int64_t)world * capacity > (1 << 20) || H > INT32_MAX / 2 || I > INT32_MAX / 64 || T_shared < 0 ||
      T_shared > (1 << 16) || (has_shared && I_shared != I)) {
    set_last_error("%s: invalid geometry", fn);
    return GLM53_ERR_INVALID;
  }
  const int64_t R = (int64_t)world * capacity;
  if (!buffer || !gate_up_w || !gate_up_s || !down_w || !down_s || !peer_base || !status || !workspace ||
      workspace_bytes < glm53_routes_decode_workspace_bytes(R + (has_shared ? T_shared : 0), H, I) ||
      (has_shared && (!shared_x || !shared_gate_w || !shared_gate_s || !shared_up_w || !shared_up_s ||
                      !shared_down_w || !shared_down_s || !shared_out))) {
    set_last_error("%s: missing pointer or workspace too small", fn);
    return GLM53_ERR_INVALID;
  }
  const EpLayout lay = ep_layout(world, (int)capacity, H);
  char* b = (char*)buffer;
  DecodeArgs a{};
  a.x = (const uint16_t*)(b + lay.recv_x);
  a.H = (int)H;
  a.I = (int)I;
  a.Is = 0;
  a.top_k = (int)R;
  a.E = (int)std::min<int64_t>(E, INT32_MAX);
  a.ids = (const uint32_t*)(b + lay.recv_e);
  a.gu_w = gate_up_w;
  a.gu_s = gate_up_s;
  a.d_w = down_w;
  a.d_s = down_s;
  a.limit = limit;
  a.hidden = (uint16_t*)workspace;
  a.status = status;
  a.x_stride = H;
  a.route_out = (uint16_t*)(b + lay.back);  // marks per-route mode; rows go to the homes
  a.arrivals = (const unsigned long long*)(b + lay.cnt_dispatch);
  a.epoch = (const unsigned long long*)(b + lay.epoch);
  a.arrivals_per_step = (unsigned long long)R;
  a.wait_ns = ep_wait_limit_ns();
  a.peer_base = peer_base;
  a.back_off = (int64_t)lay.back;
  a.back_cnt_off = (int64_t)lay.cnt_back;
  a.rank = rank;
  a.cap = (int)capacity;
  a.shared_first = true;  // owner grid order (see DecodeArgs)
  a.pdl_owner = true;     // launched right after glm53_ep_dispatch_p2p (see DecodeArgs)
  if (has_shared) {  // the home tokens' shared expert rides in the same launches
    a.Is = (int)I_shared;
    a.n_shared = (int)T_shared;
    a.shared_x = (const uint16_t*)shared_x;
    a.shared_out = (uint16_t*)shared_out;
    a.sg_w = shared_gate_w;
    a.sg_s = shared_gate_s;
    a.su_w = shared_up_w;
    a.su_s = shared_up_s;
    a.sd_w = shared_down_w;
    a.sd_s = shared_down_s;
  }
  if (!tensor_core_shape(a) || (has_shared && (((uintptr_t)shared_x | (uintptr_t)shared_out) & 15) != 0)) {
    set_last_error("%s: H and I must be multiples of 128 with 16-byte aligned tensors", fn);
    return GLM53_ERR_INVALID;
  }
  return packed_decode(a, (cudaStream_t)stream, false, flags);
}

// ---------------------------------------------------------------------------
// Packed decode with a fixed, statically allocated scratch area.
//
// For callers that must not allocate device memory at call time: an engine
// whose own pool already owns all of HBM, or a latency-critical loop where an
// allocation (which may synchronise the device) is not acceptable.  The
// scratch lives in one file-scope device array per device; its address is
// looked up once per device and then reused, so a call allocates nothing.
// Every call on a device shares the array: calls whose GPU work overlaps
// (different streams, or other host threads) race on it.
// ---------------------------------------------------------------------------

namespace glm53 {
constexpr size_t kStaticScratchBytes = GLM53_STATIC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

constexpr int kMaxScratchDevices = 64;
static std::mutex g_scratch_mutex;
static void* g_scratch_ptr[kMaxScratchDevices];

// Address of this device's scratch array; the caller's device is current.
static int static_scratch(int device, void** out) {
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[device]) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (err != cudaSuccess || !p) {
      set_last_error("glm53_packed_decode_moe_static_scratch: cudaGetSymbolAddress failed on device %d: %s",
                     device, cudaGetErrorString(err));
      return GLM53_ERR_CUDA;
    }
    g_scratch_ptr[device] = p;
  }
  *out = g_scratch_ptr[device];
  return GLM53_OK;
}
}  // namespace glm53

extern "C" int glm53_packed_decode_moe_static_scratch(
    const void* x, int64_t H, const uint32_t* expert_ids, const float* scores, int top_k, const uint8_t* gate_up_w,
    const float* gate_up_s, const uint8_t* down_w, const float* down_s, int64_t E, int64_t I,
    const uint8_t* shared_gate_w, const float* shared_gate_s, const uint8_t* shared_up_w, const float* shared_up_s,
    const uint8_t* shared_down_w, const float* shared_down_s, int64_t I_shared, float limit, void* out,
    uint32_t* status, uint32_t flags, void* stream) {
  const char* fn = "glm53_packed_decode_moe_static_scratch";
  int rc = check_geometry(fn, H, I, top_k, I_shared);
  if (rc) return rc;
  const bool has_shared = I_shared > 0;
  if (E <= 0 || !x || !expert_ids || !scores || !gate_up_w || !gate_up_s || !down_w || !down_s || !out || !status ||
      (has_shared && (!shared_gate_w || !shared_gate_s || !shared_up_w || !shared_up_s || !shared_down_w ||
                      !shared_down_s))) {
    set_last_error("%s: missing pointer or E <= 0", fn);
    return GLM53_ERR_INVALID;
  }
  if (flags & GLM53_FLAG_AFTER_ROUTER) {
    // the counter clear below is a stream operation between the router and the
    // decode, so the decode cannot be the router's programmatic dependent
    set_last_error("%s: GLM53_FLAG_AFTER_ROUTER is not supported (the scratch counters are cleared on the stream "
                   "before the decode); call without it", fn);
    return GLM53_ERR_INVALID;
  }
  const DecodeWorkspace wl = decode_workspace(top_k, H, I, I_shared);
  if (wl.bytes > kStaticScratchBytes) {
    set_last_error("%s: needs %zu scratch bytes for top_k=%d H=%lld I=%lld I_shared=%lld, above the fixed maximum "
                   "of %zu; use glm53_packed_decode_moe with a caller-provided workspace",
                   fn, wl.bytes, top_k, (long long)H, (long long)I, (long long)I_shared, kStaticScratchBytes);
    return GLM53_ERR_INVALID;
  }
  int device = -1;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess || device < 0 || device >= kMaxScratchDevices) {
    set_last_error("%s: no usable current device (%d): %s", fn, device, cudaGetErrorString(err));
    return GLM53_ERR_CUDA;
  }
  void* scratch = nullptr;
  rc = static_scratch(device, &scratch);
  if (rc) return rc;
  // The completion counters must start at zero; a call that ended early
  // (invalid expert id, launch error) may have left them set.  Everything
  // else in the scratch area is written before it is read.
  err = cudaMemsetAsync((char*)scratch + wl.counters, 0, wl.bytes - wl.counters, (cudaStream_t)stream);
  if (err != cudaSuccess) {
    set_last_error("%s: clearing the completion counters failed: %s", fn, cudaGetErrorString(err));
    return GLM53_ERR_CUDA;
  }
  DecodeArgs a{};
  fill_common(a, x, H, scores, top_k, I, shared_gate_w, shared_gate_s, shared_up_w, shared_up_s, shared_down_w,
              shared_down_s, I_shared, limit, out, scratch, status);
  a.E = (int)std::min<int64_t>(E, INT32_MAX);
  a.ids = expert_ids;
  a.gu_w = gate_up_w;
  a.gu_s = gate_up_s;
  a.d_w = down_w;
  a.d_s = down_s;
  return packed_decode(a, (cudaStream_t)stream, false, flags);
}

// ---------------------------------------------------------------------------
// Bind-time E4M3 scan
// ---------------------------------------------------------------------------

namespace glm53 {
__global__ void e4m3_nan_scan_kernel(const uint8_t* __restrict__ w, int64_t n, uint32_t* __restrict__ count) {
  uint32_t c = 0;
  const int64_t n16 = n >> 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride) {
    const uint4 v = reinterpret_cast<const uint4*>(w)[i];
    const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      // a code whose low 7 bits are all ones becomes 0xFF after | 0x80, i.e. a
      // zero byte of z; the classic zero-byte test then flags it
      const uint32_t z = ~(words[t] | 0x80808080u);
      c += ((z - 0x01010101u) & ~z & 0x80808080u) ? 1u : 0u;
    }
  }
  for (int64_t i = (n16 << 4) + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    c += ((w[i] & 0x7Fu) == 0x7Fu) ? 1u : 0u;
  c = __reduce_add_sync(0xffffffffu, c);
  if ((threadIdx.x & 31) == 0 && c) atomicAdd(count, c);
}
}  // namespace glm53

extern "C" int glm53_e4m3_scan(const uint8_t* w, int64_t n, uint32_t* nan_count, void* stream) {
  if (n < 0 || (n > 0 && (!w || !nan_count)) || (((uintptr_t)w) & 15) != 0) {
    set_last_error("glm53_e4m3_scan: invalid arguments (16-byte aligned weights required)");
    return GLM53_ERR_INVALID;
  }
  if (n == 0) return GLM53_OK;
  const int blocks = std::max(1, std::min(sm_count() * 8, (int)((n / 16 + 255) / 256)));
  e4m3_nan_scan_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(w, n, nan_count);
  return check_launch("e4m3_nan_scan_kernel");
}
