// Grouped block-FP8 GEMM on the 5th-generation tensor cores (tcgen05, TMEM,
// TMA) for expert-sorted routes: the prefill projections of the grouped MoE
// (glm53_flash_mlx/grouped_fp8.py:206-321, Metal kernel K12 at
// grouped_fp8.py:30-154) and the dense shared expert.
//
// One CTA computes D = W . X^T for one tile of 128 weight rows x up to 128
// routes over the whole K, for one route descriptor (expert, first route,
// routes <= 128).  For the gate/up projection the 128 rows are 64 gate rows
// stacked on the matching 64 up rows, so one M=128 MMA produces both halves
// of 64 hidden rows.  Roles (persistent CTA, one per SM):
//   warp 0      TMA producer: raw E4M3 weight tiles [128 rows x 128 K] and
//               activation tiles [routes x 128 K] (FP16, two 64-K boxes,
//               128-byte swizzle) into two rings of their own depths;
//   warps 1, 14 issue tcgen05.mma (kind::f16, M128, N = 128, or 64 for a tile
//               of <= 64 routes; A from TMEM, B from shared memory, FP32
//               accumulation in TMEM), warp 1 the even k-blocks and warp 14
//               the odd ones: consecutive k-blocks write different
//               accumulators, and one thread's barrier waits and commit
//               (~300 cycles each) would leave the tensor core idle between
//               its k-blocks; per k-block an issuer checks that the
//               activations landed, that the epilogue has read the
//               accumulator, and that the A operand is decoded, then commits
//               once; warp 1 also allocates TMEM;
//   warps 2-5   decode each weight row exactly to FP16 (lut(c), or lut(c)/256
//               on the bit-exact path for banks holding 0x7F/0xFF) into a
//               4-deep TMEM ring (A operand, one TMEM lane per weight row);
//   warps 6-13  epilogue (two warps per TMEM lane quarter, 64 routes each):
//               after every 128-K block, read the block's partial product
//               from TMEM and promote it in FP32 with the 128x128 block scale
//               (tot += s_kb * P_kb), then apply the route's activation range
//               scale and store BF16 rows (gate/up tiles: the reference's BF16
//               gate and up values, [R][gate I | up I]; swiglu_rows applies
//               its BF16 SwiGLU).  The output phase is kept short: the
//               accumulator of the next tile's third k-block waits for it
//               (a trace put the SwiGLU epilogue formerly done here at ~17,000
//               cycles per tile, a third of the kernel).
// Products of FP16 weights (4 significant bits) and FP16 activations are
// exact in FP32, so each 128-K block sum differs from the reference's FP32
// sum only in summation order.  Activations are the BF16 inputs converted to
// FP16 after multiplication by a power of two 2^-e per route (e chosen so the
// row's largest magnitude stays below 2^15); the epilogue multiplies by 2^e.
// swiglu_rows takes the BF16 sigmoid from a 64K-entry table built on the
// device by sigmoid_bf16 itself (bit-identical, without the FP64 exponential).
//
// Measured tcgen05 cost on B200 (one thread issuing back-to-back M128 K16
// kind::f16 MMAs, A from TMEM or shared memory alike): 47 cycles at N=64, 64 at
// N=128, 128 at N=256 -- N=64 runs at two thirds of the tensor-core rate,
// hence the 128-route tiles.
//
// Every wait on an mbarrier is bounded (a deadline on the global timer); a
// CTA that gives up sets GLM53_STATUS_WAIT_TIMEOUT, lets its copies and MMAs
// drain, frees its TMEM and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gemv_tile.cuh"
#include "kernels.cuh"

namespace glm53 {
namespace tc {

constexpr int kM = 128;         // weight rows per tile (MMA M)
constexpr int kN = 128;         // routes per tile (MMA N: 128, or 64 for short tiles)
constexpr int kKB = 128;        // K per block-scale block
// Ring depths: a clock64 trace of one CTA per role put the k-block period at
// ~1,100 cycles with the MMA issuer waiting ~450 of them for activations; a
// 4-deep activation ring with a 4-deep weight ring (whose copies then queue
// less: ~3,100 cycles from issue to landing instead of ~6,500) measured 3%
// faster than 7 + 3.
constexpr int kRawStages = 4;   // weight ring (E4M3, 16 KB per stage)
constexpr int kActStages = 4;   // activation ring (FP16, 32 KB per stage), mostly L2 hits
constexpr int kRing = 4;        // decoded A operands in TMEM = k-block completion slots
constexpr int kThreads = 480;   // 15 warps
constexpr int kEpiWarps = 8;    // two per TMEM lane quarter, 64 routes each
constexpr int kRawBytes = kM * kKB;      // 16 KB of E4M3 per stage
constexpr int kActBox = kN * 64 * 2;     // one 64-K box of up to 128 routes (FP16)
constexpr int kActBytes = 2 * kActBox;   // 32 KB per stage
constexpr int kTmemCols = 512;
// TMEM columns: accumulators [2][kN] at 0, A operands [kRing][64] at 256
constexpr int kAccCol = 0;
constexpr int kACol = 256;
constexpr uint64_t kWaitNs = 200ull * 1000 * 1000;  // longest single wait

struct TcArgs {
  const uint32_t* tile_experts;
  const uint32_t* tile_starts;
  const uint32_t* tile_lengths;
  int dense;             // descriptors implicit: (0, kN d, min(kN, R - kN d))
  int R;                 // activation rows
  int K;                 // reduction length
  int E;
  int w_rows;            // gate (or plain) weight-map rows per expert
  int u_rows;            // up weight-map rows per expert
  int u_off;             // row offset of the up projection inside an expert
  const float* s_gate;   // block-scale rows of the gate (or plain) tile
  const float* s_up;     // block-scale rows of the up tile
  int64_t s_expert;      // floats between experts in both scale tables
  const float* xscale;   // per activation row multiplier 2^e
  float limit;
  int out_cols;          // columns of out (SwiGLU: I, plain: N)
  uint16_t* out;         // SwiGLU: FP16 hidden rows; plain: BF16 rows
  uint32_t* status;
  int splits;            // k-block ranges per tile (plain dense only)
  float* partial;        // [splits][R][out_cols] FP32 partial sums when splits > 1
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.b32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false when the CTA has aborted, or when this wait has run
// for longer than kWaitNs (which aborts the CTA).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if (mbar_try(bar, parity)) return true;
    if ((it & 63u) == 63u) {
      if (*abort_flag) return false;
      const uint64_t now = global_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kWaitNs) {
        *abort_flag = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] . B[smem]^T, kind::f16, cta_group::1.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T, kind::f16, cta_group::1.
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// Instruction descriptor: FP32 accumulate, FP16 A and B, both K-major,
// N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t make_idesc(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Shared-memory matrix descriptor of a K-major tile with 128-byte swizzle:
// rows of 128 bytes, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;            // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;  // stride byte offset
  d |= (uint64_t)1u << 46;            // descriptor version
  d |= (uint64_t)2u << 61;            // SWIZZLE_128B
  return d;
}

// ---------------------------------------------------------------------------
// SwiGLU sigmoid table
// ---------------------------------------------------------------------------

// sigmoid_bf16 of every BF16 bit pattern (built once per device).
__device__ uint16_t g_sigmoid_tab[65536];

__global__ void sigmoid_table_kernel() {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < 65536) g_sigmoid_tab[i] = f32_to_bf16_bits(sigmoid_bf16((uint16_t)i));
}

// swiglu_bf16 with the sigmoid looked up: the same operations and roundings.
__device__ __forceinline__ uint16_t swiglu_bf16_tab(float gate_total, float up_total, float limit) {
  const float gate_t = bf16_round(gate_total);
  const float up_t = bf16_round(up_total);
  const uint16_t ga = f32_to_bf16_bits(fminf(gate_t, limit));
  const float ua = bf16_round(fminf(fmaxf(up_t, -limit), limit));
  const float sig = bf16_bits_to_f32(__ldg(g_sigmoid_tab + ga));
  const float silu = bf16_round(__fmul_rn(bf16_bits_to_f32(ga), sig));
  return f32_to_bf16_bits(__fmul_rn(silu, ua));
}

// ---------------------------------------------------------------------------
// Kernel
// ---------------------------------------------------------------------------

// Barriers.  k-block g uses raw stage g % kRawStages and ring slot g % kRing
// (activation stage, A operand, completion barrier kb_done) and accumulator
// g % 2; kb_done[j] completes when the MMAs of k-block g = j (mod kRing) have
// finished: the slot's activations and A operand are free again and the
// accumulator holds the block's partial product.
struct __align__(8) Bars {
  uint64_t raw_full[kRawStages], raw_empty[kRawStages], act_full[kActStages], a_full[kRing], kb_done[kRing];
  uint64_t acc_empty[2], drain;
  uint32_t tmem_base;
  int abort_flag;
};

template <bool SWIGLU>
constexpr size_t smem_bytes() {
  return 1024 /* alignment slack */ + (size_t)kRawStages * kRawBytes + (size_t)kActStages * kActBytes +
         sizeof(Bars);
}

// Tile t of the persistent schedule: descriptor d = t / (mtiles * zsub), then
// the weight tile, then the route sub-chunk (weight tiles innermost, so the
// CTAs in flight share activation rows and an expert's chunks share weights
// through L2).  len == 0 marks an unused slot.
struct Tile {
  uint32_t e, start, len;
  int mt;
  int ks, kb0, kb1;  // split index and its k-block range [kb0, kb1)
};

template <bool SPLIT>
__device__ __forceinline__ Tile tile_at(const TcArgs& a, int t, int mtiles, int zsub) {
  Tile tl;
  const int nkb = a.K / kKB;
  if constexpr (SPLIT) {
    // the split index is innermost, so the CTAs of one tile's ranges run side
    // by side and share its activation rows through L2
    tl.ks = t % a.splits;
    tl.kb0 = (int)((int64_t)tl.ks * nkb / a.splits);
    tl.kb1 = (int)((int64_t)(tl.ks + 1) * nkb / a.splits);
    t /= a.splits;
  } else {
    tl.ks = 0;
    tl.kb0 = 0;
    tl.kb1 = nkb;
  }
  const int d = t / (mtiles * zsub);
  const int rem = t - d * mtiles * zsub;
  tl.mt = rem / zsub;
  const int z = rem - tl.mt * zsub;
  if (a.dense) {
    tl.e = 0;
    tl.start = (uint32_t)d * kN;
    tl.len = tl.start < (uint32_t)a.R ? min((uint32_t)kN, (uint32_t)a.R - tl.start) : 0u;
  } else {
    tl.e = __ldg(a.tile_experts + d);
    const uint32_t dstart = __ldg(a.tile_starts + d), dlen = __ldg(a.tile_lengths + d);
    const uint32_t off = (uint32_t)z * kN;
    tl.start = dstart + off;
    tl.len = dlen > off ? min((uint32_t)kN, dlen - off) : 0u;
    if (tl.len && tl.e >= (uint32_t)a.E) tl.len = 0;  // flagged once by the producer
  }
  return tl;
}

// Weight rows of tile mt: SwiGLU tiles hold hidden rows [64 mt, 64 mt + 64)
// (gate rows in TMEM lanes 0-63, up rows in lanes 64-127); plain tiles hold
// rows [128 mt, 128 mt + 128).
template <bool SWIGLU>
__device__ __forceinline__ int tile_row0(int mt) {
  return SWIGLU ? 64 * mt : kM * mt;
}

// Tensor maps: w (and u) boxes of 64 rows (SwiGLU) or 128 rows (plain) x 128
// K codes; x boxes of 128 routes and, for tiles of <= 64 routes, x64 boxes of
// 64 routes, each x 64 K.
template <bool SWIGLU, bool FINITE, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap umap,
                      const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap xmap64, TcArgs a,
                      int ntiles, int mtiles, int zsub) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* raw = smem;                                      // [stage][128][128] E4M3, swizzled
  uint8_t* act = raw + (size_t)kRawStages * kRawBytes;      // [stage][box 2][routes][128 B] FP16, swizzled
  Bars* bars = reinterpret_cast<Bars*>(act + (size_t)kActStages * kActBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = a.K / kKB;

  auto bar = [&](uint64_t* p) { return smem_addr(p); };
  if (threadIdx.x == 0) {
    for (int s = 0; s < kRawStages; ++s) {
      mbar_init(bar(&bars->raw_full[s]), 1);
      mbar_init(bar(&bars->raw_empty[s]), 4);
    }
    for (int s = 0; s < kActStages; ++s) mbar_init(bar(&bars->act_full[s]), 1);
    for (int s = 0; s < kRing; ++s) {
      mbar_init(bar(&bars->a_full[s]), 4);  // the four decode warps
      mbar_init(bar(&bars->kb_done[s]), 1);
    }
    for (int s = 0; s < 2; ++s) mbar_init(bar(&bars->acc_empty[s]), kEpiWarps);
    mbar_init(bar(&bars->drain), 2);      // one commit per MMA issuer
    bars->abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
    if (SWIGLU) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&umap)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap64)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(&bars->tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = bars->tmem_base;
  volatile int* abort_flag = &bars->abort_flag;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    // Two independent cursors over the same (tile, k-block) sequence: the
    // weight ring refills as soon as a stage is decoded, the activation ring
    // as soon as its MMAs completed.
    if (lane == 0) {
      struct Cursor {
        int t, kb;
        uint32_t g;  // k-blocks issued
        Tile tl;
      };
      auto first = [&](Cursor& c, int t) {
        for (c.t = t; c.t < ntiles; c.t += gridDim.x) {
          c.tl = tile_at<SPLIT>(a, c.t, mtiles, zsub);
          if (c.tl.len) {
            c.kb = c.tl.kb0;
            return;
          }
        }
      };
      auto advance = [&](Cursor& c) {
        ++c.g;
        if (++c.kb == c.tl.kb1) first(c, c.t + gridDim.x);
      };
      // flag used descriptors whose expert is out of range (skipped as empty)
      if (!a.dense) {  // (splits == 1 here)
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
          const int d = t / (mtiles * zsub);
          if ((t % (mtiles * zsub)) == 0 && __ldg(a.tile_lengths + d) && __ldg(a.tile_experts + d) >= (uint32_t)a.E)
            atomicOr(a.status, kStatusBadExpert);
          // a descriptor longer than the launch's sub-tiles cover is not computed past them
          if ((t % (mtiles * zsub)) == 0 && __ldg(a.tile_lengths + d) > (uint32_t)(zsub * kN))
            atomicOr(a.status, kStatusBadGeometry);
        }
      }
      Cursor cr{0, 0, 0u, Tile{}}, ca{0, 0, 0u, Tile{}};  // first() sets kb
      first(cr, blockIdx.x);
      first(ca, blockIdx.x);
      uint64_t t_idle = 0;
      while ((cr.t < ntiles || ca.t < ntiles) && !*abort_flag) {
        bool progress = false;
        if (cr.t < ntiles) {
          const int s = cr.g % kRawStages;
          if (mbar_try(bar(&bars->raw_empty[s]), ((cr.g / kRawStages) & 1u) ^ 1u)) {
            const uint32_t rf = bar(&bars->raw_full[s]);
            mbar_expect_tx(rf, kRawBytes);
            uint8_t* rs = raw + (size_t)s * kRawBytes;
            const int row0 = tile_row0<SWIGLU>(cr.tl.mt);
            tma_load_2d(smem_addr(rs), &wmap, cr.kb * kKB, (int)cr.tl.e * a.w_rows + row0, rf);
            if (SWIGLU)
              tma_load_2d(smem_addr(rs + kRawBytes / 2), &umap, cr.kb * kKB, (int)cr.tl.e * a.u_rows + a.u_off + row0,
                          rf);
            advance(cr);
            progress = true;
          }
        }
        // stage ca.g % kActStages is free once k-block ca.g - kActStages has completed
        const uint32_t prev = ca.g - kActStages;
        if (ca.t < ntiles &&
            (ca.g < (uint32_t)kActStages || mbar_try(bar(&bars->kb_done[prev % kRing]), (prev / kRing) & 1u))) {
          const int s = ca.g % kActStages;
          {
            const uint32_t af = bar(&bars->act_full[s]);
            const bool wide = ca.tl.len > 64;
            mbar_expect_tx(af, wide ? kActBytes : kActBytes / 2);
            uint8_t* as = act + (size_t)s * kActBytes;
            const CUtensorMap* xm = wide ? &xmap : &xmap64;
            tma_load_2d(smem_addr(as), xm, ca.kb * kKB, (int)ca.tl.start, af);
            tma_load_2d(smem_addr(as + kActBox), xm, ca.kb * kKB + 64, (int)ca.tl.start, af);
            advance(ca);
            progress = true;
          }
        }
        if (progress) {
          t_idle = 0;
        } else {
          const uint64_t now = global_ns();
          if (t_idle == 0) {
            t_idle = now;
          } else if (now - t_idle > kWaitNs) {
            *abort_flag = 1;
          }
        }
      }
      // let every issued copy land before the CTA can exit
      int zero = 0;
      for (uint32_t k = cr.g > (uint32_t)kRawStages ? cr.g - kRawStages : 0u; k < cr.g; ++k)
        mbar_wait(bar(&bars->raw_full[k % kRawStages]), (k / kRawStages) & 1u, &zero);
      for (uint32_t k = ca.g > (uint32_t)kActStages ? ca.g - kActStages : 0u; k < ca.g; ++k)
        mbar_wait(bar(&bars->act_full[k % kActStages]), (k / kActStages) & 1u, &zero);
    }
  } else if (warp == 1 || warp == 14) {
    // ---------------- MMA issuers (even / odd k-blocks) ----------------
    if (lane == 0) {
      const uint32_t parity = warp == 1 ? 0u : 1u;
      uint32_t g = 0;
      bool stop = false;
      for (int t = blockIdx.x; t < ntiles && !stop; t += gridDim.x) {
        const Tile tl = tile_at<SPLIT>(a, t, mtiles, zsub);
        if (tl.len == 0) continue;
        const uint32_t idesc = tl.len > 64 ? make_idesc(kM, kN) : make_idesc(kM, 64);
        for (int kb = tl.kb0; kb < tl.kb1; ++kb, ++g) {
          if ((g & 1u) != parity) continue;
          const int s = g % kRing;
          const int as = g % kActStages;
          const int cb = g & 1;
          if (!mbar_wait(bar(&bars->act_full[as]), (g / kActStages) & 1u, abort_flag) ||
              !mbar_wait(bar(&bars->acc_empty[g & 1]), ((g >> 1) & 1u) ^ 1u, abort_flag) ||
              !mbar_wait(bar(&bars->a_full[s]), (g / kRing) & 1u, abort_flag)) {
            stop = true;
            break;
          }
          tmem_fence_after();
          const uint32_t act_s = smem_addr(act + (size_t)as * kActBytes);
          const uint32_t d_t = tmem + kAccCol + cb * kN;
#pragma unroll
          for (int k16 = 0; k16 < kKB / 16; ++k16) {
            const uint32_t a_t = tmem + kACol + s * 64 + k16 * 8;
            const uint64_t b_desc = make_sw128_desc(act_s + (k16 >> 2) * kActBox + (k16 & 3) * 32);
            mma_f16_ts(d_t, a_t, b_desc, idesc, k16 > 0 ? 1u : 0u);
          }
          mma_commit(bar(&bars->kb_done[s]));
        }
      }
      // every MMA of both issuers has completed once both commits arrived
      int zero = 0;
      mma_commit(bar(&bars->drain));
      mbar_wait(bar(&bars->drain), 0, &zero);
    }
    __syncwarp();
  } else if (warp < 6) {
    // ---------------- weight decode into TMEM (A operand) ----------------
    const int q = warp & 3;       // TMEM lane quarter this warp may access
    const int r = q * 32 + lane;  // weight row of this thread = TMEM lane
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint32_t g = 0;
    bool stop = false;
    for (int t = blockIdx.x; t < ntiles && !stop; t += gridDim.x) {
      const Tile tl = tile_at<SPLIT>(a, t, mtiles, zsub);
      if (tl.len == 0) continue;
      for (int kb = tl.kb0; kb < tl.kb1; ++kb, ++g) {
        const int s = g % kRawStages;
        const int ab = g % kRing;
        const uint32_t ring_ph = (g / kRing) & 1u;
        // the whole warp waits and leaves together (tcgen05.st is warp-wide);
        // the A slot is free once k-block g - kRing has completed
        bool ok = __all_sync(0xffffffffu, mbar_wait(bar(&bars->raw_full[s]), (g / kRawStages) & 1u, abort_flag));
        ok = ok && __all_sync(0xffffffffu, mbar_wait(bar(&bars->kb_done[ab]), ring_ph ^ 1u, abort_flag));
        if (!ok) {
          stop = true;
          break;
        }
        tmem_fence_after();
        const uint8_t* line = raw + (size_t)s * kRawBytes + r * 128;
#pragma unroll
        for (int half = 0; half < 4; ++half) {  // 32 K codes -> 16 TMEM columns
          uint32_t v[16];
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const int c = half * 2 + cc;  // 16-byte chunk (16 codes) of the 128-byte row
            const uint4 w = *reinterpret_cast<const uint4*>(line + 16 * (c ^ (r & 7)));
            e4m3x4_frag<FINITE>(w.x, v[cc * 8 + 0], v[cc * 8 + 1]);
            e4m3x4_frag<FINITE>(w.y, v[cc * 8 + 2], v[cc * 8 + 3]);
            e4m3x4_frag<FINITE>(w.z, v[cc * 8 + 4], v[cc * 8 + 5]);
            e4m3x4_frag<FINITE>(w.w, v[cc * 8 + 6], v[cc * 8 + 7]);
          }
          tmem_st16(tmem + lane_base + kACol + ab * 64 + half * 16, v);
        }
        tmem_wait_st();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(&bars->raw_empty[s]));
        tmem_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(&bars->a_full[ab]));
      }
    }
  } else {
    // ---------------- epilogue: per-block promotion, then output ----------------
    // warp pair (w, w + 4) shares a TMEM lane quarter; half h takes routes
    // [64 h, 64 h + 64) of the tile
    const int q = warp & 3;
    const int h = (warp - 6) >> 2;
    const int r = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const bool up_rows = SWIGLU && q >= 2;  // TMEM lanes 64-127 hold the up rows
    uint32_t g = 0;
    bool stop = false;
    for (int t = blockIdx.x; t < ntiles && !stop; t += gridDim.x) {
      const Tile tl = tile_at<SPLIT>(a, t, mtiles, zsub);
      if (tl.len == 0) continue;
      const int row0 = tile_row0<SWIGLU>(tl.mt);
      const float* srow = (up_rows ? a.s_up : a.s_gate) + (size_t)tl.e * a.s_expert + (size_t)(row0 >> 7) * nkb;
      WarpScales sc;
      sc.load(srow, nkb, true);
      const uint32_t n0 = (uint32_t)h * 64;
      const bool active = n0 < tl.len;  // this half has routes
      // route range multipliers of this half: lane l holds routes n0 + l and
      // n0 + 32 + l (loaded ahead of the output phase)
      const float xa = (a.xscale && n0 + lane < tl.len) ? __ldg(a.xscale + tl.start + n0 + lane) : 1.0f;
      const float xb = (a.xscale && n0 + 32 + lane < tl.len) ? __ldg(a.xscale + tl.start + n0 + 32 + lane) : 1.0f;
      float tot[64];
#pragma unroll
      for (int n = 0; n < 64; ++n) tot[n] = 0.f;
      for (int kb = tl.kb0; kb < tl.kb1; ++kb, ++g) {
        const int cb = g & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(bar(&bars->kb_done[g % kRing]), (g / kRing) & 1u, abort_flag))) {
          stop = true;
          break;
        }
        tmem_fence_after();
        const float sk = sc.at(kb) * decode_unscale<FINITE>();
        if (active) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_base + kAccCol + cb * kN + n0, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) tot[i] = fmaf(sk, __uint_as_float(v[i]), tot[i]);
          tmem_ld32(tmem + lane_base + kAccCol + cb * kN + n0 + 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) tot[32 + i] = fmaf(sk, __uint_as_float(v[i]), tot[32 + i]);
        }
        tmem_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(&bars->acc_empty[cb]));
      }
      if (stop) break;
      if (!SWIGLU && SPLIT) {
        // this range's FP32 partial sums; the reduce kernel adds the ranges in
        // order and applies the route multiplier
        const int col = row0 + r;
        float* dst = a.partial + (size_t)tl.ks * a.R * a.out_cols;
#pragma unroll
        for (int n = 0; n < 64; ++n)
          if (n0 + n < tl.len && col < a.out_cols) dst[(size_t)(tl.start + n0 + n) * a.out_cols + col] = tot[n];
      } else {
        // BF16 output rows.  Plain tiles: column row0 + r.  SwiGLU tiles write
        // the [R, 2I] gate/up rows that swiglu_rows applies the activation to:
        // TMEM lanes 0-63 are gate rows (columns row0 + r), lanes 64-127 the
        // matching up rows (columns I + row0 + r - 64).
        const int col = SWIGLU ? (r < 64 ? row0 + r : (a.out_cols >> 1) + row0 + r - 64) : row0 + r;
        if ((reinterpret_cast<uintptr_t>(a.out) & 3u) == 0) {
          // lane pairs exchange values so that each store writes two adjacent
          // columns (out_cols is a multiple of 8): half the store instructions
          // of the output phase, which the next tile's accumulators wait for
          const uint32_t odd = lane & 1u;
          const int colw = col - (int)odd;
#pragma unroll
          for (int n = 0; n < 64; n += 2) {
            const float x0 = __shfl_sync(0xffffffffu, n < 32 ? xa : xb, n & 31);
            const float x1 = __shfl_sync(0xffffffffu, n < 32 ? xa : xb, (n + 1) & 31);
            const uint32_t b0 = f32_to_bf16_bits(tot[n] * x0), b1 = f32_to_bf16_bits(tot[n + 1] * x1);
            const uint32_t got = __shfl_xor_sync(0xffffffffu, odd ? b0 : b1, 1);
            const uint32_t word = odd ? (got | (b1 << 16)) : (b0 | (got << 16));
            const uint32_t rn = n + odd;
            // the last weight tile of a plain GEMM may extend past N (TMA zero-fills those rows)
            if (n0 + rn < tl.len && colw < a.out_cols)
              *reinterpret_cast<uint32_t*>(a.out + (size_t)(tl.start + n0 + rn) * a.out_cols + colw) = word;
          }
        } else {
#pragma unroll
          for (int n = 0; n < 64; ++n) {
            const float x = __shfl_sync(0xffffffffu, n < 32 ? xa : xb, n & 31);
            if (n0 + n < tl.len && col < a.out_cols)
              a.out[(size_t)(tl.start + n0 + n) * a.out_cols + col] = f32_to_bf16_bits(tot[n] * x);
          }
        }
      }
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && bars->abort_flag) atomicOr(a.status, kStatusWaitTimeout);
  if (warp == 1) {
    tmem_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// FP8 tensor-core variant (tcgen05.mma kind::f8f6f4)
// ---------------------------------------------------------------------------
//
// The E4M3 weight tiles feed the MMA straight from shared memory: no decode
// warps and no A operand in TMEM.  Each activation row arrives as two E4M3
// terms of x * 2^-e (hi = E4M3(x 2^-e), lo = E4M3(x 2^-e - hi), written by
// split_rows_kernel), with the row maximum scaled into [128, 256).  A BF16
// value has 8 significant bits and hi holds the top 4, so hi + lo = x 2^-e
// exactly for every element within 2^9 of its row maximum (lo then stays a
// normal or subnormal E4M3 multiple of 2^-9); a smaller element keeps an
// absolute error below 2^-10 in the scaled domain.  Products of two E4M3
// values are exact in FP32, so every 128-K block sum is a sum of exact
// products, as in the kind::f16 kernel.
//
// A CTA tile is two 128-row weight sub-tiles against one activation tile of
// up to 128 routes: SwiGLU gate rows [128 mt, +128) and the matching up rows
// (TMEM lane r then holds the gate and the up total of hidden row 128 mt + r,
// so the epilogue needs no exchange), or plain output rows [256 mt, +128) and
// [256 mt + 128, +128).  Per 128-K block: 2 sub-tiles x 2 terms x 4 MMAs of
// M128 x N x K32 into the k-block's accumulator pair; TMEM holds two pairs
// (512 columns), so the epilogue's per-block promotion overlaps the next
// block's MMAs.  Each activation tile serves 256 weight rows, half the
// activation traffic per weight byte of the kind::f16 kernel.
// Roles: warp 0 TMA producer (weight ring and activation ring, two cursors);
// warps 1 and 2 issue the even and odd k-blocks; warps 3-18 epilogue (four
// per TMEM lane quarter, 32 routes each).
namespace f8 {
constexpr int kWStages = 4;                     // weight ring: two 128x128 E4M3 sub-tiles per stage
constexpr int kAStages = 3;                     // activation ring: hi and lo tiles of up to 128 routes
constexpr int kDone = 4;                        // k-block completion barriers
constexpr int kSub = kM * kKB;                  // 16 KB: one sub-tile, or one term tile of 128 routes
constexpr int kWBytes = 2 * kSub;
constexpr int kABytes = 2 * kSub;
constexpr int kEpiWarps = 16;
constexpr int kThreads = (3 + kEpiWarps) * 32;  // 608
static_assert(kWStages == kDone, "weight stages are released by the completion barrier of the same slot");
static_assert(kAStages < kDone, "an activation stage is released by an older completion barrier");

struct __align__(8) Bars {
  uint64_t w_full[kWStages], a_full[kAStages], kb_done[kDone], acc_empty[2], drain;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t smem_bytes() {
  return 1024 /* alignment slack */ + (size_t)kWStages * kWBytes + (size_t)kAStages * kABytes + sizeof(Bars);
}
static_assert(smem_bytes() <= 232448, "F8 tile rings exceed the shared memory of one CTA");

// D[tmem] (+)= A[smem] . B[smem]^T, kind::f8f6f4 (E4M3 x E4M3, FP32 accumulation), cta_group::1.
__device__ __forceinline__ void mma_f8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// First weight row of sub-tile `sub` of tile mt inside one expert's rows.
template <bool SWIGLU>
__device__ __forceinline__ int sub_row0(const TcArgs& a, int mt, int sub) {
  return SWIGLU ? (sub ? a.u_off : 0) + kM * mt : 2 * kM * mt + sub * kM;
}
}  // namespace f8

// Tensor maps: w and u boxes of 128 rows x 128 codes; x and x64 boxes of 128
// and 64 routes x 128 bytes over the [R][hi K | lo K] term rows.
template <bool SWIGLU>
__global__ void __launch_bounds__(f8::kThreads, 1)
    grouped_f8_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap umap,
                      const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap xmap64, TcArgs a,
                      int ntiles, int mtiles, int zsub) {
  using f8::kWStages;
  using f8::kAStages;
  using f8::kDone;
  using f8::kSub;
  using f8::kWBytes;
  using f8::kABytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* wring = smem;                                  // [stage][sub 2][128 rows][128 B], swizzled
  uint8_t* aring = wring + (size_t)kWStages * kWBytes;    // [stage][term 2][routes][128 B], swizzled
  f8::Bars* bars = reinterpret_cast<f8::Bars*>(aring + (size_t)kAStages * kABytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = a.K / kKB;

  auto bar = [&](uint64_t* p) { return smem_addr(p); };
  if (threadIdx.x == 0) {
    for (int s = 0; s < kWStages; ++s) mbar_init(bar(&bars->w_full[s]), 1);
    for (int s = 0; s < kAStages; ++s) mbar_init(bar(&bars->a_full[s]), 1);
    for (int s = 0; s < kDone; ++s) mbar_init(bar(&bars->kb_done[s]), 1);
    for (int s = 0; s < 2; ++s) mbar_init(bar(&bars->acc_empty[s]), f8::kEpiWarps);
    mbar_init(bar(&bars->drain), 2);  // one commit per MMA issuer
    bars->abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
    if (SWIGLU) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&umap)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap64)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(&bars->tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = bars->tmem_base;
  volatile int* abort_flag = &bars->abort_flag;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    // k-block g uses weight stage g % kWStages and activation stage
    // g % kAStages; a stage is free again once the k-block that last used it
    // (g - kWStages, g - kAStages) has completed.  Completion barrier j
    // serves k-blocks j, j + kDone, ...: k-block p + kDone cannot complete
    // before both cursors have seen p complete (it needs the stages they
    // refill after p), so one parity bit identifies p.
    if (lane == 0) {
      struct Cursor {
        int t, kb;
        uint32_t g;
        Tile tl;
      };
      auto first = [&](Cursor& c, int t) {
        for (c.t = t; c.t < ntiles; c.t += gridDim.x) {
          c.tl = tile_at<false>(a, c.t, mtiles, zsub);
          if (c.tl.len) {
            c.kb = c.tl.kb0;
            return;
          }
        }
      };
      auto advance = [&](Cursor& c) {
        ++c.g;
        if (++c.kb == c.tl.kb1) first(c, c.t + gridDim.x);
      };
      auto done = [&](uint32_t p) { return mbar_try(bar(&bars->kb_done[p % kDone]), (p / kDone) & 1u); };
      if (!a.dense) {
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
          const int d = t / (mtiles * zsub);
          if ((t % (mtiles * zsub)) == 0 && __ldg(a.tile_lengths + d) && __ldg(a.tile_experts + d) >= (uint32_t)a.E)
            atomicOr(a.status, kStatusBadExpert);
          if ((t % (mtiles * zsub)) == 0 && __ldg(a.tile_lengths + d) > (uint32_t)(zsub * kN))
            atomicOr(a.status, kStatusBadGeometry);
        }
      }
      Cursor cw{0, 0, 0u, Tile{}}, ca{0, 0, 0u, Tile{}};
      first(cw, blockIdx.x);
      first(ca, blockIdx.x);
      uint64_t t_idle = 0;
      while ((cw.t < ntiles || ca.t < ntiles) && !*abort_flag) {
        bool progress = false;
        if (cw.t < ntiles && (cw.g < (uint32_t)kWStages || done(cw.g - kWStages))) {
          const int s = cw.g % kWStages;
          const uint32_t wf = bar(&bars->w_full[s]);
          mbar_expect_tx(wf, kWBytes);
          uint8_t* ws = wring + (size_t)s * kWBytes;
          tma_load_2d(smem_addr(ws), &wmap, cw.kb * kKB,
                      (int)cw.tl.e * a.w_rows + f8::sub_row0<SWIGLU>(a, cw.tl.mt, 0), wf);
          if (SWIGLU)
            tma_load_2d(smem_addr(ws + kSub), &umap, cw.kb * kKB,
                        (int)cw.tl.e * a.u_rows + f8::sub_row0<SWIGLU>(a, cw.tl.mt, 1), wf);
          else
            tma_load_2d(smem_addr(ws + kSub), &wmap, cw.kb * kKB,
                        (int)cw.tl.e * a.w_rows + f8::sub_row0<SWIGLU>(a, cw.tl.mt, 1), wf);
          advance(cw);
          progress = true;
        }
        if (ca.t < ntiles && (ca.g < (uint32_t)kAStages || done(ca.g - kAStages))) {
          const int s = ca.g % kAStages;
          const uint32_t af = bar(&bars->a_full[s]);
          const bool wide = ca.tl.len > 64;
          mbar_expect_tx(af, wide ? 2 * kSub : kSub);
          uint8_t* as = aring + (size_t)s * kABytes;
          const CUtensorMap* xm = wide ? &xmap : &xmap64;
          tma_load_2d(smem_addr(as), xm, ca.kb * kKB, (int)ca.tl.start, af);               // hi terms
          tma_load_2d(smem_addr(as + kSub), xm, a.K + ca.kb * kKB, (int)ca.tl.start, af);  // lo terms
          advance(ca);
          progress = true;
        }
        if (progress) {
          t_idle = 0;
        } else {
          const uint64_t now = global_ns();
          if (t_idle == 0) {
            t_idle = now;
          } else if (now - t_idle > kWaitNs) {
            *abort_flag = 1;
          }
        }
      }
      int zero = 0;
      for (uint32_t k = cw.g > (uint32_t)kWStages ? cw.g - kWStages : 0u; k < cw.g; ++k)
        mbar_wait(bar(&bars->w_full[k % kWStages]), (k / kWStages) & 1u, &zero);
      for (uint32_t k = ca.g > (uint32_t)kAStages ? ca.g - kAStages : 0u; k < ca.g; ++k)
        mbar_wait(bar(&bars->a_full[k % kAStages]), (k / kAStages) & 1u, &zero);
    }
  } else if (warp == 1 || warp == 2) {
    // ---------------- MMA issuers (even / odd k-blocks) ----------------
    if (lane == 0) {
      const uint32_t parity = (uint32_t)(warp - 1);
      uint32_t g = 0;
      bool stop = false;
      for (int t = blockIdx.x; t < ntiles && !stop; t += gridDim.x) {
        const Tile tl = tile_at<false>(a, t, mtiles, zsub);
        if (tl.len == 0) continue;
        // E4M3 A and B: format code 0 in both fields, as F16 is for kind::f16
        const uint32_t idesc = tl.len > 64 ? make_idesc(kM, kN) : make_idesc(kM, 64);
        for (int kb = tl.kb0; kb < tl.kb1; ++kb, ++g) {
          if ((g & 1u) != parity) continue;
          const int ws = g % kWStages, as = g % kAStages, cb = g & 1;
          if (!mbar_wait(bar(&bars->w_full[ws]), (g / kWStages) & 1u, abort_flag) ||
              !mbar_wait(bar(&bars->a_full[as]), (g / kAStages) & 1u, abort_flag) ||
              !mbar_wait(bar(&bars->acc_empty[cb]), ((g >> 1) & 1u) ^ 1u, abort_flag)) {
            stop = true;
            break;
          }
          tmem_fence_after();
          const uint32_t w_s = smem_addr(wring + (size_t)ws * kWBytes);
          const uint32_t a_s = smem_addr(aring + (size_t)as * kABytes);
#pragma unroll
          for (int sub = 0; sub < 2; ++sub) {
            const uint32_t d_t = tmem + cb * (2 * kN) + sub * kN;
#pragma unroll
            for (int term = 0; term < 2; ++term) {
#pragma unroll
              for (int k32 = 0; k32 < kKB / 32; ++k32) {
                const uint64_t a_desc = make_sw128_desc(w_s + sub * kSub + k32 * 32);
                const uint64_t b_desc = make_sw128_desc(a_s + term * kSub + k32 * 32);
                f8::mma_f8_ss(d_t, a_desc, b_desc, idesc, (term | k32) ? 1u : 0u);
              }
            }
          }
          mma_commit(bar(&bars->kb_done[g % kDone]));
        }
      }
      int zero = 0;
      mma_commit(bar(&bars->drain));
      mbar_wait(bar(&bars->drain), 0, &zero);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: per-block promotion, then output ----------------
    const int q = warp & 3;         // TMEM lane quarter
    const int h = (warp - 3) >> 2;  // routes [32 h, 32 h + 32) of the tile
    const int r = q * 32 + lane;    // weight row of each sub-tile = TMEM lane
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint32_t g = 0;
    bool stop = false;
    for (int t = blockIdx.x; t < ntiles && !stop; t += gridDim.x) {
      const Tile tl = tile_at<false>(a, t, mtiles, zsub);
      if (tl.len == 0) continue;
      const size_t sbase = (size_t)tl.e * a.s_expert;
      const float* srow0 = a.s_gate + sbase + (size_t)(SWIGLU ? tl.mt : 2 * tl.mt) * nkb;
      const float* srow1 = SWIGLU ? a.s_up + sbase + (size_t)tl.mt * nkb : a.s_gate + sbase + (size_t)(2 * tl.mt + 1) * nkb;
      WarpScales sc0, sc1;
      sc0.load(srow0, nkb, true);
      sc1.load(srow1, nkb, true);
      const uint32_t n0 = (uint32_t)h * 32;
      const bool active = n0 < tl.len;
      // lane l holds the range multiplier of route n0 + l (loaded ahead of the output phase)
      const float xl = (a.xscale && n0 + lane < tl.len) ? __ldg(a.xscale + tl.start + n0 + lane) : 1.0f;
      float t0[32], t1[32];
#pragma unroll
      for (int n = 0; n < 32; ++n) t0[n] = t1[n] = 0.f;
      for (int kb = tl.kb0; kb < tl.kb1; ++kb, ++g) {
        const int cb = g & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(bar(&bars->kb_done[g % kDone]), (g / kDone) & 1u, abort_flag))) {
          stop = true;
          break;
        }
        tmem_fence_after();
        const float s0 = sc0.at(kb), s1 = sc1.at(kb);
        if (active) {
          const uint32_t acc = tmem + lane_base + cb * (2 * kN) + n0;
          uint32_t v[16];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tmem_ld16(acc + c * 16, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) t0[c * 16 + i] = fmaf(s0, __uint_as_float(v[i]), t0[c * 16 + i]);
            tmem_ld16(acc + kN + c * 16, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) t1[c * 16 + i] = fmaf(s1, __uint_as_float(v[i]), t1[c * 16 + i]);
          }
        }
        tmem_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(&bars->acc_empty[cb]));
      }
      if (stop) break;
      // Output: BF16 rows.  The accumulator pair of the next tile's third
      // k-block waits for this phase, so it is kept short: no activation here
      // (gate/up tiles write the reference's BF16 gate and up values to the
      // [R][gate I | up I] rows that swiglu_split applies the SwiGLU to), and
      // lane pairs exchange values so that each store writes two adjacent
      // columns.  Sub-tile 0 goes to column col0, sub-tile 1 to col0 + c1.
      const uint32_t odd = lane & 1u;
      {
        const int col0 = (SWIGLU ? kM * tl.mt : 2 * kM * tl.mt) + r - (int)odd;
        const int c1 = SWIGLU ? (a.out_cols >> 1) : kM;
#pragma unroll
        for (int n = 0; n < 32; n += 2) {
          const float x0 = __shfl_sync(0xffffffffu, xl, n), x1 = __shfl_sync(0xffffffffu, xl, n + 1);
#pragma unroll
          for (int sub = 0; sub < 2; ++sub) {
            const float* tt = sub ? t1 : t0;
            const uint32_t b0 = f32_to_bf16_bits(tt[n] * x0), b1 = f32_to_bf16_bits(tt[n + 1] * x1);
            const uint32_t got = __shfl_xor_sync(0xffffffffu, odd ? b0 : b1, 1);
            const uint32_t word = odd ? (got | (b1 << 16)) : (b0 | (got << 16));
            const uint32_t rn = n + odd;
            const int col = col0 + sub * c1;
            if (n0 + rn < tl.len && col < a.out_cols)
              *reinterpret_cast<uint32_t*>(a.out + (size_t)(tl.start + n0 + rn) * a.out_cols + col) = word;
          }
        }
      }
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && bars->abort_flag) atomicOr(a.status, kStatusWaitTimeout);
  if (warp == 1) {
    tmem_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}


// ---------------------------------------------------------------------------
// FP32 router logits on the tensor cores (T > 32 tokens)
// ---------------------------------------------------------------------------
//
// logits[t][e] = x[t] . w[e] with x BF16 [T, H] and w FP32 [E, H].  Every FP32
// weight is the exact sum of three BF16 numbers (planes [3][E][H], split once
// per call), and BF16 x BF16 products are exact in FP32, so the logit is a sum
// of exact products.  A CTA tile is 128 expert rows x 64 tokens over one
// range of K: per 128-K block, 3 planes x 8 tcgen05.mma kind::f16 (BF16,
// M128 x N64 x K16) accumulate into one TMEM accumulator, and the epilogue
// adds the block's sum into a double-FP32 total (TwoSum: ~48 significant
// bits).  A product's path thus holds at most 24 FP32 additions inside the
// block and the exact-to-2^-48 block total; each range stores its total as
// FP64 and router_logits_reduce adds the ranges in range order.  (The
// mma.sync kernel it replaces for T > 32 sums 16-wide slices the same way, at
// ~130 TFLOP/s on B200.)
// Roles: warp 0 TMA producer (4-stage ring of 64-K stages: the three planes'
// 128-row tiles and the token tile); warp 1 MMA issuer (and TMEM owner);
// warps 2-17 epilogue (four per TMEM lane quarter, 16 tokens each: the
// double-FP32 totals of 32 tokens per thread did not fit the registers).
namespace rt {
constexpr int kStages = 4;
constexpr int kStageK = 64;                     // 128-byte swizzle rows of BF16
constexpr int kTokens = 64;                     // tokens per tile (MMA N)
constexpr int kTile = 128 * kStageK * 2;        // 16 KB: 128 expert rows x 64 K
constexpr int kXTile = kTokens * kStageK * 2;   // 8 KB: 64 tokens x 64 K
constexpr int kStageBytes = 3 * kTile + kXTile;
constexpr int kEpiWarps = 16;
constexpr int kThreads = (2 + kEpiWarps) * 32;  // 576
constexpr int kCols = 128;                      // two accumulators of 64 tokens

struct __align__(8) Bars {
  uint64_t full[kStages], empty[kStages], acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t smem_bytes() { return 1024 + (size_t)kStages * kStageBytes + sizeof(Bars); }
static_assert(smem_bytes() <= 232448, "router stages exceed the shared memory of one CTA");
}  // namespace rt

// Tensor maps: wmap over the planes as [3E, H] rows (box 64 K x 128 rows;
// rows past a plane's E belong to the next plane or are zero-filled and only
// reach logits of experts >= E, which are not stored), xmap over [T, H].
__global__ void __launch_bounds__(rt::kThreads, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, int T, int H,
                     int E, int nkb, int splits, double* __restrict__ partial, uint32_t* abort_out) {
  using namespace rt;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  rt::Bars* bars = reinterpret_cast<rt::Bars*>(smem + (size_t)kStages * kStageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // tile: expert block ey, token block tx, K range z
  const int z = blockIdx.x % splits;
  const int tile = blockIdx.x / splits;
  const int ey = tile % ((E + 127) / 128), tx = tile / ((E + 127) / 128);
  const int e0 = ey * 128, t0 = tx * rt::kTokens;
  // this range's 128-K blocks [kb0, kb1) and 64-K stages
  const int kb0 = (int)((int64_t)z * nkb / splits), kb1 = (int)((int64_t)(z + 1) * nkb / splits);
  const int nstage = 2 * (kb1 - kb0);
  auto bar = [&](uint64_t* p) { return smem_addr(p); };
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(&bars->full[s]), 1);
      mbar_init(bar(&bars->empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(&bars->acc_full[s]), 1);
      mbar_init(bar(&bars->acc_empty[s]), rt::kEpiWarps);
    }
    bars->abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(&bars->tmem_base)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = bars->tmem_base;
  volatile int* abort_flag = &bars->abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      int zero = 0;
      for (int i = 0; i < nstage && !*abort_flag; ++i) {
        const int s = i % kStages;
        if (i >= kStages && !mbar_wait(bar(&bars->empty[s]), ((i / kStages) - 1) & 1u, abort_flag)) break;
        const uint32_t f = bar(&bars->full[s]);
        mbar_expect_tx(f, kStageBytes);
        uint8_t* st = smem + (size_t)s * kStageBytes;
        const int k = (2 * kb0 + i) * kStageK;
#pragma unroll
        for (int p = 0; p < 3; ++p) tma_load_2d(smem_addr(st + p * kTile), &wmap, k, p * E + e0, f);
        tma_load_2d(smem_addr(st + 3 * kTile), &xmap, k, t0, f);  // tokens past T: zero-filled
      }
      // let every issued copy land before the CTA can exit
      for (int i = nstage > kStages ? nstage - kStages : 0; i < nstage; ++i)
        mbar_wait(bar(&bars->full[i % kStages]), (i / kStages) & 1u, &zero);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // BF16 A and B (format code 1 in both fields), FP32 accumulation
      const uint32_t idesc = make_idesc(128, kTokens) | (1u << 7) | (1u << 10);
      bool stop = false;
      for (int b = 0; b < kb1 - kb0 && !stop; ++b) {
        const int cb = b & 1;
        if (!mbar_wait(bar(&bars->acc_empty[cb]), ((b >> 1) & 1u) ^ 1u, abort_flag)) break;
        tmem_fence_after();
        const uint32_t d_t = tmem + cb * kTokens;
        for (int h = 0; h < 2; ++h) {
          const int i = 2 * b + h, s = i % kStages;
          if (!mbar_wait(bar(&bars->full[s]), (i / kStages) & 1u, abort_flag)) {
            stop = true;
            break;
          }
          tmem_fence_after();
          const uint32_t st = smem_addr(smem + (size_t)s * kStageBytes);
#pragma unroll
          for (int p = 0; p < 3; ++p)
#pragma unroll
            for (int k16 = 0; k16 < kStageK / 16; ++k16)
              mma_f16_ss(d_t, make_sw128_desc(st + p * kTile + k16 * 32),
                             make_sw128_desc(st + 3 * kTile + k16 * 32), idesc, (h | p | k16) ? 1u : 0u);
          mma_commit(bar(&bars->empty[s]));
        }
        if (!stop) mma_commit(bar(&bars->acc_full[cb]));
      }
    }
    __syncwarp();
  } else {
    // epilogue: TMEM lane = expert row e0 + r; tokens [16 h, 16 h + 16)
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;
    const int r = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    float s_[16], c_[16];
#pragma unroll
    for (int n = 0; n < 16; ++n) s_[n] = c_[n] = 0.f;
    bool ok = true;
    for (int b = 0; b < kb1 - kb0; ++b) {
      const int cb = b & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(bar(&bars->acc_full[cb]), (b >> 1) & 1u, abort_flag))) {
        ok = false;
        break;
      }
      tmem_fence_after();
      uint32_t v[16];
      tmem_ld16(tmem + lane_base + cb * kTokens + 16 * h, v);
      tmem_wait_ld();
#pragma unroll
      for (int n = 0; n < 16; ++n) {  // TwoSum(s, v): s + v = t + (error, added to c)
        const float vv = __uint_as_float(v[n]);
        const float t = __fadd_rn(s_[n], vv);
        const float bp = __fsub_rn(t, s_[n]);
        const float e = __fadd_rn(__fsub_rn(s_[n], __fsub_rn(t, bp)), __fsub_rn(vv, bp));
        c_[n] = __fadd_rn(c_[n], e);
        s_[n] = t;
      }
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(&bars->acc_empty[cb]));
    }
    if (ok) {
      const int e = e0 + r;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const int t = t0 + 16 * h + n;
        if (e < E && t < T) partial[((size_t)z * T + t) * E + e] = (double)s_[n] + (double)c_[n];
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && bars->abort_flag) atomicExch(abort_out, 1u);
  if (warp == 1) {
    tmem_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// Host: tensor maps and launch
// ---------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D map over a row-major [rows, cols] tensor, box [box_rows, box_cols],
// 128-byte swizzle, zero fill outside.
static int make_map(CUtensorMap* map, const void* base, CUtensorMapDataType type, int elem_bytes, uint64_t cols,
                    uint64_t rows, uint32_t box_cols, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) {
    set_last_error("grouped_tc: cuTensorMapEncodeTiled is unavailable");
    return GLM53_ERR_CUDA;
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("grouped_tc: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return GLM53_ERR_CUDA;
  }
  return GLM53_OK;
}

// Fill g_sigmoid_tab once per device, on the caller's stream.  Under stream
// capture the fill is recorded into the graph (ahead of the kernel that needs
// it) and the device is not marked, so a later eager call fills it too.
static int ensure_sigmoid_table(cudaStream_t st) {
  static std::mutex mu;
  static bool done[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_last_error("grouped_tc: no current CUDA device");
    return GLM53_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev]) return GLM53_OK;
  sigmoid_table_kernel<<<65536 / 256, 256, 0, st>>>();
  int rc = check_launch("sigmoid_table_kernel");
  if (rc) return rc;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusNone) done[dev] = true;
  return GLM53_OK;
}

}  // namespace tc

bool router_tc_supported(int64_t T, int64_t H, int64_t E) {
  return T > 0 && T <= INT32_MAX / 2 && H > 0 && H % 128 == 0 && H <= 8192 && E > 0 && E <= 1024;
}

// K ranges per tile: about two CTAs per SM (one is resident at a time; the
// second wave covers the first's uneven finish), at most 8.
int router_tc_splits(int64_t T, int64_t E) {
  const int64_t tiles = ((E + 127) / 128) * ((T + tc::rt::kTokens - 1) / tc::rt::kTokens);
  return (int)std::max<int64_t>(1, std::min<int64_t>(8, (2 * sm_count() + tiles / 2) / tiles));
}

int router_logits_tc(const uint16_t* x, int64_t T, int64_t H, const uint16_t* planes, int64_t E, double* partial,
                     int splits, uint32_t* abort_out, cudaStream_t st) {
  using namespace tc;
  if (!router_tc_supported(T, H, E) || splits < 1 || splits > (int)(H / 128) ||
      (((uintptr_t)x | (uintptr_t)planes) & 15) != 0) {
    set_last_error("router_logits_tc: unsupported geometry");
    return GLM53_ERR_INVALID;
  }
  CUtensorMap wmap, xmap;
  int rc = make_map(&wmap, planes, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)H, (uint64_t)(3 * E), 64, 128);
  if (rc) return rc;
  rc = make_map(&xmap, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)H, (uint64_t)T, 64, rt::kTokens);
  if (rc) return rc;
  const int64_t tiles = ((E + 127) / 128) * ((T + rt::kTokens - 1) / rt::kTokens);
  const size_t smem = rt::smem_bytes();
  rc = ensure_max_smem((const void*)router_tc_kernel, smem);
  if (rc) return rc;
  router_tc_kernel<<<(unsigned)(tiles * splits), rt::kThreads, smem, st>>>(wmap, xmap, (int)T, (int)H, (int)E,
                                                                         (int)(H / 128), splits, partial, abort_out);
  return check_launch("router_tc_kernel");
}

// Sum of the split-K ranges' FP32 partials in range order, times the route
// multiplier, rounded to BF16: out[r][c] = BF16(xscale[r] * sum_ks p[ks][r][c]).
__global__ void splitk_reduce_kernel(const float* __restrict__ partial, int splits, int64_t R, int64_t N,
                                     const float* __restrict__ xscale, uint16_t* __restrict__ out) {
  const int64_t n4 = N >> 2;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= R * n4) return;
  const int64_t r = i / n4;
  const size_t plane = (size_t)R * N;
  float4 t = reinterpret_cast<const float4*>(partial)[i];
  for (int ks = 1; ks < splits; ++ks) {
    const float4 v = reinterpret_cast<const float4*>(partial + ks * plane)[i];
    t.x += v.x;
    t.y += v.y;
    t.z += v.z;
    t.w += v.w;
  }
  const float x = xscale ? __ldg(xscale + r) : 1.0f;
  const uint32_t lo = (uint32_t)f32_to_bf16_bits(t.x * x) | ((uint32_t)f32_to_bf16_bits(t.y * x) << 16);
  const uint32_t hi = (uint32_t)f32_to_bf16_bits(t.z * x) | ((uint32_t)f32_to_bf16_bits(t.w * x) << 16);
  reinterpret_cast<uint2*>(out)[i] = make_uint2(lo, hi);
}

int grouped_tc_splits(int64_t tiles, int64_t nkb) {
  const int64_t sms = sm_count();
  if (tiles <= 0 || tiles * 2 > sms) return 1;
  return (int)std::max<int64_t>(1, std::min<int64_t>(sms / tiles, nkb / 4));
}

size_t grouped_tc_splitk_bytes(int64_t R, int64_t N, int splits) {
  return splits > 1 ? align_up((size_t)splits * R * N * sizeof(float), 256) : 0;
}

bool grouped_tc_supported(int64_t K, int64_t N, float limit, bool swiglu) {
  // SwiGLU tiles are 64 hidden rows inside one 128-row scale block; plain tiles
  // are 128 output rows, the last one cut at N (8-row granularity)
  if (K % tc::kKB != 0 || N <= 0 || N % (swiglu ? 64 : 8) != 0 || K <= 0) return false;
  // FP16 hidden rows: |SwiGLU| <= limit^2 must stay inside FP16 range
  if (swiglu && !(limit > 0.0f && limit <= 128.0f)) return false;
  return true;
}

bool grouped_f8_supported(int64_t K, int64_t N, bool swiglu) {
  // SwiGLU tiles are 128 hidden rows, plain tiles 256 output rows (no tile
  // crosses an expert); the activation split holds a row of K <= 4096
  return K > 0 && K % tc::kKB == 0 && K <= 16 * 256 && N > 0 && N % (swiglu ? 128 : 256) == 0;
}

static int grouped_f8(const TcGemm& g, cudaStream_t st) {
  using namespace tc;
  const int64_t cols = g.swiglu ? g.I : g.N;
  if (!grouped_f8_supported(g.K, cols, g.swiglu) || !g.finite || g.splits > 1 || g.R <= 0 || g.max_rows <= 0 ||
      !g.x8 || (((uintptr_t)g.x8 | (uintptr_t)g.w | (uintptr_t)(g.swiglu ? g.w_up : g.w)) & 15) != 0) {
    set_last_error("grouped_f8: unsupported geometry");
    return GLM53_ERR_INVALID;
  }
  if (g.capacity == 0) return GLM53_OK;
  CUtensorMap wmap, umap, xmap, xmap64;
  int rc = make_map(&wmap, g.w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)g.K, (uint64_t)(g.E * g.w_rows), kKB, kM);
  if (rc) return rc;
  if (g.swiglu) {
    rc = make_map(&umap, g.w_up, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)g.K, (uint64_t)(g.E * g.u_rows), kKB,
                  kM);
    if (rc) return rc;
  } else {
    umap = wmap;
  }
  // term rows [R][hi K | lo K]: the lo tile of k-block kb starts at column K + 128 kb
  rc = make_map(&xmap, g.x8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)(2 * g.K), (uint64_t)g.R, kKB, kN);
  if (rc) return rc;
  rc = make_map(&xmap64, g.x8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)(2 * g.K), (uint64_t)g.R, kKB, kN / 2);
  if (rc) return rc;
  TcArgs a{};
  a.tile_experts = g.tile_experts;
  a.tile_starts = g.tile_starts;
  a.tile_lengths = g.tile_lengths;
  a.dense = g.dense ? 1 : 0;
  a.R = (int)g.R;
  a.K = (int)g.K;
  a.E = (int)g.E;
  a.w_rows = (int)g.w_rows;
  a.u_rows = (int)g.u_rows;
  a.u_off = (int)g.u_off;
  a.s_gate = g.s_gate;
  a.s_up = g.s_up ? g.s_up : g.s_gate;
  a.s_expert = g.s_expert;
  a.xscale = g.xscale;
  a.limit = g.limit;
  a.out_cols = (int)(g.swiglu ? 2 * cols : cols);  // gate/up tiles write [R][gate I | up I]
  a.out = g.out;
  a.status = g.status;
  a.splits = 1;
  a.partial = nullptr;
  const int mtiles = (int)(g.swiglu ? cols / kM : cols / (2 * kM));
  const int zsub = g.dense ? 1 : (int)((g.max_rows + kN - 1) / kN);
  const int64_t ntiles = g.capacity * mtiles * zsub;
  if (ntiles > INT32_MAX) {
    set_last_error("grouped_f8: too many tiles");
    return GLM53_ERR_INVALID;
  }
  const int grid = (int)std::min<int64_t>(ntiles, sm_count());
  void (*kern)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, TcArgs, int, int, int);
  kern = g.swiglu ? grouped_f8_kernel<true> : grouped_f8_kernel<false>;
  const size_t smem = f8::smem_bytes();
  rc = ensure_max_smem((const void*)kern, smem);
  if (rc) return rc;
  kern<<<grid, f8::kThreads, smem, st>>>(wmap, umap, xmap, xmap64, a, (int)ntiles, mtiles, zsub);
  return check_launch("grouped_f8_kernel");
}

int grouped_tc(const TcGemm& g, cudaStream_t st) {
  using namespace tc;
  if (g.f8) return grouped_f8(g, st);
  const int64_t cols = g.swiglu ? g.I : g.N;
  // a plain tile cut at N needs the rows past N to be out of the map (one expert)
  const bool cut_ok = g.swiglu || g.N % kM == 0 || g.E == 1;
  if (!grouped_tc_supported(g.K, cols, g.limit, g.swiglu) || !cut_ok || g.R <= 0 || g.max_rows <= 0 ||
      (((uintptr_t)g.x16 | (uintptr_t)g.w | (uintptr_t)(g.swiglu ? g.w_up : g.w)) & 15) != 0) {
    set_last_error("grouped_tc: unsupported geometry");
    return GLM53_ERR_INVALID;
  }
  if (g.capacity == 0) return GLM53_OK;
  CUtensorMap wmap, umap, xmap, xmap64;
  const uint32_t wbox = g.swiglu ? kM / 2 : kM;  // SwiGLU: 64 gate rows + 64 up rows per tile
  int rc = make_map(&wmap, g.w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)g.K, (uint64_t)(g.E * g.w_rows), kKB,
                    wbox);
  if (rc) return rc;
  if (g.swiglu) {
    rc = make_map(&umap, g.w_up, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)g.K, (uint64_t)(g.E * g.u_rows), kKB,
                  wbox);
    if (rc) return rc;
  } else {
    umap = wmap;
  }
  rc = make_map(&xmap, g.x16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)g.K, (uint64_t)g.R, 64, kN);
  if (rc) return rc;
  rc = make_map(&xmap64, g.x16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)g.K, (uint64_t)g.R, 64, kN / 2);
  if (rc) return rc;
  TcArgs a{};
  a.tile_experts = g.tile_experts;
  a.tile_starts = g.tile_starts;
  a.tile_lengths = g.tile_lengths;
  a.dense = g.dense ? 1 : 0;
  a.R = (int)g.R;
  a.K = (int)g.K;
  a.E = (int)g.E;
  a.w_rows = (int)g.w_rows;
  a.u_rows = (int)g.u_rows;
  a.u_off = (int)g.u_off;
  a.s_gate = g.s_gate;
  a.s_up = g.s_up ? g.s_up : g.s_gate;
  a.s_expert = g.s_expert;
  a.xscale = g.xscale;
  a.limit = g.limit;
  a.out_cols = (int)(g.swiglu ? 2 * cols : cols);  // gate/up tiles write [R][gate I | up I]
  a.out = g.out;
  a.status = g.status;
  const int splits = (g.splits > 1 && g.dense && !g.swiglu && g.partial && (cols % 4) == 0) ? g.splits : 1;
  if (splits > g.K / kKB) {
    set_last_error("grouped_tc: %d K ranges for %lld k-blocks", splits, (long long)(g.K / kKB));
    return GLM53_ERR_INVALID;
  }
  a.splits = splits;
  a.partial = g.partial;
  const int mtiles = (int)((cols + wbox - 1) / wbox);
  const int zsub = g.dense ? 1 : (int)((g.max_rows + kN - 1) / kN);
  const int64_t ntiles = g.capacity * mtiles * zsub * splits;
  if (ntiles > INT32_MAX) {
    set_last_error("grouped_tc: too many tiles");
    return GLM53_ERR_INVALID;
  }
  const int grid = (int)std::min<int64_t>(ntiles, sm_count());
  void (*kern)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, TcArgs, int, int, int);
  size_t smem;
  if (g.swiglu) {
    kern = g.finite ? grouped_tc_kernel<true, true, false> : grouped_tc_kernel<true, false, false>;
    smem = smem_bytes<true>();
  } else if (splits > 1) {
    kern = g.finite ? grouped_tc_kernel<false, true, true> : grouped_tc_kernel<false, false, true>;
    smem = smem_bytes<false>();
  } else {
    kern = g.finite ? grouped_tc_kernel<false, true, false> : grouped_tc_kernel<false, false, false>;
    smem = smem_bytes<false>();
  }
  rc = ensure_max_smem((const void*)kern, smem);
  if (rc) return rc;
  kern<<<grid, kThreads, smem, st>>>(wmap, umap, xmap, xmap64, a, (int)ntiles, mtiles, zsub);
  rc = check_launch("grouped_tc_kernel");
  if (rc || splits == 1) return rc;
  const int64_t n4 = g.R * (cols / 4);
  glm53::splitk_reduce_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(g.partial, splits, g.R, cols, g.xscale,
                                                                             g.out);
  return check_launch("splitk_reduce_kernel");
}

// ---------------------------------------------------------------------------
// Activations: BF16 rows (optionally gathered through the route order) ->
// FP16 * 2^-e with 2^e per row.
// ---------------------------------------------------------------------------

__global__ void to_f16_rows_kernel(const uint16_t* __restrict__ x, int64_t H, const uint32_t* __restrict__ order,
                                   int div, int64_t rows, __half* __restrict__ y, float* __restrict__ scale) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t src = order ? (int64_t)(order[row] / (uint32_t)div) : row;
  const uint4* xr = reinterpret_cast<const uint4*>(x + src * H);
  const int n8 = (int)(H >> 3);
  float m = 0.f;
  for (int i = lane; i < n8; i += 32) {
    const uint4 v = xr[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      m = fmaxf(m, fabsf(__uint_as_float(w[t] << 16)));
      m = fmaxf(m, fabsf(__uint_as_float(w[t] & 0xFFFF0000u)));
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  int e = 0;
  if (m >= 16384.0f) {  // keep |x| * 2^-e < 2^15
    int ex;
    frexpf(m, &ex);
    e = ex - 14;
  }
  const float down = ldexpf(1.0f, -e);
  uint4* yr = reinterpret_cast<uint4*>(y + row * H);
  for (int i = lane; i < n8; i += 32) {
    const uint4 v = xr[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      __half2 h = __floats2half2_rn(__uint_as_float(w[t] << 16) * down, __uint_as_float(w[t] & 0xFFFF0000u) * down);
      o[t] = *reinterpret_cast<uint32_t*>(&h);
    }
    yr[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (lane == 0) scale[row] = ldexpf(1.0f, e);
}

int rows_to_f16(const uint16_t* x, int64_t H, const uint32_t* order, int div, int64_t rows, __half* y, float* scale,
                cudaStream_t st) {
  if (rows <= 0) return GLM53_OK;
  if (H % 8 != 0 || (((uintptr_t)x | (uintptr_t)y) & 15) != 0) {
    set_last_error("rows_to_f16: 16-byte aligned rows required");
    return GLM53_ERR_INVALID;
  }
  to_f16_rows_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(x, H, order, div, rows, y, scale);
  return check_launch("to_f16_rows_kernel");
}

// ---------------------------------------------------------------------------
// Activations for the kind::f8f6f4 kernel: BF16 row x (optionally gathered
// through the route order) -> [hi K | lo K] E4M3 terms of x * 2^-e, the row
// maximum scaled into [128, 256), scale[r] = 2^e.  One warp per row holds the
// whole row in registers before it writes, so y may alias x (the two term
// rows take the bytes of the BF16 row).  A row whose maximum is infinite gets
// scale NaN (its outputs become NaN); NaN elements stay NaN in both terms.
// ---------------------------------------------------------------------------

constexpr int kSplitChunks = 16;  // 16 x 256 elements per row at most

// E4M3 pair, round to nearest even, saturating: e0 in the low byte.
__device__ __forceinline__ uint32_t e4m3x2_rn(float e0, float e1) {
  uint16_t d;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(d) : "f"(e1), "f"(e0));
  return d;
}

__device__ __forceinline__ float2 e4m3x2_value(uint32_t p) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"((uint16_t)p));
  const __half2 v = *reinterpret_cast<const __half2*>(&h);
  return __half22float2(v);
}

// One warp writes the [hi K | lo K] terms of a BF16 row held as 8-element
// chunks v[j] (lane + 32 j) with row maximum m (already reduced over the
// warp), and the row's scale.
__device__ __forceinline__ void write_terms(const uint4 (&v)[kSplitChunks], int n8, float m, int64_t K, uint8_t* yr,
                                            float* scale) {
  const int lane = threadIdx.x & 31;
  int e = 0;
  if (m > 0.f && m <= 3.402823466e38f) {
    int ex;
    frexpf(m, &ex);  // m in [2^(ex-1), 2^ex)
    e = max(ex - 8, -126);
  }
  const float mul = ldexpf(1.0f, -e);
#pragma unroll
  for (int j = 0; j < kSplitChunks; ++j) {
    const int i = lane + 32 * j;
    if (i < n8) {
      const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
      uint32_t hi[2] = {0u, 0u}, lo[2] = {0u, 0u};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float f0 = __uint_as_float(w[t] << 16) * mul;
        const float f1 = __uint_as_float(w[t] & 0xFFFF0000u) * mul;
        const uint32_t ph = e4m3x2_rn(f0, f1);
        const float2 hv = e4m3x2_value(ph);
        const uint32_t pl = e4m3x2_rn(f0 - hv.x, f1 - hv.y);
        hi[t >> 1] |= ph << (16 * (t & 1));
        lo[t >> 1] |= pl << (16 * (t & 1));
      }
      *reinterpret_cast<uint2*>(yr + 8 * i) = make_uint2(hi[0], hi[1]);
      *reinterpret_cast<uint2*>(yr + K + 8 * i) = make_uint2(lo[0], lo[1]);
    }
  }
  if (lane == 0) *scale = m > 3.402823466e38f ? __int_as_float(0x7fc00000) : ldexpf(1.0f, e);
}

__global__ void split_rows_kernel(const uint16_t* x, int64_t K, const uint32_t* __restrict__ order, int div,
                                  int64_t rows, uint8_t* y, float* __restrict__ scale) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t src = order ? (int64_t)(__ldg(order + row) / (uint32_t)div) : row;
  const uint4* xr = reinterpret_cast<const uint4*>(x + src * K);
  const int n8 = (int)(K >> 3);
  uint4 v[kSplitChunks];
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < kSplitChunks; ++j) {
    const int i = lane + 32 * j;
    if (i < n8) {
      v[j] = xr[i];
      const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        m = fmaxf(m, fabsf(__uint_as_float(w[t] << 16)));
        m = fmaxf(m, fabsf(__uint_as_float(w[t] & 0xFFFF0000u)));
      }
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __syncwarp();  // every lane's row chunks are in registers before any term is written
  write_terms(v, n8, m, K, y + row * 2 * K, scale + row);
}

int rows_to_e4m3_split(const uint16_t* x, int64_t K, const uint32_t* order, int div, int64_t rows, uint8_t* y,
                       float* scale, cudaStream_t st) {
  if (rows <= 0) return GLM53_OK;
  if (K % 8 != 0 || K > 32 * 8 * kSplitChunks || (((uintptr_t)x | (uintptr_t)y) & 15) != 0 ||
      (order && (const void*)x == (const void*)y)) {
    set_last_error("rows_to_e4m3_split: 16-byte aligned rows of K <= %d required", 32 * 8 * kSplitChunks);
    return GLM53_ERR_INVALID;
  }
  split_rows_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(x, K, order, div, rows, y, scale);
  return check_launch("split_rows_kernel");
}


// ---------------------------------------------------------------------------
// SwiGLU of the grouped gate/up rows [R][gate I | up I] (BF16, the reference's
// gate and up values): the reference's BF16 SwiGLU (swiglu_bf16, sigmoid from
// the table), as FP16 hidden rows for the kind::f16 down projection
// (swiglu_rows) or as the E4M3 terms of the BF16 hidden rows for the
// kind::f8f6f4 one (swiglu_split).
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint4 swiglu8(uint4 g, uint4 u, float limit) {
  const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, uw[4] = {u.x, u.y, u.z, u.w};
  uint32_t o[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const uint32_t h0 = tc::swiglu_bf16_tab(__uint_as_float(gw[t] << 16), __uint_as_float(uw[t] << 16), limit);
    const uint32_t h1 =
        tc::swiglu_bf16_tab(__uint_as_float(gw[t] & 0xFFFF0000u), __uint_as_float(uw[t] & 0xFFFF0000u), limit);
    o[t] = h0 | (h1 << 16);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void swiglu_rows_kernel(const uint16_t* __restrict__ gu, int64_t R, int64_t I, float limit,
                                   __half* __restrict__ hidden) {
  const int64_t n8 = I >> 3;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < R * n8; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / n8, c = i - r * n8;
    const uint4 g = *reinterpret_cast<const uint4*>(gu + r * 2 * I + 8 * c);
    const uint4 u = *reinterpret_cast<const uint4*>(gu + r * 2 * I + I + 8 * c);
    const uint4 h = swiglu8(g, u, limit);
    const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const __half2 hh = __floats2half2_rn(__uint_as_float(hw[t] << 16), __uint_as_float(hw[t] & 0xFFFF0000u));
      o[t] = *reinterpret_cast<const uint32_t*>(&hh);
    }
    *reinterpret_cast<uint4*>(hidden + r * I + 8 * c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void swiglu_split_kernel(const uint16_t* __restrict__ gu, int64_t R, int64_t I, float limit,
                                    uint8_t* __restrict__ terms, float* __restrict__ scale) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= R) return;
  const uint16_t* gr = gu + row * 2 * I;
  const int n8 = (int)(I >> 3);
  uint4 v[kSplitChunks];
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < kSplitChunks; ++j) {
    const int i = lane + 32 * j;
    if (i < n8) {
      v[j] = swiglu8(*reinterpret_cast<const uint4*>(gr + 8 * i), *reinterpret_cast<const uint4*>(gr + I + 8 * i),
                     limit);
      const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        m = fmaxf(m, fabsf(__uint_as_float(w[t] << 16)));
        m = fmaxf(m, fabsf(__uint_as_float(w[t] & 0xFFFF0000u)));
      }
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  write_terms(v, n8, m, I, terms + row * 2 * I, scale + row);
}

int swiglu_rows(const uint16_t* gu, int64_t R, int64_t I, float limit, __half* hidden, cudaStream_t st) {
  if (R <= 0) return GLM53_OK;
  if (I % 8 != 0 || (((uintptr_t)gu | (uintptr_t)hidden) & 15) != 0) {
    set_last_error("swiglu_rows: 16-byte aligned rows required");
    return GLM53_ERR_INVALID;
  }
  int rc = tc::ensure_sigmoid_table(st);
  if (rc) return rc;
  const int64_t n = R * (I / 8);
  const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 16);
  swiglu_rows_kernel<<<blocks, 256, 0, st>>>(gu, R, I, limit, hidden);
  return check_launch("swiglu_rows_kernel");
}

int swiglu_split(const uint16_t* gu, int64_t R, int64_t I, float limit, uint8_t* terms, float* scale,
                 cudaStream_t st) {
  if (R <= 0) return GLM53_OK;
  if (I % 8 != 0 || I > 32 * 8 * kSplitChunks || (((uintptr_t)gu | (uintptr_t)terms) & 15) != 0) {
    set_last_error("swiglu_split: 16-byte aligned rows of I <= %d required", 32 * 8 * kSplitChunks);
    return GLM53_ERR_INVALID;
  }
  int rc = tc::ensure_sigmoid_table(st);
  if (rc) return rc;
  swiglu_split_kernel<<<(unsigned)((R + 7) / 8), 256, 0, st>>>(gu, R, I, limit, terms, scale);
  return check_launch("swiglu_split_kernel");
}

}  // namespace glm53
