/*
 * CPU oracle for the GLM-5.3 FP8 MoE hot path.  TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the arithmetic of the reference's Metal
 * kernels so that the CUDA path can be checked against it.  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs
 * may load it; the product path never does.
 *
 * Parity pins (checked by tests/test_oracle_golden.py):
 *   - E4M3 table: every one of the 256 codes against ml_dtypes.float8_e4m3fn,
 *     which differs from the reference table only at 0x7F/0xFF (+-480 here).
 *   - BF16 SwiGLU sigmoid: SHA-256 over all 33,346 finite BF16 values in
 *     [-10, 10] equals the reference artifact's hash ef6da17a... (see
 *     orc_sigmoid_bf16 for the one pinned input).
 *   - Tile descriptors: the 31/32/33-route known answer of the reference tests.
 *   - Router score recompute: the sigmoid -> normalise -> scale known answer.
 * Floating-point sums whose order the Apple GPU defines (simd_sum, simdgroup
 * MMA) are restated as the butterfly tree / sequential order named at each
 * function; those are compared with the tolerance the tests state.
 *
 * Build: gcc -O2 -ffp-contract=off -fPIC -shared -pthread (oracle/Makefile).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_BLOCK 128
#define ORC_THREADS 256

/* ------------------------------------------------------------------------ */
/* Scalar helpers                                                           */
/* ------------------------------------------------------------------------ */

/* glm53_flash_mlx/fp8.py:22-27 (_e4m3_value): subnormal m*2^-9, normal
 * (1+m/8)*2^(e-7); codes 0x7F/0xFF decode to +-480 (no NaN). */
float orc_e4m3(uint8_t code) {
  float sign = (code & 0x80) ? -1.0f : 1.0f;
  int e = (code >> 3) & 15;
  int m = code & 7;
  float v = (e == 0) ? (float)m * ldexpf(1.0f, -9)
                     : (1.0f + (float)m / 8.0f) * ldexpf(1.0f, e - 7);
  return sign * v;
}

static float g_lut[256];
static int g_lut_ready = 0;
static void lut_init(void) {
  if (g_lut_ready) return;
  for (int c = 0; c < 256; ++c) g_lut[c] = orc_e4m3((uint8_t)c);
  g_lut_ready = 1;
}

void orc_e4m3_table(float* out) {
  lut_init();
  memcpy(out, g_lut, sizeof(g_lut));
}

static inline float f32_from_bf16(uint16_t b) {
  uint32_t u = ((uint32_t)b) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* Round-to-nearest-even float -> bfloat16 (Metal/MLX conversion). */
static inline uint16_t bf16_from_f32(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) {
    return (uint16_t)((u >> 16) | 0x0040u); /* quiet NaN */
  }
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

uint16_t orc_bf16_from_f32(float f) { return bf16_from_f32(f); }
float orc_f32_from_bf16(uint16_t b) { return f32_from_bf16(b); }

static inline float bfr(float f) { return f32_from_bf16(bf16_from_f32(f)); }

/* BF16 sigmoid with the per-op rounding of the reference's SwiGLU epilogue
 * (glm53_flash_mlx/packed.py:155-160, MLX's BF16 sigmoid): every operation
 * is done in FP32 and rounded to BF16:
 *   tail = 1 / (1 + exp(|g|));  sig = g < 0 ? tail : 1 - tail.
 * exp is the correctly rounded exponential.  The reference's JIT exponential
 * differs from it at exactly one BF16 input in [-10, 10]: g = -6.84375
 * (0xC0DB), where the reference yields 0x3A8C instead of 0x3A8B
 * (bench-results/m3ultra512-native-routed-sigmoid-formula-sweep-20260907.json,
 * results.standard_bf16.first_difference).  That input is pinned here. */
uint16_t orc_sigmoid_bf16(uint16_t g_bits) {
  if (g_bits == 0xC0DBu) return 0x3A8Cu;
  float g = f32_from_bf16(g_bits);
  float a = fabsf(g);
  float e = bfr((float)exp((double)a));
  float den = bfr(1.0f + e);
  float tail = bfr(1.0f / den);
  float sig = (g < 0.0f) ? tail : bfr(1.0f - tail);
  return bf16_from_f32(sig);
}

/* The K7/K9 epilogue (glm53_flash_mlx/packed.py:146-163): BF16 stores of the
 * two FP32 dot products, clamp in FP32, BF16, sigmoid, SiLU, times up. */
uint16_t orc_swiglu_bf16(float gate_total, float up_total, float limit) {
  float gate_t = bfr(gate_total);
  float up_t = bfr(up_total);
  float gate_value = fminf(gate_t, limit);
  float up_value = fminf(fmaxf(up_t, -limit), limit);
  uint16_t ga = bf16_from_f32(gate_value);
  float ua = bfr(up_value);
  float sig = f32_from_bf16(orc_sigmoid_bf16(ga));
  float silu = bfr(f32_from_bf16(ga) * sig);
  return bf16_from_f32(silu * ua);
}

/* Butterfly reduction over 32 lanes (the restated simd_sum order). */
static float simd_sum32(const float* v) {
  float a[32];
  memcpy(a, v, sizeof(a));
  for (int off = 16; off >= 1; off >>= 1) {
    float b[32];
    for (int i = 0; i < 32; ++i) b[i] = a[i] + a[i ^ off];
    memcpy(a, b, sizeof(a));
  }
  return a[0];
}

/* Two-stage threadgroup reduction of 256 per-thread partials
 * (glm53_flash_mlx/fp8.py:59-71): simd_sum per 32-thread group, then a
 * simd_sum over the 8 group partials (other lanes contribute 0). */
static float tg_reduce256(const float* partial) {
  float groups[32];
  for (int g = 0; g < 32; ++g) groups[g] = 0.0f;
  for (int g = 0; g < ORC_THREADS / 32; ++g) groups[g] = simd_sum32(partial + 32 * g);
  return simd_sum32(groups);
}

/* ------------------------------------------------------------------------ */
/* Thread pool (parallel-for over rows)                                     */
/* ------------------------------------------------------------------------ */

typedef void (*row_fn)(void* ctx, int64_t row);
typedef struct {
  row_fn fn;
  void* ctx;
  int64_t n;
  int nthreads;
  int index;
} pf_arg;

static void* pf_worker(void* p) {
  pf_arg* a = (pf_arg*)p;
  int64_t per = (a->n + a->nthreads - 1) / a->nthreads;
  int64_t lo = per * a->index;
  int64_t hi = lo + per < a->n ? lo + per : a->n;
  for (int64_t r = lo; r < hi; ++r) a->fn(a->ctx, r);
  return NULL;
}

static void parallel_for(int64_t n, int nthreads, row_fn fn, void* ctx) {
  if (nthreads <= 1 || n < 2) {
    for (int64_t r = 0; r < n; ++r) fn(ctx, r);
    return;
  }
  if (nthreads > 512) nthreads = 512;
  pthread_t th[512];
  pf_arg args[512];
  for (int i = 0; i < nthreads; ++i) {
    args[i].fn = fn;
    args[i].ctx = ctx;
    args[i].n = n;
    args[i].nthreads = nthreads;
    args[i].index = i;
    pthread_create(&th[i], NULL, pf_worker, &args[i]);
  }
  for (int i = 0; i < nthreads; ++i) pthread_join(th[i], NULL);
}

/* ------------------------------------------------------------------------ */
/* K1 / K2: block-128 E4M3 linear                                           */
/* ------------------------------------------------------------------------ */

/* K1 expression tree (glm53_flash_mlx/fp8.py:55-58): thread t sums
 * (x[k] * lut[w[k]]) * s over k = t, t+256, ...; then tg_reduce256. */
static float k1_dot(const uint16_t* x, const uint8_t* wr, const float* srow,
                    int64_t K) {
  float partial[ORC_THREADS];
  for (int t = 0; t < ORC_THREADS; ++t) {
    float acc = 0.0f;
    for (int64_t k = t; k < K; k += ORC_THREADS) {
      float scale = srow[k / ORC_BLOCK];
      float prod = f32_from_bf16(x[k]) * g_lut[wr[k]];
      prod = prod * scale;
      acc = acc + prod;
    }
    partial[t] = acc;
  }
  return tg_reduce256(partial);
}

/* K2 expression tree (glm53_flash_mlx/fp8.py:88-97): decoded = lut*s first,
 * then acc += x * decoded. */
static float k2_dot(const uint16_t* x, const uint8_t* wr, const float* srow,
                    int64_t K) {
  float partial[ORC_THREADS];
  for (int t = 0; t < ORC_THREADS; ++t) {
    float acc = 0.0f;
    for (int64_t k = t; k < K; k += ORC_THREADS) {
      float decoded = g_lut[wr[k]] * srow[k / ORC_BLOCK];
      float prod = f32_from_bf16(x[k]) * decoded;
      acc = acc + prod;
    }
    partial[t] = acc;
  }
  return tg_reduce256(partial);
}

typedef struct {
  const uint16_t* x;
  int64_t M, K, N, scale_cols;
  const uint8_t* w;
  const float* s;
  uint16_t* y;
} lin_ctx;

static void lin_row(void* p, int64_t n) {
  lin_ctx* c = (lin_ctx*)p;
  const uint8_t* wr = c->w + n * c->K;
  const float* srow = c->s + (n / ORC_BLOCK) * c->scale_cols;
  for (int64_t m = 0; m < c->M; ++m) {
    const uint16_t* xr = c->x + m * c->K;
    float v = (c->M == 1) ? k1_dot(xr, wr, srow, c->K) : k2_dot(xr, wr, srow, c->K);
    c->y[m * c->N + n] = bf16_from_f32(v);
  }
}

/* block_fp8_linear (glm53_flash_mlx/fp8.py:254-299): y = x @ dequant(W)^T.
 * One batch row uses the K1 tree, more rows the K2 tree. */
int orc_block_fp8_linear(const uint16_t* x, int64_t M, int64_t K,
                         const uint8_t* w, int64_t N, const float* s,
                         uint16_t* y, int nthreads) {
  lut_init();
  if (M < 0 || K <= 0 || N <= 0) return 1;
  lin_ctx c = {x, M, K, N, (K + ORC_BLOCK - 1) / ORC_BLOCK, w, s, y};
  parallel_for(N, nthreads, lin_row, &c);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Packed L=1 decode MoE (K7, K6, K8, K9, shared down K1, BF16 add)         */
/* ------------------------------------------------------------------------ */

typedef struct {
  const uint16_t* x;
  int64_t H, I, E, Is;
  int top_k;
  const uint32_t* ids;
  const uint8_t* gu_w;
  const float* gu_s;
  const uint8_t* d_w;
  const float* d_s;
  const uint8_t* sg_w;
  const float* sg_s;
  const uint8_t* su_w;
  const float* su_s;
  float limit;
  uint16_t* hidden;        /* [top_k * I] */
  uint16_t* shared_hidden; /* [Is] */
  uint16_t* down;          /* [top_k * H] */
} dec_ctx;

/* K7 (glm53_flash_mlx/packed.py:100-166): one output row of one slot. */
static void dec_gate_up_row(void* p, int64_t item) {
  dec_ctx* c = (dec_ctx*)p;
  int64_t slot = item / c->I, row = item % c->I;
  int64_t e = c->ids[slot];
  int64_t H = c->H, I = c->I;
  int64_t scale_cols = (H + ORC_BLOCK - 1) / ORC_BLOCK;
  int64_t half = (I + ORC_BLOCK - 1) / ORC_BLOCK;
  const uint8_t* gw = c->gu_w + (e * 2 * I + row) * H;
  const uint8_t* uw = c->gu_w + (e * 2 * I + I + row) * H;
  const float* gs = c->gu_s + (e * 2 * half + row / ORC_BLOCK) * scale_cols;
  const float* us = c->gu_s + (e * 2 * half + half + row / ORC_BLOCK) * scale_cols;
  float g = k1_dot(c->x, gw, gs, H);
  float u = k1_dot(c->x, uw, us, H);
  c->hidden[slot * I + row] = orc_swiglu_bf16(g, u, c->limit);
}

/* K9 (glm53_flash_mlx/packed.py:181-235): the shared expert. */
static void dec_shared_row(void* p, int64_t row) {
  dec_ctx* c = (dec_ctx*)p;
  int64_t H = c->H;
  int64_t scale_cols = (H + ORC_BLOCK - 1) / ORC_BLOCK;
  const float* gs = c->sg_s + (row / ORC_BLOCK) * scale_cols;
  const float* us = c->su_s + (row / ORC_BLOCK) * scale_cols;
  float g = k1_dot(c->x, c->sg_w + row * H, gs, H);
  float u = k1_dot(c->x, c->su_w + row * H, us, H);
  c->shared_hidden[row] = orc_swiglu_bf16(g, u, c->limit);
}

/* K6 (glm53_flash_mlx/packed.py:66-98): down projection of one slot row. */
static void dec_down_row(void* p, int64_t item) {
  dec_ctx* c = (dec_ctx*)p;
  int64_t slot = item / c->H, h = item % c->H;
  int64_t e = c->ids[slot];
  int64_t H = c->H, I = c->I;
  int64_t scale_rows = (H + ORC_BLOCK - 1) / ORC_BLOCK;
  int64_t scale_cols = (I + ORC_BLOCK - 1) / ORC_BLOCK;
  const uint8_t* wr = c->d_w + (e * H + h) * I;
  const float* srow = c->d_s + (e * scale_rows + h / ORC_BLOCK) * scale_cols;
  c->down[slot * H + h] = bf16_from_f32(k1_dot(c->hidden + slot * I, wr, srow, I));
}

/* PackedFP8MoE.__call__ decode (glm53_flash_mlx/packed.py:896-923).
 * Returns 0, or 3 when an expert id is out of range.  hidden_out may be NULL;
 * when given it receives the [top_k*I] routed hidden (then [Is] shared). */
int orc_packed_decode_moe(const uint16_t* x, int64_t H, const uint32_t* ids,
                          const float* scores, int top_k, const uint8_t* gu_w,
                          const float* gu_s, const uint8_t* d_w,
                          const float* d_s, int64_t E, int64_t I,
                          const uint8_t* sg_w, const float* sg_s,
                          const uint8_t* su_w, const float* su_s,
                          const uint8_t* sd_w, const float* sd_s, int64_t Is,
                          float limit, uint16_t* out, uint16_t* hidden_out,
                          int nthreads) {
  lut_init();
  for (int j = 0; j < top_k; ++j)
    if ((int64_t)ids[j] >= E) return 3;
  dec_ctx c;
  memset(&c, 0, sizeof(c));
  c.x = x; c.H = H; c.I = I; c.E = E; c.Is = Is; c.top_k = top_k; c.ids = ids;
  c.gu_w = gu_w; c.gu_s = gu_s; c.d_w = d_w; c.d_s = d_s;
  c.sg_w = sg_w; c.sg_s = sg_s; c.su_w = su_w; c.su_s = su_s; c.limit = limit;
  c.hidden = (uint16_t*)malloc(sizeof(uint16_t) * top_k * I);
  c.down = (uint16_t*)malloc(sizeof(uint16_t) * top_k * H);
  c.shared_hidden = Is > 0 ? (uint16_t*)malloc(sizeof(uint16_t) * Is) : NULL;
  parallel_for(top_k * I, nthreads, dec_gate_up_row, &c);
  parallel_for(top_k * H, nthreads, dec_down_row, &c);
  uint16_t* shared_out = NULL;
  if (Is > 0 && sg_w) {
    parallel_for(Is, nthreads, dec_shared_row, &c);
    shared_out = (uint16_t*)malloc(sizeof(uint16_t) * H);
    orc_block_fp8_linear(c.shared_hidden, 1, Is, sd_w, H, sd_s, shared_out, nthreads);
  }
  /* K8 (glm53_flash_mlx/packed.py:168-179): FP32 slot-ordered weighted sum. */
  for (int64_t h = 0; h < H; ++h) {
    float total = 0.0f;
    for (int j = 0; j < top_k; ++j) {
      float contribution = f32_from_bf16(c.down[j * H + h]) * scores[j];
      total = total + contribution;
    }
    uint16_t r = bf16_from_f32(total);
    if (shared_out) r = bf16_from_f32(f32_from_bf16(r) + f32_from_bf16(shared_out[h]));
    out[h] = r;
  }
  if (hidden_out) {
    memcpy(hidden_out, c.hidden, sizeof(uint16_t) * top_k * I);
    if (c.shared_hidden) memcpy(hidden_out + top_k * I, c.shared_hidden, sizeof(uint16_t) * Is);
  }
  free(c.hidden);
  free(c.down);
  free(c.shared_hidden);
  free(shared_out);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Router: Float32Gate + group_expert_select                                */
/* ------------------------------------------------------------------------ */

typedef struct {
  const uint16_t* x;
  int64_t T, H, E;
  const float* w;
  const float* bias;
  int top_k, n_group, topk_group, norm;
  float scale;
  double* logits64;
  float* logits32;
  uint32_t* idx;
  float* score;
  float* margin;
} rt_ctx;

/* logits = f32(x) @ f32(W)^T (glm53_flash_mlx/patch.py:133), computed here
 * in FP64 (the accuracy reference) and in FP32 sequential order. */
static void rt_row(void* p, int64_t t) {
  rt_ctx* c = (rt_ctx*)p;
  const uint16_t* xr = c->x + t * c->H;
  int64_t E = c->E;
  double* l64 = c->logits64 + t * E;
  for (int64_t e = 0; e < E; ++e) {
    const float* wr = c->w + e * c->H;
    double acc = 0.0;
    float acc32 = 0.0f;
    for (int64_t k = 0; k < c->H; ++k) {
      float xv = f32_from_bf16(xr[k]);
      acc += (double)xv * (double)wr[k];
      acc32 = acc32 + xv * wr[k];
    }
    l64[e] = acc;
    if (c->logits32) c->logits32[t * E + e] = acc32;
  }
  /* group_expert_select (mlx-vlm deepseek_v32, restated): s = sigmoid(l);
   * choice = s + bias; optional group mask; top-k of choice; scores = s[idx];
   * normalise; times routed_scaling_factor.  Slot order: descending choice,
   * ties to the lower expert id (the build's canonical order). */
  double* sig = (double*)malloc(sizeof(double) * E);
  double* choice = (double*)malloc(sizeof(double) * E);
  for (int64_t e = 0; e < E; ++e) {
    sig[e] = 1.0 / (1.0 + exp(-l64[e]));
    choice[e] = sig[e] + (double)c->bias[e];
  }
  if (c->n_group > 1) {
    int64_t per = E / c->n_group;
    double* gscore = (double*)malloc(sizeof(double) * c->n_group);
    for (int g = 0; g < c->n_group; ++g) {
      double b1 = -INFINITY, b2 = -INFINITY;
      for (int64_t e = g * per; e < (g + 1) * per; ++e) {
        double v = choice[e];
        if (v > b1) { b2 = b1; b1 = v; } else if (v > b2) { b2 = v; }
      }
      gscore[g] = b1 + b2;
    }
    /* drop the n_group - topk_group lowest groups (ties: higher index dropped first) */
    int drop = c->n_group - c->topk_group;
    char* dropped = (char*)calloc(c->n_group, 1);
    for (int d = 0; d < drop; ++d) {
      int worst = -1;
      for (int g = 0; g < c->n_group; ++g) {
        if (dropped[g]) continue;
        if (worst < 0 || gscore[g] < gscore[worst] ||
            (gscore[g] == gscore[worst] && g > worst))
          worst = g;
      }
      dropped[worst] = 1;
    }
    for (int g = 0; g < c->n_group; ++g)
      if (dropped[g])
        for (int64_t e = g * per; e < (g + 1) * per; ++e) choice[e] = 0.0;
    free(dropped);
    free(gscore);
  }
  char* taken = (char*)calloc(E, 1);
  double picked[64];
  double sum = 0.0;
  float fsc[64];
  for (int j = 0; j < c->top_k; ++j) {
    int64_t best = -1;
    for (int64_t e = 0; e < E; ++e) {
      if (taken[e]) continue;
      if (best < 0 || choice[e] > choice[best]) best = e;
    }
    taken[best] = 1;
    c->idx[t * c->top_k + j] = (uint32_t)best;
    picked[j] = sig[best];
  }
  if (c->margin) {
    double next = -INFINITY;
    for (int64_t e = 0; e < E; ++e)
      if (!taken[e] && choice[e] > next) next = choice[e];
    double last = choice[c->idx[t * c->top_k + c->top_k - 1]];
    c->margin[t] = (float)(last - next);
  }
  for (int j = 0; j < c->top_k; ++j) sum += picked[j];
  for (int j = 0; j < c->top_k; ++j) {
    double v = picked[j];
    if (c->top_k > 1 && c->norm) v = v / sum;
    fsc[j] = (float)(v * (double)c->scale);
    c->score[t * c->top_k + j] = fsc[j];
  }
  free(taken);
  free(sig);
  free(choice);
}

int orc_router(const uint16_t* x, int64_t T, int64_t H, const float* w,
               int64_t E, const float* bias, int top_k, int n_group,
               int topk_group, int norm, float scale, uint32_t* idx,
               float* score, double* logits64, float* logits32, float* margin,
               int nthreads) {
  if (top_k <= 0 || top_k > 64 || top_k > E) return 1;
  if (n_group > 1 && (E % n_group != 0 || topk_group < 1 || topk_group > n_group)) return 1;
  rt_ctx c = {x, T, H, E, w, bias, top_k, n_group, topk_group, norm, scale,
              logits64, logits32, idx, score, margin};
  parallel_for(T, nthreads, rt_row, &c);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Route plan and tile plan                                                  */
/* ------------------------------------------------------------------------ */

/* build_route_plan (glm53_flash_mlx/grouped_fp8.py:157-170) as a stable
 * counting sort (native_execution/native_indexer_plan.metal:1880-1939):
 * routes ordered by expert id, ties by route index.  Ids >= E are counted in
 * *invalid and placed after every valid route, in route order. */
int orc_route_plan(const uint32_t* ids, int64_t R, int64_t E,
                   const float* scores, uint32_t* order, uint32_t* inverse,
                   uint32_t* sorted_experts, float* sorted_scores,
                   uint32_t* expert_offsets, uint32_t* invalid) {
  uint32_t* counts = (uint32_t*)calloc(E + 1, sizeof(uint32_t));
  uint32_t bad = 0;
  for (int64_t r = 0; r < R; ++r) {
    if (ids[r] < (uint32_t)E) counts[ids[r]]++;
    else bad++;
  }
  expert_offsets[0] = 0;
  for (int64_t e = 0; e < E; ++e) expert_offsets[e + 1] = expert_offsets[e] + counts[e];
  uint32_t* cursor = (uint32_t*)malloc(sizeof(uint32_t) * (E + 1));
  for (int64_t e = 0; e < E; ++e) cursor[e] = expert_offsets[e];
  uint32_t tail = expert_offsets[E];
  for (int64_t r = 0; r < R; ++r) {
    uint32_t pos = ids[r] < (uint32_t)E ? cursor[ids[r]]++ : tail++;
    order[pos] = (uint32_t)r;
    inverse[r] = pos;
    sorted_experts[pos] = ids[r];
    if (scores && sorted_scores) sorted_scores[pos] = scores[r];
  }
  *invalid = bad;
  free(counts);
  free(cursor);
  return 0;
}

/* build_grouped_tile_plan (glm53_flash_mlx/grouped_fp8.py:173-203) with the
 * tile height as a parameter (the reference uses 32).  capacity =
 * ceil(R/tile_rows) + E.  Valid descriptors: (expert, start, min(rows left,
 * tile_rows)); invalid slots are the sentinel (0, R, 0). */
int orc_tile_plan(const uint32_t* sorted_experts, int64_t R, int64_t E,
                  int64_t tile_rows, uint32_t* tile_experts,
                  uint32_t* tile_starts, uint32_t* tile_lengths,
                  uint32_t* route_offsets, uint32_t* tile_offsets,
                  uint32_t* descriptor_count) {
  uint32_t* counts = (uint32_t*)calloc(E, sizeof(uint32_t));
  for (int64_t r = 0; r < R; ++r)
    if (sorted_experts[r] < (uint32_t)E) counts[sorted_experts[r]]++;
  route_offsets[0] = 0;
  tile_offsets[0] = 0;
  for (int64_t e = 0; e < E; ++e) {
    route_offsets[e + 1] = route_offsets[e] + counts[e];
    tile_offsets[e + 1] = tile_offsets[e] + (counts[e] + tile_rows - 1) / tile_rows;
  }
  int64_t cap = (R + tile_rows - 1) / tile_rows + E;
  int64_t owner = 0;
  for (int64_t d = 0; d < cap; ++d) {
    if (d < (int64_t)tile_offsets[E]) {
      while ((int64_t)tile_offsets[owner + 1] <= d) ++owner;
      uint32_t start = route_offsets[owner] + (uint32_t)((d - tile_offsets[owner]) * tile_rows);
      uint32_t remaining = route_offsets[owner + 1] - start;
      tile_experts[d] = (uint32_t)owner;
      tile_starts[d] = start;
      tile_lengths[d] = remaining < tile_rows ? remaining : (uint32_t)tile_rows;
    } else {
      tile_experts[d] = 0;
      tile_starts[d] = (uint32_t)R;
      tile_lengths[d] = 0;
    }
  }
  *descriptor_count = tile_offsets[E];
  free(counts);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Grouped prefill (K12, activate_gate_up, restore_and_reduce)               */
/* ------------------------------------------------------------------------ */

typedef struct {
  const uint16_t* x; /* [R, K] sorted rows */
  int64_t R, K, N, E;
  const uint32_t* experts; /* per sorted row */
  const uint8_t* w;        /* [E, N, K] */
  const float* s;          /* [E, ceil(N/128), ceil(K/128)] */
  uint16_t* out;           /* [R, N] */
} grp_ctx;

/* K12 (glm53_flash_mlx/grouped_fp8.py:70-139): FP32 x times FP32
 * (lut * scale) weights; accumulation per 8-wide K fragment (the simdgroup
 * MMA granule), fragments in K order; BF16 output. */
static void grp_row(void* p, int64_t r) {
  grp_ctx* c = (grp_ctx*)p;
  int64_t e = c->experts[r];
  if (e >= c->E) return;
  int64_t sr = (c->N + ORC_BLOCK - 1) / ORC_BLOCK, sc = (c->K + ORC_BLOCK - 1) / ORC_BLOCK;
  const uint16_t* xr = c->x + r * c->K;
  for (int64_t n = 0; n < c->N; ++n) {
    const uint8_t* wr = c->w + (e * c->N + n) * c->K;
    const float* srow = c->s + (e * sr + n / ORC_BLOCK) * sc;
    float acc = 0.0f;
    for (int64_t k0 = 0; k0 < c->K; k0 += 8) {
      float frag = 0.0f;
      for (int64_t k = k0; k < k0 + 8 && k < c->K; ++k) {
        float wd = g_lut[wr[k]] * srow[k / ORC_BLOCK];
        frag = frag + f32_from_bf16(xr[k]) * wd;
      }
      acc = acc + frag;
    }
    c->out[r * c->N + n] = bf16_from_f32(acc);
  }
}

int orc_grouped_linear(const uint16_t* x, int64_t R, int64_t K,
                       const uint32_t* sorted_experts, const uint8_t* w,
                       int64_t E, int64_t N, const float* s, uint16_t* out,
                       int nthreads) {
  lut_init();
  grp_ctx c = {x, R, K, N, E, sorted_experts, w, s, out};
  parallel_for(R, nthreads, grp_row, &c);
  return 0;
}

/* activate_gate_up (glm53_flash_mlx/grouped_fp8.py:265-270): MLX BF16 ops,
 * the same rounding sequence as the K7 epilogue. */
void orc_activate_gate_up(const uint16_t* gate_up, int64_t R, int64_t I,
                          float limit, uint16_t* hidden) {
  for (int64_t r = 0; r < R; ++r)
    for (int64_t i = 0; i < I; ++i)
      hidden[r * I + i] = orc_swiglu_bf16(f32_from_bf16(gate_up[r * 2 * I + i]),
                                          f32_from_bf16(gate_up[r * 2 * I + I + i]), limit);
}

/* restore_and_reduce (glm53_flash_mlx/grouped_fp8.py:273-276): FP32
 * out*score, restored by inverse order, summed over the top_k slots in slot
 * order, then BF16. */
void orc_restore_and_reduce(const uint16_t* sorted_out, const float* sorted_scores,
                            const uint32_t* inverse, int64_t T, int top_k,
                            int64_t H, uint16_t* out) {
  for (int64_t t = 0; t < T; ++t)
    for (int64_t h = 0; h < H; ++h) {
      float total = 0.0f;
      for (int j = 0; j < top_k; ++j) {
        uint32_t pos = inverse[t * top_k + j];
        float v = f32_from_bf16(sorted_out[(int64_t)pos * H + h]) * sorted_scores[pos];
        total = total + v;
      }
      out[t * H + h] = bf16_from_f32(total);
    }
}

/* BF16 elementwise add, MLX semantics: BF16(f32(a) + f32(b)). */
void orc_bf16_add(const uint16_t* a, const uint16_t* b, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = bf16_from_f32(f32_from_bf16(a[i]) + f32_from_bf16(b[i]));
}

/* Vector forms used by the Python wrapper. */
void orc_sigmoid_bf16_vec(const uint16_t* g, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = orc_sigmoid_bf16(g[i]);
}

void orc_swiglu_bf16_vec(const uint16_t* gate, const uint16_t* up, int64_t n,
                         float limit, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i)
    out[i] = orc_swiglu_bf16(f32_from_bf16(gate[i]), f32_from_bf16(up[i]), limit);
}

/* ------------------------------------------------------------------------ */
/* FFN boundary: mHC collapse + post-attention RMSNorm, and hc expand       */
/* ------------------------------------------------------------------------ */

/* The FFN half of a GLM-5.3 layer (scripts/trace_grouped_fp8_route_amplification.py:
 * 178-214, scripts/profile_native_prefill_ffn_entry_seam.py:79-87):
 *   collapsed, post, comb = layer.ffn_hc(state)        # mHC collapse
 *   normalized = layer.post_attention_layernorm(collapsed)
 *   moe = mlp(normalized)                                # router + MoE
 *   state' = hc_expand(moe, state, post, comb)
 *
 * ffn_hc is mlx-vlm's deepseek_v4 hyper-connection module (mlx-vlm 0.6.17
 * @ e82d557d, absent here).  It is restated from the published mHC
 * algorithm (DeepSeek-V4 inference hc_pre / hc_split_sinkhorn) with the
 * parameter dtypes the reference loads (hc fn BF16 [(2+n)n, nH]; hc scale
 * FP32 [3] and base FP32 [(2+n)n], glm53_flash_mlx/patch.py:296-318):
 *   x = f32(state[t]) flattened (n*H);  r = 1/sqrt(mean(x^2) + norm_eps)
 *   m = (x . fn^T) * r
 *   pre  = sigmoid(m[0:n] * scale[0] + base[0:n]) + eps
 *   post = 2 * sigmoid(m[n:2n] * scale[1] + base[n:2n])
 *   comb = softmax_j(m[2n:] * scale[2] + base[2n:]) + eps   (n x n, [src][dst])
 *   comb /= colsum + eps; then (iters-1) x (comb /= rowsum + eps; comb /= colsum + eps)
 *   collapsed = BF16(sum_b pre[b] * x[b])
 * PARITY UNPINNED for the collapse: no golden vector of mlx-vlm's module
 * exists in the reference.  Dot products and the mean square accumulate in
 * double here (the GPU's FP32 split sums are compared with a tolerance);
 * the 4-term sums are pairwise, (a0 + a1) + (a2 + a3).
 * post_attention_layernorm is MLX's fast RMSNorm:
 *   out = BF16(f32(w) * BF16(x * (1 / sqrt(mean(x^2) + eps)))). */
typedef struct {
  const uint16_t* state;
  int64_t H;
  const uint16_t* fn;
  const float* scale;
  const float* base;
  int iters;
  float eps, norm_eps;
  const uint16_t* norm_w;
  float rms_eps;
  uint16_t *collapsed, *normalized;
  float *post, *comb, *mixes;
} hc_ctx;

static inline float orc_sigmoidf(float z) { return 1.0f / (1.0f + expf(-z)); }
static inline float sum4(const float* v, int stride) {
  return (v[0] + v[stride]) + (v[2 * stride] + v[3 * stride]);
}

static void hc_row(void* p, int64_t t) {
  const hc_ctx* c = (const hc_ctx*)p;
  const int n = 4;
  const int64_t H = c->H, K = n * H;
  const uint16_t* x = c->state + t * K;
  double ss = 0.0;
  for (int64_t k = 0; k < K; ++k) {
    double v = f32_from_bf16(x[k]);
    ss += v * v;
  }
  float r = 1.0f / sqrtf((float)ss / (float)K + c->norm_eps);
  float m[24];
  for (int j = 0; j < (2 + n) * n; ++j) {
    const uint16_t* w = c->fn + (int64_t)j * K;
    double acc = 0.0;
    for (int64_t k = 0; k < K; ++k) acc += (double)f32_from_bf16(x[k]) * (double)f32_from_bf16(w[k]);
    m[j] = (float)acc * r;
    if (c->mixes) c->mixes[t * (2 + n) * n + j] = m[j];
  }
  float pre[4], cm[16];
  for (int b = 0; b < n; ++b) {
    pre[b] = orc_sigmoidf(m[b] * c->scale[0] + c->base[b]) + c->eps;
    c->post[t * n + b] = 2.0f * orc_sigmoidf(m[n + b] * c->scale[1] + c->base[n + b]);
  }
  for (int i = 0; i < n; ++i) {
    float z[4], mx = -INFINITY;
    for (int j = 0; j < n; ++j) {
      z[j] = m[2 * n + i * n + j] * c->scale[2] + c->base[2 * n + i * n + j];
      if (z[j] > mx) mx = z[j];
    }
    for (int j = 0; j < n; ++j) z[j] = expf(z[j] - mx);
    float s = sum4(z, 1);
    for (int j = 0; j < n; ++j) cm[i * n + j] = z[j] / s + c->eps;
  }
  for (int it = 0; it < c->iters; ++it) {
    if (it > 0) {
      for (int i = 0; i < n; ++i) {
        float s = sum4(cm + i * n, 1) + c->eps;
        for (int j = 0; j < n; ++j) cm[i * n + j] = cm[i * n + j] / s;
      }
    }
    float cs[4];
    for (int j = 0; j < n; ++j) cs[j] = sum4(cm + j, n) + c->eps;
    for (int i = 0; i < n; ++i)
      for (int j = 0; j < n; ++j) cm[i * n + j] = cm[i * n + j] / cs[j];
  }
  memcpy(c->comb + t * n * n, cm, sizeof(cm));
  double ss2 = 0.0;
  uint16_t* col = c->collapsed + t * H;
  for (int64_t d = 0; d < H; ++d) {
    float y = pre[0] * f32_from_bf16(x[d]);
    y = y + pre[1] * f32_from_bf16(x[H + d]);
    y = y + pre[2] * f32_from_bf16(x[2 * H + d]);
    y = y + pre[3] * f32_from_bf16(x[3 * H + d]);
    col[d] = bf16_from_f32(y);
    double v = f32_from_bf16(col[d]);
    ss2 += v * v;
  }
  if (c->norm_w && c->normalized) {
    float inv = 1.0f / sqrtf((float)ss2 / (float)H + c->rms_eps);
    for (int64_t d = 0; d < H; ++d)
      c->normalized[t * H + d] =
          bf16_from_f32(f32_from_bf16(c->norm_w[d]) * bfr(f32_from_bf16(col[d]) * inv));
  }
}

/* Returns 0, or 1 for an unsupported geometry (branches != 4). */
int orc_hc_collapse_norm(const uint16_t* state, int64_t T, int64_t H, int branches,
                         const uint16_t* fn, const float* scale, const float* base,
                         int sinkhorn_iters, float eps, float norm_eps,
                         const uint16_t* norm_w, float rms_eps, uint16_t* collapsed,
                         uint16_t* normalized, float* post, float* comb, float* mixes,
                         int threads) {
  if (branches != 4 || H <= 0 || sinkhorn_iters < 1) return 1;
  hc_ctx c = {state, H, fn, scale, base, sinkhorn_iters, eps, norm_eps, norm_w, rms_eps,
              collapsed, normalized, post, comb, mixes};
  parallel_for(T, threads, hc_row, &c);
  return 0;
}

/* MLX fast RMSNorm on BF16 rows (post_attention_layernorm), as above. */
void orc_rms_norm_bf16(const uint16_t* x, int64_t T, int64_t H, const uint16_t* w,
                       float rms_eps, uint16_t* out) {
  for (int64_t t = 0; t < T; ++t) {
    double ss = 0.0;
    for (int64_t d = 0; d < H; ++d) {
      double v = f32_from_bf16(x[t * H + d]);
      ss += v * v;
    }
    float inv = 1.0f / sqrtf((float)ss / (float)H + rms_eps);
    for (int64_t d = 0; d < H; ++d)
      out[t * H + d] = bf16_from_f32(f32_from_bf16(w[d]) * bfr(f32_from_bf16(x[t * H + d]) * inv));
  }
}

/* hc expand after the MoE, restating the reference's own kernel
 * glm53_native_prefill_post_attention_hc_expand
 * (native_execution/native_indexer_plan.metal:2362-2389), used on the MoE
 * output by NativePrefillMoEPlan::finish_hc (native_prefill_moe_plan.cpp:
 * 136-161):
 *   mixed = fma chain over source s = 0..3 of comb[t][s][b] * residual[t][s][d]
 *   out[t][b][d] = BF16(post[t][b] * moe[t][d] + mixed)   (product rounded,
 *   then the add; no contraction). */
void orc_hc_expand(const uint16_t* moe, const uint16_t* residual, const float* post,
                   const float* comb, int64_t T, int64_t H, uint16_t* out) {
  const int n = 4;
  for (int64_t t = 0; t < T; ++t)
    for (int b = 0; b < n; ++b)
      for (int64_t d = 0; d < H; ++d) {
        float mixed = 0.0f;
        for (int s = 0; s < n; ++s)
          mixed = fmaf(comb[(t * n + s) * n + b], f32_from_bf16(residual[(t * n + s) * H + d]), mixed);
        float branch = post[t * n + b] * f32_from_bf16(moe[t * H + d]);
        out[(t * n + b) * H + d] = bf16_from_f32(branch + mixed);
      }
}

/* ------------------------------------------------------------------------ */
/* Rounding envelopes (tolerance certificates for the parity tests)         */
/* ------------------------------------------------------------------------ */

/* A routed expert's BF16 down rows computed by ANY FP32 evaluation order of
 * its dot products lie inside the envelope computed here; the parity tests
 * accept a layer output beyond max-abs 2e-2 only when it lies inside the
 * envelope propagated through the final combine (a proven rounding flip).
 *
 * Error model.  A dot product z = sum_k t_k (t_k = x_k * lut(w_k) * s_k) is
 * computed exactly here in double (every product is exact in double: 8 + 4 +
 * 24 significant bits, and the double sum's own error is below K * 2^-53 *
 * sum|t_k|).  A kernel that evaluates it with FP32 additions (and FP32 block
 * scale products), at most `depth` roundings of relative size u = 2^-24 on
 * the path from any term to the result, returns a value within
 * gamma(depth) * sum|t_k| of z (gamma(n) = n u / (1 - n u), the standard
 * bound for recursive summation).  The tensor-core kernels sum 16 exact
 * products per MMA into the FP32 accumulator; each MMA is taken to round at
 * most twice (its product sum and the add into the accumulator), so a 128-K
 * block of 8 MMAs adds 16 to the depth, the block-scale product 1 and the
 * FP32 sum over blocks one per block: depth <= 16 + 1 + K/128 (65 at K =
 * 4096), rounded up to the `depth` the caller states.  The CUDA kernels
 * stage activations as FP16 times 2^-e (e = 0 unless the row's largest
 * magnitude reaches 2^14); a BF16 value is then exact unless it falls below
 * FP16's normal range (|x| 2^-e < 2^-14), where it is off by at most 2^-25
 * 2^e: those terms add 2^-25 2^e |lut(w) s| each to the bound.
 *
 * The value rounded to BF16 is then one of the BF16 values between the
 * roundings of the envelope's ends (rounding is monotone).  The SwiGLU of the
 * reference (BF16 per-op rounding) is evaluated on every candidate pair of
 * gate / up BF16 values; the down projection is linear in the hidden row, so
 * its envelope is the exact sum over the hidden intervals plus the same
 * FP32 evaluation bound. */

/* The CUDA kernels' FP16 staging of a row with largest magnitude mx:
 * values below *tiny (FP16 subnormal after the 2^-e scale) may be off by
 * *err. */
static void env_f16_staging(double mx, double* tiny, double* err) {
  int e = 0;
  if (mx >= 16384.0) {
    int ex;
    frexp(mx, &ex);
    e = ex - 14;
  }
  *tiny = ldexp(1.0, -14 + e);
  *err = ldexp(1.0, -25 + e);
}

static double env_gamma(int depth) {
  const double u = ldexp(1.0, -24);
  return depth * u / (1.0 - depth * u) + ldexp(1.0, -45);
}

/* bit pattern order of BF16 values as integers: +0 < ... , -0 just below +0 */
static inline int32_t bf16_ord(uint16_t b) { return (b & 0x8000u) ? -(int32_t)(b & 0x7FFFu) - 1 : (int32_t)b; }
static inline uint16_t bf16_from_ord(int32_t o) { return o < 0 ? (uint16_t)(0x8000u | (uint32_t)(-(o + 1))) : (uint16_t)o; }

/* BF16 value interval reachable by rounding any FP32 value in [lo, hi]
 * (conservative: the double ends are rounded to the nearest FP32 first). */
static void bf16_range(double lo, double hi, uint16_t* rlo, uint16_t* rhi) {
  *rlo = bf16_from_f32((float)lo);
  *rhi = bf16_from_f32((float)hi);
}

typedef struct {
  const uint16_t* x;      /* [R, H] route rows */
  const uint32_t* order;  /* routes sorted by expert */
  const int64_t* start;   /* [E + 1] offsets into order */
  int64_t H, I, E, R;
  const uint8_t* gu_w;
  const float* gu_s;
  const uint8_t* d_w;
  const float* d_s;
  float limit;
  double g_gu, g_d;       /* gamma(depth) of the two projections */
  float* h_lo;            /* [R, I] hidden envelope */
  float* h_hi;
  float* d_lo;            /* [R, H] down envelope (BF16 values as floats) */
  float* d_hi;
  int64_t wide;           /* candidate sets that were cut off (should be 0) */
  pthread_mutex_t mu;
} env_ctx;

#define ENV_MAX_CAND 16384

/* one (expert, hidden row): gate and up envelopes of every route of the
 * expert, then the hidden envelope over all candidate pairs */
static void env_gate_up_item(void* p, int64_t item) {
  env_ctx* c = (env_ctx*)p;
  const int64_t e = item / c->I, row = item % c->I;
  const int64_t H = c->H, I = c->I;
  const int64_t scale_cols = (H + ORC_BLOCK - 1) / ORC_BLOCK;
  const int64_t half = (I + ORC_BLOCK - 1) / ORC_BLOCK;
  const uint8_t* gw = c->gu_w + (e * 2 * I + row) * H;
  const uint8_t* uw = c->gu_w + (e * 2 * I + I + row) * H;
  const float* gs = c->gu_s + (e * 2 * half + row / ORC_BLOCK) * scale_cols;
  const float* us = c->gu_s + (e * 2 * half + half + row / ORC_BLOCK) * scale_cols;
  int64_t wide = 0;
  for (int64_t q = c->start[e]; q < c->start[e + 1]; ++q) {
    const int64_t r = c->order[q];
    const uint16_t* xr = c->x + r * H;
    double mx = 0;
    for (int64_t k = 0; k < H; ++k) mx = fmax(mx, fabs((double)f32_from_bf16(xr[k])));
    double tiny, serr;
    env_f16_staging(mx, &tiny, &serr);
    double gz = 0, ga = 0, uz = 0, ua = 0, gs16 = 0, us16 = 0;
    for (int64_t k = 0; k < H; ++k) {
      const double xv = (double)f32_from_bf16(xr[k]);
      const double wg = (double)g_lut[gw[k]] * (double)gs[k / ORC_BLOCK];
      const double wu = (double)g_lut[uw[k]] * (double)us[k / ORC_BLOCK];
      const double tg = xv * wg, tu = xv * wu;
      gz += tg; ga += fabs(tg);
      uz += tu; ua += fabs(tu);
      if (xv != 0 && fabs(xv) < tiny) { gs16 += serr * fabs(wg); us16 += serr * fabs(wu); }
    }
    uint16_t g0, g1, u0, u1;
    bf16_range(gz - c->g_gu * ga - gs16, gz + c->g_gu * ga + gs16, &g0, &g1);
    bf16_range(uz - c->g_gu * ua - us16, uz + c->g_gu * ua + us16, &u0, &u1);
    /* The result is monotone in the up value for a fixed gate (the clip and
     * the final product are), so the up envelope's two ends suffice.  Gate
     * candidates are enumerated, except inside |g| < 2^-9, where the BF16
     * sigmoid is exactly 0.5 and silu = g / 2, so the result is monotone in
     * g there and that band's two ends suffice. */
    const float uend[2] = {f32_from_bf16(u0), f32_from_bf16(u1)};
    const int32_t go0 = bf16_ord(g0), go1 = bf16_ord(g1);
    const int32_t tneg = bf16_ord(0xBB00u), tpos = bf16_ord(0x3B00u);  /* -2^-9, +2^-9 */
    float lo = INFINITY, hi = -INFINITY;
    int32_t n = 0;
    for (int32_t go = go0; go <= go1; ++go) {
      if (go > tneg && go < tpos) {  /* tiny band: its ends only */
        const int32_t band_hi = go1 < tpos - 1 ? go1 : tpos - 1;
        if (go != band_hi) {
          for (int t = 0; t < 2; ++t) {
            const float h = f32_from_bf16(orc_swiglu_bf16(f32_from_bf16(bf16_from_ord(go)), uend[t], c->limit));
            lo = fminf(lo, h);
            hi = fmaxf(hi, h);
          }
          go = band_hi;
        }
      }
      if (++n > ENV_MAX_CAND) { ++wide; break; }
      for (int t = 0; t < 2; ++t) {
        const float h = f32_from_bf16(orc_swiglu_bf16(f32_from_bf16(bf16_from_ord(go)), uend[t], c->limit));
        lo = fminf(lo, h);
        hi = fmaxf(hi, h);
      }
    }
    c->h_lo[r * I + row] = lo;
    c->h_hi[r * I + row] = hi;
  }
  if (wide) {
    pthread_mutex_lock(&c->mu);
    c->wide += wide;
    pthread_mutex_unlock(&c->mu);
  }
}

/* one (expert, output row): the down envelope of every route of the expert */
static void env_down_item(void* p, int64_t item) {
  env_ctx* c = (env_ctx*)p;
  const int64_t e = item / c->H, h = item % c->H;
  const int64_t H = c->H, I = c->I;
  const int64_t scale_rows = (H + ORC_BLOCK - 1) / ORC_BLOCK;
  const int64_t scale_cols = (I + ORC_BLOCK - 1) / ORC_BLOCK;
  const uint8_t* wr = c->d_w + (e * H + h) * I;
  const float* srow = c->d_s + (e * scale_rows + h / ORC_BLOCK) * scale_cols;
  for (int64_t q = c->start[e]; q < c->start[e + 1]; ++q) {
    const int64_t r = c->order[q];
    const float* hl = c->h_lo + r * I;
    const float* hh = c->h_hi + r * I;
    double mx = 0;
    for (int64_t k = 0; k < I; ++k) mx = fmax(mx, fmax(fabs((double)hl[k]), fabs((double)hh[k])));
    double tiny, serr;
    env_f16_staging(mx, &tiny, &serr);
    double lo = 0, hi = 0, a = 0, s16 = 0;
    for (int64_t k = 0; k < I; ++k) {
      const double ws = (double)g_lut[wr[k]] * (double)srow[k / ORC_BLOCK];
      const double p0 = (double)hl[k] * ws, p1 = (double)hh[k] * ws;
      lo += p0 < p1 ? p0 : p1;
      hi += p0 < p1 ? p1 : p0;
      a += fabs(p0) > fabs(p1) ? fabs(p0) : fabs(p1);
      if (fmin(fabs((double)hl[k]), fabs((double)hh[k])) < tiny && (hl[k] != 0 || hh[k] != 0)) s16 += serr * fabs(ws);
    }
    uint16_t d0, d1;
    bf16_range(lo - c->g_d * a - s16, hi + c->g_d * a + s16, &d0, &d1);
    c->d_lo[r * H + h] = f32_from_bf16(d0);
    c->d_hi[r * H + h] = f32_from_bf16(d1);
  }
}

/* Envelopes of the BF16 down rows of R routes (row r = expert ids[r] applied
 * to x[r]) through a packed bank (layout of orc_packed_decode_moe), with the
 * gate/up and down projections evaluated at FP32 depth depth_gu / depth_d.
 * d_lo / d_hi [R, H] (and optionally h_lo / h_hi [R, I]) receive the
 * envelope ends.  Returns the number of candidate sets that had to be cut
 * (0 means the envelope is complete), or -1 for a bad expert id. */
int64_t orc_rows_envelope(const uint16_t* x, int64_t R, int64_t H, const uint32_t* ids,
                          const uint8_t* gu_w, const float* gu_s, const uint8_t* d_w, const float* d_s,
                          int64_t E, int64_t I, float limit, int depth_gu, int depth_d,
                          float* d_lo, float* d_hi, float* h_lo_out, float* h_hi_out, int nthreads) {
  lut_init();
  for (int64_t r = 0; r < R; ++r)
    if ((int64_t)ids[r] >= E) return -1;
  int64_t* start = (int64_t*)calloc((size_t)E + 1, sizeof(int64_t));
  uint32_t* order = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(R > 0 ? R : 1));
  for (int64_t r = 0; r < R; ++r) start[ids[r] + 1]++;
  for (int64_t e = 0; e < E; ++e) start[e + 1] += start[e];
  int64_t* fill = (int64_t*)malloc(sizeof(int64_t) * (size_t)E);
  for (int64_t e = 0; e < E; ++e) fill[e] = start[e];
  for (int64_t r = 0; r < R; ++r) order[fill[ids[r]]++] = (uint32_t)r;
  free(fill);
  env_ctx c;
  memset(&c, 0, sizeof(c));
  c.x = x; c.order = order; c.start = start; c.H = H; c.I = I; c.E = E; c.R = R;
  c.gu_w = gu_w; c.gu_s = gu_s; c.d_w = d_w; c.d_s = d_s; c.limit = limit;
  c.g_gu = env_gamma(depth_gu);
  c.g_d = env_gamma(depth_d);
  c.h_lo = h_lo_out ? h_lo_out : (float*)malloc(sizeof(float) * (size_t)(R * I > 0 ? R * I : 1));
  c.h_hi = h_hi_out ? h_hi_out : (float*)malloc(sizeof(float) * (size_t)(R * I > 0 ? R * I : 1));
  c.d_lo = d_lo; c.d_hi = d_hi;
  pthread_mutex_init(&c.mu, NULL);
  parallel_for(E * I, nthreads, env_gate_up_item, &c);
  if (d_lo && d_hi) parallel_for(E * H, nthreads, env_down_item, &c);
  pthread_mutex_destroy(&c.mu);
  if (!h_lo_out) free(c.h_lo);
  if (!h_hi_out) free(c.h_hi);
  free(start);
  free(order);
  return c.wide;
}

typedef struct {
  const float* h;          /* [R, I] the kernel's hidden rows */
  const uint32_t* order;
  const int64_t* start;
  int64_t H, I;
  const uint8_t* d_w;
  const float* d_s;
  double g;
  double* lo;              /* [R, H] */
  double* hi;
} down_ctx;

static void down_interval_item(void* p, int64_t item) {
  down_ctx* c = (down_ctx*)p;
  const int64_t e = item / c->H, h = item % c->H;
  const int64_t H = c->H, I = c->I;
  const int64_t scale_rows = (H + ORC_BLOCK - 1) / ORC_BLOCK;
  const int64_t scale_cols = (I + ORC_BLOCK - 1) / ORC_BLOCK;
  const uint8_t* wr = c->d_w + (e * H + h) * I;
  const float* srow = c->d_s + (e * scale_rows + h / ORC_BLOCK) * scale_cols;
  for (int64_t q = c->start[e]; q < c->start[e + 1]; ++q) {
    const int64_t r = c->order[q];
    const float* hr = c->h + r * I;
    double mx = 0;
    for (int64_t k = 0; k < I; ++k) mx = fmax(mx, fabs((double)hr[k]));
    double tiny, serr;
    env_f16_staging(mx, &tiny, &serr);
    double z = 0, a = 0, s16 = 0;
    for (int64_t k = 0; k < I; ++k) {
      const double ws = (double)g_lut[wr[k]] * (double)srow[k / ORC_BLOCK];
      const double t = (double)hr[k] * ws;
      z += t;
      a += fabs(t);
      if (hr[k] != 0 && fabs((double)hr[k]) < tiny) s16 += serr * fabs(ws);
    }
    c->lo[r * H + h] = z - c->g * a - s16;
    c->hi[r * H + h] = z + c->g * a + s16;
  }
}

/* Real interval [lo, hi] that contains every FP32 evaluation (at most `depth`
 * roundings on a term's path) of the down projection of route r's hidden row
 * h[r] (given values, e.g. the kernel's own) through expert ids[r]: the exact
 * dot product plus / minus gamma(depth) * sum |terms| (plus the FP16 staging
 * allowance of orc_rows_envelope for hidden values below FP16's normal range).  The parity tests
 * check the kernel's FP32 or BF16 down values against it. */
int orc_down_interval(const float* h, int64_t R, int64_t I, const uint32_t* ids, const uint8_t* d_w,
                      const float* d_s, int64_t E, int64_t H, int depth, double* lo, double* hi, int nthreads) {
  lut_init();
  for (int64_t r = 0; r < R; ++r)
    if ((int64_t)ids[r] >= E) return 3;
  int64_t* start = (int64_t*)calloc((size_t)E + 1, sizeof(int64_t));
  uint32_t* order = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(R > 0 ? R : 1));
  for (int64_t r = 0; r < R; ++r) start[ids[r] + 1]++;
  for (int64_t e = 0; e < E; ++e) start[e + 1] += start[e];
  int64_t* fill = (int64_t*)malloc(sizeof(int64_t) * (size_t)E);
  for (int64_t e = 0; e < E; ++e) fill[e] = start[e];
  for (int64_t r = 0; r < R; ++r) order[fill[ids[r]]++] = (uint32_t)r;
  free(fill);
  down_ctx c = {h, order, start, H, I, d_w, d_s, env_gamma(depth), lo, hi};
  parallel_for(E * H, nthreads, down_interval_item, &c);
  free(start);
  free(order);
  return 0;
}
