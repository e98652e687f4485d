/*
 * C form of the CPU oracle -- TEST INFRASTRUCTURE ONLY (the timed CPU baseline of bench.py and the
 * `--impl reference` arm, and a cross-check of the numpy oracle). Nothing in the product links it.
 *
 * It restates strata-mlx's block decoders (strata_mlx/blocks.py:40-193, unpack32 with the same float32
 * operations in the same order), the matvec's per-run sums (blocks.py:196-220), mlx-lm's swiglu as
 * blocks.py:230-238 states it, the router product (fused.py:334-354), top-k with ties to the lower index
 * (fused.py:400-418), the softmax over the chosen logits (fused.py:491) and moe_combine's order
 * (fused.py:448-462). Parallel over rows with OpenMP.
 *
 * Build: oracle/build.py (gcc -O3 -march=native -fopenmp -ffp-contract=off -shared).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#include "iq_tables_ref.h"

enum { Q2_0 = 0, IQ4_NL, IQ4_XS, IQ3_S, IQ3_XXS, IQ2_S, IQ2_XS, IQ2_XXS, IQ1_M, Q3_K, Q8_0 };
static const int PER_BLOCK[] = {64, 32, 256, 256, 256, 256, 256, 256, 256, 256, 32};
static const int BLOCK_BYTES[] = {18, 18, 136, 110, 98, 82, 74, 66, 56, 110, 34};
static const int8_t KVAL[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

static float half_bits(uint32_t h) {
  _Float16 v;
  uint16_t b = (uint16_t)h;
  memcpy(&v, &b, 2);
  return (float)v;
}
static uint32_t u16_at(const uint8_t* b) { return (uint32_t)b[0] | ((uint32_t)b[1] << 8); }
static uint32_t u32_at(const uint8_t* b) { return u16_at(b) | (u16_at(b + 2) << 16); }
static float half_at(const uint8_t* b) { return half_bits(u16_at(b)); }
static float neg_if(float v, uint32_t bit) { return bit ? -v : v; }

static float q3k_scale(const uint8_t* s, uint32_t k) {
  uint32_t p = k % 4, word = k / 4;
  uint32_t low = word < 2 ? ((uint32_t)s[4 * word + p] & 15) : ((uint32_t)s[4 * (word - 2) + p] >> 4);
  return (float)((int)(low | ((((uint32_t)s[8 + p] >> (2 * word)) & 3) << 4)) - 32);
}

/* run n (32 weights) of a row: blocks.py:57-193 */
void ref_unpack32(int kind, const uint8_t* row, int n, float* w) {
  if (kind == Q2_0) {
    const uint8_t* b = row + (n / 2) * 18;
    const uint8_t* q = b + 2 + 8 * (n % 2);
    float d = half_at(b);
    for (int i = 0; i < 8; ++i)
      for (int j = 0; j < 4; ++j) w[4 * i + j] = d * ((float)((q[i] >> (2 * j)) & 3) - 1.0f);
  } else if (kind == IQ4_NL) {
    const uint8_t* b = row + n * 18;
    float d = half_at(b);
    for (int i = 0; i < 16; ++i) {
      w[i] = d * (float)KVAL[b[2 + i] & 15];
      w[16 + i] = d * (float)KVAL[b[2 + i] >> 4];
    }
  } else if (kind == IQ4_XS) {
    const uint8_t* b = row + (n / 8) * 136;
    uint32_t ib = n % 8;
    uint32_t ls = (((uint32_t)b[4 + ib / 2] >> (4 * (ib % 2))) & 15) | (((u16_at(b + 2) >> (2 * ib)) & 3) << 4);
    float d = half_at(b) * ((float)ls - 32.0f);
    const uint8_t* q = b + 8 + 16 * ib;
    for (int i = 0; i < 16; ++i) {
      w[i] = d * (float)KVAL[q[i] & 15];
      w[16 + i] = d * (float)KVAL[q[i] >> 4];
    }
  } else if (kind == IQ3_S) {
    const uint8_t* b = row + (n / 8) * 110;
    uint32_t ib = n % 8;
    float d = half_at(b) * (float)(1 + 2 * (((uint32_t)b[106 + ib / 2] >> (4 * (ib % 2))) & 15));
    uint32_t high = b[66 + ib];
    for (int l = 0; l < 8; ++l) {
      const uint8_t* g = ref_iq3s_grid[(uint32_t)b[2 + 8 * ib + l] | (((high >> l) & 1) << 8)];
      uint32_t sign = (uint32_t)b[74 + 4 * ib + l / 2] >> (4 * (l % 2));
      for (int j = 0; j < 4; ++j) w[4 * l + j] = neg_if(d * (float)g[j], (sign >> j) & 1);
    }
  } else if (kind == IQ3_XXS) {
    const uint8_t* b = row + (n / 8) * 98;
    uint32_t ib = n % 8;
    uint32_t aux = u32_at(b + 66 + 4 * ib);
    float d = half_at(b) * (0.5f + (float)(aux >> 28)) * 0.5f;
    for (int l = 0; l < 8; ++l) {
      const uint8_t* g = ref_iq3xxs_grid[b[2 + 8 * ib + l]];
      uint32_t sign = (uint32_t)ref_ksigns[(aux >> (7 * (l / 2))) & 127] >> (4 * (l % 2));
      for (int j = 0; j < 4; ++j) w[4 * l + j] = neg_if(d * (float)g[j], (sign >> j) & 1);
    }
  } else if (kind == IQ2_S) {
    const uint8_t* b = row + (n / 8) * 82;
    uint32_t ib = n % 8;
    float d = half_at(b) * 0.25f;
    uint32_t high = b[66 + ib], scales = b[74 + ib];
    for (int l = 0; l < 4; ++l) {
      const uint8_t* g = ref_iq2s_grid[(uint32_t)b[2 + 4 * ib + l] | (((high >> (2 * l)) & 3) << 8)];
      uint32_t sign = b[34 + 4 * ib + l];
      float dl = d * (0.5f + (float)(l < 2 ? scales & 15 : scales >> 4));
      for (int j = 0; j < 8; ++j) w[8 * l + j] = neg_if(dl * (float)g[j], (sign >> j) & 1);
    }
  } else if (kind == IQ2_XS) {
    const uint8_t* b = row + (n / 8) * 74;
    uint32_t ib = n % 8;
    float d = half_at(b) * 0.25f;
    uint32_t scales = b[66 + ib];
    for (int l = 0; l < 4; ++l) {
      uint32_t q = u16_at(b + 2 + 2 * (4 * ib + l));
      const uint8_t* g = ref_iq2xs_grid[q & 511];
      uint32_t sign = ref_ksigns[q >> 9];
      float dl = d * (0.5f + (float)(l < 2 ? scales & 15 : scales >> 4));
      for (int j = 0; j < 8; ++j) w[8 * l + j] = neg_if(dl * (float)g[j], (sign >> j) & 1);
    }
  } else if (kind == IQ2_XXS) {
    const uint8_t* b = row + (n / 8) * 66;
    const uint8_t* q = b + 2 + 8 * (n % 8);
    uint32_t aux = u32_at(q + 4);
    float d = half_at(b) * (0.5f + (float)(aux >> 28)) * 0.25f;
    for (int l = 0; l < 4; ++l) {
      const uint8_t* g = ref_iq2xxs_grid[q[l]];
      uint32_t sign = ref_ksigns[(aux >> (7 * l)) & 127];
      for (int j = 0; j < 8; ++j) w[8 * l + j] = neg_if(d * (float)g[j], (sign >> j) & 1);
    }
  } else if (kind == Q3_K) {
    const uint8_t* b = row + (n / 8) * 110;
    uint32_t r = n % 8;
    const uint8_t* q = b + 32 + 32 * (r / 4);
    uint32_t shift = 2 * (r % 4);
    float d = half_at(b + 108);
    float s0 = d * q3k_scale(b + 96, 2 * r), s1 = d * q3k_scale(b + 96, 2 * r + 1);
    for (int i = 0; i < 32; ++i) {
      int v = (int)(((uint32_t)q[i] >> shift) & 3) - ((((uint32_t)b[i] >> r) & 1) ? 0 : 4);
      w[i] = (i < 16 ? s0 : s1) * (float)v;
    }
  } else if (kind == IQ1_M) {
    const uint8_t* b = row + (n / 8) * 56;
    uint32_t ib = n % 8;
    uint32_t packed = (u16_at(b + 48) >> 12) | ((u16_at(b + 50) >> 8) & 0x00f0) | ((u16_at(b + 52) >> 4) & 0x0f00) |
                      (u16_at(b + 54) & 0xf000);
    float d = half_bits(packed);
    uint32_t scales = u16_at(b + 48 + 2 * (ib / 2)) >> (6 * (ib % 2));
    for (int l = 0; l < 4; ++l) {
      uint32_t high = ((uint32_t)b[32 + 2 * ib + l / 2] >> (4 * (l % 2))) & 15;
      const uint8_t* g = ref_iq1_grid[(uint32_t)b[4 * ib + l] | ((high & 7) << 8)];
      float dl = d * (float)(2 * ((scales >> (3 * (l / 2))) & 7) + 1);
      float delta = (high & 8) ? -1.125f : -0.875f;
      for (int j = 0; j < 8; ++j) w[8 * l + j] = dl * ((float)g[j] + delta);
    }
  } else if (kind == Q8_0) {
    const uint8_t* b = row + n * 34;
    float d = half_at(b);
    for (int i = 0; i < 32; ++i) w[i] = d * (float)(int8_t)b[2 + i];
  }
}

int64_t ref_row_bytes(int kind, int64_t cols) {
  if (kind < 0 || kind > Q8_0 || cols % PER_BLOCK[kind]) return -1;
  return cols / PER_BLOCK[kind] * BLOCK_BYTES[kind];
}

int ref_dequant(int kind, const uint8_t* blocks, int64_t mats, int rows, int cols, float* out) {
  int64_t rb = ref_row_bytes(kind, cols);
  if (rb < 0) return -2;
  int64_t total = mats * rows;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < total; ++r)
    for (int n = 0; n < cols / 32; ++n) ref_unpack32(kind, blocks + r * rb, n, out + r * cols + 32 * n);
  return 0;
}

/* one row . x with the reference matvec's order: a float32 sum per run, added to the row's sum */
static float row_dot(int kind, const uint8_t* row, int cols, const float* x) {
  float w[32], sum = 0.0f;
  for (int n = 0; n < cols / 32; ++n) {
    ref_unpack32(kind, row, n, w);
    float s = 0.0f;
    for (int j = 0; j < 32; ++j) s += w[j] * x[32 * n + j];
    sum += s;
  }
  return sum;
}

/* out[r] = W[r] . x for a matrix of rows x cols blocks */
void ref_matvec(int kind, const uint8_t* w, int rows, int cols, const float* x, float* out) {
  int64_t rb = ref_row_bytes(kind, cols);
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) out[r] = row_dot(kind, w + r * rb, cols, x);
}

/* rounding to the activations' type: 1 float16, 2 bfloat16 (nearest even), else none */
static float round_to(float v, int dtype) {
  if (dtype == 1) return (float)(_Float16)v;
  if (dtype == 2) {
    uint32_t u;
    memcpy(&u, &v, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) return v;
    u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
    memcpy(&v, &u, 4);
  }
  return v;
}

static float swiglu_mlx(float g, float u, int dt) {
  g = round_to(g, dt);
  u = round_to(u, dt);
  float y = 1.0f / (1.0f + expf(fabsf(g)));
  float sig = round_to(g < 0.0f ? y : 1.0f - y, dt);
  float a = round_to(g * sig, dt);
  return round_to(a * u, dt);
}

typedef struct ref_layer {
  int hidden, inter, experts, top_k, dtype;
  int kind_gate, kind_up, kind_down;
  const uint8_t *gate, *up, *down;
  const uint16_t* router;
  int shared_inter, kind_sgate, kind_sup, kind_sdown;
  const uint8_t *sgate, *sup, *sdown;
  const uint16_t* shared_gate;
} ref_layer;

static void expert_glu(int kg, const uint8_t* g, int ku, const uint8_t* u, int kd, const uint8_t* d, int H, int I,
                       const float* x, int dt, float* h, float* y) {
  int64_t rbg = ref_row_bytes(kg, H), rbu = ref_row_bytes(ku, H), rbd = ref_row_bytes(kd, I);
#pragma omp parallel for schedule(static)
  for (int r = 0; r < I; ++r)
    h[r] = swiglu_mlx(row_dot(kg, g + r * rbg, H, x), row_dot(ku, u + r * rbu, H, x), dt);
#pragma omp parallel for schedule(static)
  for (int r = 0; r < H; ++r) y[r] = round_to(row_dot(kd, d + r * rbd, I, h), dt);
}

/* One MoE block (fused.py:487-497) for T tokens x (T, H) float32 holding values of the activations' type.
 * out (T, H); idx, w (T, K) the routes. Returns 0, or a negative code for a shape it does not take. */
int ref_moe_layer(const ref_layer* L, const float* x, int T, float* out, uint32_t* idx, float* wts) {
  const int H = L->hidden, I = L->inter, E = L->experts, K = L->top_k, Is = L->shared_inter, dt = L->dtype;
  if (K > 16 || K > E) return -2;
  float* xr = malloc(sizeof(float) * H);
  float* logits = malloc(sizeof(float) * E);
  float* h = malloc(sizeof(float) * (I > Is ? I : Is));
  float* y = malloc(sizeof(float) * (size_t)K * H);
  float* s = malloc(sizeof(float) * H);
  for (int t = 0; t < T; ++t) {
    for (int c = 0; c < H; ++c) xr[c] = round_to(x[(size_t)t * H + c], dt);
#pragma omp parallel for schedule(static)
    for (int e = 0; e < E; ++e) {
      float acc = 0.0f;
      for (int c = 0; c < H; ++c) acc += half_bits(L->router[(size_t)e * H + c]) * xr[c];
      logits[e] = acc;
    }
    uint32_t* it = idx + (size_t)t * K;
    float sel[16];
    for (int k = 0; k < K; ++k) {
      int best = -1;
      for (int e = 0; e < E; ++e) {
        int taken = 0;
        for (int q = 0; q < k; ++q) taken |= (it[q] == (uint32_t)e);
        if (!taken && (best < 0 || logits[e] > logits[best])) best = e;
      }
      it[k] = (uint32_t)best;
      sel[k] = logits[best];
    }
    float sum = 0.0f, ex[16];
    for (int k = 0; k < K; ++k) sum += (ex[k] = expf(sel[k] - sel[0]));
    float* wt = wts + (size_t)t * K;
    for (int k = 0; k < K; ++k) wt[k] = ex[k] / sum;
    const int64_t gstride = (int64_t)I * ref_row_bytes(L->kind_gate, H);
    const int64_t ustride = (int64_t)I * ref_row_bytes(L->kind_up, H);
    const int64_t dstride = (int64_t)H * ref_row_bytes(L->kind_down, I);
    for (int k = 0; k < K; ++k) {
      const int64_t e = it[k];
      expert_glu(L->kind_gate, L->gate + e * gstride, L->kind_up, L->up + e * ustride, L->kind_down,
                 L->down + e * dstride, H, I, xr, dt, h, y + (size_t)k * H);
    }
    float g = -INFINITY;
    if (Is) {
      float acc = 0.0f;
      for (int c = 0; c < H; ++c) acc += half_bits(L->shared_gate[c]) * xr[c];
      g = round_to(acc, dt);
      expert_glu(L->kind_sgate, L->sgate, L->kind_sup, L->sup, L->kind_sdown, L->sdown, H, Is, xr, dt, h, s);
    } else {
      memset(s, 0, sizeof(float) * H);
    }
    const float gate = round_to(1.0f / (1.0f + expf(-g)), dt);
#pragma omp parallel for schedule(static)
    for (int i = 0; i < H; ++i) {
      float acc = 0.0f;
      for (int j = 0; j < 8 && j < K; ++j) {
        float part = 0.0f;
        for (int k = j; k < K; k += 8) part = y[(size_t)k * H + i] * wt[k] + part;
        acc = j == 0 ? part : part + acc;
      }
      out[(size_t)t * H + i] = round_to(round_to(acc, dt) + round_to(gate * s[i], dt), dt);
    }
  }
  free(xr);
  free(logits);
  free(h);
  free(y);
  free(s);
  return 0;
}

int ref_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
#else
  (void)n;
  return 1;
#endif
}
