/*
 * kvq_oracle.c — CPU restatement of mlx-bun's quantized-KV attention path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library and the timed CPU baseline; nothing in the product path links it.
 *
 * What it restates (paths are inside the mlx-bun project):
 *   - MLX affine group quantize as called by ops.quantize
 *     (src/mlx/ops.ts:615-637 -> mlx_quantize).  MLX itself is a third-party
 *     dependency absent here (pinned by the project at mlx 0.31.2,
 *     CLAUDE.md:31-32); the rule below was recovered from, and is checked
 *     bit-exactly against, goldens/rotating-kvq.bin (bf16, gs 32, 8 bit):
 *       per group, in f32:  anchor = (|min| > |max|) ? min : max
 *                           s0     = (max - min) / (2^bits - 1), negated when
 *                                    the anchor is max
 *                           q0     = round_half_away(anchor / s0)
 *                           scale  = anchor / q0        (q0 != 0)
 *                           code   = clamp(round_half_away((w - anchor) /
 *                                    scale), 0, 2^bits - 1)
 *                           stored = (dtype(scale), dtype(anchor))
 *     Codes use the UNROUNDED f32 scale (rounding it first reproduces only
 *     ~52% of the golden codes).  Unpinned edge: a group whose range is
 *     below KVQO_EPS (constant group) uses s0 = +-KVQO_EPS, and q0 == 0 gives
 *     (scale = s0, bias = 0).  Both implementations share this choice.
 *   - Packing (src/model/fused-decode-kernel.ts:102-114): element e of a row
 *     sits in word e / (32/bits) at bit bits*(e % (32/bits)), LSB first.
 *   - The unfused SDPA op graph quantizedSdpaUnfused
 *     (src/model/gemma4-base.ts:1273-1342) with its rounding points:
 *       q * dtype(scale) rounded to dtype            (:1285, ops.ts:47-60)
 *       scores = quantized_matmul(q, K^T) -> dtype   (:1307)
 *       masked with dtype finfo.min                  (:1310-1330, :1263-1267)
 *       softmax(precise) in f32 -> dtype             (:1332)
 *       out = quantized_matmul(P, V) -> dtype        (:1334)
 *     GQA maps query head h to kv head h / (Hq/Hkv) (:1289-1305).
 *     Masks: bottom-right aligned causal, optional window
 *     (createCausalMask :1595-1614; causal string path :1312-1319).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define KVQO_F16 9
#define KVQO_BF16 12
#define KVQO_EPS 1e-7f

/* ---------------- 16-bit float conversions (IEEE RNE, own code) -------- */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float kvqo_half_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ffu;
  if (exp == 0) {
    if (man == 0) return u2f(sign);
    /* subnormal: value = man * 2^-24 */
    float v = (float)man * 5.9604644775390625e-08f;
    return sign ? -v : v;
  }
  if (exp == 31) return u2f(sign | 0x7f800000u | (man << 13));
  return u2f(sign | ((exp + 112) << 23) | (man << 13));
}

uint16_t kvqo_f32_to_half(float f) {
  uint32_t u = f2u(f);
  uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
  uint32_t a = u & 0x7fffffffu;
  if (a >= 0x7f800000u) /* inf / nan */
    return (uint16_t)(sign | 0x7c00u | (a > 0x7f800000u ? 0x200u : 0u));
  if (a >= 0x477ff000u) /* rounds to >= 65520 -> inf */
    return (uint16_t)(sign | 0x7c00u);
  if (a < 0x38800000u) { /* below 2^-14: subnormal half (or zero) */
    if (a < 0x33000000u) return sign; /* < 2^-25 rounds to 0 (tie at 2^-25 -> even = 0) */
    uint32_t e = a >> 23;                 /* biased f32 exponent */
    uint32_t m = (a & 0x7fffffu) | 0x800000u;
    uint32_t shift = 126 - e;             /* 14 + 113 - e - 1 ... result = m >> (shift) */
    /* value = m * 2^(e-150); half subnormal unit = 2^-24 -> units = m * 2^(e-126) */
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  /* normal range */
  uint32_t e = (a >> 23) - 112;          /* half biased exponent (1..30) */
  uint32_t m = a & 0x7fffffu;
  uint32_t q = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++; /* carry may bump exponent */
  return (uint16_t)(sign | q);
}

float kvqo_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

uint16_t kvqo_f32_to_bf16(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet nan */
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

static inline float to_f32(uint16_t v, int dtype) {
  return dtype == KVQO_BF16 ? kvqo_bf16_to_f32(v) : kvqo_half_to_f32(v);
}
static inline uint16_t from_f32(float v, int dtype) {
  return dtype == KVQO_BF16 ? kvqo_f32_to_bf16(v) : kvqo_f32_to_half(v);
}
static inline float round_dt(float v, int dtype) { return to_f32(from_f32(v, dtype), dtype); }

/* dtype finfo.min (src/model/gemma4-base.ts:1263-1267) */
static inline float finfo_min(int dtype) {
  return dtype == KVQO_BF16 ? -3.3895313892515355e38f : -65504.0f;
}

/* ---------------- affine group quantize ---------------- */

/* One group of gs f32 values -> codes[gs], (scale, bias) in f32 before the
 * dtype rounding of the stored scale. */
static void quantize_group(const float* w, int gs, int bits, uint32_t* codes,
                           float* scale_out, float* bias_out) {
  const float nbins = (float)((1 << bits) - 1);
  float mn = w[0], mx = w[0];
  for (int i = 1; i < gs; i++) {
    mn = w[i] < mn ? w[i] : mn;
    mx = w[i] > mx ? w[i] : mx;
  }
  float s0 = (mx - mn) / nbins;
  if (!(s0 >= KVQO_EPS)) s0 = KVQO_EPS;
  const int neg = fabsf(mn) > fabsf(mx);
  const float anchor = neg ? mn : mx;
  s0 = neg ? s0 : -s0;
  const float q0 = roundf(anchor / s0);
  float scale, bias;
  if (q0 != 0.0f) {
    scale = anchor / q0;
    bias = anchor;
  } else {
    scale = s0;
    bias = 0.0f;
  }
  for (int i = 0; i < gs; i++) {
    float c = roundf((w[i] - bias) / scale);
    c = c < 0.0f ? 0.0f : (c > nbins ? nbins : c);
    codes[i] = (uint32_t)c;
  }
  *scale_out = scale;
  *bias_out = bias;
}

/* Quantize `rows` contiguous rows of D dtype values. */
void kvqo_quantize_rows(const uint16_t* x, int64_t rows, int D, int gs, int bits, int dtype,
                        uint32_t* packed, uint16_t* scales, uint16_t* biases) {
  const int per = 32 / bits;
  const int words = D / per;
  const int ngroups = D / gs;
  float* w = (float*)malloc(sizeof(float) * (size_t)gs);
  uint32_t* codes = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)D);
  for (int64_t r = 0; r < rows; r++) {
    for (int g = 0; g < ngroups; g++) {
      for (int i = 0; i < gs; i++) w[i] = to_f32(x[r * D + g * gs + i], dtype);
      float sc, bi;
      quantize_group(w, gs, bits, codes + g * gs, &sc, &bi);
      scales[r * ngroups + g] = from_f32(sc, dtype);
      biases[r * ngroups + g] = from_f32(bi, dtype);
    }
    for (int wd = 0; wd < words; wd++) {
      uint32_t v = 0;
      for (int j = 0; j < per; j++) v |= codes[wd * per + j] << (bits * j);
      packed[r * words + wd] = v;
    }
  }
  free(w);
  free(codes);
}

/* Dequantize rows to f32: w = scale * code + bias (f32). */
void kvqo_dequantize_rows(const uint32_t* packed, const uint16_t* scales, const uint16_t* biases,
                          int64_t rows, int D, int gs, int bits, int dtype, float* out) {
  const int per = 32 / bits;
  const uint32_t mask = (1u << bits) - 1u;
  for (int64_t r = 0; r < rows; r++)
    for (int e = 0; e < D; e++) {
      const uint32_t c = (packed[r * (D / per) + e / per] >> (bits * (e % per))) & mask;
      const float sc = to_f32(scales[r * (D / gs) + e / gs], dtype);
      const float bi = to_f32(biases[r * (D / gs) + e / gs], dtype);
      out[r * D + e] = sc * (float)c + bi;
    }
}

/* ---------------- unfused SDPA op graph ---------------- */

typedef struct kvqo_view {
  const uint32_t* packed;
  const uint16_t* scales;
  const uint16_t* biases;
  int64_t batch_stride; /* rows */
  int64_t head_stride;  /* rows */
} kvqo_view;

static void dequant_row(const kvqo_view* t, int64_t row, int D, int gs, int bits, int dtype,
                        float* out) {
  kvqo_dequantize_rows(t->packed + row * (D * bits / 32), t->scales + row * (D / gs),
                       t->biases + row * (D / gs), 1, D, gs, bits, dtype, out);
}

/*
 * q   [B, Hq, L, D] dtype, contiguous.  out [B, Hq, L, D] dtype.
 * K/V views are [B, Hkv, N, *] with row strides.  seq_lens (nullable) gives
 * a per-batch key count N_b <= N (rows [0, N_b) are attended).
 * mask_mode 0: none; 1: bottom-right aligned causal; window > 0 adds the
 * sliding-window condition j > (N_b - L + i) - window (createCausalMask).
 * scores_out (nullable) receives the dtype-rounded masked logits
 * [B, Hq, L, N] as f32 (entries beyond N_b are left untouched).
 */
int kvqo_sdpa_unfused(const uint16_t* q, const kvqo_view* K, const kvqo_view* V, int B, int Hq,
                      int Hkv, int L, int N, int D, int gs, int bits, int dtype, float scale,
                      int mask_mode, int window, const int32_t* seq_lens, uint16_t* out,
                      float* scores_out, int threads) {
  if (Hkv <= 0 || Hq % Hkv != 0) return -1;
  const int nrep = Hq / Hkv;
  const float scale_dt = round_dt(scale, dtype);
  const float neg = finfo_min(dtype);
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
  int64_t total = (int64_t)B * Hq;
#pragma omp parallel
  {
    float* kd = (float*)malloc(sizeof(float) * (size_t)D);
    float* qs = (float*)malloc(sizeof(float) * (size_t)D);
    float* s = (float*)malloc(sizeof(float) * (size_t)(N > 0 ? N : 1));
    float* acc = (float*)malloc(sizeof(float) * (size_t)D);
#pragma omp for schedule(dynamic, 1)
    for (int64_t bh = 0; bh < total; bh++) {
      const int b = (int)(bh / Hq), h = (int)(bh % Hq), kvh = h / nrep;
      const int Nb = seq_lens ? seq_lens[b] : N;
      const int64_t kbase = b * K->batch_stride + kvh * K->head_stride;
      const int64_t vbase = b * V->batch_stride + kvh * V->head_stride;
      for (int l = 0; l < L; l++) {
        const uint16_t* qrow = q + (((int64_t)b * Hq + h) * L + l) * D;
        for (int d = 0; d < D; d++) qs[d] = round_dt(to_f32(qrow[d], dtype) * scale_dt, dtype);
        const int qpos = Nb - L + l; /* bottom-right aligned query position */
        for (int n = 0; n < Nb; n++) {
          dequant_row(K, kbase + n, D, gs, bits, dtype, kd);
          float a = 0.0f;
          for (int d = 0; d < D; d++) a += qs[d] * kd[d];
          float sv = round_dt(a, dtype);
          if (mask_mode == 1) {
            int ok = n <= qpos;
            if (window > 0) ok = ok && (qpos < n + window);
            if (!ok) sv = neg;
          }
          s[n] = sv;
          if (scores_out) scores_out[(((int64_t)b * Hq + h) * L + l) * N + n] = sv;
        }
        /* softmax(precise): f32 internally, rounded to dtype */
        float m = -INFINITY;
        for (int n = 0; n < Nb; n++) m = s[n] > m ? s[n] : m;
        float sum = 0.0f;
        for (int n = 0; n < Nb; n++) {
          s[n] = expf(s[n] - m);
          sum += s[n];
        }
        for (int n = 0; n < Nb; n++) s[n] = round_dt(s[n] / sum, dtype);
        for (int d = 0; d < D; d++) acc[d] = 0.0f;
        for (int n = 0; n < Nb; n++) {
          if (s[n] == 0.0f) continue;
          dequant_row(V, vbase + n, D, gs, bits, dtype, kd);
          for (int d = 0; d < D; d++) acc[d] += s[n] * kd[d];
        }
        uint16_t* orow = out + (((int64_t)b * Hq + h) * L + l) * D;
        for (int d = 0; d < D; d++) orow[d] = from_f32(acc[d], dtype);
      }
    }
    free(kd);
    free(qs);
    free(s);
    free(acc);
  }
  return 0;
}

/* Number of OpenMP threads the baseline will use. */
int kvqo_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
