/*
 * fmha_oracle.c -- CPU restatement of the reference's decode attention.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the thing measured or
 * shipped). The product CUDA path in fmha_b200/ does not link this file.
 *
 * Follows fmha_host.cpp:158-244 (do_validation) of HGLiu1998/fmha:
 *   scores[s] = sum_d float(q[d]) * float(k[s][d])     (fmha_host.cpp:179-197)
 *   scores[s] *= 1/sqrtf(D)                             (fmha_host.cpp:210-212)
 *   max, sumExp += expf(s - max), p = expf(s - max)/sumExp
 *                                                       (fmha_host.cpp:215-226)
 *   o[d] = sum_s p[s] * float(v[s][d]), cast to fp16    (fmha_host.cpp:230-243)
 * with two deliberate changes for the B200 library's contract:
 *   - K/V are indexed in the [B,H,S,D] layout (the reference packs them as
 *     [sum S, Hkv, D]); the packed form is kept in fmha_oracle_decode_thd();
 *   - the kv head of query head h is h / (Hq/Hkv) (the reference indexes K/V
 *     with the query head, fmha_host.cpp:190-191, which is not GQA).
 * P stays fp32 in "exact" mode; "ref-faithful" mode rounds it to bf16 as
 * fmha_host.cpp:225 does.
 *
 * Build: -O2 -ffp-contract=off (no FMA contraction, like the reference's
 * x86-64 build) and -fopenmp for the batch-parallel loop.
 */
#include "fmha_oracle.h"

#include <math.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- numbers */

float fmha_oracle_bf16_to_f32(uint16_t x) {
  uint32_t u = (uint32_t)x << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

uint16_t fmha_oracle_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
    return (uint16_t)((u >> 16) | 0x0040u); /* quiet NaN */
  }
  u += 0x7fffu + ((u >> 16) & 1u); /* round to nearest even */
  return (uint16_t)(u >> 16);
}

uint16_t fmha_oracle_f32_to_f16(float f) {
  _Float16 h = (_Float16)f; /* IEEE RNE conversion */
  uint16_t r;
  memcpy(&r, &h, 2);
  return r;
}

float fmha_oracle_f16_to_f32(uint16_t x) {
  _Float16 h;
  memcpy(&h, &x, 2);
  return (float)h;
}

static inline float bf(uint16_t x) { return fmha_oracle_bf16_to_f32(x); }

/* -------------------------------------------------------------- generator */

/* splitmix64 finaliser (Steele, Lea, Flood, "Fast splittable pseudorandom
 * number generators", OOPSLA 2014). */
static inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

void fmha_oracle_gen_bf16(uint16_t* out, int64_t n, uint64_t seed,
                          uint32_t tensor_id, int64_t offset) {
  const uint64_t key = mix64(seed ^ mix64(((uint64_t)tensor_id << 32) | 0x5bd1e995u));
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t e = (uint64_t)(offset + i);
    int64_t t = 0;
    for (int j = 0; j < 3; ++j) {
      const uint64_t h = mix64(key + e * 3u + (uint64_t)j);
      t += (int64_t)(h & 0xffffu) + (int64_t)((h >> 16) & 0xffffu) +
           (int64_t)((h >> 32) & 0xffffu) + (int64_t)(h >> 48);
    }
    /* sum of 12 uniforms (v+0.5)/65536 minus 6: mean 0, variance ~1. */
    const int64_t num = 2 * t + 12 - 12 * 65536;
    const float x = (float)num * (1.0f / 131072.0f); /* exact */
    out[i] = fmha_oracle_f32_to_bf16(x);
  }
}

/* -------------------------------------------------------------- attention */

/* One (batch row, query head): q[D], rows k_s = K + s*kstride, v_s likewise. */
static void attend_row(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                       int64_t row_stride, int S, int D, int p_bf16,
                       float* o_f32, uint16_t* o_f16) {
  float scores[16];
  float p[16];
  for (int s = 0; s < S; ++s) {
    float sum = 0.0f;
    const uint16_t* ks = k + (int64_t)s * row_stride;
    for (int d = 0; d < D; ++d) sum += bf(q[d]) * bf(ks[d]);
    scores[s] = sum;
  }
  for (int s = 0; s < S; ++s) scores[s] *= (1.0f / sqrtf((float)D));
  float max_val = -INFINITY;
  for (int s = 0; s < S; ++s) max_val = fmaxf(max_val, scores[s]);
  float sum_exp = 0.0f;
  for (int s = 0; s < S; ++s) sum_exp += expf(scores[s] - max_val);
  for (int s = 0; s < S; ++s) {
    float ps = expf(scores[s] - max_val) / sum_exp;
    p[s] = p_bf16 ? bf(fmha_oracle_f32_to_bf16(ps)) : ps;
  }
  for (int d = 0; d < D; ++d) {
    float sum = 0.0f;
    for (int s = 0; s < S; ++s) sum += p[s] * bf(v[(int64_t)s * row_stride + d]);
    if (o_f32) o_f32[d] = sum;
    if (o_f16) o_f16[d] = fmha_oracle_f32_to_f16(sum);
  }
}

void fmha_oracle_decode_bhsd(const uint16_t* Q, const uint16_t* K,
                             const uint16_t* V, int64_t batch, int Hq, int Hkv,
                             int S, int D, int p_bf16, float* O_f32,
                             uint16_t* O_f16) {
  const int G = Hq / Hkv;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < batch; ++b) {
    for (int h = 0; h < Hq; ++h) {
      const int kvh = h / G;
      const int64_t qo = (b * Hq + h) * (int64_t)D;
      const int64_t ko = ((b * Hkv + kvh) * (int64_t)S) * D;
      attend_row(Q + qo, K + ko, V + ko, D, S, D, p_bf16,
                 O_f32 ? O_f32 + qo : 0, O_f16 ? O_f16 + qo : 0);
    }
  }
}

void fmha_oracle_decode_thd(const uint16_t* Q, const uint16_t* K,
                            const uint16_t* V, const int32_t* cu, int64_t batch,
                            int Hq, int Hkv, int D, int p_bf16, float* O_f32,
                            uint16_t* O_f16) {
  const int G = Hq / Hkv;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < batch; ++b) {
    const int S = cu[b + 1] - cu[b];
    const int64_t row_stride = (int64_t)Hkv * D;
    for (int h = 0; h < Hq; ++h) {
      const int kvh = h / G;
      const int64_t qo = (b * Hq + h) * (int64_t)D;
      const int64_t ko = (int64_t)cu[b] * row_stride + (int64_t)kvh * D;
      attend_row(Q + qo, K + ko, V + ko, row_stride, S, D, p_bf16,
                 O_f32 ? O_f32 + qo : 0, O_f16 ? O_f16 + qo : 0);
    }
  }
}

int fmha_oracle_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void fmha_oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
