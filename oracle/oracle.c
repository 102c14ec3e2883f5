/*
 * CPU oracle for the llminfer attention hot path — TEST INFRASTRUCTURE ONLY.
 * See oracle.h for the contract of every function and the reference lines it
 * restates.  Built by oracle/Makefile into oracle/build/liboracle.so.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- binary16 conversion (round to nearest, ties to even) ---------------- */

/* Drops the low `shift` bits of `v` with round-to-nearest-even. */
static uint32_t shift_round_even(uint32_t v, unsigned shift) {
  if (shift == 0)
    return v;
  if (shift > 31)
    return 0;
  uint32_t kept = v >> shift;
  uint32_t dropped = v & ((1u << shift) - 1u);
  uint32_t half = 1u << (shift - 1u);
  if (dropped > half || (dropped == half && (kept & 1u)))
    kept += 1u;
  return kept;
}

uint16_t oracle_f32_to_f16(float value) {
  uint32_t bits;
  memcpy(&bits, &value, sizeof bits);
  uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
  uint32_t magnitude = bits & 0x7fffffffu;
  uint32_t biased = magnitude >> 23; /* float exponent field */
  uint32_t fraction = magnitude & 0x7fffffu;
  if (biased == 0xffu) /* inf stays inf; NaN becomes a quiet NaN */
    return (uint16_t)(sign | 0x7c00u | (fraction ? 0x200u : 0u));
  int exponent = (int)biased - 127;
  if (exponent > 15)
    return (uint16_t)(sign | 0x7c00u);
  if (exponent >= -14) {
    /* Normal half; a carry out of the fraction bumps the exponent, which is
     * exactly the rounding to the next binade (or to infinity). */
    uint32_t h = ((uint32_t)(exponent + 15) << 10) + shift_round_even(fraction, 13);
    return (uint16_t)(sign | h);
  }
  if (exponent < -25)
    return sign;
  /* Subnormal half: value / 2^-24 = (1.fraction) * 2^(exponent + 24). */
  uint32_t significand = fraction | 0x800000u;
  return (uint16_t)(sign | shift_round_even(significand, (unsigned)(-exponent - 1)));
}

float oracle_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exponent = (h >> 10) & 0x1fu;
  uint32_t fraction = h & 0x3ffu;
  float out;
  if (exponent == 0) {
    out = ldexpf((float)fraction, -24);
    return sign ? -out : out;
  }
  uint32_t bits = sign | ((exponent == 31 ? 255u : exponent + 112u) << 23) | (fraction << 13);
  memcpy(&out, &bits, sizeof out);
  return out;
}

void oracle_f32_to_f16_array(const float *in, uint16_t *out, size_t n) {
  for (size_t i = 0; i < n; ++i)
    out[i] = oracle_f32_to_f16(in[i]);
}

void oracle_f16_to_f32_array(const uint16_t *in, float *out, size_t n) {
  for (size_t i = 0; i < n; ++i)
    out[i] = oracle_f16_to_f32(in[i]);
}

static inline float round_half(float x) { return oracle_f16_to_f32(oracle_f32_to_f16(x)); }

/* ---- inputs --------------------------------------------------------------- */

void oracle_lcg_fill(uint32_t *state, uint16_t *out, size_t n) {
  uint32_t s = *state;
  for (size_t i = 0; i < n; ++i) {
    s = s * 1664525u + 1013904223u;
    out[i] = oracle_f32_to_f16((float)((int)(s >> 24) - 128) / 64.0f);
  }
  *state = s;
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

static int pick_threads(int threads) {
  int most = oracle_max_threads();
  return threads <= 0 || threads > most ? most : threads;
}

/* ---- GQA ------------------------------------------------------------------ */

/* One query row of the dense fp64 check (FlashAttentionTest.mm:53-85): the
 * row's scores against keys [0, visible), exact softmax, weighted values.
 * k and v point at the row's kv head in a cache of kv_row-element rows;
 * weights holds `visible` doubles. */
static void dense_row(const uint16_t *qr, const uint16_t *ks, const uint16_t *vs,
                      size_t kv_row, unsigned D, unsigned visible, double *weights,
                      double *o) {
  const double inv_sqrt = 1.0 / sqrt((double)D);
  double top = -INFINITY;
  for (unsigned i = 0; i < visible; ++i) {
    double dot = 0.0;
    for (unsigned d = 0; d < D; ++d)
      dot += (double)oracle_f16_to_f32(qr[d]) * oracle_f16_to_f32(ks[i * kv_row + d]);
    weights[i] = dot * inv_sqrt;
    if (weights[i] > top)
      top = weights[i];
  }
  double total = 0.0;
  for (unsigned i = 0; i < visible; ++i) {
    weights[i] = exp(weights[i] - top);
    total += weights[i];
  }
  for (unsigned d = 0; d < D; ++d) {
    double acc = 0.0;
    for (unsigned i = 0; i < visible; ++i)
      acc += weights[i] * oracle_f16_to_f32(vs[i * kv_row + d]);
    o[d] = acc / total;
  }
}

void oracle_gqa_dense(const oracle_gqa_params *p, unsigned batch,
                      const uint16_t *q, size_t q_stride, const uint16_t *k,
                      const uint16_t *v, size_t kv_stride, double *out,
                      int threads) {
  const unsigned D = p->headDim, Hq = p->queryHeads;
  const unsigned group = p->queryHeads / p->kvHeads;
  const size_t kv_row = (size_t)p->kvHeads * D;
  const long rows = (long)batch * p->tokens * Hq;
#pragma omp parallel num_threads(pick_threads(threads))
  {
    double *weights = (double *)malloc(sizeof(double) * (p->past + p->tokens + 1));
#pragma omp for schedule(dynamic, 1)
    for (long r = 0; r < rows; ++r) {
      unsigned seq = (unsigned)(r / ((long)p->tokens * Hq));
      unsigned row = (unsigned)(r % ((long)p->tokens * Hq)); /* token*Hq + head */
      unsigned token = row / Hq, head = row % Hq;
      dense_row(q + seq * q_stride + (size_t)row * D,
                k + seq * kv_stride + (size_t)(head / group) * D,
                v + seq * kv_stride + (size_t)(head / group) * D, kv_row, D,
                p->past + token + 1, weights,
                out + ((size_t)seq * p->tokens * Hq + row) * D);
    }
    free(weights);
  }
}

void oracle_gqa_dense_rows(const oracle_gqa_params *p, const uint16_t *q_rows,
                           const uint16_t *k, const uint16_t *v,
                           const unsigned *token, const unsigned *head, unsigned n,
                           double *out, int threads) {
  const unsigned D = p->headDim;
  const unsigned group = p->queryHeads / p->kvHeads;
  const size_t kv_row = (size_t)p->kvHeads * D;
#pragma omp parallel num_threads(pick_threads(threads))
  {
    double *weights = (double *)malloc(sizeof(double) * (p->past + p->tokens + 1));
#pragma omp for schedule(dynamic, 1)
    for (long r = 0; r < (long)n; ++r)
      dense_row(q_rows + (size_t)r * D, k + (size_t)(head[r] / group) * D,
                v + (size_t)(head[r] / group) * D, kv_row, D, p->past + token[r] + 1,
                weights, out + (size_t)r * D);
    free(weights);
  }
}

void oracle_gqa_eager_f16(const oracle_gqa_params *p, unsigned batch,
                          const uint16_t *q, size_t q_stride,
                          const uint16_t *k, const uint16_t *v,
                          size_t kv_stride, uint16_t *out, int threads) {
  const unsigned D = p->headDim, Hq = p->queryHeads;
  const unsigned group = p->queryHeads / p->kvHeads;
  const size_t kv_row = (size_t)p->kvHeads * D;
  const long rows = (long)batch * p->tokens * Hq;
  const float score_scale = 1.0f / sqrtf((float)D);
#pragma omp parallel num_threads(pick_threads(threads))
  {
    float *prob = (float *)malloc(sizeof(float) * (p->past + p->tokens + 1));
#pragma omp for schedule(dynamic, 1)
    for (long r = 0; r < rows; ++r) {
      unsigned seq = (unsigned)(r / ((long)p->tokens * Hq));
      unsigned row = (unsigned)(r % ((long)p->tokens * Hq));
      unsigned token = row / Hq, head = row % Hq;
      unsigned visible = p->past + token + 1;
      const uint16_t *qr = q + seq * q_stride + (size_t)row * D;
      const uint16_t *ks = k + seq * kv_stride + (size_t)(head / group) * D;
      const uint16_t *vs = v + seq * kv_stride + (size_t)(head / group) * D;
      /* gqaScores: fp32 fma dot, rounded to half, scaled, rounded again. */
      float top = -INFINITY;
      for (unsigned i = 0; i < visible; ++i) {
        float dot = 0.0f;
        for (unsigned d = 0; d < D; ++d)
          dot = fmaf(oracle_f16_to_f32(qr[d]), oracle_f16_to_f32(ks[i * kv_row + d]), dot);
        prob[i] = round_half(round_half(dot) * score_scale);
        if (prob[i] > top)
          top = prob[i];
      }
      /* gqaSoftmax: fp32 normaliser, probabilities stored as half. */
      float total = 0.0f;
      for (unsigned i = 0; i < visible; ++i)
        total += expf(prob[i] - top);
      for (unsigned i = 0; i < visible; ++i)
        prob[i] = round_half(expf(prob[i] - top) / total);
      /* gqaValue: fp32 fma over keys, rounded to half. */
      uint16_t *o = out + ((size_t)seq * p->tokens * Hq + row) * D;
      for (unsigned d = 0; d < D; ++d) {
        float acc = 0.0f;
        for (unsigned i = 0; i < visible; ++i)
          acc = fmaf(prob[i], oracle_f16_to_f32(vs[i * kv_row + d]), acc);
        o[d] = oracle_f32_to_f16(acc);
      }
    }
    free(prob);
  }
}

void oracle_cache_append(unsigned count, unsigned offset, unsigned batch,
                         const uint16_t *input, size_t in_stride,
                         uint16_t *cache, size_t cache_stride) {
  for (unsigned s = 0; s < batch; ++s)
    memcpy(cache + s * cache_stride + offset, input + s * in_stride,
           sizeof(uint16_t) * count);
}

/* ---- Gated DeltaNet --------------------------------------------------------- */

void oracle_delta_update(const oracle_delta_params *p, unsigned batch,
                         const float *q, const float *k, const uint16_t *v,
                         const float *beta, const float *decay, float *state,
                         uint16_t *out, int threads) {
  const unsigned T = p->tokens, Hk = p->keyHeads, dk = p->keyDim;
  const unsigned Hv = p->valueHeads, dv = p->valueDim;
  const unsigned group = Hv / Hk;
  const size_t key_width = (size_t)Hk * dk, value_width = (size_t)Hv * dv;
  const long columns = (long)batch * Hv * dv;
#pragma omp parallel for num_threads(pick_threads(threads)) schedule(static)
  for (long c = 0; c < columns; ++c) {
    unsigned seq = (unsigned)(c / value_width);
    unsigned column = (unsigned)(c % value_width);
    unsigned vh = column / dv, j = column % dv, kh = vh / group;
    float *S = state + ((size_t)seq * Hv + vh) * dk * dv + j; /* stride dv */
    for (unsigned t = 0; t < T; ++t) {
      const size_t tok = (size_t)seq * T + t;
      const float *qt = q + tok * key_width + (size_t)kh * dk;
      const float *kt = k + tok * key_width + (size_t)kh * dk;
      const float a = decay[tok * Hv + vh], b = beta[tok * Hv + vh];
      const float x = oracle_f16_to_f32(v[tok * value_width + column]);
      float pred = 0.0f;
      for (unsigned i = 0; i < dk; ++i)
        pred = fmaf(S[(size_t)i * dv] * a, kt[i], pred);
      const float delta = (x - pred) * b;
      float y = 0.0f;
      for (unsigned i = 0; i < dk; ++i) {
        float next = fmaf(kt[i], delta, S[(size_t)i * dv] * a);
        S[(size_t)i * dv] = next;
        y = fmaf(next, qt[i], y);
      }
      out[tok * value_width + column] = oracle_f32_to_f16(y);
    }
  }
}

void oracle_l2norm(const float *in, float *out, size_t rows, unsigned width,
                   float epsilon, float scale) {
  for (size_t r = 0; r < rows; ++r) {
    const float *x = in + r * width;
    float sum = 0.0f;
    for (unsigned i = 0; i < width; ++i)
      sum = fmaf(x[i], x[i], sum);
    float factor = (1.0f / sqrtf(sum + epsilon)) * scale;
    for (unsigned i = 0; i < width; ++i)
      out[r * width + i] = x[i] * factor;
  }
}

/* softplus(x) = log(1 + e^x) evaluated without overflow; for tiny e^-|x| the
 * two-term series e - e^2/2 keeps full precision. */
static float softplus_stable(float x) {
  float e = expf(-fabsf(x));
  float tail = e < 1e-4f ? e * (1.0f - 0.5f * e) : logf(1.0f + e);
  return (x > 0.0f ? x : 0.0f) + tail;
}

void oracle_delta_gates(const float *a, const float *b, const float *aLog,
                        const float *dtBias, size_t rows, unsigned heads,
                        float *beta, float *decay) {
  for (size_t r = 0; r < rows; ++r)
    for (unsigned h = 0; h < heads; ++h) {
      size_t i = r * heads + h;
      beta[i] = round_half(1.0f / (1.0f + expf(-b[i])));
      decay[i] = expf(-expf(aLog[h]) * softplus_stable(a[i] + dtBias[h]));
    }
}

/* ---- q/k norm and RoPE; causal conv ------------------------------------------- */

void oracle_norm_rope(const oracle_rope_params *p, unsigned batch, const uint16_t *input,
                      size_t input_stride, const float *weight, uint16_t *output,
                      size_t output_stride) {
  const unsigned D = p->headDim, half_r = p->rotaryDim / 2;
  float *x = (float *)malloc(sizeof(float) * D);
  for (unsigned s = 0; s < batch; ++s)
    for (unsigned r = 0; r < p->tokens * p->heads; ++r) {
      const uint16_t *in = input + s * input_stride + (size_t)r * p->headStride;
      uint16_t *out = output + s * output_stride + ((size_t)p->outputStart * p->heads + r) * D;
      if (weight) {
        float sum = 0.0f;
        for (unsigned i = 0; i < D; ++i) {
          const float v = oracle_f16_to_f32(in[i]);
          sum = fmaf(v, v, sum);
        }
        const float scale = 1.0f / sqrtf(sum / (float)D + p->epsilon);
        for (unsigned i = 0; i < D; ++i)
          x[i] = round_half(oracle_f16_to_f32(in[i]) * scale * (1.0f + weight[i]));
      } else {
        for (unsigned i = 0; i < D; ++i)
          x[i] = oracle_f16_to_f32(in[i]);
      }
      const float position = (float)(p->past + r / p->heads);
      for (unsigned i = 0; i < half_r; ++i) {
        const unsigned j = i + half_r;
        const float phase = position / powf(p->theta, 2.0f * (float)i / (float)p->rotaryDim);
        const float c = round_half(cosf(phase)), sn = round_half(sinf(phase));
        const float xv = x[i], yv = x[j];
        x[i] = round_half(round_half(xv * c) - round_half(yv * sn));
        x[j] = round_half(round_half(yv * c) + round_half(xv * sn));
      }
      for (unsigned i = 0; i < D; ++i)
        out[i] = oracle_f32_to_f16(x[i]);
    }
  free(x);
}

static float silu_ref(float x) { return x * (1.0f / (1.0f + expf(-x))); }

void oracle_causal_conv(const oracle_conv_params *p, unsigned batch, const uint16_t *input,
                        size_t input_stride, const uint16_t *weight, uint16_t *history,
                        size_t history_stride, uint16_t *output, size_t output_stride) {
  const unsigned H = p->kernelSize - 1;
  for (unsigned s = 0; s < batch; ++s)
    for (unsigned c = 0; c < p->channels; ++c) {
      uint16_t *recent = history + s * history_stride + (size_t)c * H;
      const uint16_t *filter = weight + (size_t)c * p->kernelSize;
      for (unsigned t = 0; t < p->tokens; ++t) {
        const size_t i = (size_t)t * p->channels + c;
        const uint16_t current = input[s * input_stride + i];
        float acc = oracle_f16_to_f32(current) * oracle_f16_to_f32(filter[H]);
        for (unsigned j = 0; j < H; ++j)
          acc = fmaf(oracle_f16_to_f32(recent[j]), oracle_f16_to_f32(filter[j]), acc);
        float y = round_half(acc);
        if (p->applySilu)
          y = round_half(silu_ref(y));
        output[s * output_stride + i] = oracle_f32_to_f16(y);
        if (H) {
          for (unsigned j = 1; j < H; ++j)
            recent[j - 1] = recent[j];
          recent[H - 1] = current;
        }
      }
    }
}

/* ---- cost model ------------------------------------------------------------- */

uint64_t oracle_gqa_pairs(uint64_t tokens, uint64_t past) {
  return tokens * past + tokens * (tokens + 1) / 2;
}

uint64_t oracle_gqa_fp_macs(uint64_t tokens, uint64_t past, uint64_t queryHeads,
                            uint64_t headDim) {
  return 2 * queryHeads * oracle_gqa_pairs(tokens, past) * headDim;
}

uint64_t oracle_delta_fp_macs(uint64_t tokens, uint64_t valueHeads,
                              uint64_t keyDim, uint64_t valueDim) {
  return 3 * tokens * valueHeads * keyDim * valueDim;
}

/* Logical bytes: operands read and written once (Cost.cpp:85-93). */
void oracle_kv_append_bytes(uint64_t tokens, uint64_t kvHeads, uint64_t headDim,
                            uint64_t *read, uint64_t *write) {
  /* new keys and values [T][Hkv][D] f16 in; the same rows written. */
  *read = 2 * tokens * kvHeads * headDim * 2;
  *write = *read;
}

void oracle_gqa_bytes(uint64_t tokens, uint64_t past, uint64_t queryHeads, uint64_t kvHeads,
                      uint64_t headDim, uint64_t *read, uint64_t *write) {
  /* q [T][Hq][D] f16 and cache rows [0, past+T) of K and V in; out like q. */
  const uint64_t q_bytes = tokens * queryHeads * headDim * 2;
  *read = q_bytes + 2 * (past + tokens) * kvHeads * headDim * 2;
  *write = q_bytes;
}

void oracle_delta_bytes(uint64_t tokens, uint64_t keyHeads, uint64_t keyDim,
                        uint64_t valueHeads, uint64_t valueDim, uint64_t *read,
                        uint64_t *write) {
  /* q, k f32; v f16; beta, decay f32; the state read once and written once;
   * out f16. */
  const uint64_t state = valueHeads * keyDim * valueDim * 4;
  *read = 2 * tokens * keyHeads * keyDim * 4 + tokens * valueHeads * valueDim * 2 +
          2 * tokens * valueHeads * 4 + state;
  *write = tokens * valueHeads * valueDim * 2 + state;
}

void oracle_set_threads(int threads) {
#ifdef _OPENMP
  if (threads > 0)
    omp_set_num_threads(threads);
#else
  (void)threads;
#endif
}
