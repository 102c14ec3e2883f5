/*
 * CPU oracle for the llminfer attention hot path — TEST INFRASTRUCTURE ONLY.
 *
 * This library is the checker, never the product: only tests/, the smoke
 * check in __graft_entry__.py and the cpu_baseline / --impl reference legs of
 * bench.py load it.  Nothing in llminfer_b200/ links or calls it.
 *
 * Each function restates, in plain C, the arithmetic of one piece of the
 * reference (GladingRay/llminfer); the citation is given beside it.  The
 * reference's own implementation of this path is Metal Shading Language and
 * Objective-C++ (no Metal on Linux), so it cannot be run here; the pins used
 * to trust this restatement are listed in tests/test_oracle.py.
 */
#ifndef LLMI_ORACLE_H
#define LLMI_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same field order and meaning as the reference's GqaParams
 * (lib/Backend/Metal/Kernels/ReferenceParams.h:53-55). */
typedef struct {
  unsigned tokens, queryHeads, kvHeads, headDim, past;
} oracle_gqa_params;

/* Same field order and meaning as the reference's GraphDeltaParams
 * (lib/Backend/Metal/Kernels/GraphParams.h:50-52). */
typedef struct {
  unsigned tokens, keyHeads, keyDim, valueHeads, valueDim;
} oracle_delta_params;

/* IEEE binary32 <-> binary16, round to nearest even (the conversion the
 * reference uses everywhere: lib/ModelFormat/Quantization.cpp:25-55). */
uint16_t oracle_f32_to_f16(float value);
float oracle_f16_to_f32(uint16_t bits);
void oracle_f32_to_f16_array(const float *in, uint16_t *out, size_t n);
void oracle_f16_to_f32_array(const uint16_t *in, float *out, size_t n);

/* The linear congruential fill of tests/FlashAttentionTest.mm:28-36:
 * state = state*1664525 + 1013904223, value = (int(state>>24) - 128) / 64
 * stored as fp16.  `state` is advanced in place. */
void oracle_lcg_fill(uint32_t *state, uint16_t *out, size_t n);

/* Dense causal GQA with fp64 accumulation and an exact softmax, the check of
 * tests/FlashAttentionTest.mm:53-85, for `batch` independent sequences.
 *   q:   [batch][tokens][queryHeads][headDim] fp16, sequence stride q_stride
 *   k,v: per sequence a cache [rows][kvHeads][headDim] fp16 holding at least
 *        past+tokens rows, sequence stride kv_stride (elements)
 *   out: [batch][tokens][queryHeads][headDim] fp64 (unrounded)
 * Query token t sees keys [0, past + t]; kv head = q head / (Hq/Hkv);
 * scores are scaled by 1/sqrt(headDim).  threads <= 0 uses every core. */
void oracle_gqa_dense(const oracle_gqa_params *p, unsigned batch,
                      const uint16_t *q, size_t q_stride, const uint16_t *k,
                      const uint16_t *v, size_t kv_stride, double *out,
                      int threads);

/* The same check for n chosen rows of ONE sequence, for shapes whose full
 * output is too large to compute on a CPU: row r is query token token[r],
 * query head head[r], with its q row at q_rows[r*headDim] and the sequence's
 * cache rows in k, v ([rows][kvHeads][headDim] fp16).  out: [n][headDim]. */
void oracle_gqa_dense_rows(const oracle_gqa_params *p, const uint16_t *q_rows,
                           const uint16_t *k, const uint16_t *v,
                           const unsigned *token, const unsigned *head, unsigned n,
                           double *out, int threads);

/* The reference's non-flash path with its fp16 rounding points:
 * gqaScores (Reference.metal:303-323): s = half(half(q.k) * rsqrt(D));
 * gqaSoftmax (Graph.metal:172-210): p = half(exp(s - max) / sum);
 * gqaValue (Graph.metal:212-230): out = half(sum p*v) with fp32 fma.
 * Same layouts as oracle_gqa_dense; out is fp16. */
void oracle_gqa_eager_f16(const oracle_gqa_params *p, unsigned batch,
                          const uint16_t *q, size_t q_stride,
                          const uint16_t *k, const uint16_t *v,
                          size_t kv_stride, uint16_t *out, int threads);

/* cacheAppend (Reference.metal:295-301) for `batch` sequences:
 * cache[s][offset + i] = input[s][i] for i < count. */
void oracle_cache_append(unsigned count, unsigned offset, unsigned batch,
                         const uint16_t *input, size_t in_stride,
                         uint16_t *cache, size_t cache_stride);

/* Token-sequential gated delta rule, graphDeltaUpdate (Graph.metal:146-170)
 * with updateDeltaColumn (Reference.metal:182-197), fp32 with the same fma
 * association:
 *   pred  = sum_i fma(S[i][j]*decay, k[i], pred)
 *   delta = (v - pred) * beta
 *   S[i][j] = fma(k[i], delta, S[i][j]*decay);  y = sum_i fma(S[i][j], q[i], y)
 * Layouts (per sequence, `batch` sequences back to back):
 *   q, k:  [tokens][keyHeads*keyDim] fp32
 *   v:     [tokens][valueHeads*valueDim] fp16
 *   beta, decay: [tokens][valueHeads] fp32
 *   state: [valueHeads][keyDim][valueDim] fp32, updated in place
 *   out:   [tokens][valueHeads*valueDim] fp16
 * Value head vh reads key head vh / (valueHeads/keyHeads). */
void oracle_delta_update(const oracle_delta_params *p, unsigned batch,
                         const float *q, const float *k, const uint16_t *v,
                         const float *beta, const float *decay, float *state,
                         uint16_t *out, int threads);

/* Producers of the DeltaUpdate inputs, used to build synthetic inputs:
 * l2NormF32 (Graph.metal:96-109): out = x * rsqrt(sum x^2 + eps) * scale per
 * group of `width`; deltaGates (Graph.metal:131-144 with stableSoftplus,
 * Reference.metal:8-12): beta = half(sigmoid(b)),
 * decay = exp(-exp(aLog[h]) * softplus(a + dtBias[h])). */
void oracle_l2norm(const float *in, float *out, size_t rows, unsigned width,
                   float epsilon, float scale);
void oracle_delta_gates(const float *a, const float *b, const float *aLog,
                        const float *dtBias, size_t rows, unsigned heads,
                        float *beta, float *decay);

/* RopeParams (ReferenceParams.h:44-47) and ConvParams (ReferenceParams.h:32-34). */
typedef struct {
  unsigned tokens, heads, headDim, rotaryDim, headStride, past, outputStart;
  float epsilon, theta;
} oracle_rope_params;
typedef struct {
  unsigned tokens, channels, kernelSize, applySilu;
} oracle_conv_params;

/* q/k RmsNorm + PartialRoPE, restating rmsNorm (Reference.metal:98-117:
 * x * rsqrt(sum x^2 / width + eps) * (1 + w), rounded to fp16), rotatePair
 * (Reference.metal:261-269: phase = position / theta^(2i/R), cos and sin
 * rounded to fp16, each product rounded to fp16) and the row addressing of
 * normRope (Reference.metal:271-293).  weight == NULL skips the norm: that
 * is partialRope (Graph.metal:111-129).  Per sequence s < batch, row r reads
 * input + s*input_stride + r*headStride and writes output + s*output_stride
 * + (outputStart*heads + r)*headDim. */
void oracle_norm_rope(const oracle_rope_params *p, unsigned batch, const uint16_t *input,
                      size_t input_stride, const float *weight, uint16_t *output,
                      size_t output_stride);

/* causalConv (Reference.metal:137-158), walked token by token per channel
 * as the reference does, the history shifting after each token; with
 * applySilu the output is half(silu(half(acc))), which is also causalConv
 * (applySilu 0) followed by siluF16 (Graph.metal:70-76).  input/output
 * [tokens][channels] and history [channels][kernelSize-1] per sequence;
 * weight [channels][kernelSize]; the history is updated in place. */
void oracle_causal_conv(const oracle_conv_params *p, unsigned batch, const uint16_t *input,
                        size_t input_stride, const uint16_t *weight, uint16_t *history,
                        size_t history_stride, uint16_t *output, size_t output_stride);

/* Logical work of one op, following the reference cost model
 * (lib/GraphIR/Cost.cpp:85-93 traffic, :180-201 math). */
uint64_t oracle_gqa_pairs(uint64_t tokens, uint64_t past);
uint64_t oracle_gqa_fp_macs(uint64_t tokens, uint64_t past, uint64_t queryHeads,
                            uint64_t headDim);
uint64_t oracle_delta_fp_macs(uint64_t tokens, uint64_t valueHeads,
                              uint64_t keyDim, uint64_t valueDim);
/* Logical bytes read and written by one sequence's op (same model). */
void oracle_kv_append_bytes(uint64_t tokens, uint64_t kvHeads, uint64_t headDim,
                            uint64_t *read, uint64_t *write);
void oracle_gqa_bytes(uint64_t tokens, uint64_t past, uint64_t queryHeads, uint64_t kvHeads,
                      uint64_t headDim, uint64_t *read, uint64_t *write);
void oracle_delta_bytes(uint64_t tokens, uint64_t keyHeads, uint64_t keyDim,
                        uint64_t valueHeads, uint64_t valueDim, uint64_t *read,
                        uint64_t *write);

/* Sets the OpenMP thread count used when a call passes threads <= 0 (a
 * launcher may have set OMP_NUM_THREADS=1 for the process). */
void oracle_set_threads(int threads);

/* Number of threads oracle_* would use for `threads` <= 0. */
int oracle_max_threads(void);

#ifdef __cplusplus
}
#endif

#endif
