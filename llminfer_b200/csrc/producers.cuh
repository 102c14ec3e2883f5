// Producers on either side of the attention path: the kernels that turn the
// projections' outputs into the operands of cacheAppend / gqaFlashAttention
// (q and k: RmsNorm with (1 + w), partial RoPE, the k rows straight into the
// KV cache) and of graphDeltaUpdate (causal conv1d, SiLU, q/k L2 norm; the
// gates).  All of them are HBM-bound elementwise or row-reduction work: one
// warp per row, 16-byte loads where the layout allows, no shared memory
// beyond a row buffer.
//
// Rounding follows the reference op by op (each fp16 boundary of the unfused
// graph is kept): rmsNorm (Reference.metal:98-118), rotatePair and normRope
// (Reference.metal:261-293), partialRope (Graph.metal:111-129), causalConv
// (Reference.metal:137-158), siluF16 (Graph.metal:70-76), l2NormF32
// (Graph.metal:96-109), deltaGates (Graph.metal:131-144).  Reductions run as
// warp trees, so sums differ from the reference's serial fma order in the
// last bits of fp32.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"

namespace llmi {
namespace producers {

__device__ __forceinline__ float logistic(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float silu(float x) { return x * logistic(x); }
__device__ __forceinline__ float stable_softplus(float x) {
  const float e = expf(-fabsf(x));
  const float tail = e < 1e-4f ? e * (1.0f - 0.5f * e) : logf(1.0f + e);
  return fmaxf(x, 0.0f) + tail;
}
__device__ __forceinline__ float round_half(float x) { return __half2float(__float2half_rn(x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
    v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// ---- q/k: RmsNorm (1 + w) and partial RoPE -----------------------------------

constexpr int kRopeMaxDim = 1024;
constexpr int kRopeWarps = 8;

struct RopeArgs {
  const __half *input;
  size_t input_stride;  // elements between sequences
  const float *weight;  // RmsNorm weight [head_dim], or null: rope only
  __half *output;
  size_t output_stride;
  unsigned batch, tokens, heads, head_dim, rotary_dim, head_stride, past, output_start;
  float epsilon, theta;
};

// One warp per (sequence, token, head) row.  Row r of a sequence reads
// input + r * head_stride and writes output + (output_start * heads + r) *
// head_dim (for k, the cache rows of this step).  kVec: head_dim % 8 == 0
// and 16-byte aligned rows (uint4 loads and stores).
template <bool kVec>
__global__ void __launch_bounds__(32 * kRopeWarps) norm_rope(const RopeArgs a) {
  __shared__ __align__(16) __half rows[kRopeWarps][kRopeMaxDim];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t rows_per_seq = uint64_t(a.tokens) * a.heads;
  const uint64_t g = uint64_t(blockIdx.x) * kRopeWarps + warp;
  if (g >= rows_per_seq * a.batch)
    return;  // whole warps only
  const uint32_t seq = uint32_t(g / rows_per_seq), row = uint32_t(g % rows_per_seq);
  const __half *in = a.input + seq * a.input_stride + size_t(row) * a.head_stride;
  __half *out = a.output + seq * a.output_stride +
                (size_t(a.output_start) * a.heads + row) * a.head_dim;
  __half *x = rows[warp];
  const unsigned D = a.head_dim;

  // Normalised row (fp16, as rmsNorm writes it) into the warp's row buffer.
  if (a.weight) {
    float sum = 0.f;
    if (kVec) {
      for (unsigned i = lane * 8; i < D; i += 256) {
        const uint4 w = *reinterpret_cast<const uint4 *>(in + i);
        const __half *h = reinterpret_cast<const __half *>(&w);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float v = __half2float(h[e]);
          sum = fmaf(v, v, sum);
        }
        *reinterpret_cast<uint4 *>(x + i) = w;
      }
    } else {
      for (unsigned i = lane; i < D; i += 32) {
        const float v = __half2float(in[i]);
        sum = fmaf(v, v, sum);
        x[i] = in[i];
      }
    }
    sum = warp_sum(sum);
    const float scale = rsqrtf(sum / float(D) + a.epsilon);
    __syncwarp();
    for (unsigned i = lane; i < D; i += 32)
      x[i] = __float2half_rn(__half2float(x[i]) * scale * (1.0f + a.weight[i]));
  } else {
    for (unsigned i = lane; i < D; i += 32)
      x[i] = in[i];
  }
  __syncwarp();

  // Rotary pairs (i, i + R/2), R = rotary_dim, at position past + token.
  const unsigned half_r = a.rotary_dim / 2;
  const float position = float(a.past + row / a.heads);
  for (unsigned i = lane; i < half_r; i += 32) {
    const unsigned j = i + half_r;
    const float phase = position / powf(a.theta, 2.0f * float(i) / float(a.rotary_dim));
    const float c = round_half(cosf(phase)), s = round_half(sinf(phase));
    const float xv = __half2float(x[i]), yv = __half2float(x[j]);
    // Pairs are disjoint, so each lane reads and writes only its own.
    x[i] = __float2half_rn(round_half(xv * c) - round_half(yv * s));
    x[j] = __float2half_rn(round_half(yv * c) + round_half(xv * s));
  }
  __syncwarp();
  if (kVec) {
    for (unsigned i = lane * 8; i < D; i += 256)
      *reinterpret_cast<uint4 *>(out + i) = *reinterpret_cast<const uint4 *>(x + i);
  } else {
    for (unsigned i = lane; i < D; i += 32)
      out[i] = x[i];
  }
}

// ---- DeltaNet inputs: causal conv1d, SiLU, q/k L2 norm -----------------------

struct ConvArgs {
  const __half *input;  // [tokens][channels] per sequence
  size_t input_stride;
  const __half *weight;  // [channels][kernel]
  const __half *history;  // [channels][kernel - 1] per sequence (read only here)
  size_t history_stride;
  unsigned batch, tokens, channels, kernel;
  bool apply_silu;
};

// out(t, c) = sum_j w[c][j] x(t - (K-1) + j, c), x(t < 0) from the history,
// in the reference's order: acc = x_t w[K-1], then fma over j ascending.
// Then half(acc), and with SiLU half(silu(half(acc))).
__device__ __forceinline__ float conv_at(const ConvArgs &a, const __half *in, const __half *hist,
                                         uint32_t t, uint32_t c) {
  const unsigned K = a.kernel;
  const __half *w = a.weight + size_t(c) * K;
  float acc = __half2float(in[size_t(t) * a.channels + c]) * __half2float(w[K - 1]);
  for (unsigned j = 0; j + 1 < K; ++j) {
    const int tau = int(t) - int(K - 1) + int(j);
    const __half xv = tau >= 0 ? in[size_t(tau) * a.channels + c]
                               : hist[size_t(c) * (K - 1) + size_t(tau + int(K - 1))];
    acc = fmaf(__half2float(xv), __half2float(w[j]), acc);
  }
  float y = round_half(acc);
  if (a.apply_silu)
    y = round_half(silu(y));
  return y;
}

// Element-wise conv (the CausalConv1d op; SiLU optional).
__global__ void causal_conv(const ConvArgs a, __half *output, size_t output_stride) {
  const uint64_t per_seq = uint64_t(a.tokens) * a.channels;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < per_seq * a.batch;
       i += uint64_t(gridDim.x) * blockDim.x) {
    const uint32_t seq = uint32_t(i / per_seq);
    const uint64_t r = i % per_seq;
    const uint32_t t = uint32_t(r / a.channels), c = uint32_t(r % a.channels);
    const float y = conv_at(a, a.input + seq * a.input_stride, a.history + seq * a.history_stride,
                            t, c);
    output[seq * output_stride + r] = __float2half_rn(y);
  }
}

// The history after the step: the last K-1 inputs (older rows shift in
// from the previous history when the step is shorter).  One thread per
// (sequence, channel), ascending j, so every read precedes the write that
// could replace it.  Launched after every output has read the old history.
__global__ void conv_history(const ConvArgs a, __half *history) {
  const uint64_t n = uint64_t(a.batch) * a.channels;
  const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n)
    return;
  const uint32_t seq = uint32_t(i / a.channels), c = uint32_t(i % a.channels);
  const unsigned H = a.kernel - 1;
  const __half *in = a.input + seq * a.input_stride;
  __half *h = history + seq * a.history_stride + size_t(c) * H;
  for (unsigned j = 0; j < H; ++j) {
    const long src = long(a.tokens) - long(H) + long(j);
    h[j] = src >= 0 ? in[size_t(src) * a.channels + c] : h[j + a.tokens];
  }
}

struct PrepArgs {
  ConvArgs conv;  // channels = qkv width, apply_silu = true
  unsigned key_heads, key_dim, value_heads, value_dim;
  float epsilon;
  float *q, *k;  // [tokens][key_heads * key_dim] per sequence (fp32)
  __half *v;     // [tokens][value_heads * value_dim] per sequence
};

// One warp per (sequence, token, head of the qkv row): q heads, then k
// heads, then v heads, as the Slice ops of the DeltaNet block cut them.  q
// and k rows are L2-normalised (q also by 1/sqrt(key_dim)) into fp32; v rows
// stay fp16.  Requires key_dim, value_dim <= 256.
__global__ void __launch_bounds__(256) delta_prepare(const PrepArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned heads = 2 * a.key_heads + a.value_heads;
  const uint64_t rows_per_seq = uint64_t(a.conv.tokens) * heads;
  const uint64_t g = uint64_t(blockIdx.x) * 8 + warp;
  if (g >= rows_per_seq * a.conv.batch)
    return;  // whole warps only
  const uint32_t seq = uint32_t(g / rows_per_seq);
  const uint32_t r = uint32_t(g % rows_per_seq);
  const uint32_t t = r / heads, h = r % heads;
  const __half *in = a.conv.input + seq * a.conv.input_stride;
  const __half *hist = a.conv.history + seq * a.conv.history_stride;
  const bool is_v = h >= 2 * a.key_heads;
  const unsigned width = is_v ? a.value_dim : a.key_dim;
  const uint32_t c0 = is_v ? 2 * a.key_heads * a.key_dim + (h - 2 * a.key_heads) * a.value_dim
                           : h * a.key_dim;
  float y[8];
  float sum = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const unsigned i = lane + 32 * e;
    y[e] = i < width ? conv_at(a.conv, in, hist, t, c0 + i) : 0.f;
    sum = fmaf(y[e], y[e], sum);
  }
  if (is_v) {
    __half *out = a.v + (size_t(seq) * a.conv.tokens + t) * a.value_heads * a.value_dim +
                  (h - 2 * a.key_heads) * a.value_dim;
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (lane + 32 * e < width)
        out[lane + 32 * e] = __float2half_rn(y[e]);
    return;
  }
  sum = warp_sum(sum);
  const bool is_q = h < a.key_heads;
  const float factor = rsqrtf(sum + a.epsilon) * (is_q ? rsqrtf(float(a.key_dim)) : 1.0f);
  float *out = (is_q ? a.q : a.k) +
               (size_t(seq) * a.conv.tokens + t) * a.key_heads * a.key_dim +
               (is_q ? h : h - a.key_heads) * a.key_dim;
#pragma unroll
  for (int e = 0; e < 8; ++e)
    if (lane + 32 * e < width)
      out[lane + 32 * e] = y[e] * factor;
}

// ---- L2Norm (fp16 rows -> fp32) and DeltaGates ---------------------------------

__global__ void __launch_bounds__(256) l2_norm(const __half *input, float *output, unsigned rows,
                                                unsigned width, float epsilon, float scale) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t row = uint64_t(blockIdx.x) * 8 + warp;
  if (row >= rows)
    return;
  const __half *x = input + row * width;
  float sum = 0.f;
  for (unsigned i = lane; i < width; i += 32) {
    const float v = __half2float(x[i]);
    sum = fmaf(v, v, sum);
  }
  sum = warp_sum(sum);
  const float factor = rsqrtf(sum + epsilon) * scale;
  for (unsigned i = lane; i < width; i += 32)
    output[row * width + i] = __half2float(x[i]) * factor;
}

__global__ void delta_gates(const __half *a_in, const __half *b_in, const float *a_log,
                            const float *dt_bias, float *beta, float *decay, uint64_t count,
                            unsigned heads) {
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += uint64_t(gridDim.x) * blockDim.x) {
    const unsigned h = unsigned(i % heads);
    beta[i] = round_half(logistic(__half2float(b_in[i])));
    decay[i] = expf(-expf(a_log[h]) * stable_softplus(__half2float(a_in[i]) + dt_bias[h]));
  }
}

}  // namespace producers
}  // namespace llmi
