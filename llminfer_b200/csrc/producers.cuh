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

// 1 / (1 + e^-x): the correctly rounded reciprocal equals the IEEE quotient
// 1.0f / y bit for bit, in fewer instructions.
__device__ __forceinline__ float logistic(float x) { return __frcp_rn(1.0f + expf(-x)); }
__device__ __forceinline__ float silu(float x) { return x * logistic(x); }
__device__ __forceinline__ float stable_softplus(float x) {
  const float e = expf(-fabsf(x));
  const float tail = e < 1e-4f ? e * (1.0f - 0.5f * e) : logf(1.0f + e);
  return fmaxf(x, 0.0f) + tail;
}
__device__ __forceinline__ float round_half(float x) { return __half2float(__float2half_rn(x)); }

// half(silu(half(x))) for every fp16 value of half(x): the conv's SiLU
// epilogue takes an fp16 input and rounds its output to fp16, so it is a
// function of 65536 inputs.  The table is filled once per device by
// silu_table_init from the same silu() as above (so a lookup equals the
// computed value bit for bit) and replaces about 25 instructions per element
// (expf, a correctly rounded reciprocal, two conversions) by one load from
// the copy delta_prepare_resident keeps in shared memory.
__device__ __half g_silu_half[65536];

__global__ void silu_table_init() {
  const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < 65536u)
    g_silu_half[i] =
        __float2half_rn(silu(__half2float(__ushort_as_half(static_cast<unsigned short>(i)))));
}

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

// One warp per (sequence, token): the token's rotary angles are computed
// once (pair i by lane i % 32, so at most kRopeMaxPairs / 32 per lane, in
// registers) and then every head row of the token is processed.  Head h of
// the token reads input + (token * heads + h) * head_stride and writes
// output + ((output_start + token) * heads + h) * head_dim (for k, the
// cache rows of this step).  kVec: head_dim % 8 == 0 and 16-byte aligned
// rows (uint4 loads and stores).
constexpr int kRopeMaxRotary = 256;  // rotary dims (Qwen3.5 rotates 64)
constexpr int kRopeMaxPairs = kRopeMaxRotary / 2;
// Head rows in flight per warp (head_dim <= 256): at the C5 shape 1 took
// 0.603 ms, 3 0.576 ms, 4 0.586 ms (a few registers spilled).
constexpr int kRopeAhead = 3;
template <bool kVec, int kChunks = 1>
__global__ void __launch_bounds__(32 * kRopeWarps, kChunks == 1 ? 4 : 2)
    norm_rope(const RopeArgs a) {
  __shared__ __align__(16) __half rows[kRopeWarps][kRopeMaxDim];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t g = uint64_t(blockIdx.x) * kRopeWarps + warp;
  if (g >= uint64_t(a.tokens) * a.batch)
    return;  // whole warps only
  const uint32_t seq = uint32_t(g / a.tokens), token = uint32_t(g % a.tokens);
  __half *x = rows[warp];
  const unsigned D = a.head_dim, half_r = a.rotary_dim / 2;

  // cos and sin of this lane's pairs, rounded to fp16 (rotatePair).
  constexpr int kPerLane = kRopeMaxPairs / 32;
  float cs[kPerLane], sn[kPerLane];
  const float position = float(a.past + token);
#pragma unroll
  for (int k = 0; k < kPerLane; ++k) {
    const unsigned i = lane + 32 * k;
    if (i < half_r) {
      const float phase = position / powf(a.theta, 2.0f * float(i) / float(a.rotary_dim));
      cs[k] = round_half(cosf(phase));
      sn[k] = round_half(sinf(phase));
    }
  }

  auto row_in = [&](unsigned h) {
    return a.input + seq * a.input_stride + (uint64_t(token) * a.heads + h) * a.head_stride;
  };
  if constexpr (kVec) {
    // Lane l holds elements 8l + 256k .. +8 (k < kChunks, head_dim <= 256
    // kChunks) of every row in registers, with (1 + w) for them.  The rows of
    // the next kAhead - 1 heads are in flight while one is processed: a ring
    // of kAhead rows, slot u refilled with head h + kAhead as soon as head h
    // has been copied out of it (one row ahead left each SM about 16 KB of
    // loads in flight, far below what HBM latency needs).
    constexpr int kAhead = kChunks == 1 ? kRopeAhead : 2;
    float wp1[kChunks][8];
#pragma unroll
    for (int k = 0; k < kChunks; ++k)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const unsigned i = 256 * k + 8 * lane + e;
        wp1[k][e] = (a.weight && i < D) ? 1.0f + a.weight[i] : 1.0f;
      }
    uint4 ring[kAhead][kChunks];
    auto load = [&](unsigned h, uint4 (&r)[kChunks]) {
      const __half *in = row_in(h);
#pragma unroll
      for (int k = 0; k < kChunks; ++k)
        if (256 * k + 8 * lane < D)
          r[k] = *reinterpret_cast<const uint4 *>(in + 256 * k + 8 * lane);
    };
#pragma unroll
    for (int u = 0; u < kAhead; ++u)
      if (unsigned(u) < a.heads)
        load(u, ring[u]);
    for (unsigned h0 = 0; h0 < a.heads; h0 += kAhead) {
#pragma unroll
      for (int u = 0; u < kAhead; ++u) {
        const unsigned h = h0 + u;
        if (h >= a.heads)
          break;
        uint4 (&cur)[kChunks] = ring[u];
        float scale = 1.f;
        if (a.weight) {
          float sum = 0.f;
#pragma unroll
          for (int k = 0; k < kChunks; ++k)
            if (256 * k + 8 * lane < D) {
              const __half *hv = reinterpret_cast<const __half *>(&cur[k]);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float v = __half2float(hv[e]);
                sum = fmaf(v, v, sum);
              }
            }
          sum = warp_sum(sum);
          scale = rsqrtf(sum / float(D) + a.epsilon);
        }
#pragma unroll
        for (int k = 0; k < kChunks; ++k)
          if (256 * k + 8 * lane < D) {
            uint4 o = cur[k];
            if (a.weight) {
              const __half *hv = reinterpret_cast<const __half *>(&cur[k]);
              float v[8];
#pragma unroll
              for (int e = 0; e < 8; ++e)
                v[e] = __half2float(hv[e]) * scale * wp1[k][e];
              o = make_uint4(pack_half2(v[0], v[1]), pack_half2(v[2], v[3]),
                             pack_half2(v[4], v[5]), pack_half2(v[6], v[7]));
            }
            *reinterpret_cast<uint4 *>(x + 256 * k + 8 * lane) = o;
          }
        if (h + kAhead < a.heads)
          load(h + kAhead, cur);
        __syncwarp();
#pragma unroll
        for (int k = 0; k < kPerLane; ++k) {
          const unsigned i = lane + 32 * k;
          if (i < half_r) {
            const unsigned j = i + half_r;
            const float xv = __half2float(x[i]), yv = __half2float(x[j]);
            x[i] = __float2half_rn(round_half(xv * cs[k]) - round_half(yv * sn[k]));
            x[j] = __float2half_rn(round_half(yv * cs[k]) + round_half(xv * sn[k]));
          }
        }
        __syncwarp();
        __half *out = a.output + seq * a.output_stride +
                      (uint64_t(a.output_start) * a.heads + uint64_t(token) * a.heads + h) * D;
#pragma unroll
        for (int k = 0; k < kChunks; ++k)
          if (256 * k + 8 * lane < D)
            *reinterpret_cast<uint4 *>(out + 256 * k + 8 * lane) =
                *reinterpret_cast<const uint4 *>(x + 256 * k + 8 * lane);
        __syncwarp();  // the row buffer is reused by the next head
      }
    }
  } else {
  for (unsigned h = 0; h < a.heads; ++h) {
    const __half *in = row_in(h);
    __half *out = a.output + seq * a.output_stride +
                  (uint64_t(a.output_start) * a.heads + uint64_t(token) * a.heads + h) * D;
    if (a.weight) {
      float sum = 0.f;
      for (unsigned i = lane; i < D; i += 32) {
        const float v = __half2float(in[i]);
        sum = fmaf(v, v, sum);
      }
      sum = warp_sum(sum);
      const float scale = rsqrtf(sum / float(D) + a.epsilon);
      for (unsigned i = lane; i < D; i += 32)
        x[i] = __float2half_rn(__half2float(in[i]) * scale * (1.0f + a.weight[i]));
    } else {
      for (unsigned i = lane; i < D; i += 32)
        x[i] = in[i];
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < kPerLane; ++k) {
      const unsigned i = lane + 32 * k;
      if (i < half_r) {
        const unsigned j = i + half_r;
        const float xv = __half2float(x[i]), yv = __half2float(x[j]);
        x[i] = __float2half_rn(round_half(xv * cs[k]) - round_half(yv * sn[k]));
        x[j] = __float2half_rn(round_half(yv * cs[k]) + round_half(xv * sn[k]));
      }
    }
    __syncwarp();
    for (unsigned i = lane; i < D; i += 32)
      out[i] = x[i];
    __syncwarp();  // the row buffer is reused by the next head
  }
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
  const float factor = rsqrtf(sum + a.epsilon) * (is_q ? 1.0f / sqrtf(float(a.key_dim)) : 1.0f);
  float *out = (is_q ? a.q : a.k) +
               (size_t(seq) * a.conv.tokens + t) * a.key_heads * a.key_dim +
               (is_q ? h : h - a.key_heads) * a.key_dim;
#pragma unroll
  for (int e = 0; e < 8; ++e)
    if (lane + 32 * e < width)
      out[lane + 32 * e] = y[e] * factor;
}

// Tiled form for 128-wide heads and 4 conv taps (the Qwen3.5 shape): one warp
// owns one head for kPrepTokens consecutive tokens.  Lane l holds channels
// 4l..4l+3 of the head: their 4 x 4 taps in registers, and a sliding window
// of the last three input rows (8-byte loads), so every input row is read
// once per tile and every weight once per warp.  The tap sums keep the
// reference's order; SiLU comes from the per-device fp16 table, read through
// `silu` (a copy of it in shared memory, below).
constexpr int kPrepTokens = 32;
template <typename Silu>
__device__ __forceinline__ void prepare_tile(const PrepArgs &a, uint32_t seq, uint32_t t0,
                                             unsigned h, int lane, Silu silu) {
  const uint32_t W = a.conv.channels;
  const uint32_t t1 = min(t0 + uint32_t(kPrepTokens), a.conv.tokens);
  const bool is_v = h >= 2 * a.key_heads;
  const uint32_t c = (is_v ? 2 * a.key_heads * 128 + (h - 2 * a.key_heads) * 128 : h * 128) +
                     4 * lane;
  const __half *in = a.conv.input + seq * a.conv.input_stride;
  const __half *hist = a.conv.history + seq * a.conv.history_stride;

  float w[4][4];  // [channel][tap]
  {
    const uint4 *wp = reinterpret_cast<const uint4 *>(a.conv.weight + size_t(c) * 4);
    const uint4 w0 = wp[0], w1 = wp[1];
    const __half *h0 = reinterpret_cast<const __half *>(&w0);
    const __half *h1 = reinterpret_cast<const __half *>(&w1);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      w[j / 4][j % 4] = __half2float(h0[j]);
      w[2 + j / 4][j % 4] = __half2float(h1[j]);
    }
  }
  auto load_row = [&](int tau, float (&r)[4]) {
    if (tau >= 0) {
      const uint2 v = *reinterpret_cast<const uint2 *>(in + size_t(tau) * W + c);
      const __half *hv = reinterpret_cast<const __half *>(&v);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        r[e] = __half2float(hv[e]);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        r[e] = __half2float(hist[size_t(c + e) * 3 + size_t(tau + 3)]);
    }
  };
  float x3[4], x2[4], x1[4];  // rows t-3, t-2, t-1
  load_row(int(t0) - 3, x3);
  load_row(int(t0) - 2, x2);
  load_row(int(t0) - 1, x1);
  const bool is_q = h < a.key_heads;
  const float scale = is_q ? 1.0f / sqrtf(float(a.key_dim)) : 1.0f;
  // Rows are loaded kPrepAhead tokens at a time, so that many loads are in
  // flight per lane before the first is used.
  constexpr int kPrepAhead = 4;
  uint2 ahead[kPrepAhead];
  for (uint32_t t = t0; t < t1; ++t) {
    const uint32_t slot = (t - t0) % kPrepAhead;
    if (slot == 0) {
#pragma unroll
      for (int u = 0; u < kPrepAhead; ++u)
        if (t + u < t1)
          ahead[u] = *reinterpret_cast<const uint2 *>(in + size_t(t + u) * W + c);
    }
    float x0[4];
    {
      uint2 v = ahead[0];
#pragma unroll
      for (int u = 1; u < kPrepAhead; ++u)
        if (slot == uint32_t(u))
          v = ahead[u];
      const __half *hv = reinterpret_cast<const __half *>(&v);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        x0[e] = __half2float(hv[e]);
    }
    float y[4], sum = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float acc = x0[e] * w[e][3];
      acc = fmaf(x3[e], w[e][0], acc);
      acc = fmaf(x2[e], w[e][1], acc);
      acc = fmaf(x1[e], w[e][2], acc);
      y[e] = silu(acc);
      sum = fmaf(y[e], y[e], sum);
    }
    const size_t tok = size_t(seq) * a.conv.tokens + t;
    if (is_v) {
      uint2 o;
      o.x = pack_half2(y[0], y[1]);
      o.y = pack_half2(y[2], y[3]);
      *reinterpret_cast<uint2 *>(a.v + tok * a.value_heads * 128 +
                                 (h - 2 * a.key_heads) * 128 + 4 * lane) = o;
    } else {
      sum = warp_sum(sum);
      const float factor = rsqrtf(sum + a.epsilon) * scale;
      float *out = (is_q ? a.q : a.k) + tok * a.key_heads * 128 +
                   (is_q ? h : h - a.key_heads) * 128 + 4 * lane;
      *reinterpret_cast<float4 *>(out) =
          make_float4(y[0] * factor, y[1] * factor, y[2] * factor, y[3] * factor);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      x3[e] = x2[e];
      x2[e] = x1[e];
      x1[e] = x0[e];
    }
  }
}

// Persistent form: one 1024-thread CTA per SM copies the SiLU table (128 KB)
// into shared memory once, then its warps walk (sequence, token tile, head)
// items, heads fastest, so that the 32 warps of a round read neighbouring
// heads of the same input rows.  A lookup is then a shared-memory load: the
// 32 lanes' random fp16 inputs cost a few bank conflicts, where the global
// table's L1 gather touched about 26 sectors per request (C5 layer shape,
// with the gates: 1.434 -> 1.321 ms).  768 threads with eight rows in flight
// per lane instead of four (more bytes in flight per SM) ran slower.  Grid: at
// most one CTA per SM; kPrepResidentSmem bytes of dynamic shared memory.
constexpr int kPrepResidentThreads = 1024;
constexpr size_t kPrepResidentSmem = 65536 * sizeof(__half);
__global__ void __launch_bounds__(kPrepResidentThreads, 1) delta_prepare_resident(const PrepArgs a) {
  extern __shared__ __align__(16) __half silu_tab[];
  {
    const uint4 *src = reinterpret_cast<const uint4 *>(g_silu_half);
    uint4 *dst = reinterpret_cast<uint4 *>(silu_tab);
    for (unsigned i = threadIdx.x; i < kPrepResidentSmem / 16; i += kPrepResidentThreads)
      dst[i] = __ldg(src + i);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned heads = 2 * a.key_heads + a.value_heads;
  const uint32_t tiles = (a.conv.tokens + kPrepTokens - 1) / kPrepTokens;
  const uint64_t items = uint64_t(a.conv.batch) * tiles * heads;
  const uint64_t step = uint64_t(gridDim.x) * (kPrepResidentThreads / 32);
  auto silu = [&](float acc) {
    return __half2float(silu_tab[__half_as_ushort(__float2half_rn(acc))]);
  };
  for (uint64_t item = uint64_t(blockIdx.x) * (kPrepResidentThreads / 32) + warp; item < items;
       item += step) {
    const unsigned h = unsigned(item % heads);
    const uint64_t rest = item / heads;
    const uint32_t tile = uint32_t(rest % tiles), seq = uint32_t(rest / tiles);
    prepare_tile(a, seq, tile * kPrepTokens, h, lane, silu);
  }
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
