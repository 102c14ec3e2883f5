// Gated DeltaNet recurrent update, token by token, with the state held in
// registers for the whole call.  Semantics of graphDeltaUpdate
// (Graph.metal:146-170) with updateDeltaColumn (Reference.metal:182-197):
//   S = decay*S;  pred = S^T k;  delta = beta*(v - pred);
//   S += k delta^T;  y = S^T q   (y rounded to fp16)
// with the same per-element fma forms; only the order in which the dk-long
// sums are added differs (per-warp partial sums, then across warps).
//
// The reference walks the state column by column from device memory twice
// per token.  Here one CTA owns one (sequence, value head): its dk x 128 fp32
// state (64 KiB for dk = 128) is read once with 128-bit streaming loads,
// lives in registers (warp w holds rows w, w+8, ...; lane j holds columns
// 4j..4j+3, so every row is one coalesced 512-byte access), and is written
// back once after the last token.  For one token this is the HBM-bound
// decode step; every byte of state crosses HBM exactly twice.
#pragma once

#include "common.cuh"

namespace llmi {
namespace delta {

struct Args {
  const float *q, *k;      // [batch][tokens][Hk*dk]
  const __half *v;         // [batch][tokens][Hv*dv]
  const float *beta, *decay;  // [batch][tokens][Hv]
  float *state;            // [batch][Hv][dk][dv]
  __half *out;             // [batch][tokens][Hv*dv]
  uint32_t batch, tokens, key_heads, key_dim, value_heads, value_dim, group;
  // Nonzero when the caller guarantees that no work still in flight writes
  // the state (LLMI_FLAG_SETTLED): recurrent_v32 then loads it into
  // registers before wait_primary(), while the kernel ahead still runs.
  uint32_t settled;
};

constexpr int kRecWarps = 8;
// recurrent_v32 comes in two register budgets.  A grid that fits on the GPU
// in one wave (B = 2: 256 CTAs) takes the unbounded form, whose address
// arithmetic stays ahead of the wait (56 registers, four CTAs per SM).  A
// grid that runs in waves (B = 16: 2048 CTAs) takes five CTAs per SM (at
// most 51 registers a thread), which keeps those waves at three.
constexpr int kRecV32OneWave = 4;  // CTAs per SM of the unbounded form
constexpr int kRecV32Waves = 5;

// dv == 128, dk == DK (multiple of 8, <= 128).  Grid (Hv, batch), 256 threads.
template <int DK>
__global__ void __launch_bounds__(kRecWarps * 32) recurrent_v128(const Args a) {
  constexpr int R = DK / kRecWarps;  // state rows per warp
  constexpr int DV = 128;
  __shared__ float4 red_pred[kRecWarps][32];
  __shared__ float4 red_out[kRecWarps][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t vh = blockIdx.x, seq = blockIdx.y;
  const uint32_t kh = vh / a.group;
  float *S = a.state + (size_t(seq) * a.value_heads + vh) * DK * DV;
  // No L2 warm-up here (recurrent_v32 has one): this form runs when many
  // CTAs stream the state in waves, HBM-bound, and prefetches by the CTAs
  // resident ahead of their wait only re-read lines the kernel ahead is
  // about to write (1.8 % slower at C4).
  pdl_enter();

  float4 s[R];
#pragma unroll
  for (int r = 0; r < R; ++r)
    s[r] = ld_stream_f4(S + size_t(warp + kRecWarps * r) * DV + lane * 4);

  const size_t key_width = size_t(a.key_heads) * DK;
  const size_t value_width = size_t(a.value_heads) * DV;
  for (uint32_t t = 0; t < a.tokens; ++t) {
    const size_t tok = size_t(seq) * a.tokens + t;
    const float *kt = a.k + tok * key_width + size_t(kh) * DK;
    const float *qt = a.q + tok * key_width + size_t(kh) * DK;
    const float dec = __ldg(a.decay + tok * a.value_heads + vh);
    const float bet = __ldg(a.beta + tok * a.value_heads + vh);
    const uint2 vraw = __ldg(reinterpret_cast<const uint2 *>(a.v + tok * value_width + vh * DV) + lane);
    const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&vraw.x));
    const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&vraw.y));

    float kr[R], qr[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      kr[r] = __ldg(kt + warp + kRecWarps * r);
      qr[r] = __ldg(qt + warp + kRecWarps * r);
    }
    float4 pp = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      pp.x = fmaf(s[r].x * dec, kr[r], pp.x);
      pp.y = fmaf(s[r].y * dec, kr[r], pp.y);
      pp.z = fmaf(s[r].z * dec, kr[r], pp.z);
      pp.w = fmaf(s[r].w * dec, kr[r], pp.w);
    }
    red_pred[warp][lane] = pp;
    __syncthreads();
    float4 pred = red_pred[0][lane];
#pragma unroll
    for (int w = 1; w < kRecWarps; ++w) {
      const float4 x = red_pred[w][lane];
      pred.x += x.x;
      pred.y += x.y;
      pred.z += x.z;
      pred.w += x.w;
    }
    const float4 delta = make_float4((v01.x - pred.x) * bet, (v01.y - pred.y) * bet,
                                     (v23.x - pred.z) * bet, (v23.y - pred.w) * bet);
    float4 yp = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      s[r].x = fmaf(kr[r], delta.x, s[r].x * dec);
      s[r].y = fmaf(kr[r], delta.y, s[r].y * dec);
      s[r].z = fmaf(kr[r], delta.z, s[r].z * dec);
      s[r].w = fmaf(kr[r], delta.w, s[r].w * dec);
      yp.x = fmaf(s[r].x, qr[r], yp.x);
      yp.y = fmaf(s[r].y, qr[r], yp.y);
      yp.z = fmaf(s[r].z, qr[r], yp.z);
      yp.w = fmaf(s[r].w, qr[r], yp.w);
    }
    red_out[warp][lane] = yp;
    __syncthreads();
    if (warp == 0) {
      float4 y = red_out[0][lane];
#pragma unroll
      for (int w = 1; w < kRecWarps; ++w) {
        const float4 x = red_out[w][lane];
        y.x += x.x;
        y.y += x.y;
        y.z += x.z;
        y.w += x.w;
      }
      uint2 packed;
      *reinterpret_cast<__half2 *>(&packed.x) = __floats2half2_rn(y.x, y.y);
      *reinterpret_cast<__half2 *>(&packed.y) = __floats2half2_rn(y.z, y.w);
      reinterpret_cast<uint2 *>(a.out + tok * value_width + vh * DV)[lane] = packed;
    }
  }

#pragma unroll
  for (int r = 0; r < R; ++r)
    st_stream_f4(S + size_t(warp + kRecWarps * r) * DV + lane * 4, s[r]);
}

// The same update with the value columns split into blocks of 32: one CTA
// per (sequence, value head, block), 16 KiB of state for dk = 128, so small
// batches still give every SM several CTAs (at batch 16 the 128-column form
// has 512 CTAs and runs at a third of HBM bandwidth).  Lane l holds columns
// 4(l % 8)..+3 of the block for rows w*4 + l/8 + 32p; each warp load covers
// four 128-byte row segments.  Row sums: per lane, then across the four row
// lanes of a warp (shuffles), then across warps (shared memory).
// Grid (Hv * dv / 32, batch), 256 threads; dk multiple of 32, <= 128.
template <int DK, int MIN_CTAS>
__global__ void __launch_bounds__(kRecWarps * 32, MIN_CTAS) recurrent_v32(const Args a) {
  constexpr int R = DK / 32;  // row passes per thread
  constexpr int DV = 128, kCols = 32;
  __shared__ float4 red_pred[kRecWarps][8];
  __shared__ float4 red_out[kRecWarps][8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cg = lane & 7, rs = lane >> 3;
  const uint32_t vh = blockIdx.x / (DV / kCols), blk = blockIdx.x % (DV / kCols);
  const uint32_t seq = blockIdx.y, kh = vh / a.group;
  const uint32_t col = blk * kCols + 4 * cg;  // this lane's first column within the head
  float *S = a.state + (size_t(seq) * a.value_heads + vh) * DK * DV;
  // A settled state is loaded into registers before the wait.  Otherwise
  // this block's state goes into L2 while the kernel ahead still runs (a
  // prefetch never changes what a later load returns; one 128-byte row
  // segment per thread) and is loaded after the wait.
  auto row_of = [&](int p) { return warp * 4 + rs + 32 * p; };
  // This CTA's key and query rows of token 0; the operands below keep the
  // address arithmetic (a division by the group) ahead of the wait.
  const float *k0 = a.k + size_t(seq) * a.tokens * a.key_heads * DK + size_t(kh) * DK;
  const float *q0 = a.q + (k0 - a.k);
  asm volatile("" ::"l"(k0), "l"(q0));
  float4 s[R];
  if (a.settled) {
#pragma unroll
    for (int p = 0; p < R; ++p)
      s[p] = ld_stream_f4(S + size_t(row_of(p)) * DV + col);
    pdl_enter();
  } else {
    if (threadIdx.x < DK)
      prefetch_l2(S + size_t(threadIdx.x) * DV + blk * kCols, kCols * 4);
    pdl_enter();
#pragma unroll
    for (int p = 0; p < R; ++p)
      s[p] = ld_stream_f4(S + size_t(row_of(p)) * DV + col);
  }

  const size_t key_width = size_t(a.key_heads) * DK;
  const size_t value_width = size_t(a.value_heads) * DV;
  for (uint32_t t = 0; t < a.tokens; ++t) {
    const size_t tok = size_t(seq) * a.tokens + t;
    const float *kt = k0 + t * key_width;
    const float *qt = q0 + t * key_width;
    const float dec = __ldg(a.decay + tok * a.value_heads + vh);
    const float bet = __ldg(a.beta + tok * a.value_heads + vh);
    const uint2 vraw = __ldg(reinterpret_cast<const uint2 *>(a.v + tok * value_width + vh * DV + col));
    const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&vraw.x));
    const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&vraw.y));
    float kr[R], qr[R];
#pragma unroll
    for (int p = 0; p < R; ++p) {
      kr[p] = __ldg(kt + row_of(p));
      qr[p] = __ldg(qt + row_of(p));
    }
    float4 pp = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < R; ++p) {
      pp.x = fmaf(s[p].x * dec, kr[p], pp.x);
      pp.y = fmaf(s[p].y * dec, kr[p], pp.y);
      pp.z = fmaf(s[p].z * dec, kr[p], pp.z);
      pp.w = fmaf(s[p].w * dec, kr[p], pp.w);
    }
#pragma unroll
    for (int off = 8; off < 32; off <<= 1) {
      pp.x += __shfl_xor_sync(0xffffffffu, pp.x, off);
      pp.y += __shfl_xor_sync(0xffffffffu, pp.y, off);
      pp.z += __shfl_xor_sync(0xffffffffu, pp.z, off);
      pp.w += __shfl_xor_sync(0xffffffffu, pp.w, off);
    }
    if (rs == 0)
      red_pred[warp][cg] = pp;
    __syncthreads();
    float4 pred = red_pred[0][cg];
#pragma unroll
    for (int w = 1; w < kRecWarps; ++w) {
      const float4 x = red_pred[w][cg];
      pred.x += x.x;
      pred.y += x.y;
      pred.z += x.z;
      pred.w += x.w;
    }
    const float4 delta = make_float4((v01.x - pred.x) * bet, (v01.y - pred.y) * bet,
                                     (v23.x - pred.z) * bet, (v23.y - pred.w) * bet);
    float4 yp = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < R; ++p) {
      s[p].x = fmaf(kr[p], delta.x, s[p].x * dec);
      s[p].y = fmaf(kr[p], delta.y, s[p].y * dec);
      s[p].z = fmaf(kr[p], delta.z, s[p].z * dec);
      s[p].w = fmaf(kr[p], delta.w, s[p].w * dec);
      yp.x = fmaf(s[p].x, qr[p], yp.x);
      yp.y = fmaf(s[p].y, qr[p], yp.y);
      yp.z = fmaf(s[p].z, qr[p], yp.z);
      yp.w = fmaf(s[p].w, qr[p], yp.w);
    }
#pragma unroll
    for (int off = 8; off < 32; off <<= 1) {
      yp.x += __shfl_xor_sync(0xffffffffu, yp.x, off);
      yp.y += __shfl_xor_sync(0xffffffffu, yp.y, off);
      yp.z += __shfl_xor_sync(0xffffffffu, yp.z, off);
      yp.w += __shfl_xor_sync(0xffffffffu, yp.w, off);
    }
    if (rs == 0)
      red_out[warp][cg] = yp;
    __syncthreads();
    if (warp == 0 && rs == 0) {
      float4 y = red_out[0][cg];
#pragma unroll
      for (int w = 1; w < kRecWarps; ++w) {
        const float4 x = red_out[w][cg];
        y.x += x.x;
        y.y += x.y;
        y.z += x.z;
        y.w += x.w;
      }
      uint2 packed;
      *reinterpret_cast<__half2 *>(&packed.x) = __floats2half2_rn(y.x, y.y);
      *reinterpret_cast<__half2 *>(&packed.y) = __floats2half2_rn(y.z, y.w);
      *reinterpret_cast<uint2 *>(a.out + tok * value_width + vh * DV + col) = packed;
    }
    // The reduction buffers are reused by the next token.
    if (t + 1 < a.tokens)
      __syncthreads();
  }

#pragma unroll
  for (int p = 0; p < R; ++p)
    st_stream_f4(S + size_t(row_of(p)) * DV + col, s[p]);
}

// Any (dk, dv): one thread per (sequence, value column), state in global
// memory, the reference's column walk.  Used only for shapes outside the
// fast kernels.
__global__ void __launch_bounds__(128) recurrent_generic(const Args a) {
  pdl_enter();
  const uint32_t value_width = a.value_heads * a.value_dim;
  const uint64_t total = uint64_t(a.batch) * value_width;
  const uint64_t c = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x;
  if (c >= total)
    return;
  const uint32_t seq = uint32_t(c / value_width), column = uint32_t(c % value_width);
  const uint32_t vh = column / a.value_dim, j = column % a.value_dim, kh = vh / a.group;
  const uint32_t dk = a.key_dim, dv = a.value_dim;
  float *S = a.state + (size_t(seq) * a.value_heads + vh) * dk * dv + j;
  const size_t key_width = size_t(a.key_heads) * dk;
  for (uint32_t t = 0; t < a.tokens; ++t) {
    const size_t tok = size_t(seq) * a.tokens + t;
    const float *kt = a.k + tok * key_width + size_t(kh) * dk;
    const float *qt = a.q + tok * key_width + size_t(kh) * dk;
    const float dec = a.decay[tok * a.value_heads + vh], bet = a.beta[tok * a.value_heads + vh];
    const float x = __half2float(a.v[tok * value_width + column]);
    float pred = 0.f;
    for (uint32_t i = 0; i < dk; ++i)
      pred = fmaf(S[size_t(i) * dv] * dec, kt[i], pred);
    const float delta = (x - pred) * bet;
    float y = 0.f;
    for (uint32_t i = 0; i < dk; ++i) {
      const float next = fmaf(kt[i], delta, S[size_t(i) * dv] * dec);
      S[size_t(i) * dv] = next;
      y = fmaf(next, qt[i], y);
    }
    a.out[tok * value_width + column] = __float2half_rn(y);
  }
}

}  // namespace delta
}  // namespace llmi
