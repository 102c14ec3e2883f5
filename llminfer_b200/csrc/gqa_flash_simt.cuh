// Causal GQA flash attention on CUDA cores, for shapes outside the
// tensor-core prefill kernel (head_dim not a multiple of 16 or above 256).
// Same contract as gqaFlashAttention (FlashAttention.metal:1-83): query token
// t sees keys [0, past + t], online softmax in fp32, probabilities and
// accumulation in fp32, output rounded to fp16.
//
// One CTA = 4 query tokens of one query head of one sequence (a warp per
// token).  Keys are staged 32 at a time in shared memory as fp32; lane i
// scores key i of the tile (conflict-free: key rows are padded to D+1 words),
// then every lane accumulates its output dimensions over the tile.
#pragma once

#include "common.cuh"

namespace llmi {
namespace flash_simt {

constexpr int kWarps = 4;
constexpr int kKeys = 32;
constexpr int kMaxPerLane = 8;  // head_dim <= 256

struct Args {
  const __half *q;  // [batch][tokens][Hq][D]
  const __half *k, *v;
  size_t cache_stride;
  __half *out;
  uint32_t tokens, q_heads, kv_heads, head_dim, past, group;
  float scale_log2;
};

inline size_t smem_bytes(uint32_t D) {
  return sizeof(float) * (size_t(kKeys) * (D + 1) + size_t(kKeys) * D + size_t(kWarps) * D);
}

__global__ void __launch_bounds__(kWarps * 32) gqa_prefill_simt(const Args a) {
  extern __shared__ float sm[];
  const uint32_t D = a.head_dim, ldk = D + 1;
  float *ks = sm;
  float *vs = ks + kKeys * ldk;
  float *qs = vs + kKeys * D;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t first = blockIdx.x * kWarps;
  const uint32_t token = first + warp, head = blockIdx.y, seq = blockIdx.z;
  const uint32_t kvh = head / a.group;
  const bool active = token < a.tokens;
  const uint32_t visible = active ? a.past + token + 1 : 0;
  const uint32_t needed = a.past + min(first + kWarps, a.tokens);

  const __half *qrow = a.q + ((size_t(seq) * a.tokens + token) * a.q_heads + head) * D;
  for (uint32_t d = lane; d < D; d += 32)
    qs[warp * D + d] = active ? __half2float(qrow[d]) : 0.f;

  const size_t row = size_t(a.kv_heads) * D;
  const __half *kseq = a.k + seq * a.cache_stride + size_t(kvh) * D;
  const __half *vseq = a.v + seq * a.cache_stride + size_t(kvh) * D;

  float m = -INFINITY, l = 0.f, o[kMaxPerLane];
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i)
    o[i] = 0.f;

  for (uint32_t base = 0; base < needed; base += kKeys) {
    const uint32_t n = min(uint32_t(kKeys), needed - base);
    __syncthreads();  // the previous tile is consumed
    for (uint32_t i = threadIdx.x; i < n * D; i += blockDim.x) {
      const uint32_t key = i / D, d = i % D;
      ks[key * ldk + d] = __half2float(kseq[(base + key) * row + d]);
      vs[key * D + d] = __half2float(vseq[(base + key) * row + d]);
    }
    __syncthreads();
    if (base >= visible)
      continue;  // warp-uniform; the tile barriers above are shared
    const uint32_t valid = min(n, visible - base);
    float x = -INFINITY;
    if (uint32_t(lane) < valid) {
      float dot = 0.f;
      for (uint32_t d = 0; d < D; ++d)
        dot = fmaf(qs[warp * D + d], ks[lane * ldk + d], dot);
      x = dot * a.scale_log2;
    }
    float top = x;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
      top = fmaxf(top, __shfl_xor_sync(0xffffffffu, top, off));
    const float next = fmaxf(m, top);
    const float rescale = fast_exp2(m - next);
    const float p = uint32_t(lane) < valid ? fast_exp2(x - next) : 0.f;
    float sum = p;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
      sum += __shfl_xor_sync(0xffffffffu, sum, off);
    l = l * rescale + sum;
    m = next;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i)
      o[i] *= rescale;
    for (uint32_t key = 0; key < valid; ++key) {
      const float w = __shfl_sync(0xffffffffu, p, key);
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i) {
        const uint32_t d = lane + 32 * i;
        if (d < D)
          o[i] = fmaf(w, vs[key * D + d], o[i]);
      }
    }
  }

  if (!active)
    return;
  __half *orow = a.out + ((size_t(seq) * a.tokens + token) * a.q_heads + head) * D;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const uint32_t d = lane + 32 * i;
    if (d < D)
      orow[d] = __float2half_rn(o[i] / l);
  }
}

}  // namespace flash_simt
}  // namespace llmi
