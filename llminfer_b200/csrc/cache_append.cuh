// cacheAppend: copies a step's new keys (or values) into each sequence's
// cache at rows [past, past + tokens).  Semantics of the reference kernel
// lib/Backend/Metal/Kernels/Reference.metal:295-301, batched over sequences.
#pragma once

#include "common.cuh"

namespace llmi {

struct AppendArgs {
  const uint16_t *input;
  uint16_t *cache;
  size_t input_stride, cache_stride;  // elements between sequences
  uint32_t count, offset, batch;
};

// 16-byte path: count, offset, strides and both bases are multiples of 8
// halves.  One grid-stride loop over (sequence, vector).
__global__ void __launch_bounds__(256) cache_append_v8(AppendArgs a) {
  pdl_enter();
  const uint32_t vectors = a.count / 8;
  const uint64_t total = uint64_t(vectors) * a.batch;
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < total;
       i += uint64_t(gridDim.x) * blockDim.x) {
    const uint64_t seq = i / vectors, j = i % vectors;
    const uint4 *src = reinterpret_cast<const uint4 *>(a.input + seq * a.input_stride) + j;
    uint4 *dst = reinterpret_cast<uint4 *>(a.cache + seq * a.cache_stride + a.offset) + j;
    *dst = *src;
  }
}

__global__ void __launch_bounds__(256) cache_append_scalar(AppendArgs a) {
  pdl_enter();
  const uint64_t total = uint64_t(a.count) * a.batch;
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < total;
       i += uint64_t(gridDim.x) * blockDim.x) {
    const uint64_t seq = i / a.count, j = i % a.count;
    a.cache[seq * a.cache_stride + a.offset + j] = a.input[seq * a.input_stride + j];
  }
}

}  // namespace llmi
