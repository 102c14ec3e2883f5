// Chunk-parallel first pass of the tensor-core DeltaNet prefill: the
// chunk-local triangular system of the WY / UT form, for every chunk at once.
//
// For one chunk of C = 64 tokens of one (sequence, value head), with G_t the
// within-chunk cumulative log-decay and beta_t the write strengths (the terms
// of Graph.metal:146-170 / Reference.metal:182-197 unrolled over a chunk):
//   A[t][s] = beta_t (k_t . k_s) e^{G_t - G_s}   (s < t, else 0)
//   T       = (I + A)^-1                          (unit lower triangular)
// and the pass writes Tu = T diag(beta) in fp16.  Nothing of this depends on
// the state, so unlike the state recurrence it has no order across chunks:
// the grid is every (chunk, key head, sequence), each CTA computes k k^T of
// its chunk once and solves the system of each value head that shares the
// key head.  The second pass (delta_chunk_tc.cuh, Presolved) loads Tu with
// one bulk copy per chunk and derives Tw = T diag(beta e^G) = Tu diag(e^G).
//
// Output layout: per (sequence, value head, chunk) an 8 KB image of Tu
// [64 t][64 s] fp16 in the 128-byte-swizzled K-major layout the second
// pass's tcgen05 MMAs read (row t at t * 128 bytes, 16-byte chunk c of a row
// at position c ^ (t & 7)), so the image is copied verbatim into shared
// memory.  The pass also writes, per (sequence, key head, chunk), the k rows
// it converted to fp16 as a 16 KB image in the second pass's [K; Q] operand
// layout (two 8 KB blocks of 64 keys, the same swizzle), which replaces the
// second pass's own fp32 staging and conversion at no extra HBM traffic (it
// reads 16 KB of fp16 there instead of 32 KB of fp32).  Requires
// key_dim == 128.
//
// Warp MMAs (m16n8k16, fp16 in, fp32 accumulation) do k k^T and the blocked
// substitution; the 16x16 diagonal blocks are inverted by forward
// substitution in fp32.  A 128-thread CTA holds no tensor memory and about
// 35 KB of shared memory and 80 registers, so six run on each SM.
#pragma once

#include "common.cuh"
#include "delta_recurrent.cuh"
#include "tcgen05.cuh"

namespace llmi {
namespace delta_solve {

constexpr int C = 64, DK = 128;
constexpr int kThreads = 128;
constexpr int kLdK = DK + 8;  // fp16 row stride of the k tile (conflict-free ldmatrix)
constexpr int kLdA = 72;      // fp16 row stride of A
constexpr int kLdT = 24;      // fp16 row stride of the diagonal-block inverses
constexpr int kMaxGroup = 4;                    // value heads per key head held at once
constexpr uint32_t kImageBytes = C * C * 2;     // one Tu image
constexpr uint32_t kKImageBytes = C * DK * 2;   // one chunk's k rows

struct Smem {
  // The k rows are read only up to k k^T, which every warp finishes before
  // the first barrier of the value-head loop; the Tu image, written two
  // barriers later, takes their place.  35 KB in all: six CTAs per SM.
  union {
    __half k[C * kLdK];                    // k rows of the chunk, fp16
    alignas(128) uint8_t tu[kImageBytes];  // the Tu image
  };
  __half am[C * kLdA];      // A, fp16 (blocks below the diagonal are read)
  float ad[4 * 16 * 16];    // diagonal blocks of A, fp32, [block][s][t]
  __half td[C * kLdT];      // inverses of the diagonal blocks of I + A, fp16
  float g2[kMaxGroup][C];   // per value head of the key head: G_t in log2 units
  float bet[kMaxGroup][C];  // beta_t (0 past the last token)
};
static_assert(sizeof(Smem) + 1024 <= 232448 / 6, "six solve CTAs per SM");

// One 16x16 fp16 tile of a row-major array as an m16n8k16 A fragment.
__device__ __forceinline__ void frag_a(uint32_t (&f)[4], const __half *base, int ld, int m0,
                                       int k0, int lane) {
  ldmatrix_x4(f, smem_u32(base + (m0 + (lane & 15)) * ld + k0 + (lane >> 4) * 8));
}

// Grid (chunks, key heads, batch), kThreads threads, sizeof(Smem) bytes of
// dynamic shared memory.  tu_out: [batch][value heads][chunks] Tu images;
// k_out: [batch][key heads][chunks] k-row images.
__global__ void __launch_bounds__(kThreads, 6)
    solve_pass(const delta::Args a, uint8_t *__restrict__ tu_out, uint8_t *__restrict__ k_out) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t chunk = blockIdx.x, kh = blockIdx.y, seq = blockIdx.z;
  const uint32_t n_chunks = gridDim.x;
  const uint32_t t0 = chunk * C;
  const int valid = int(min(uint32_t(C), a.tokens - t0));

  // Gates of value head vh into slot j: G (log2 units, inclusive cumulative
  // sum of log2 decay; pad tokens decay 1, beta 0).  A decay of exactly 0
  // gets log2 -1e4, so every factor across it is 0.  One warp.
  auto gates = [&](uint32_t vh, int j) {
    const size_t tok0 = size_t(seq) * a.tokens + t0;
    float la[2], bb[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int t = 2 * lane + i;
      const bool in = t < valid;
      const float d = in ? a.decay[(tok0 + t) * a.value_heads + vh] : 1.f;
      la[i] = in ? (d > 0.f ? fast_log2(d) : -1e4f) : 0.f;
      bb[i] = in ? a.beta[(tok0 + t) * a.value_heads + vh] : 0.f;
    }
    const float pair = la[0] + la[1];
    float incl = pair;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off)
        incl += y;
    }
    sm.g2[j][2 * lane] = incl - pair + la[0];
    sm.g2[j][2 * lane + 1] = incl;
    sm.bet[j][2 * lane] = bb[0];
    sm.bet[j][2 * lane + 1] = bb[1];
  };
  // k rows of the chunk (fp32, 512 B each) into the fp16 tile, in two
  // rounds of loads; rows past the last token are zero.  The gates of up to
  // kMaxGroup value heads are derived while the first round is in flight.
  {
    const float *src = a.k + (size_t(seq) * a.tokens + t0) * a.key_heads * DK + size_t(kh) * DK;
    const size_t row_stride = size_t(a.key_heads) * DK;
#pragma unroll
    for (int round = 0; round < 2; ++round) {
      float4 r[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int idx = tid + kThreads * (8 * round + i), t = idx >> 5, c4 = idx & 31;
        r[i] = t < valid ? ld_stream_f4(src + size_t(t) * row_stride + 4 * c4)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      if (round == 0 && a.group <= uint32_t(kMaxGroup) && warp < int(a.group))
        gates(kh * a.group + warp, warp);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int idx = tid + kThreads * (8 * round + i), t = idx >> 5, c4 = idx & 31;
        *reinterpret_cast<uint2 *>(sm.k + t * kLdK + 4 * c4) =
            make_uint2(pack_half2(r[i].x, r[i].y), pack_half2(r[i].z, r[i].w));
      }
    }
  }
  __syncthreads();
  // The k rows' image for the second pass: 16-byte chunk ch of row t to
  // block ch / 8, swizzled position (ch % 8) ^ (t % 8).
  {
    uint8_t *dst = k_out + ((size_t(seq) * a.key_heads + kh) * n_chunks + chunk) * kKImageBytes;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = tid + kThreads * i, t = idx >> 4, ch = idx & 15;
      *reinterpret_cast<uint4 *>(dst + (ch >> 3) * (kKImageBytes / 2) + sw128_chunk(t, ch & 7)) =
          *reinterpret_cast<const uint4 *>(sm.k + t * kLdK + 8 * ch);
    }
  }

  // k k^T on the blocks at or below the diagonal: warp w owns rows
  // 16w..16w+15 and the column tiles 0..2w+1.
  float dots[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e)
      dots[j][e] = 0.f;
#pragma unroll
  for (int ks = 0; ks < DK / 16; ++ks) {
    uint32_t fa[4];
    frag_a(fa, sm.k, kLdK, 16 * warp, 16 * ks, lane);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      if (np <= warp) {
        // Two column tiles of 8 tokens: rows s of the k tile are the columns
        // of k^T, so a plain ldmatrix gives the B fragments.
        uint32_t fb[4];
        const int row = 16 * np + ((lane >> 4) << 3) + (lane & 7);
        const int col = 16 * ks + ((lane >> 3) & 1) * 8;
        ldmatrix_x4(fb, smem_u32(sm.k + row * kLdK + col));
        mma_f16_16816(dots[2 * np], fa, fb[0], fb[1]);
        mma_f16_16816(dots[2 * np + 1], fa, fb[2], fb[3]);
      }
    }
  }

  const int g = lane >> 2;
  const bool gates_ahead = a.group <= uint32_t(kMaxGroup);
  for (uint32_t vh = kh * a.group; vh < (kh + 1) * a.group; ++vh) {
    const int j = gates_ahead ? int(vh - kh * a.group) : 0;
    if (!gates_ahead) {
      if (warp == 0)
        gates(vh, 0);
      __syncthreads();
    }
    const float *g2 = sm.g2[j], *bet = sm.bet[j];

    // A from the dot products: beta_t (k_t . k_s) 2^(G_t - G_s) for s < t.
    // fp16 rows into am, the diagonal blocks also in fp32 (column-major).
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int t = 16 * warp + g + 8 * half;
      const float g_t = g2[t], b_t = bet[t];
#pragma unroll
      for (int jt = 0; jt < 8; ++jt) {
        if (jt < 2 * warp + 2) {
          const int s = 8 * jt + 2 * (lane & 3);
          float v[2];
#pragma unroll
          for (int e = 0; e < 2; ++e)
            v[e] = s + e < t ? b_t * dots[jt][2 * half + e] * fast_exp2(g_t - g2[s + e]) : 0.f;
          *reinterpret_cast<uint32_t *>(sm.am + t * kLdA + s) = pack_half2(v[0], v[1]);
          if (jt >= 2 * warp) {  // the diagonal block
#pragma unroll
            for (int e = 0; e < 2; ++e)
              sm.ad[warp * 256 + ((s + e) & 15) * 16 + (t & 15)] = v[e];
          }
        }
      }
    }
    __syncthreads();

    // Diagonal blocks of (I + A)^-1 by column-oriented forward substitution
    // in fp32 (warp i = block i, lane = column).
    if (lane < 16) {
      const float4 *ab = reinterpret_cast<const float4 *>(sm.ad + warp * 256);
      float x[16];
#pragma unroll
      for (int r = 0; r < 16; ++r)
        x[r] = r == lane ? 1.f : 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float col[16];  // column j of the block: A[r][j]
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 c = ab[4 * j + i];
          col[4 * i] = c.x;
          col[4 * i + 1] = c.y;
          col[4 * i + 2] = c.z;
          col[4 * i + 3] = c.w;
        }
#pragma unroll
        for (int r = j + 1; r < 16; ++r)
          x[r] = fmaf(-col[r], x[j], x[r]);
      }
#pragma unroll
      for (int r = 0; r < 16; ++r)
        sm.td[(warp * 16 + r) * kLdT + lane] = __float2half_rn(x[r]);
    }
    __syncthreads();

    // Block rows T_i = T_ii (I_i - sum_{k<i} A_ik T_k): warp w owns the 16
    // columns of diagonal block w (zero above it); Tu = T diag(beta).
    {
      float su[2][2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e)
          su[nt][e] = bet[16 * warp + 8 * nt + 2 * (lane & 3) + e];
      uint32_t xb[4][2][2];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float x[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        if (i >= warp) {
          float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
          for (int kb = 0; kb < i; ++kb) {
            if (kb >= warp) {
              uint32_t fa[4];
              frag_a(fa, sm.am, kLdA, 16 * i, 16 * kb, lane);
#pragma unroll
              for (int nt = 0; nt < 2; ++nt)
                mma_f16_16816(acc[nt], fa, xb[kb][nt][0], xb[kb][nt][1]);
            }
          }
          uint32_t ft[4];
          frag_a(ft, sm.td, kLdT, 16 * i, 0, lane);
          const int r0 = 16 * i + g;
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const int c0 = 16 * warp + 8 * nt + 2 * (lane & 3);
            const uint32_t rb0 = movmatrix_trans(
                pack_half2(float(r0 == c0) - acc[nt][0], float(r0 == c0 + 1) - acc[nt][1]));
            const uint32_t rb1 = movmatrix_trans(pack_half2(float(r0 + 8 == c0) - acc[nt][2],
                                                            float(r0 + 8 == c0 + 1) - acc[nt][3]));
            mma_f16_16816(x[nt], ft, rb0, rb1);
            xb[i][nt][0] = movmatrix_trans(pack_half2(x[nt][0], x[nt][1]));
            xb[i][nt][1] = movmatrix_trans(pack_half2(x[nt][2], x[nt][3]));
          }
        }
        const int r = 16 * i + g;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int c0 = 16 * warp + 8 * nt + 2 * (lane & 3);
          const uint32_t o0 = sw128_chunk(r, c0 >> 3) + (c0 & 7) * 2;
          const uint32_t o1 = sw128_chunk(r + 8, c0 >> 3) + (c0 & 7) * 2;
          *reinterpret_cast<uint32_t *>(sm.tu + o0) =
              pack_half2(x[nt][0] * su[nt][0], x[nt][1] * su[nt][1]);
          *reinterpret_cast<uint32_t *>(sm.tu + o1) =
              pack_half2(x[nt][2] * su[nt][0], x[nt][3] * su[nt][1]);
        }
      }
    }
    __syncthreads();

    // The image to global memory (8 KB, 16-byte stores).
    uint4 *dst = reinterpret_cast<uint4 *>(
        tu_out + ((size_t(seq) * a.value_heads + vh) * n_chunks + chunk) * kImageBytes);
    const uint4 *srcv = reinterpret_cast<const uint4 *>(sm.tu);
#pragma unroll
    for (int i = 0; i < int(kImageBytes / 16 / kThreads); ++i)
      dst[tid + kThreads * i] = srcv[tid + kThreads * i];
    __syncthreads();
  }
}

}  // namespace delta_solve
}  // namespace llmi
