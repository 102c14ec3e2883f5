// Gated DeltaNet multi-token update in chunks of 64 tokens.
//
// Same result as the token-sequential graphDeltaUpdate
// (Graph.metal:146-170, Reference.metal:182-197) up to rounding, computed
// with the chunkwise (WY / UT) form of the gated delta rule (Yang, Kautz,
// Hatamizadeh, "Gated Delta Networks", 2024).  With S the [dk][dv] state at
// the start of a chunk, G_t the within-chunk cumulative log-decay
// (sum_{s<=t} log decay_s) and e^{x} = exp:
//   A[t][s] = beta_t (k_t . k_s) e^{G_t - G_s}            (s < t, else 0)
//   (I + A) [W | U] = [diag(beta e^{G}) K | diag(beta) V]  (unit lower-triangular solve)
//   V'     = U - W S                                       (the chunk's deltas)
//   y_t    = e^{G_t} q_t^T S + sum_{s<=t} (q_t . k_s) e^{G_t - G_s} V'_s
//   S     <- e^{G_C} S + sum_s e^{G_C - G_s} k_s V'_s^T
// Unrolling the per-token recurrence S_t = decay_t (I - beta_t k_t k_t^T)
// S_{t-1} + beta_t k_t v_t^T over a chunk gives exactly these terms.
//
// One CTA (8 warps) owns one (sequence, value head) for the whole call and
// walks its chunks in order.  The fp32 state lives in mma accumulator
// fragments (warp w holds key rows 16w..16w+15, all 128 value columns) and,
// rounded to fp16, in shared memory as the B operand of W S and Q S.  Every
// product is a warp-level m16n8k16 MMA (fp16 operands, fp32 accumulation).
// The triangular solve is blocked by 16 tokens: the four 16x16 diagonal
// blocks are inverted by forward substitution in fp32, and block row i of
// [W | U] = T_ii (RHS_i - sum_{k<i} A_ik [W | U]_k) runs on the MMAs.
// The next chunk's raw rows are staged into shared memory with cp.async
// while the current chunk's last two phases run, so global latency is off the
// per-chunk critical path.
// Requires key_dim == value_dim == 128.
#pragma once

#include "common.cuh"
#include "delta_recurrent.cuh"

namespace llmi {
namespace delta_chunk {

constexpr int C = 64;       // tokens per chunk
constexpr int DK = 128, DV = 128;
constexpr int kThreads = 256;
constexpr int kLd128 = 136;  // fp16 row stride of 128-wide tiles (+8: conflict-free ldmatrix)
constexpr int kLd64 = 72;    // fp16 row stride of 64-wide tiles
constexpr int kLd16 = 24;    // fp16 row stride of the 16x16 diagonal inverses
constexpr int kLdD = 17;     // fp32 row stride of the 16x16 diagonal blocks of A

struct Smem {
  static constexpr int tile128 = C * kLd128 * 2;
  static constexpr int Ks = 0;                       // K
  static constexpr int Kg = Ks + tile128;            // K * e^{G_C - G}
  static constexpr int Qs = Kg + tile128;            // Q
  static constexpr int Rk = Qs + tile128;            // K * beta e^{G}   (right-hand side for W)
  static constexpr int Rv = Rk + tile128;            // V * beta         (right-hand side for U)
  static constexpr int Wm = Rv + tile128;            // W
  static constexpr int Um = Wm + tile128;            // U
  static constexpr int Vp = Um + tile128;            // V'
  static constexpr int Sm = Vp + tile128;            // S (fp16), DK rows
  static constexpr int Pm = Sm + DK * kLd128 * 2;    // (Q K^T) masked, decayed
  static constexpr int Am = Pm + C * kLd64 * 2;      // A (fp16)
  static constexpr int Td = Am + C * kLd64 * 2;      // diagonal-block inverses (fp16)
  static constexpr int Ad = Td + C * kLd16 * 2;      // diagonal blocks of A (fp32)
  static constexpr int vec = Ad + 4 * 16 * kLdD * 4; // g[64], beta[64], glast
  static constexpr int gates = vec + (2 * C + 4) * 4; // next chunk's decay[64], beta[64]
  static constexpr int total = gates + 2 * C * 4;
  // The next chunk's raw rows are staged (cp.async) in buffers that are dead
  // during the last two phases of a chunk: K and Q (fp32) over Rk..Um, V
  // (fp16) over Am..Ad.
  static constexpr int rawK = Rk;
  static constexpr int rawQ = Rk + C * DK * 4;
  static constexpr int rawV = Am;
};
static_assert(Smem::rawQ + C * DK * 4 <= Smem::Vp, "raw K/Q staging overlaps V'");
static_assert(Smem::rawV + C * DV * 2 <= Smem::vec, "raw V staging overlaps the gates");

// ---- warp-level fragments (m16n8k16) ------------------------------------------------

// A tile 16x16 of a row-major [m][k] array.
__device__ __forceinline__ void load_a(uint32_t (&f)[4], const __half *base, int ld, int m0, int k0,
                                       int lane) {
  ldmatrix_x4(f, smem_u32(base + (m0 + (lane & 15)) * ld + k0 + (lane >> 4) * 8));
}

// A tile 16x16 where A[m][k] = X[k][m] and X is row-major [k][m].
__device__ __forceinline__ void load_a_trans(uint32_t (&f)[4], const __half *x, int ld, int m0,
                                             int k0, int lane) {
  const int j = lane >> 3;
  ldmatrix_x4_trans(f, smem_u32(x + (k0 + (lane & 7) + 8 * (j >> 1)) * ld + m0 + 8 * (j & 1)));
}

// B fragments of two n8 tiles (n0..n0+15, k0..k0+15) from Y row-major [n][k].
__device__ __forceinline__ void load_b_nk(uint32_t (&b)[4], const __half *y, int ld, int n0, int k0,
                                          int lane) {
  const int j = lane >> 3;
  ldmatrix_x4(b, smem_u32(y + (n0 + (lane & 7) + 8 * (j >> 1)) * ld + k0 + 8 * (j & 1)));
}

// B fragments of two n8 tiles (k0..k0+15, n0..n0+15) from Z row-major [k][n].
__device__ __forceinline__ void load_b_kn(uint32_t (&b)[4], const __half *z, int ld, int k0, int n0,
                                          int lane) {
  const int j = lane >> 3;
  ldmatrix_x4_trans(b, smem_u32(z + (k0 + (lane & 7) + 8 * (j & 1)) * ld + n0 + 8 * (j >> 1)));
}

__device__ __forceinline__ void mma2(float (&c0)[4], float (&c1)[4], const uint32_t (&a)[4],
                                     const uint32_t (&b)[4]) {
  mma_f16_16816(c0, a, b[0], b[1]);
  mma_f16_16816(c1, a, b[2], b[3]);
}

template <int N>
__device__ __forceinline__ void zero(float (&acc)[N][4]) {
#pragma unroll
  for (int i = 0; i < N; ++i)
    acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
}

// cp.async of 16 (or 4) bytes global -> shared; `bytes_valid` 0 writes zeros
// without reading.
__device__ __forceinline__ void cp_async16(void *dst, const void *src, uint32_t bytes_valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(bytes_valid)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src, uint32_t bytes_valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(bytes_valid)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// Grid (valueHeads, batch), kThreads threads, Smem::total bytes.
__global__ void __launch_bounds__(kThreads, 1) chunked(const delta::Args a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __half *Ks = reinterpret_cast<__half *>(smem + Smem::Ks);
  __half *Kg = reinterpret_cast<__half *>(smem + Smem::Kg);
  __half *Qs = reinterpret_cast<__half *>(smem + Smem::Qs);
  __half *Rk = reinterpret_cast<__half *>(smem + Smem::Rk);
  __half *Rv = reinterpret_cast<__half *>(smem + Smem::Rv);
  __half *Wm = reinterpret_cast<__half *>(smem + Smem::Wm);
  __half *Um = reinterpret_cast<__half *>(smem + Smem::Um);
  __half *Vp = reinterpret_cast<__half *>(smem + Smem::Vp);
  __half *Sm = reinterpret_cast<__half *>(smem + Smem::Sm);
  __half *Pm = reinterpret_cast<__half *>(smem + Smem::Pm);
  __half *Am = reinterpret_cast<__half *>(smem + Smem::Am);
  __half *Td = reinterpret_cast<__half *>(smem + Smem::Td);
  float *Ad = reinterpret_cast<float *>(smem + Smem::Ad);
  float *g = reinterpret_cast<float *>(smem + Smem::vec);  // cumulative log-decay
  float *bet = g + C;                                       // beta
  float *glast = bet + C;                                   // G of the chunk's last token

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const uint32_t vh = blockIdx.x, seq = blockIdx.y;
  const uint32_t kh = vh / a.group;
  const size_t key_width = size_t(a.key_heads) * DK, value_width = size_t(a.value_heads) * DV;
  float *S = a.state + (size_t(seq) * a.value_heads + vh) * DK * DV;
  const int fr = lane >> 2, fc = (lane & 3) * 2;  // accumulator fragment row / column

  // State fragments: key rows 16*warp.., all value columns.
  float sf[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int r = 16 * warp + fr, c = nt * 8 + fc;
    const float2 lo = *reinterpret_cast<const float2 *>(S + r * DV + c);
    const float2 hi = *reinterpret_cast<const float2 *>(S + (r + 8) * DV + c);
    sf[nt][0] = lo.x;
    sf[nt][1] = lo.y;
    sf[nt][2] = hi.x;
    sf[nt][3] = hi.y;
    *reinterpret_cast<uint32_t *>(Sm + r * kLd128 + c) = pack_half2(lo.x, lo.y);
    *reinterpret_cast<uint32_t *>(Sm + (r + 8) * kLd128 + c) = pack_half2(hi.x, hi.y);
  }

  const uint32_t n_chunks = (a.tokens + C - 1) / C;
  const int m0 = 16 * (warp & 3);  // this warp's token rows in 64-row products
  float *rawK = reinterpret_cast<float *>(smem + Smem::rawK);
  float *rawQ = reinterpret_cast<float *>(smem + Smem::rawQ);
  __half *rawV = reinterpret_cast<__half *>(smem + Smem::rawV);
  float *gates = reinterpret_cast<float *>(smem + Smem::gates);  // decay[64], beta[64]

  // Stages a chunk's raw rows (zeros past the last token) with cp.async.
  auto stage = [&](uint32_t chunk) {
    const uint32_t t0 = chunk * C;
    const int valid = int(min(uint32_t(C), a.tokens - t0));
    const size_t tok0 = size_t(seq) * a.tokens + t0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = tid + i * kThreads, t = idx >> 5, c = (idx & 31) * 4;
      const bool in = t < valid;
      const size_t row = (tok0 + (in ? t : 0)) * key_width + kh * DK + c;
      cp_async16(rawK + t * DK + c, a.k + row, in ? 16u : 0u);
      cp_async16(rawQ + t * DK + c, a.q + row, in ? 16u : 0u);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = tid + i * kThreads, t = idx >> 4, c = (idx & 15) * 8;
      const bool in = t < valid;
      cp_async16(rawV + t * DV + c, a.v + (tok0 + (in ? t : 0)) * value_width + vh * DV + c,
                 in ? 16u : 0u);
    }
    if (tid < 2 * C) {
      const int t = tid & (C - 1);
      const bool in = t < valid;
      const float *src = (tid < C ? a.decay : a.beta) + (tok0 + (in ? t : 0)) * a.value_heads + vh;
      cp_async4(gates + tid, src, in ? 4u : 0u);
    }
    cp_async_commit();
  };
  stage(0);

  for (uint32_t chunk = 0; chunk < n_chunks; ++chunk) {
    const uint32_t t0 = chunk * C;
    const int valid = int(min(uint32_t(C), a.tokens - t0));
    const size_t tok0 = size_t(seq) * a.tokens + t0;

    // 1. The chunk's raw rows were staged during the previous chunk (or
    //    before the loop): read them into registers.
    cp_async_wait_all();
    __syncthreads();
    float4 kr[8], qr[8];
    uint4 vr[4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = tid + i * kThreads, t = idx >> 5, c = (idx & 31) * 4;
      kr[i] = *reinterpret_cast<const float4 *>(rawK + t * DK + c);
      qr[i] = *reinterpret_cast<const float4 *>(rawQ + t * DK + c);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = tid + i * kThreads, t = idx >> 4, c = (idx & 15) * 8;
      vr[i] = *reinterpret_cast<const uint4 *>(rawV + t * DV + c);
    }
    // Gates: g = inclusive cumsum of log(decay), beta; pad tokens decay 1, beta 0.
    if (warp == 0) {
      float la[2], b[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int t = 2 * lane + i;
        const bool in = t < valid;
        la[i] = in ? logf(gates[t]) : 0.f;
        b[i] = in ? gates[C + t] : 0.f;
      }
      const float pair = la[0] + la[1];
      float incl = pair;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off)
          incl += y;
      }
      const float excl = incl - pair;
      g[2 * lane] = excl + la[0];
      g[2 * lane + 1] = incl;
      bet[2 * lane] = b[0];
      bet[2 * lane + 1] = b[1];
      if (lane == 31)
        *glast = incl;
    }
    __syncthreads();
    const float gl = *glast;

    // 2. Operands: K, K e^{G_C - G}, K beta e^{G}, Q (fp16), V beta.
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = tid + i * kThreads, t = idx >> 5, c = (idx & 31) * 4;
      const float4 kv = kr[i], qv = qr[i];
      const float sd = bet[t] * expf(g[t]), sg = expf(gl - g[t]);
      uint2 w;
      w.x = pack_half2(kv.x, kv.y);
      w.y = pack_half2(kv.z, kv.w);
      *reinterpret_cast<uint2 *>(Ks + t * kLd128 + c) = w;
      w.x = pack_half2(kv.x * sg, kv.y * sg);
      w.y = pack_half2(kv.z * sg, kv.w * sg);
      *reinterpret_cast<uint2 *>(Kg + t * kLd128 + c) = w;
      w.x = pack_half2(kv.x * sd, kv.y * sd);
      w.y = pack_half2(kv.z * sd, kv.w * sd);
      *reinterpret_cast<uint2 *>(Rk + t * kLd128 + c) = w;
      w.x = pack_half2(qv.x, qv.y);
      w.y = pack_half2(qv.z, qv.w);
      *reinterpret_cast<uint2 *>(Qs + t * kLd128 + c) = w;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = tid + i * kThreads, t = idx >> 4, c = (idx & 15) * 8;
      const __half2 b2 = __float2half2_rn(bet[t]);
      uint4 raw = vr[i];
      __half2 *h = reinterpret_cast<__half2 *>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        h[j] = __hmul2(h[j], b2);
      *reinterpret_cast<uint4 *>(Rv + t * kLd128 + c) = raw;
    }
    __syncthreads();

    // 3. A = beta_t (K K^T) e^{G_t - G_s} (s < t);  P = (Q K^T) e^{G_t - G_s} (s <= t).
    {
      const int n0 = 32 * (warp >> 2);
      float kk[4][4], qk[4][4];
      zero(kk);
      zero(qk);
#pragma unroll
      for (int ks = 0; ks < DK / 16; ++ks) {
        uint32_t fk[4], fq[4];
        load_a(fk, Ks, kLd128, m0, ks * 16, lane);
        load_a(fq, Qs, kLd128, m0, ks * 16, lane);
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          uint32_t b[4];
          load_b_nk(b, Ks, kLd128, n0 + 16 * p, ks * 16, lane);
          mma2(kk[2 * p], kk[2 * p + 1], fk, b);
          mma2(qk[2 * p], qk[2 * p + 1], fq, b);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = m0 + fr + (e >> 1) * 8, c = n0 + nt * 8 + fc + (e & 1);
          const float dec = c <= r ? expf(g[r] - g[c]) : 0.f;
          const float av = c < r ? bet[r] * kk[nt][e] * dec : 0.f;
          Am[r * kLd64 + c] = __float2half_rn(av);
          if ((r >> 4) == (c >> 4))
            Ad[((r >> 4) * 16 + (r & 15)) * kLdD + (c & 15)] = av;
          Pm[r * kLd64 + c] = __float2half_rn(qk[nt][e] * dec);
        }
    }
    __syncthreads();

    // 4. Diagonal blocks: T_ii = (I + A_ii)^-1 by forward substitution in fp32
    //    (warp i, lane = column).
    if (warp < 4 && lane < 16) {
      const float *ab = Ad + warp * 16 * kLdD;
      float col[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < r; ++j)
          acc = fmaf(ab[r * kLdD + j], col[j], acc);
        col[r] = r == lane ? 1.f : (r > lane ? -acc : 0.f);
      }
#pragma unroll
      for (int r = 0; r < 16; ++r)
        Td[(warp * 16 + r) * kLd16 + lane] = __float2half_rn(col[r]);
    }
    __syncthreads();

    // 5. Block rows of (I + A) [W | U] = [Rk | Rv]:
    //      X_i = T_ii (RHS_i - sum_{k<i} A_ik X_k)
    //    warp w solves columns 32w..32w+31 of [W | U] (W for w < 4).
    {
      const __half *rhs = warp < 4 ? Rk : Rv;
      __half *sol = warp < 4 ? Wm : Um;
      const int nc = 32 * (warp & 3);
#pragma unroll 1
      for (int i = 0; i < 4; ++i) {
        float acc[4][4];
        zero(acc);
        for (int kb = 0; kb < i; ++kb) {
          uint32_t fa[4];
          load_a(fa, Am, kLd64, 16 * i, 16 * kb, lane);
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            uint32_t b[4];
            load_b_kn(b, sol, kLd128, 16 * kb, nc + 16 * p, lane);
            mma2(acc[2 * p], acc[2 * p + 1], fa, b);
          }
        }
        // Residual R = RHS_i - acc, moved from accumulator layout (row =
        // token) to B-operand layout (k = token) with movmatrix.
        uint32_t rb[4][2];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const int r = 16 * i + fr, c = nc + nt * 8 + fc;
          const __half2 lo = *reinterpret_cast<const __half2 *>(rhs + r * kLd128 + c);
          const __half2 hi = *reinterpret_cast<const __half2 *>(rhs + (r + 8) * kLd128 + c);
          rb[nt][0] = movmatrix_trans(pack_half2(__low2float(lo) - acc[nt][0], __high2float(lo) - acc[nt][1]));
          rb[nt][1] = movmatrix_trans(pack_half2(__low2float(hi) - acc[nt][2], __high2float(hi) - acc[nt][3]));
        }
        uint32_t ft[4];
        load_a(ft, Td, kLd16, 16 * i, 0, lane);
        float x[4][4];
        zero(x);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
          mma_f16_16816(x[nt], ft, rb[nt][0], rb[nt][1]);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const int r = 16 * i + fr, c = nc + nt * 8 + fc;
          *reinterpret_cast<uint32_t *>(sol + r * kLd128 + c) = pack_half2(x[nt][0], x[nt][1]);
          *reinterpret_cast<uint32_t *>(sol + (r + 8) * kLd128 + c) = pack_half2(x[nt][2], x[nt][3]);
        }
        __syncthreads();
      }
    }

    // 6. V' = U - W S;  Y = e^{G_t} (Q S).
    const int n0 = 64 * (warp >> 2);
    float y[8][4];
    {
      float ws[8][4];
      zero(ws);
      zero(y);
#pragma unroll
      for (int ks = 0; ks < DK / 16; ++ks) {
        uint32_t fw[4], fq[4];
        load_a(fw, Wm, kLd128, m0, ks * 16, lane);
        load_a(fq, Qs, kLd128, m0, ks * 16, lane);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          uint32_t b[4];
          load_b_kn(b, Sm, kLd128, ks * 16, n0 + 16 * p, lane);
          mma2(ws[2 * p], ws[2 * p + 1], fw, b);
          mma2(y[2 * p], y[2 * p + 1], fq, b);
        }
      }
      const float e0 = expf(g[m0 + fr]), e1 = expf(g[m0 + fr + 8]);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int r = m0 + fr, c = n0 + nt * 8 + fc;
        const __half2 lo = *reinterpret_cast<const __half2 *>(Um + r * kLd128 + c);
        const __half2 hi = *reinterpret_cast<const __half2 *>(Um + (r + 8) * kLd128 + c);
        *reinterpret_cast<uint32_t *>(Vp + r * kLd128 + c) =
            pack_half2(__low2float(lo) - ws[nt][0], __high2float(lo) - ws[nt][1]);
        *reinterpret_cast<uint32_t *>(Vp + (r + 8) * kLd128 + c) =
            pack_half2(__low2float(hi) - ws[nt][2], __high2float(hi) - ws[nt][3]);
        y[nt][0] *= e0;
        y[nt][1] *= e0;
        y[nt][2] *= e1;
        y[nt][3] *= e1;
      }
    }
    __syncthreads();

    // The next chunk's raw rows into the buffers this chunk no longer reads.
    if (chunk + 1 < n_chunks)
      stage(chunk + 1);

    // 7. Y += P V';  write the chunk's outputs.
#pragma unroll
    for (int ks = 0; ks < C / 16; ++ks) {
      uint32_t fp[4];
      load_a(fp, Pm, kLd64, m0, ks * 16, lane);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        uint32_t b[4];
        load_b_kn(b, Vp, kLd128, ks * 16, n0 + 16 * p, lane);
        mma2(y[2 * p], y[2 * p + 1], fp, b);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int r = m0 + fr, c = n0 + nt * 8 + fc;
      if (r < valid)
        *reinterpret_cast<uint32_t *>(a.out + (tok0 + r) * value_width + vh * DV + c) =
            pack_half2(y[nt][0], y[nt][1]);
      if (r + 8 < valid)
        *reinterpret_cast<uint32_t *>(a.out + (tok0 + r + 8) * value_width + vh * DV + c) =
            pack_half2(y[nt][2], y[nt][3]);
    }

    // 8. S <- e^{G_C} S + (K e^{G_C - G})^T V'  (this warp's 16 key rows).
    {
      const float el = expf(gl);
#pragma unroll
      for (int nt = 0; nt < 16; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          sf[nt][e] *= el;
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks) {
        uint32_t fk[4];
        load_a_trans(fk, Kg, kLd128, 16 * warp, ks * 16, lane);
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          uint32_t b[4];
          load_b_kn(b, Vp, kLd128, ks * 16, 16 * p, lane);
          mma2(sf[2 * p], sf[2 * p + 1], fk, b);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        const int r = 16 * warp + fr, c = nt * 8 + fc;
        *reinterpret_cast<uint32_t *>(Sm + r * kLd128 + c) = pack_half2(sf[nt][0], sf[nt][1]);
        *reinterpret_cast<uint32_t *>(Sm + (r + 8) * kLd128 + c) = pack_half2(sf[nt][2], sf[nt][3]);
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int r = 16 * warp + fr, c = nt * 8 + fc;
    *reinterpret_cast<float2 *>(S + r * DV + c) = make_float2(sf[nt][0], sf[nt][1]);
    *reinterpret_cast<float2 *>(S + (r + 8) * DV + c) = make_float2(sf[nt][2], sf[nt][3]);
  }
}

}  // namespace delta_chunk
}  // namespace llmi
