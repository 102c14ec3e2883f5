// Causal GQA flash-attention prefill on 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), head_dim 256.  Same contract as
// gqaFlashAttention (FlashAttention.metal:1-83): query token t sees keys
// [0, past + t], fp32 online softmax, fp32 accumulation, fp16 output.
//
// Tiling.  One CTA owns 128 query rows of one (sequence, kv head): the G
// query heads of the group stacked over 128/G consecutive tokens
// (row r = token (r / G), head (r % G)), so each K/V tile is fetched once for
// the whole group.  Keys stream in tiles of 64.
//
// Q lives in TMEM.  Both MMAs read their A operand from TMEM, so only K and
// V cross shared memory: S_j = Q K_j^T as a TS MMA (M128 N64 K256) streams
// 64 B of K per clock, where an SS form would stream Q too (192 B/clk, more
// than shared memory feeds the tensor core).  This also frees the 64 KiB a
// shared-memory Q tile would take for deeper K/V rings.
//
// Roles (320 threads, one CTA per SM):
//   warps 0-7  softmax.  Warps w and w+4 share TMEM lanes 32*(w%4).. (query
//              rows).  At the start each writes its half of the rows' Q into
//              TMEM.  Per tile both read the row's 64 scores with tcgen05.ld
//              and apply the causal mask, so both derive the same row maximum
//              without exchanging it; after a pair barrier (both have read S)
//              warp w exponentiates keys [0,32) and warp w+4 keys [32,64) and
//              writes the probabilities as fp16 over the S buffer.  The row
//              sums are combined once, in the epilogue, where each half
//              normalises 128 of the 256 output columns.
//   warp 8     TMA producer: K tiles into a 4-slot ring and V tiles into a
//              3-slot ring, K one tile ahead.
//   warp 9     TMEM allocator; one elected thread issues the MMAs:
//                S_j = Q K_j^T     (TS: A = Q from TMEM, B = K K-major)
//                O  += P_j V_j     (TS: A = P from TMEM, B = V MN-major)
//              and commits them to mbarriers.
// TMEM columns: O [0,256), Q [256,384), S/P buffers [384,448) and [448,512).
//
// Rescaling O.  The running maximum used for the exponentials only moves
// when a row's tile maximum exceeds it by more than 8 (log2 units), so
// probabilities stay below 2^8; then that row waits for the P.V of the
// previous tile to retire and rescales its O row in TMEM.  This keeps the
// 256-column O accumulator out of the common path.
//
// Every wait is bounded; a wait that gives up raises the device error word
// and sets a CTA abort flag that makes every role leave its loop, drain its
// copies and MMAs (bounded), free TMEM and return.
#pragma once

#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "tcgen05.cuh"

namespace llmi {
namespace prefill_tc {

constexpr int kD = 256;
constexpr int kRows = 128;
constexpr int kKeys = 64;
constexpr int kSoftmaxWarps = 8;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr int kSoftmaxThreads = kSoftmaxWarps * 32;
// Every kPolyEvery-th exponential of a fully visible tile runs on the FMA
// pipe (exp2_fma) instead of MUFU; 0 disables it.
constexpr int kPolyEvery = 0;
constexpr int kKVBytes = kKeys * kD * 2;  // 32 KiB, 4 boxes of 8 KiB
// K and V have separate rings: K_j is released as soon as S_j retires, V_j
// after P_j V_j, so the K ring runs a tile ahead of V and the next S MMA
// does not wait behind the previous P.V.
constexpr int kKStages = 4;
constexpr int kVStages = 3;
constexpr int kSBuffers = 2;  // S/P buffers in TMEM
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0, kColQ = 256, kColS = 384;
constexpr float kRescaleThreshold = 8.0f;

struct Smem {
  // Offsets from the 1024-byte aligned base.
  static constexpr int k = 0;
  static constexpr int v = k + kKStages * kKVBytes;
  static constexpr int bars = v + kVStages * kKVBytes;
  static constexpr int row_sum = bars + 256;  // [2 halves][128 rows] fp32
  static constexpr int total = row_sum + 2 * kRows * 4;
  static constexpr int alloc = total + 1024;  // alignment slack
};
static_assert(Smem::alloc <= 232448, "shared memory budget of one sm_100 CTA");

struct Args {
  const __half *q;  // [batch][tokens][Hq][D]
  __half *out;      // [batch][tokens][Hq][D]
  uint32_t tokens, q_heads, kv_heads, group, past, tok_per_tile, tiles_per_head;
  float scale_log2;
};

// ---- the kernel --------------------------------------------------------------------

// Rendezvous of the two softmax warps that share a TMEM lane quarter: every
// thread arrives (count 64) and waits, bounded and abort-aware, so a partner
// that has left on a failed wait cannot strand the other.
__device__ __forceinline__ bool pair_sync(uint64_t *bar, unsigned parity,
                                          volatile uint32_t *abort) {
  tc_fence_before();
  mbar_arrive(bar);
  const bool ok = __all_sync(0xffffffffu, wait_or_abort(bar, parity, abort));
  tc_fence_after();
  return ok;
}

__global__ void __launch_bounds__(kThreads, 1)
    gqa_prefill_tcgen05(const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Smem::bars);
  uint64_t *q_ready = bars + 0;     // Q written to TMEM (softmax threads)
  uint64_t *bar_k = bars + 1;       // [kKStages] K tile landed
  uint64_t *k_empty = bars + 5;     // [kKStages] S MMA done with the K slot
  uint64_t *bar_v = bars + 9;       // [kVStages] V tile landed
  uint64_t *v_empty = bars + 12;    // [kVStages] P.V MMA done with the V slot
  uint64_t *s_full = bars + 15;     // [kSBuffers]
  uint64_t *p_ready = bars + 17;    // [kSBuffers]
  uint64_t *o_done = bars + 19;
  uint64_t *o_final = bars + 20;
  uint64_t *drain = bars + 21;
  uint64_t *pair_bar = bars + 22;   // [4] softmax warp pairs
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 26);
  volatile uint32_t *abort = reinterpret_cast<volatile uint32_t *>(bars + 27);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Heaviest (latest-token) tiles first.
  const uint32_t tile = a.tiles_per_head - 1 - blockIdx.x;
  const uint32_t kvh = blockIdx.y, seq = blockIdx.z;
  const uint32_t t0 = tile * a.tok_per_tile;
  const uint32_t t_last = min(t0 + a.tok_per_tile, a.tokens) - 1;
  const uint32_t n_tiles = (a.past + t_last + 1 + kKeys - 1) / kKeys;

  if (threadIdx.x == 0) {
    mbar_init(q_ready, kSoftmaxThreads);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&bar_k[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&bar_v[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < kSBuffers; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_ready[s], kSoftmaxThreads);
    }
    mbar_init(o_done, 1);
    mbar_init(o_final, 1);
    mbar_init(drain, 1);
    for (int i = 0; i < 4; ++i)
      mbar_init(&pair_bar[i], 64);
    *abort = 0u;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducerWarp) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_map(&map_k);
      prefetch_map(&map_v);
      // Issue order K_0, then per tile j: K_{j+1}, V_j (K runs a tile ahead).
      auto load_k = [&](uint32_t j) -> bool {
        const int s = j % kKStages;
        if (j >= kKStages && !wait_or_abort(&k_empty[s], ((j / kKStages) - 1) & 1, abort))
          return false;
        mbar_arrive_expect_tx(&bar_k[s], kKVBytes);
        for (int b = 0; b < 4; ++b)
          tma_load_4d(smem + Smem::k + s * kKVBytes + b * (kKVBytes / 4), &map_k, b * 64, int(kvh),
                      int(j * kKeys), int(seq), &bar_k[s]);
        return true;
      };
      auto load_v = [&](uint32_t j) -> bool {
        const int s = j % kVStages;
        if (j >= kVStages && !wait_or_abort(&v_empty[s], ((j / kVStages) - 1) & 1, abort))
          return false;
        mbar_arrive_expect_tx(&bar_v[s], kKVBytes);
        for (int b = 0; b < 4; ++b)
          tma_load_4d(smem + Smem::v + s * kKVBytes + b * (kKVBytes / 4), &map_v, b * 64, int(kvh),
                      int(j * kKeys), int(seq), &bar_v[s]);
        return true;
      };
      uint32_t k_issued = 0, v_issued = 0;
      if (n_tiles > 0 && load_k(0))
        k_issued = 1;
      for (uint32_t j = 0; k_issued > j && j < n_tiles; ++j) {
        if (j + 1 < n_tiles) {
          if (!load_k(j + 1))
            break;
          k_issued = j + 2;
        }
        if (!load_v(j))
          break;
        v_issued = j + 1;
      }
      // Let every issued copy land before shared memory can be released.
      for (uint32_t j = k_issued > kKStages ? k_issued - kKStages : 0; j < k_issued; ++j)
        mbar_wait(&bar_k[j % kKStages], (j / kKStages) & 1);
      for (uint32_t j = v_issued > kVStages ? v_issued - kVStages : 0; j < v_issued; ++j)
        mbar_wait(&bar_v[j % kVStages], (j / kVStages) & 1);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(kRows, kKeys, false);
      constexpr uint32_t idesc_o = idesc_f16(kRows, kD, true);
      const uint32_t k_base = smem_u32(smem + Smem::k);
      const uint32_t v_base = smem_u32(smem + Smem::v);
      bool ok = wait_or_abort(q_ready, 0, abort);
      tc_fence_after();
      auto issue_pv = [&](uint32_t i) -> bool {
        const int sb = i % kSBuffers, sv = i % kVStages;
        if (!wait_or_abort(&p_ready[sb], (i / kSBuffers) & 1, abort))
          return false;
        if (!wait_or_abort(&bar_v[sv], (i / kVStages) & 1, abort))
          return false;
        tc_fence_after();
        const uint32_t p_tmem = tmem + kColS + sb * kKeys;  // P over the S buffer
#pragma unroll
        for (int ks = 0; ks < kKeys / 16; ++ks) {
          const uint64_t b = smem_desc(v_base + sv * kKVBytes + ks * 2048, kKVBytes / 4, 1024);
          mma_ts(tmem + kColO, p_tmem + ks * 8, b, idesc_o, (i > 0 || ks > 0) ? 1u : 0u);
        }
        mma_commit(&v_empty[sv]);
        mma_commit(o_done);
        return true;
      };
      for (uint32_t j = 0; ok && j < n_tiles; ++j) {
        const int sk = j % kKStages, sb = j % kSBuffers;
        if (!wait_or_abort(&bar_k[sk], (j / kKStages) & 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kD / 16; ++ks) {
          const uint32_t box = ks >> 2, off = (ks & 3) * 32;
          const uint64_t kb = smem_desc(k_base + sk * kKVBytes + box * (kKVBytes / 4) + off, 16, 1024);
          mma_ts(tmem + kColS + sb * kKeys, tmem + kColQ + ks * 8, kb, idesc_s, ks > 0 ? 1u : 0u);
        }
        mma_commit(&k_empty[sk]);
        mma_commit(&s_full[sb]);
        if (j >= 1 && !issue_pv(j - 1))
          ok = false;
      }
      if (ok && n_tiles > 0)
        ok = issue_pv(n_tiles - 1);
      mma_commit(o_final);
      // Every MMA issued so far has retired once `drain` completes.
      mma_commit(drain);
      mbar_wait(drain, 0);
    }
    __syncwarp();
  } else {
    // ---------------- softmax warps 0-7 ----------------
    const int quarter = warp & 3, half = warp >> 2;
    const uint32_t row = uint32_t(quarter) * 32u + uint32_t(lane);  // TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t(quarter) * 32u) << 16);
    const uint32_t token = t0 + row / a.group;
    const uint32_t head = kvh * a.group + row % a.group;
    const bool valid = token < a.tokens;
    const uint32_t limit = a.past + min(token, a.tokens - 1);  // last visible key
    const uint32_t first_masked_tile = (a.past + t0) / kKeys;   // tiles before are fully visible
    constexpr int kHalf = kKeys / 2;
    uint64_t *my_pair = &pair_bar[quarter];
    uint32_t pair_phase = 0;

    // Q -> TMEM: this warp writes dims [128*half, 128*half + 128) of its row
    // (fp16 pairs, 64 columns); rows past the last token are zero.
    {
      const uint4 *src = reinterpret_cast<const uint4 *>(
          a.q + ((size_t(seq) * a.tokens + token) * a.q_heads + head) * kD + half * (kD / 2));
#pragma unroll
      for (int chunk = 0; chunk < 2; ++chunk) {
        uint32_t r[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint4 w = valid ? __ldg(src + chunk * 8 + i) : make_uint4(0u, 0u, 0u, 0u);
          r[4 * i + 0] = w.x;
          r[4 * i + 1] = w.y;
          r[4 * i + 2] = w.z;
          r[4 * i + 3] = w.w;
        }
        tmem_st32(lane_base + kColQ + half * 64 + chunk * 32, r);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(q_ready);
    }

    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (uint32_t j = 0; j < n_tiles; ++j) {
      const int s = j % kSBuffers;
      // tcgen05.ld/st are warp-collective: every decision below is warp-uniform.
      if (!__all_sync(0xffffffffu, wait_or_abort(&s_full[s], (j / kSBuffers) & 1, abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t raw[2][32];
      tmem_ld32(lane_base + kColS + s * kKeys, raw[0]);
      tmem_ld32(lane_base + kColS + s * kKeys + 32, raw[1]);
      tmem_wait_ld();
      // Raw scores; the 1/sqrt(D) * log2(e) scale is folded into the
      // exponent's FFMA below (it is positive, so the max commutes with it).
      float x[kKeys];
#pragma unroll
      for (int c = 0; c < kKeys; ++c)
        x[c] = __uint_as_float(raw[c >> 5][c & 31]);
      const bool masked_tile = j >= first_masked_tile;
      if (masked_tile) {
        const int lim = int(limit) - int(j * kKeys);
#pragma unroll
        for (int c = 0; c < kKeys; ++c)
          if (c > lim)
            x[c] = -INFINITY;
      }
      // Both warps of the pair have read S_j before either overwrites it with P.
      if (!pair_sync(my_pair, (pair_phase++) & 1, abort)) {
        ok = false;
        break;
      }
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        mx[i] = x[i];
#pragma unroll
      for (int c = 8; c < kKeys; ++c)
        mx[c & 7] = fmaxf(mx[c & 7], x[c]);
      const float tmax =
          fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * a.scale_log2;
      const bool need = tmax > m + kRescaleThreshold;
      if (__any_sync(0xffffffffu, need)) {
        const float next = need ? tmax : m;
        const float alpha = need ? fast_exp2(m - next) : 1.f;  // 0 when m = -inf
        if (j > 0) {
          // O holds P_0..P_{j-1} V: wait for the last of those MMAs, then
          // rescale this warp's half of the O row.
          if (!__all_sync(0xffffffffu, wait_or_abort(o_done, (j - 1) & 1, abort))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = half * (kD / 2); c < (half + 1) * (kD / 2); c += 32) {
            uint32_t o[32];
            tmem_ld32(lane_base + kColO + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i)
              o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(lane_base + kColO + c, o);
          }
        }
        l *= alpha;
        m = next;
      }
      // p = 2^(s*scale - m) for this warp's 32 keys.  With kPolyEvery > 0,
      // that share of the exponentials of fully visible tiles runs on the FMA
      // pipe (exp2_fma); tiles with masked (-inf) scores use ex2 throughout.
      uint32_t packed[kHalf / 2];
      float sums[4] = {0.f, 0.f, 0.f, 0.f};
      const float neg_m = -m, scale = a.scale_log2;
      // The half is chosen with a compile-time offset so x[] stays in registers.
      auto exponentiate = [&](auto offset) {
        constexpr int kOff = decltype(offset)::value;
#pragma unroll
        for (int c = 0; c < kHalf; c += 2) {
          const float a0 = fmaf(x[kOff + c], scale, neg_m);
          const float a1 = fmaf(x[kOff + c + 1], scale, neg_m);
          const bool poly =
              kPolyEvery > 0 && !masked_tile && ((c / 2) % kPolyEvery) == kPolyEvery - 1;
          const float p0 = fast_exp2(a0);
          const float p1 = poly ? exp2_fma(a1) : fast_exp2(a1);
          sums[(c >> 1) & 3] += p0 + p1;
          packed[c >> 1] = pack_half2(p0, p1);
        }
      };
      if (half == 0)
        exponentiate(std::integral_constant<int, 0>{});
      else
        exponentiate(std::integral_constant<int, kHalf>{});
      l += (sums[0] + sums[1]) + (sums[2] + sums[3]);
      // P as fp16 pairs over the S buffer: keys 32*half.. -> columns 16*half..
      tmem_st16(lane_base + kColS + s * kKeys + half * (kHalf / 2), packed);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_ready[s]);
    }
    // The row's normaliser is the sum of both halves.
    float *row_sum = reinterpret_cast<float *>(smem + Smem::row_sum);
    row_sum[half * kRows + row] = l;
    if (ok && pair_sync(my_pair, pair_phase & 1, abort) &&
        __all_sync(0xffffffffu, wait_or_abort(o_final, 0, abort))) {
      tc_fence_after();
      const float inv = 1.f / (l + row_sum[(1 - half) * kRows + row]);
      __half *orow = a.out + ((size_t(seq) * a.tokens + token) * a.q_heads + head) * kD;
#pragma unroll 1
      for (int c = half * (kD / 2); c < (half + 1) * (kD / 2); c += 32) {
        uint32_t o[32];
        tmem_ld32(lane_base + kColO + c, o);
        tmem_wait_ld();
        if (valid) {
          uint4 *dst = reinterpret_cast<uint4 *>(orow + c);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 w;
            w.x = pack_half2(__uint_as_float(o[8 * i + 0]) * inv, __uint_as_float(o[8 * i + 1]) * inv);
            w.y = pack_half2(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv);
            w.z = pack_half2(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv);
            w.w = pack_half2(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv);
            dst[i] = w;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace prefill_tc
}  // namespace llmi
