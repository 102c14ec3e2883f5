// Causal GQA flash-attention prefill on CTA pairs (tcgen05 cta_group::2),
// head_dim 256.  Same contract and numerics as gqa_prefill_tcgen05
// (gqaFlashAttention, FlashAttention.metal:1-83): query token t sees keys
// [0, past + t], fp32 online softmax, fp32 accumulation, fp16 output.
//
// A cluster of two CTAs owns 256 query rows of one (sequence, kv head): CTA
// r holds rows 128r..128r+127 (the G query heads of the group stacked over
// 128/G tokens), its own Q (64 KiB in shared memory), its S/P buffers and its
// 128 rows of O in its own tensor memory.  One thread of the even CTA issues
// M=256 MMAs for both:
//   S = Q K^T   M256 N128 K256 (SS): each CTA holds 64 of the tile's 128 keys;
//   O += P V    M256 N256 K128 (TS): each CTA holds 128 of the 256 value dims.
// So each CTA stages half of every K and V tile, and the same shared memory
// holds three K tiles and two V tiles of lookahead.
//
// The MMA-issuing thread waits twice per 128-key tile: once for the K tile
// (both CTAs' boxes on one barrier) and once for P and V together (both
// CTAs' V boxes and all 16 softmax warps on one barrier).  An mbarrier wait
// in that thread idles the tensor pipe for about 100 cycles once commits are
// in flight, so waits per box (nine per tile) ran at half the MMA rate.
// Slots are released per tile by multicast commits, which cost nothing.
//
// Every mbarrier wait is bounded (abort flag per CTA).  The only unbounded
// synchronisation is the cluster barrier at start and end and the pair's TMEM
// allocation, which both CTAs reach on every path.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "gqa_prefill_tc.cuh"
#include "tcgen05.cuh"

namespace llmi {
namespace prefill_tc2 {

constexpr int kD = 256;
constexpr int kRows = 128;               // query rows per CTA
constexpr int kKeys = 128;               // keys per tile (the S MMA's N)
constexpr int kHalfKeys = kKeys / 2;     // keys of a tile staged by each CTA
constexpr int kHalfDims = kD / 2;        // value dims staged by each CTA
constexpr int kSoftmaxWarps = 8;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr int kKBox = kHalfKeys * 64 * 2;        // 8 KiB: 64 keys x 64 dims
constexpr int kKTile = kKBox * (kD / 64);        // 32 KiB: this CTA's keys, all dims
constexpr int kVBox = kKeys * 64 * 2;            // 16 KiB: 128 keys x 64 dims
constexpr int kVTile = kVBox * (kHalfDims / 64); // 32 KiB: all keys, this CTA's dims
constexpr int kKTiles = 3;                       // K ring (tiles)
constexpr int kVTiles = 2;                       // V ring (tiles), one per P buffer
constexpr int kSBuffers = 2;                     // S/P buffers in tensor memory
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0, kColS = 256;
constexpr float kRescaleThreshold = 8.0f;
static_assert(kVTiles == kSBuffers, "a V slot is released by the P.V commit of its buffer");

struct Smem {
  static constexpr int q = 0;                          // 4 boxes [128 rows][64 dims]
  static constexpr int k = q + kRows * kD * 2;         // [kKTiles][4 dim boxes][64 keys][64 dims]
  static constexpr int v = k + kKTiles * kKTile;       // [kVTiles][2 dim boxes][128 keys][64 dims]
  static constexpr int bars = v + kVTiles * kVTile;
  static constexpr int row_max = bars + 256;           // [2 parities][2 halves][128 rows] fp32
  static constexpr int total = row_max + 4 * kRows * 4;
  static constexpr int alloc = total;  // the dynamic shared memory starts 1024-byte aligned
};
static_assert(Smem::alloc <= 232448, "shared memory budget of one sm_100 CTA");
static_assert((1 + 2 * kKTiles + 3 * kSBuffers + 2 + 4) * 8 + 8 <= 256, "barrier area");

using Args = prefill_tc::Args;

// map_q: q [batch][tokens][Hq][D], box 64 dims x G heads x 128/G tokens;
// map_k: cache [batch][rows][Hkv][D], box 64 dims x 1 head x 64 keys;
// map_v: same cache layout, box 64 dims x 1 head x 128 keys; all 128B-swizzled.
// Grid (2 * pairs, kv heads, batch), clusters of (2, 1, 1).  a.tiles_per_head
// counts CTAs (query tiles of 128 rows), even.
__global__ void __launch_bounds__(kThreads, 1)
    gqa_prefill_pair(const __grid_constant__ CUtensorMap map_q,
                     const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const Args a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Smem::bars);
  uint64_t *q_full = bars;                    // even CTA: both Q halves landed (2 arrivals)
  uint64_t *k_full = q_full + 1;              // even CTA: [kKTiles] both K halves landed
  uint64_t *k_free = k_full + kKTiles;        // each CTA: [kKTiles] S MMAs done with the slot
  uint64_t *pv_ready = k_free + kKTiles;      // even CTA: [kSBuffers] V halves + all P rows
  uint64_t *s_full = pv_ready + kSBuffers;    // each CTA: [kSBuffers]
  uint64_t *o_done = s_full + kSBuffers;      // each CTA: [kSBuffers] P.V of the buffer done
  uint64_t *o_final = o_done + kSBuffers;
  uint64_t *drain = o_final + 1;
  uint64_t *pair_bar = drain + 1;             // [4] softmax warp pairs (local)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pair_bar + 4);
  volatile uint32_t *abort = reinterpret_cast<volatile uint32_t *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();  // 0: even CTA (issues the MMAs), 1: odd
  // Heaviest (latest-token) pairs first.
  const uint32_t pair = a.tiles_per_head / 2 - 1 - blockIdx.x / 2;
  const uint32_t kvh = blockIdx.y, seq = blockIdx.z;
  const uint32_t pair_t0 = pair * 2 * a.tok_per_tile;
  const uint32_t t0 = pair_t0 + rank * a.tok_per_tile;  // this CTA's first token
  const uint32_t pair_last = min(pair_t0 + 2 * a.tok_per_tile, a.tokens) - 1;
  const uint32_t n_tiles = (a.past + pair_last + 1 + kKeys - 1) / kKeys;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 2);
    for (int s = 0; s < kKTiles; ++s) {
      mbar_init(&k_full[s], 2);
      mbar_init(&k_free[s], 1);
    }
    for (int s = 0; s < kSBuffers; ++s) {
      mbar_init(&pv_ready[s], 2 + 2 * kSoftmaxWarps);
      mbar_init(&s_full[s], 1);
      mbar_init(&o_done[s], 1);
    }
    mbar_init(o_final, 1);
    mbar_init(drain, 1);
    for (int i = 0; i < 4; ++i)
      mbar_init(&pair_bar[i], 64);
    // 128B-swizzled tiles need 1024-byte aligned shared addresses; a
    // misaligned window fails loudly (every role skips its work).
    *abort = (smem_u32(smem) & 1023u) ? 1u : 0u;
    if (*abort)
      raise_error(kErrBadLaunch);
    fence_barrier_init();
  }
  if (warp == kMmaWarp)
    tmem_alloc_pair(tmem_slot, kTmemCols);
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers are initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool run = *abort == 0u;

  if (warp == kProducerWarp) {
    // ---------------- TMA producer (each CTA: its Q, its halves of K and V) ----------------
    if (lane == 0 && run) {
      prefetch_map(&map_q);
      prefetch_map(&map_k);
      prefetch_map(&map_v);
      const uint32_t q_full_even = cluster_addr(smem_u32(q_full), 0);
      mbar_arrive_expect_tx_cluster(q_full_even, kRows * kD * 2);
      for (int b = 0; b < kD / 64; ++b)
        tma_load_4d_pair(smem + Smem::q + b * (kRows * 64 * 2), &map_q, b * 64,
                         int(kvh * a.group), int(t0), int(seq), q_full_even);
      auto load_k = [&](uint32_t j) -> bool {
        const uint32_t s = j % kKTiles;
        if (j >= kKTiles && !wait_or_abort_cluster(&k_free[s], ((j / kKTiles) - 1) & 1, abort))
          return false;
        const uint32_t full = cluster_addr(smem_u32(&k_full[s]), 0);
        mbar_arrive_expect_tx_cluster(full, kKTile);
        for (int b = 0; b < kD / 64; ++b)
          tma_load_4d_pair(smem + Smem::k + s * kKTile + b * kKBox, &map_k, b * 64, int(kvh),
                           int(j * kKeys + rank * kHalfKeys), int(seq), full);
        return true;
      };
      auto load_v = [&](uint32_t j) -> bool {
        const uint32_t s = j % kVTiles;
        // The slot's previous tile j - kVTiles was read by the P.V MMAs of
        // buffer s, whose completion o_done[s] announces.
        if (j >= kVTiles && !wait_or_abort_cluster(&o_done[s], ((j / kVTiles) - 1) & 1, abort))
          return false;
        const uint32_t ready = cluster_addr(smem_u32(&pv_ready[s]), 0);
        mbar_arrive_expect_tx_cluster(ready, kVTile);
        for (int d = 0; d < kHalfDims / 64; ++d)
          tma_load_4d_pair(smem + Smem::v + s * kVTile + d * kVBox, &map_v,
                           int(rank * kHalfDims + d * 64), int(kvh), int(j * kKeys), int(seq),
                           ready);
        return true;
      };
      // Issue order K_0, K_1, then per tile j: K_{j+2}, V_j.  Each wait is on
      // a release that precedes, in the MMA order, the one the next wait
      // needs, so the producer never blocks on a later event first.
      bool fine = load_k(0) && (n_tiles < 2 || load_k(1));
      for (uint32_t j = 0; fine && j < n_tiles; ++j)
        fine = (j + 2 >= n_tiles || load_k(j + 2)) && load_v(j);
      // This CTA's copies count on the even CTA's barriers: before the CTA
      // may exit, wait until the last MMA (which read every copy) has
      // retired.  The MMA thread commits o_final on every path.
      wait_or_abort_cluster(o_final, 0, abort);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer (even CTA only) ----------------
    if (lane == 0 && rank == 0 && run) {
      constexpr uint32_t idesc_s = idesc_f16(2 * kRows, kKeys, false);
      constexpr uint32_t idesc_o = idesc_f16(2 * kRows, kD, true);
      // Descriptors are built once; per MMA only the start address moves.
      const uint64_t q_desc = smem_desc(smem_u32(smem + Smem::q), 16, 1024);
      const uint64_t k_desc = smem_desc(smem_u32(smem + Smem::k), 16, 1024);
      const uint64_t v_desc = smem_desc(smem_u32(smem + Smem::v), kVBox, 1024);
      bool ok = wait_or_abort_cluster(q_full, 0, abort);
      tc_fence_after();
      auto issue_pv = [&](uint32_t i) -> bool {
        const int sb = i % kSBuffers;
        if (!wait_or_abort_cluster(&pv_ready[sb], (i / kSBuffers) & 1, abort))
          return false;
        tc_fence_after();
        const uint32_t p_tmem = tmem + kColS + sb * kKeys;  // P (fp16 pairs) over the S buffer
        const uint64_t v_tile = desc_add(v_desc, sb * kVTile);
#pragma unroll
        for (int ks = 0; ks < kKeys / 16; ++ks)
          mma_ts_pair(tmem + kColO, p_tmem + ks * 8, desc_add(v_tile, ks * 2048), idesc_o,
                      (i > 0 || ks > 0) ? 1u : 0u);
        mma_commit_pair(&o_done[sb]);
        return true;
      };
      for (uint32_t j = 0; ok && j < n_tiles; ++j) {
        const int sb = j % kSBuffers;
        const uint32_t s = j % kKTiles;
        if (!wait_or_abort_cluster(&k_full[s], (j / kKTiles) & 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t k_tile = desc_add(k_desc, s * kKTile);
#pragma unroll
        for (int b = 0; b < kD / 64; ++b) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ss_pair(tmem + kColS + sb * kKeys, desc_add(q_desc, b * (kRows * 64 * 2) + kk * 32),
                        desc_add(k_tile, b * kKBox + kk * 32), idesc_s, (b > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit_pair(&k_free[s]);
        mma_commit_pair(&s_full[sb]);
        if (j >= 1 && !issue_pv(j - 1))
          ok = false;
      }
      if (ok)
        ok = issue_pv(n_tiles - 1);
      mma_commit_pair(o_final);
      // Every MMA issued so far has retired once `drain` completes (in both
      // CTAs' tensor memory).
      mma_commit_pair(drain);
      mbar_wait(drain, 0);
    }
    __syncwarp();
  } else if (run) {
    // ---------------- softmax warps 0-7 (each CTA, its 128 rows) ----------------
    const int quarter = warp & 3, half = warp >> 2;
    const uint32_t row = uint32_t(quarter) * 32u + uint32_t(lane);  // TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t(quarter) * 32u) << 16);
    const uint32_t token = t0 + row / a.group;
    const uint32_t head = kvh * a.group + row % a.group;
    const bool valid = token < a.tokens;
    const uint32_t limit = a.past + min(token, a.tokens - 1);  // last visible key
    const uint32_t first_masked_tile = (a.past + t0) / kKeys;   // tiles before are fully visible
    constexpr int kHalf = kKeys / 2;                            // keys per warp of the pair
    uint64_t *my_pair = &pair_bar[quarter];
    uint32_t pair_phase = 0;
    float *row_max = reinterpret_cast<float *>(smem + Smem::row_max);
    const uint32_t pv_ready_even0 = cluster_addr(smem_u32(&pv_ready[0]), 0);
    const uint32_t pv_ready_even1 = cluster_addr(smem_u32(&pv_ready[1]), 0);

    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (uint32_t j = 0; j < n_tiles; ++j) {
      const int s = j % kSBuffers;
      if (!__all_sync(0xffffffffu, wait_or_abort_cluster(&s_full[s], (j / kSBuffers) & 1, abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t raw[2][32];
      const uint32_t s_cols = lane_base + kColS + s * kKeys + half * kHalf;
      tmem_ld32(s_cols, raw[0]);
      tmem_ld32(s_cols + 32, raw[1]);
      tmem_wait_ld();
      float x[kHalf];
#pragma unroll
      for (int c = 0; c < kHalf; ++c)
        x[c] = __uint_as_float(raw[c >> 5][c & 31]);
      if (j >= first_masked_tile) {
        const int lim = int(limit) - int(j * kKeys + half * kHalf);
#pragma unroll
        for (int c = 0; c < kHalf; ++c)
          if (c > lim)
            x[c] = -INFINITY;
      }
      // Row maximum with three-input max (eight independent chains).
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        mx[i] = x[i];
#pragma unroll
      for (int c = 8; c < kHalf; c += 2)
        mx[(c >> 1) & 7] = max3f(mx[(c >> 1) & 7], x[c], x[c + 1]);
      const float pmax = max3f(max3f(mx[0], mx[1], mx[2]), max3f(mx[3], mx[4], mx[5]),
                               fmaxf(mx[6], mx[7]));
      float *slot = row_max + (j & 1) * 2 * kRows;
      slot[half * kRows + row] = pmax;
      if (!prefill_tc::pair_sync(my_pair, (pair_phase++) & 1, abort)) {
        ok = false;
        break;
      }
      const float tmax = fmaxf(pmax, slot[(1 - half) * kRows + row]) * a.scale_log2;
      const bool need = tmax > m + kRescaleThreshold;
      if (__any_sync(0xffffffffu, need)) {
        const float next = need ? tmax : m;
        const float alpha = need ? fast_exp2(m - next) : 1.f;  // 0 when m = -inf
        if (j > 0) {
          // P.V of tile j-1 (buffer (j-1)%2) must have retired before O is
          // rescaled; P.V of tile j+1 cannot start before this tile's P.
          const int pb = (j - 1) % kSBuffers;
          if (!__all_sync(0xffffffffu,
                          wait_or_abort_cluster(&o_done[pb], ((j - 1) / kSBuffers) & 1, abort))) {
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
      // p = 2^(x * scale - m): the argument and the row sums in packed fp32
      // pairs (each lane rounds as fmaf / + would), the exponential on the
      // MUFU, the pack to fp16 pairs for the P.V MMA.
      uint32_t packed[kHalf / 2];
      float2 sums[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      const float2 neg_m = make_float2(-m, -m), scale = make_float2(a.scale_log2, a.scale_log2);
#pragma unroll
      for (int c = 0; c < kHalf; c += 2) {
        const float2 arg = fma2(make_float2(x[c], x[c + 1]), scale, neg_m);
        const float2 p = make_float2(fast_exp2(arg.x), fast_exp2(arg.y));
        sums[(c >> 1) & 1] = add2(sums[(c >> 1) & 1], p);
        packed[c >> 1] = pack_half2(p.x, p.y);
      }
      l += (sums[0].x + sums[1].x) + (sums[0].y + sums[1].y);
      tmem_st32(lane_base + kColS + s * kKeys + half * (kHalf / 2), packed);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0)
        mbar_arrive_cluster(s ? pv_ready_even1 : pv_ready_even0);
    }
    float *row_sum = row_max + (n_tiles & 1) * 2 * kRows;
    row_sum[half * kRows + row] = l;
    if (ok && prefill_tc::pair_sync(my_pair, pair_phase & 1, abort) &&
        __all_sync(0xffffffffu, wait_or_abort_cluster(o_final, 0, abort))) {
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

  // Neither CTA frees tensor memory while the other's rows may still be
  // written by the pair's MMAs or read by its softmax.
  tc_fence_before();
  cluster_sync();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

}  // namespace prefill_tc2
}  // namespace llmi
