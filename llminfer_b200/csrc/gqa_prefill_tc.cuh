// Causal GQA flash-attention prefill on 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), head_dim 256.  Same contract as
// gqaFlashAttention (FlashAttention.metal:1-83): query token t sees keys
// [0, past + t], fp32 online softmax, fp32 accumulation, fp16 output.
//
// Tiling.  One CTA owns 128 query rows of one (sequence, kv head): the G
// query heads of the group stacked over 128/G consecutive tokens
// (row r = token (r / G), head (r % G)), so each K/V tile is fetched once for
// the whole group.  Keys stream in tiles of 128, so S = Q K^T runs as
// M128 N128 instructions: N = 64 instructions reach only ~70 % of the
// tensor pipe's rate on sm_100, N >= 128 the full rate.
//
// Operands.  Q (fp16, 64 KiB) sits in shared memory for the whole CTA, so
// S = Q K^T is an SS MMA; with N = 128 its 8 KiB of operands per
// instruction match what shared memory feeds the tensor core.  K streams
// through a ring of 16 KiB boxes (128 keys x 64 dims), V through a ring of
// 16 KiB groups (32 keys x 256 dims as four 64-dim boxes); each slot is
// released as soon as the MMAs reading it retire.  O += P V is a TS MMA
// (P from TMEM, V MN-major), M128 N256.
//
// Roles (320 threads, one CTA per SM):
//   warps 0-7  softmax.  Warps w and w+4 share TMEM lanes 32*(w%4).. (query
//              rows); per tile warp w+4h reads keys [64h, 64h+64) of its
//              rows, the pair exchanges row maxima through shared memory,
//              and each warp writes its 64 probabilities as fp16 pairs over
//              the S columns it read (after the exchange both have read).
//              The row sums are combined once, in the epilogue, where each
//              half normalises 128 of the 256 output columns.
//   warp 8     TMA producer: Q once, then K one tile ahead of V.
//   warp 9     TMEM allocator; one elected thread issues the MMAs and
//              commits them to mbarriers.
// TMEM columns: O [0,256), S/P buffers [256,384) and [384,512).
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
constexpr int kKeys = 128;            // keys per tile
constexpr int kSoftmaxWarps = 8;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr int kSoftmaxThreads = kSoftmaxWarps * 32;
constexpr int kBoxBytes = 16384;      // one K box (128 keys x 64 dims) or V group (32 keys x 256)
constexpr int kKBoxesPerTile = kD / 64;
constexpr int kVKeys = 32;            // keys per V group
constexpr int kVGroupsPerTile = kKeys / kVKeys;
constexpr int kKSlots = 5;
constexpr int kVSlots = 4;
constexpr int kSBuffers = 2;          // S/P buffers in TMEM
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0, kColS = 256;
constexpr float kRescaleThreshold = 8.0f;

struct Smem {
  // Offsets from the 1024-byte aligned base.
  static constexpr int q = 0;                              // 4 boxes [128 rows][64 dims]
  static constexpr int k = q + kRows * kD * 2;
  static constexpr int v = k + kKSlots * kBoxBytes;
  static constexpr int bars = v + kVSlots * kBoxBytes;
  static constexpr int row_max = bars + 256;               // [2 tiles][2 halves][128 rows] fp32
  static constexpr int row_sum = row_max + 4 * kRows * 4;  // [2 halves][128 rows] fp32
  static constexpr int total = row_sum + 2 * kRows * 4;
  static constexpr int alloc = total + 1024;  // alignment slack
};
static_assert(Smem::alloc <= 232448, "shared memory budget of one sm_100 CTA");

struct Args {
  __half *out;  // [batch][tokens][Hq][D]
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

// map_q: q [batch][tokens][Hq][D], box 64 dims x G heads x 128/G tokens;
// map_k: cache [batch][rows][Hkv][D], box 64 dims x 1 head x 128 keys;
// map_v: same cache layout, box 64 dims x 1 head x 32 keys; all 128B-swizzled.
__global__ void __launch_bounds__(kThreads, 1)
    gqa_prefill_tcgen05(const __grid_constant__ CUtensorMap map_q,
                        const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  // Rounded up to 1024 bytes by an offset from the shared array itself, so
  // the compiler keeps every access through `smem` a shared-memory one (a
  // round trip through an integer address would make them generic).
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Smem::bars);
  uint64_t *q_full = bars + 0;      // Q landed
  uint64_t *bar_k = bars + 1;       // [kKSlots] K box landed
  uint64_t *k_empty = bars + 6;     // [kKSlots] S MMAs done with the K slot
  uint64_t *bar_v = bars + 11;      // [kVSlots] V group landed
  uint64_t *v_empty = bars + 15;    // [kVSlots] P.V MMAs done with the V slot
  uint64_t *s_full = bars + 19;     // [kSBuffers]
  uint64_t *p_ready = bars + 21;    // [kSBuffers]
  uint64_t *o_done = bars + 23;
  uint64_t *o_final = bars + 24;
  uint64_t *drain = bars + 25;
  uint64_t *pair_bar = bars + 26;   // [4] softmax warp pairs
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 30);
  volatile uint32_t *abort = reinterpret_cast<volatile uint32_t *>(bars + 31);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Heaviest (latest-token) tiles first.
  const uint32_t tile = a.tiles_per_head - 1 - blockIdx.x;
  const uint32_t kvh = blockIdx.y, seq = blockIdx.z;
  const uint32_t t0 = tile * a.tok_per_tile;
  const uint32_t t_last = min(t0 + a.tok_per_tile, a.tokens) - 1;
  const uint32_t n_tiles = (a.past + t_last + 1 + kKeys - 1) / kKeys;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kKSlots; ++s) {
      mbar_init(&bar_k[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kVSlots; ++s) {
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
  if (warp == kMmaWarp)
    tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducerWarp) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_map(&map_q);
      prefetch_map(&map_k);
      prefetch_map(&map_v);
      mbar_arrive_expect_tx(q_full, kRows * kD * 2);
      for (int b = 0; b < kKBoxesPerTile; ++b)
        tma_load_4d(smem + Smem::q + b * kBoxBytes, &map_q, b * 64, int(kvh * a.group), int(t0),
                    int(seq), q_full);
      // K boxes and V groups are numbered in issue order; box n uses slot
      // n % slots in its (n / slots)-th round.  k_boxes / v_groups count the
      // copies issued so far.
      uint32_t k_boxes = 0, v_groups = 0;
      auto load_k = [&](uint32_t j) -> bool {
        for (int b = 0; b < kKBoxesPerTile; ++b) {
          const uint32_t n = j * kKBoxesPerTile + b, s = n % kKSlots;
          if (n >= kKSlots && !wait_or_abort(&k_empty[s], ((n / kKSlots) - 1) & 1, abort))
            return false;
          mbar_arrive_expect_tx(&bar_k[s], kBoxBytes);
          tma_load_4d(smem + Smem::k + s * kBoxBytes, &map_k, b * 64, int(kvh), int(j * kKeys),
                      int(seq), &bar_k[s]);
          k_boxes = n + 1;
        }
        return true;
      };
      auto load_v = [&](uint32_t j) -> bool {
        for (int g = 0; g < kVGroupsPerTile; ++g) {
          const uint32_t n = j * kVGroupsPerTile + g, s = n % kVSlots;
          if (n >= kVSlots && !wait_or_abort(&v_empty[s], ((n / kVSlots) - 1) & 1, abort))
            return false;
          mbar_arrive_expect_tx(&bar_v[s], kBoxBytes);
          for (int d = 0; d < kD / 64; ++d)
            tma_load_4d(smem + Smem::v + s * kBoxBytes + d * (kBoxBytes / 4), &map_v, d * 64,
                        int(kvh), int(j * kKeys + g * kVKeys), int(seq), &bar_v[s]);
          v_groups = n + 1;
        }
        return true;
      };
      // Issue order K_0, then per tile j: K_{j+1}, V_j (K runs a tile ahead).
      bool fine = n_tiles > 0 && load_k(0);
      for (uint32_t j = 0; fine && j < n_tiles; ++j) {
        if (j + 1 < n_tiles && !load_k(j + 1))
          break;
        fine = load_v(j);
      }
      // Let every issued copy land before shared memory can be released.
      mbar_wait(q_full, 0);
      for (uint32_t n = k_boxes > kKSlots ? k_boxes - kKSlots : 0; n < k_boxes; ++n)
        mbar_wait(&bar_k[n % kKSlots], (n / kKSlots) & 1);
      for (uint32_t n = v_groups > kVSlots ? v_groups - kVSlots : 0; n < v_groups; ++n)
        mbar_wait(&bar_v[n % kVSlots], (n / kVSlots) & 1);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(kRows, kKeys, false);
      constexpr uint32_t idesc_o = idesc_f16(kRows, kD, true);
      const uint32_t q_base = smem_u32(smem + Smem::q);
      const uint32_t k_base = smem_u32(smem + Smem::k);
      const uint32_t v_base = smem_u32(smem + Smem::v);
      bool ok = wait_or_abort(q_full, 0, abort);
      tc_fence_after();
      auto issue_pv = [&](uint32_t i) -> bool {
        const int sb = i % kSBuffers;
        if (!wait_or_abort(&p_ready[sb], (i / kSBuffers) & 1, abort))
          return false;
        tc_fence_after();
        const uint32_t p_tmem = tmem + kColS + sb * kKeys;  // P (fp16 pairs) over the S buffer
        for (int g = 0; g < kVGroupsPerTile; ++g) {
          const uint32_t n = i * kVGroupsPerTile + g, s = n % kVSlots;
          if (!wait_or_abort(&bar_v[s], (n / kVSlots) & 1, abort))
            return false;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kVKeys / 16; ++kk) {
            const int ks = g * (kVKeys / 16) + kk;
            const uint64_t b = smem_desc(v_base + s * kBoxBytes + kk * 2048, kBoxBytes / 4, 1024);
            mma_ts(tmem + kColO, p_tmem + ks * 8, b, idesc_o, (i > 0 || ks > 0) ? 1u : 0u);
          }
          mma_commit(&v_empty[s]);
        }
        mma_commit(o_done);
        return true;
      };
      for (uint32_t j = 0; ok && j < n_tiles; ++j) {
        const int sb = j % kSBuffers;
        for (int b = 0; ok && b < kKBoxesPerTile; ++b) {
          const uint32_t n = j * kKBoxesPerTile + b, s = n % kKSlots;
          if (!wait_or_abort(&bar_k[s], (n / kKSlots) & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t qa = smem_desc(q_base + b * kBoxBytes + kk * 32, 16, 1024);
            const uint64_t kb = smem_desc(k_base + s * kBoxBytes + kk * 32, 16, 1024);
            mma_ss(tmem + kColS + sb * kKeys, qa, kb, idesc_s, (b > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&k_empty[s]);
        }
        if (!ok)
          break;
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
    constexpr int kHalf = kKeys / 2;                            // keys per warp of the pair
    uint64_t *my_pair = &pair_bar[quarter];
    uint32_t pair_phase = 0;
    float *row_max = reinterpret_cast<float *>(smem + Smem::row_max);

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
      const uint32_t s_cols = lane_base + kColS + s * kKeys + half * kHalf;
      tmem_ld32(s_cols, raw[0]);
      tmem_ld32(s_cols + 32, raw[1]);
      tmem_wait_ld();
      // Raw scores; the 1/sqrt(D) * log2(e) scale is folded into the
      // exponent's FFMA below (it is positive, so the max commutes with it).
      float x[kHalf];
#pragma unroll
      for (int c = 0; c < kHalf; ++c)
        x[c] = __uint_as_float(raw[c >> 5][c & 31]);
      const bool masked_tile = j >= first_masked_tile;
      if (masked_tile) {
        const int lim = int(limit) - int(j * kKeys + half * kHalf);
#pragma unroll
        for (int c = 0; c < kHalf; ++c)
          if (c > lim)
            x[c] = -INFINITY;
      }
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        mx[i] = x[i];
#pragma unroll
      for (int c = 8; c < kHalf; ++c)
        mx[c & 7] = fmaxf(mx[c & 7], x[c]);
      const float pmax = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      // Exchange the partial maxima (slot by tile parity, so a fast warp
      // cannot overwrite a value its partner has yet to read).  After the
      // rendezvous both warps have also read their S columns, so either may
      // write P over them.
      float *slot = row_max + (j & 1) * 2 * kRows;
      slot[half * kRows + row] = pmax;
      if (!pair_sync(my_pair, (pair_phase++) & 1, abort)) {
        ok = false;
        break;
      }
      const float tmax = fmaxf(pmax, slot[(1 - half) * kRows + row]) * a.scale_log2;
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
      // p = 2^(s*scale - m) for this warp's 64 keys, as fp16 pairs over the
      // S buffer: keys 64*half.. -> columns 32*half..
      uint32_t packed[kHalf / 2];
      float sums[4] = {0.f, 0.f, 0.f, 0.f};
      const float neg_m = -m, scale = a.scale_log2;
#pragma unroll
      for (int c = 0; c < kHalf; c += 2) {
        const float p0 = fast_exp2(fmaf(x[c], scale, neg_m));
        const float p1 = fast_exp2(fmaf(x[c + 1], scale, neg_m));
        sums[(c >> 1) & 3] += p0 + p1;
        packed[c >> 1] = pack_half2(p0, p1);
      }
      l += (sums[0] + sums[1]) + (sums[2] + sums[3]);
      tmem_st32(lane_base + kColS + s * kKeys + half * (kHalf / 2), packed);
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
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace prefill_tc
}  // namespace llmi
