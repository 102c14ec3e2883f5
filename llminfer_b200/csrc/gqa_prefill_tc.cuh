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
// Roles (192 threads, one CTA per SM):
//   warps 0-3  softmax: thread r owns TMEM lane r = query row r.  It reads its
//              row of S (64 fp32) with tcgen05.ld, applies the causal mask and
//              the online softmax, writes P back to TMEM as fp16 (over the
//              consumed S columns) and, in the epilogue, normalises O.
//   warp 4     TMA producer: Q once (4 boxes of 64 dims), then K and V tiles
//              into a 2-stage ring.
//   warp 5     TMEM allocator; one elected thread issues the MMAs:
//                S_j = Q K_j^T     (SS, M128 N64 K256, both K-major)
//                O  += P_j V_j     (TS, A = P from TMEM, B = V MN-major)
//              and commits them to mbarriers.
// TMEM columns: O [0,256), S/P buffers [256,320) and [320,384).
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

#include "common.cuh"

namespace llmi {
namespace prefill_tc {

constexpr int kD = 256;
constexpr int kRows = 128;
constexpr int kKeys = 64;
constexpr int kThreads = 192;
constexpr int kSoftmaxThreads = 128;
constexpr int kQBytes = kRows * kD * 2;   // 64 KiB, 4 boxes of 16 KiB
constexpr int kKVBytes = kKeys * kD * 2;  // 32 KiB, 4 boxes of 8 KiB
constexpr int kStages = 2;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0, kColS = 256;
constexpr float kRescaleThreshold = 8.0f;

struct Smem {
  // Offsets from the 1024-byte aligned base.
  static constexpr int q = 0;
  static constexpr int k = kQBytes;
  static constexpr int v = k + kStages * kKVBytes;
  static constexpr int bars = v + kStages * kKVBytes;
  static constexpr int total = bars + 256;
  static constexpr int alloc = total + 1024;  // alignment slack
};

struct Args {
  __half *out;  // [batch][tokens][Hq][D]
  uint32_t tokens, q_heads, kv_heads, group, past, tok_per_tile, tiles_per_head;
  float scale_log2;
};

// ---- PTX wrappers ---------------------------------------------------------------

__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int c0, int c1, int c2,
                                            int c3, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle, sm100 version bits.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// Instruction descriptor for kind::f16: f16 A/B, f32 accumulator.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n, bool b_mn_major) {
  return (1u << 4) | (0u << 7) | (0u << 10) | (uint32_t(b_mn_major) << 16) |
         (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Bounded wait that also gives up as soon as another role has aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, unsigned parity,
                                              volatile uint32_t *abort) {
  if (mbar_try_wait(bar, parity))
    return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity))
        return true;
    if (*abort)
      return false;
    if (global_timer_ns() - start > kWaitLimitNs) {
      raise_error(kErrWaitTimeout);
      *abort = 1u;
      return false;
    }
  }
}

// ---- the kernel --------------------------------------------------------------------

__global__ void __launch_bounds__(kThreads, 1)
    attend(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
           const __grid_constant__ CUtensorMap map_v, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Smem::bars);
  uint64_t *bar_q = bars + 0;
  uint64_t *bar_k = bars + 1;       // [2]
  uint64_t *bar_v = bars + 3;       // [2]
  uint64_t *kv_empty = bars + 5;    // [2]
  uint64_t *s_full = bars + 7;      // [2]
  uint64_t *p_ready = bars + 9;     // [2]
  uint64_t *o_done = bars + 11;
  uint64_t *o_final = bars + 12;
  uint64_t *drain = bars + 13;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 16);
  volatile uint32_t *abort = reinterpret_cast<volatile uint32_t *>(bars + 17);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Heaviest (latest-token) tiles first.
  const uint32_t tile = a.tiles_per_head - 1 - blockIdx.x;
  const uint32_t kvh = blockIdx.y, seq = blockIdx.z;
  const uint32_t t0 = tile * a.tok_per_tile;
  const uint32_t t_last = min(t0 + a.tok_per_tile, a.tokens) - 1;
  const uint32_t n_tiles = (a.past + t_last + 1 + kKeys - 1) / kKeys;

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bar_k[s], 1);
      mbar_init(&bar_v[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_ready[s], kSoftmaxThreads);
    }
    mbar_init(o_done, 1);
    mbar_init(o_final, 1);
    mbar_init(drain, 1);
    *abort = 0u;
    fence_barrier_init();
  }
  if (warp == 5) {
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

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_map(&map_q);
      prefetch_map(&map_k);
      prefetch_map(&map_v);
      const int head0 = int(kvh * a.group);
      mbar_arrive_expect_tx(bar_q, kQBytes);
      for (int b = 0; b < 4; ++b)
        tma_load_4d(smem + Smem::q + b * (kQBytes / 4), &map_q, b * 64, head0, int(t0), int(seq),
                    bar_q);
      uint32_t issued = 0;
      for (uint32_t j = 0; j < n_tiles; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !wait_or_abort(&kv_empty[s], ((j / kStages) - 1) & 1, abort))
          break;
        mbar_arrive_expect_tx(&bar_k[s], kKVBytes);
        for (int b = 0; b < 4; ++b)
          tma_load_4d(smem + Smem::k + s * kKVBytes + b * (kKVBytes / 4), &map_k, b * 64, int(kvh),
                      int(j * kKeys), int(seq), &bar_k[s]);
        mbar_arrive_expect_tx(&bar_v[s], kKVBytes);
        for (int b = 0; b < 4; ++b)
          tma_load_4d(smem + Smem::v + s * kKVBytes + b * (kKVBytes / 4), &map_v, b * 64, int(kvh),
                      int(j * kKeys), int(seq), &bar_v[s]);
        issued = j + 1;
      }
      // Let every issued copy land before shared memory can be released.
      mbar_wait(bar_q, 0);
      for (uint32_t j = issued > kStages ? issued - kStages : 0; j < issued; ++j) {
        mbar_wait(&bar_k[j % kStages], (j / kStages) & 1);
        mbar_wait(&bar_v[j % kStages], (j / kStages) & 1);
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(kRows, kKeys, false);
      constexpr uint32_t idesc_o = idesc_f16(kRows, kD, true);
      const uint32_t q_base = smem_u32(smem + Smem::q);
      const uint32_t k_base = smem_u32(smem + Smem::k);
      const uint32_t v_base = smem_u32(smem + Smem::v);
      bool ok = wait_or_abort(bar_q, 0, abort);
      tc_fence_after();
      auto issue_pv = [&](uint32_t i) -> bool {
        const int s = i % kStages;
        if (!wait_or_abort(&p_ready[s], (i / kStages) & 1, abort))
          return false;
        if (!wait_or_abort(&bar_v[s], (i / kStages) & 1, abort))
          return false;
        tc_fence_after();
        const uint32_t p_tmem = tmem + kColS + s * kKeys;
#pragma unroll
        for (int ks = 0; ks < kKeys / 16; ++ks) {
          const uint64_t b = smem_desc(v_base + s * kKVBytes + ks * 2048, kKVBytes / 4, 1024);
          mma_ts(tmem + kColO, p_tmem + ks * 8, b, idesc_o, (i > 0 || ks > 0) ? 1u : 0u);
        }
        mma_commit(&kv_empty[s]);
        mma_commit(o_done);
        return true;
      };
      for (uint32_t j = 0; ok && j < n_tiles; ++j) {
        const int s = j % kStages;
        if (!wait_or_abort(&bar_k[s], (j / kStages) & 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kD / 16; ++ks) {
          const uint32_t box = ks >> 2, off = (ks & 3) * 32;
          const uint64_t qa = smem_desc(q_base + box * (kQBytes / 4) + off, 16, 1024);
          const uint64_t kb = smem_desc(k_base + s * kKVBytes + box * (kKVBytes / 4) + off, 16, 1024);
          mma_ss(tmem + kColS + s * kKeys, qa, kb, idesc_s, ks > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[s]);
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
    // ---------------- softmax warps 0-3 ----------------
    const uint32_t row = threadIdx.x;  // TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t(warp) * 32u) << 16);
    const uint32_t token = t0 + row / a.group;
    const uint32_t head = kvh * a.group + row % a.group;
    const bool valid = token < a.tokens;
    const uint32_t limit = a.past + min(token, a.tokens - 1);  // last visible key
    const uint32_t first_masked_tile = (a.past + t0) / kKeys;   // tiles before are fully visible
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    uint32_t j = 0;
    for (; j < n_tiles; ++j) {
      const int s = j % kStages;
      // tcgen05.ld/st are warp-collective: every decision below is warp-uniform.
      if (!__all_sync(0xffffffffu, wait_or_abort(&s_full[s], (j / kStages) & 1, abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t raw[2][32];
      tmem_ld32(lane_base + kColS + s * kKeys, raw[0]);
      tmem_ld32(lane_base + kColS + s * kKeys + 32, raw[1]);
      tmem_wait_ld();
      float x[kKeys];
#pragma unroll
      for (int c = 0; c < kKeys; ++c)
        x[c] = __uint_as_float(raw[c >> 5][c & 31]) * a.scale_log2;
      if (j >= first_masked_tile) {
        const int lim = int(limit) - int(j * kKeys);
#pragma unroll
        for (int c = 0; c < kKeys; ++c)
          if (c > lim)
            x[c] = -INFINITY;
      }
      float tmax = x[0];
#pragma unroll
      for (int c = 1; c < kKeys; ++c)
        tmax = fmaxf(tmax, x[c]);
      const bool need = tmax > m + kRescaleThreshold;
      if (__any_sync(0xffffffffu, need)) {
        const float next = need ? tmax : m;
        const float alpha = need ? fast_exp2(m - next) : 1.f;  // 0 when m = -inf
        if (j > 0) {
          // O holds P_0..P_{j-1} V: wait for the last of those MMAs, rescale.
          if (!__all_sync(0xffffffffu, wait_or_abort(o_done, (j - 1) & 1, abort))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < kD; c += 32) {
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
      uint32_t packed[32];
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < kKeys; c += 2) {
        const float p0 = fast_exp2(x[c] - m), p1 = fast_exp2(x[c + 1] - m);
        sum += p0 + p1;
        packed[c >> 1] = pack_half2(p0, p1);
      }
      l += sum;
      tmem_st32(lane_base + kColS + s * kKeys, packed);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_ready[s]);
    }
    if (ok && __all_sync(0xffffffffu, wait_or_abort(o_final, 0, abort))) {
      tc_fence_after();
      const float inv = 1.f / l;
      __half *orow = a.out + ((size_t(seq) * a.tokens + token) * a.q_heads + head) * kD;
#pragma unroll 1
      for (int c = 0; c < kD; c += 32) {
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
  if (warp == 5) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace prefill_tc
}  // namespace llmi
