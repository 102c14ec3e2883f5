// Decode attention (CausalGqa with one new token per sequence) as split-K
// flash decoding.
//
// The reference computes decode in three dispatches with an fp16 score
// buffer [tokens*queryHeads, past+tokens]: gqaScores
// (Reference.metal:303-323), gqaSoftmax (Graph.metal:172-210) and gqaValue
// (Graph.metal:212-230).  Here the cache is streamed exactly once:
//
//  * The key range of every unit is cut into tiles of 16 keys, and the tiles
//    of all units are laid end to end and divided evenly among workers.  A
//    worker keeps an online softmax for the GQA group of its unit and writes
//    one partial record (max, sum, unnormalised output) for every unit it
//    touches.  Because whole tiles are balanced across workers, every SM
//    streams the same number of bytes whatever the batch and context length.
//  * The merge pass combines the records of each (sequence, kv head)
//    (log-sum-exp) and writes the fp16 output.
//
// Four partial-pass kernels:
//  * partial_rows: a worker is a CTA and a unit a sequence.  A producer warp
//    fetches whole cache rows (all kv heads of one key, 2 KiB for Hkv 4 x
//    D 256) with one bulk copy each into a CTA-wide ring; warp h computes kv
//    head h.  Used for Hkv 4 x D 256 and Hkv 8 x D 128 (2 KiB rows, one CTA
//    per SM) and Hkv 2 x D 256 (1 KiB rows, two CTAs per SM).
//  * partial_mma: when Hkv equals the warps of a CTA, the CTA is a worker and
//    warp h serves kv head h, with private per-warp pipelines of 512-byte row
//    copies.
//  * partial_mma_cta: otherwise the CTA is a worker whose warps take a unit's
//    tiles in turn and combine into one record per unit.
//  * partial_simt: CUDA cores, any head_dim <= 512 and any group.
//
// Scores and the softmax stay in fp32 (log2 domain).  Probabilities enter the
// P.V product rounded to fp16, as in the reference's decode path.
//
// Tensor-core mapping of one 16-key tile (m16n8k16, f16 x f16 -> f32):
//   S^T[key][head]  = K[key][:] . Q[head][:]       A = K tile (ldmatrix),
//                                                   B = Q (registers), N = 8
//   O^T[d][head]   += V^T[d][key] . P^T[key][head] A = V tile (ldmatrix.trans),
//                                                   B = P via movmatrix.trans
// so the group's query heads (<= 8) sit in N and no row of M is wasted.
#pragma once

#include "common.cuh"

namespace llmi {
namespace decode {

constexpr int kTileKeys = 16;

// How the key tiles of all units are divided among workers.  Worker w owns
// tiles [w*tiles_per_worker, (w+1)*tiles_per_worker) of the concatenation of
// the units' tile lists and writes one record per unit it touches.
//
// Two shapes of worker:
//  * heads == 1: a worker is one warp and a unit is one (sequence, kv head);
//  * heads == Hkv: a worker is one CTA whose warp h serves kv head h, and a
//    unit is one sequence.
// Records are laid out [worker][span][heads].
struct Partition {
  uint32_t units;             // sequences * (kv heads when heads == 1)
  uint32_t tiles_per_unit;    // key tiles (or key splits) per unit
  uint32_t tiles_per_worker;
  uint32_t max_span;          // units a worker can touch
  uint32_t workers;
  uint32_t heads;             // kv heads served by one worker
  uint32_t prefetch_tiles;    // tiles a worker warms L2 with before it waits (<= 16)
};

// For a worker that holds records: its first tile, worker * tiles_per_worker,
// lies below the tile count, which the plan keeps within 32 bits.
__host__ __device__ inline uint32_t first_unit(const Partition &pt, uint32_t worker) {
  return worker * pt.tiles_per_worker / pt.tiles_per_unit;
}

__host__ __device__ inline uint64_t record_index(const Partition &pt, uint32_t worker,
                                                 uint32_t unit, uint32_t head = 0) {
  return (uint64_t(worker) * pt.max_span + (unit - first_unit(pt, worker))) * pt.heads + head;
}

// Record layout (fp32): [max: G][sum: G][out: G][D], padded to 4 floats.
__host__ __device__ inline uint32_t record_floats(uint32_t group, uint32_t head_dim) {
  return (2 * group + group * head_dim + 3) & ~3u;
}

struct Args {
  const __half *q;       // [batch][queryHeads][D]  (tokens == 1)
  const __half *k, *v;   // caches, sequence stride cache_stride
  size_t cache_stride;
  __half *out;           // [batch][queryHeads][D]
  float *records;
  Partition pt;
  uint32_t kv_heads, group, head_dim, keys;  // keys = past + 1
  uint32_t record_floats;
  float scale_log2;      // log2(e) / sqrt(D)
  // The step's KvAppend folded into the op (each may be null): the new K
  // and V rows [batch][kv_heads][D], `new_stride` halves between sequences.
  // The partial pass reads key keys - 1 from them, and the merge writes them
  // into the caches' row keys - 1, which no kernel of the op reads.
  const __half *k_new, *v_new;
  size_t new_stride;
  uint32_t batch;
  // Nonzero when the caller guarantees that no work still in flight writes
  // cache rows [0, keys - 1) (LLMI_FLAG_SETTLED): partial_rows then requests
  // its first tiles below the newest row before wait_primary().
  uint32_t settled;
};

// L2 warm-up of a CTA worker's first key tiles, issued before
// wait_primary(): the cache rows are read-only to the kernels ahead in a
// decode step except the newest, and a prefetch never changes what a later
// load returns, so the first tiles stream in while the kernel ahead (the
// appends, the previous layer) still runs.
//
// Tile t of units that are (sequence, kv head) pairs: one row of D halves
// per key and head; lane 16 (V ? 1 : 0) + r takes key row r.
template <int D>
__device__ __forceinline__ void prefetch_head_rows(const Args &a, uint32_t t, int lane) {
  const uint32_t tpu = a.pt.tiles_per_unit;
  const uint32_t unit = t / tpu, key0 = (t % tpu) * kTileKeys;
  const uint32_t seq = unit / a.kv_heads, kvh = unit % a.kv_heads;
  const uint32_t row = uint32_t(lane & 15);
  if (key0 + row >= a.keys)
    return;
  const __half *base = lane < 16 ? a.k : a.v;
  prefetch_l2(base + seq * a.cache_stride + (size_t(key0 + row) * a.kv_heads + kvh) * D, D * 2);
}

// One warp's tensor-core state for one unit: the group's queries as B
// fragments, the running max / sum for its two heads (N columns
// 2*(lane%4), +1) and the O^T accumulator fragments.
template <int D>
struct TileMath {
  static constexpr int KS = D / 16;
  uint32_t qf[KS][2];
  float o[KS][4];
  float m0, m1, l0, l1;

  __device__ __forceinline__ void start(const __half *qgroup, uint32_t group, int lane) {
    const uint32_t head = lane >> 2, head0 = (lane & 3) * 2;
    const __half *qrow = qgroup + size_t(head) * D;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      if (head < group) {
        qf[ks][0] = *reinterpret_cast<const uint32_t *>(qrow + ks * 16 + head0);
        qf[ks][1] = *reinterpret_cast<const uint32_t *>(qrow + ks * 16 + head0 + 8);
      } else {
        qf[ks][0] = qf[ks][1] = 0u;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
        o[ks][i] = 0.f;
    }
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.f;
  }

  // One 16-key tile.  kbase/vbase: shared addresses of key row 0 of this
  // head's K and V slices; rows `row_stride` bytes apart; `valid` keys.
  __device__ __forceinline__ void tile(uint32_t kbase, uint32_t vbase, uint32_t row_stride,
                                       uint32_t valid, float scale_log2, int lane) {
    const uint32_t krow = lane >> 2;
    const uint32_t k_lane = ((lane & 7) + ((lane >> 3) & 1) * 8) * row_stride + (lane >> 4) * 16;
    const uint32_t v_lane = ((lane & 7) + (lane >> 4) * 8) * row_stride + ((lane >> 3) & 1) * 16;
    float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < KS; ks += 2) {
      uint32_t fa[4];
      ldmatrix_x4(fa, kbase + k_lane + ks * 32);
      mma_f16_16816(sa, fa, qf[ks][0], qf[ks][1]);
      if (ks + 1 < KS) {
        uint32_t fb[4];
        ldmatrix_x4(fb, kbase + k_lane + (ks + 1) * 32);
        mma_f16_16816(sb, fb, qf[ks + 1][0], qf[ks + 1][1]);
      }
    }
    const float x0 = krow < valid ? (sa[0] + sb[0]) * scale_log2 : -INFINITY;
    const float x1 = krow < valid ? (sa[1] + sb[1]) * scale_log2 : -INFINITY;
    const float x2 = krow + 8 < valid ? (sa[2] + sb[2]) * scale_log2 : -INFINITY;
    const float x3 = krow + 8 < valid ? (sa[3] + sb[3]) * scale_log2 : -INFINITY;
    float t0 = fmaxf(x0, x2), t1 = fmaxf(x1, x3);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, off));
      t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, off));
    }
    const float n0 = fmaxf(m0, t0), n1 = fmaxf(m1, t1);
    const float r0 = fast_exp2(m0 - n0), r1 = fast_exp2(m1 - n1);
    m0 = n0;
    m1 = n1;
    const float p0 = fast_exp2(x0 - n0), p1 = fast_exp2(x1 - n1);
    const float p2 = fast_exp2(x2 - n0), p3 = fast_exp2(x3 - n1);
    l0 = l0 * r0 + p0 + p2;
    l1 = l1 * r1 + p1 + p3;
    const uint32_t b0 = movmatrix_trans(pack_half2(p0, p1));
    const uint32_t b1 = movmatrix_trans(pack_half2(p2, p3));
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
      o[mt][0] *= r0;
      o[mt][1] *= r1;
      o[mt][2] *= r0;
      o[mt][3] *= r1;
      uint32_t fv[4];
      ldmatrix_x4_trans(fv, vbase + v_lane + mt * 32);
      mma_f16_16816(o[mt], fv, b0, b1);
    }
  }

  // Writes this unit's record (max and sum per head, O^T as [head][D]).
  __device__ __forceinline__ void flush(float *rec, uint32_t G, int lane) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, 4);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 8);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 16);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 4);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 8);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 16);
    const uint32_t head0 = (lane & 3) * 2, krow = lane >> 2;
    if (lane < 4) {
      if (head0 < G) {
        rec[head0] = m0;
        rec[G + head0] = l0;
      }
      if (head0 + 1 < G) {
        rec[head0 + 1] = m1;
        rec[G + head0 + 1] = l1;
      }
    }
    float *out0 = rec + 2 * G + head0 * D;
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
      const uint32_t d = mt * 16 + krow;
      if (head0 < G) {
        out0[d] = o[mt][0];
        out0[d + 8] = o[mt][2];
      }
      if (head0 + 1 < G) {
        out0[D + d] = o[mt][1];
        out0[D + d + 8] = o[mt][3];
      }
    }
  }
};

// ---------------------------------------------------------------------------
// partial_rows: CTA-wide ring of whole cache rows, one producer warp.

template <int D, int HKV, int STAGES>
struct RowShape {
  static constexpr int kRowBytes = HKV * D * 2;       // one key's [Hkv][D] row
  static constexpr int kRowStride = kRowBytes + 16;   // +16 B: conflict-free ldmatrix per head
  static constexpr int kTileBytes = kTileKeys * kRowStride;
  static constexpr int kStageBytes = 2 * kTileBytes;  // K tile + V tile
  static constexpr int kThreads = (HKV + 1) * 32;
  static constexpr int kSmemBytes = STAGES * kStageBytes + 2 * STAGES * 8 + 16;
};

template <int D, int HKV, int STAGES>
__global__ void __launch_bounds__(RowShape<D, HKV, STAGES>::kThreads, 1)
    partial_rows(const Args a) {
  using Shape = RowShape<D, HKV, STAGES>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * Shape::kStageBytes);
  uint64_t *empty = full + STAGES;
  volatile uint32_t *abort = reinterpret_cast<volatile uint32_t *>(empty + STAGES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Partition pt = a.pt;  // heads == HKV, units = sequences
  const uint32_t worker = blockIdx.x;
  const uint32_t total = pt.units * pt.tiles_per_unit;
  const uint32_t begin = min(total, worker * pt.tiles_per_worker);
  const uint32_t end = min(total, begin + pt.tiles_per_worker);
  if (begin >= end) {
    pdl_enter();
    return;  // uniform over the CTA
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], HKV);
    }
    *abort = 0u;
    fence_barrier_init();
  }
  __syncthreads();
  const uint32_t tpu = pt.tiles_per_unit;

  if (warp == HKV) {
    // Producer: lanes 0-15 fetch the tile's 16 key rows, lanes 16-31 its 16
    // value rows, each row [Hkv][D] with one bulk copy.  Rows past the end of
    // the cache range repeat the last valid row (masked to -inf).
    const uint64_t policy = policy_evict_first();
    // The step's new row of this lane's K or V, when the caller folded the
    // KvAppend in: it replaces the cache's row keys - 1.
    const __half *fresh = lane < 16 ? a.k_new : a.v_new;
    uint32_t issued = 0;
    // Tile t is keys [key0, key0 + 16) of sequence seq; both advance with t
    // (no division per tile: the copies' issue is on the pipeline's path).
    uint32_t seq = begin / tpu, key0 = (begin % tpu) * kTileKeys;
    // Settled caches: the first STAGES tiles that end below the newest row
    // are requested before the wait (the newest row may come from the kernel
    // ahead: `fresh`, or a separate cacheAppend).
    bool waited = !a.settled;
    if (waited)
      pdl_enter();
    for (uint32_t t = begin; t < end; ++t) {
      const uint32_t j = t - begin;
      const int s = j % STAGES;
      if (!waited && (j >= STAGES || key0 + kTileKeys >= a.keys)) {
        pdl_enter();
        waited = true;
      }
      if (j >= STAGES &&
          !__all_sync(0xffffffffu, wait_or_abort(&empty[s], ((j / STAGES) - 1) & 1, abort)))
        break;
      const uint32_t valid = min(uint32_t(kTileKeys), a.keys - key0);
      if (lane == 0)
        mbar_arrive_expect_tx(&full[s], 2 * kTileKeys * Shape::kRowBytes);
      __syncwarp();
      const uint32_t row = lane & 15;
      const uint32_t key = key0 + min(row, valid - 1);
      const __half *src = (lane < 16 ? a.k : a.v) + seq * a.cache_stride + size_t(key) * HKV * D;
      if (fresh != nullptr && key + 1 == a.keys)
        src = fresh + seq * a.new_stride;
      uint8_t *dst = smem + s * Shape::kStageBytes + (lane < 16 ? 0 : Shape::kTileBytes) +
                     row * Shape::kRowStride;
      bulk_g2s(dst, src, Shape::kRowBytes, &full[s], policy);
      issued = j + 1;
      key0 += kTileKeys;
      if (key0 >= a.keys) {
        key0 = 0;
        ++seq;
      }
    }
    if (!waited)
      pdl_enter();
    // Every issued copy lands before the CTA can exit (bounded).
    if (lane == 0)
      for (uint32_t j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j)
        mbar_wait(&full[j % STAGES], (j / STAGES) & 1);
    __syncwarp();
    return;
  }

  // Consumer warp: kv head `warp`.
  const uint32_t h = warp;
  TileMath<D> math;
  uint32_t unit = 0xffffffffu;
  bool ok = true;
  uint32_t u = begin / tpu, key0 = (begin % tpu) * kTileKeys;  // tile t, advanced with t
  asm volatile("" ::"r"(u), "r"(key0));  // the division stays ahead of the wait
  pdl_enter();  // before the queries are read
  for (uint32_t t = begin; t < end; ++t) {
    const uint32_t j = t - begin;
    const int s = j % STAGES;
    if (u != unit) {
      if (unit != 0xffffffffu)
        math.flush(a.records + record_index(pt, worker, unit, h) * a.record_floats, a.group, lane);
      unit = u;
      math.start(a.q + (size_t(u) * HKV * a.group + h * a.group) * D, a.group, lane);
    }
    if (!__all_sync(0xffffffffu, wait_or_abort(&full[s], (j / STAGES) & 1, abort))) {
      ok = false;
      break;
    }
    const uint32_t kbase = smem_u32(smem + s * Shape::kStageBytes) + h * D * 2;
    const uint32_t valid = min(uint32_t(kTileKeys), a.keys - key0);
    math.tile(kbase, kbase + Shape::kTileBytes, Shape::kRowStride, valid, a.scale_log2, lane);
    __syncwarp();
    if (lane == 0)
      mbar_arrive(&empty[s]);
    key0 += kTileKeys;
    if (key0 >= a.keys) {
      key0 = 0;
      ++u;
    }
  }
  if (ok)
    math.flush(a.records + record_index(pt, worker, unit, h) * a.record_floats, a.group, lane);
}

// ---------------------------------------------------------------------------
// partial_mma: per-warp pipelines of 512-byte row copies.

template <int D, int WARPS, int STAGES>
struct MmaShape {
  static constexpr int kRowBytes = D * 2;
  static constexpr int kRowStride = D * 2 + 16;  // +16 B: conflict-free ldmatrix
  static constexpr int kTileBytes = kTileKeys * kRowStride;
  static constexpr int kStageBytes = 2 * kTileBytes;  // K tile + V tile
  static constexpr int kSmemBytes = WARPS * STAGES * kStageBytes + WARPS * STAGES * 8;
};

// Requires D % 16 == 0, D <= 256 and group <= 8.
template <int D, int WARPS, int STAGES>
__global__ void __launch_bounds__(WARPS * 32, 1) partial_mma(const Args a) {
  using Shape = MmaShape<D, WARPS, STAGES>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t *stages = smem + warp * STAGES * Shape::kStageBytes;
  uint64_t *bars =
      reinterpret_cast<uint64_t *>(smem + WARPS * STAGES * Shape::kStageBytes) + warp * STAGES;

  const Partition pt = a.pt;
  // heads == 1: this warp is a worker; otherwise the CTA is, and this warp
  // serves kv head `warp` of each sequence in the CTA's range.
  const bool grouped = pt.heads > 1;
  const uint32_t worker = grouped ? blockIdx.x : blockIdx.x * WARPS + warp;
  const uint32_t my_head = grouped ? uint32_t(warp) : 0u;
  const uint32_t total = pt.units * pt.tiles_per_unit;
  const uint32_t begin = min(total, worker * pt.tiles_per_worker);
  const uint32_t end = min(total, begin + pt.tiles_per_worker);
  pdl_enter();  // before the first global read
  if (begin >= end || (grouped && my_head >= pt.heads))
    return;  // warps are independent: no CTA-wide barrier below

  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s)
      mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  __syncwarp();

  const uint64_t policy = policy_evict_first();
  const uint32_t tpu = pt.tiles_per_unit;
  const __half *fresh = lane < 16 ? a.k_new : a.v_new;

  // Lanes 0-15 fetch the 16 key rows, lanes 16-31 the 16 value rows.  Rows
  // past the end of the cache range repeat the last valid row (their scores
  // are masked to -inf, so they contribute exactly zero).
  auto issue = [&](uint32_t tile, int stage) {
    const uint32_t unit = tile / tpu, key0 = (tile % tpu) * kTileKeys;
    const uint32_t seq = grouped ? unit : unit / a.kv_heads;
    const uint32_t kvh = grouped ? my_head : unit % a.kv_heads;
    const uint32_t valid = min(uint32_t(kTileKeys), a.keys - key0);
    if (lane == 0)
      mbar_arrive_expect_tx(&bars[stage], 2 * kTileKeys * Shape::kRowBytes);
    __syncwarp();
    const uint32_t row = lane & 15;
    const uint32_t key = key0 + min(row, valid - 1);
    const __half *src = (lane < 16 ? a.k : a.v) + seq * a.cache_stride +
                        (size_t(key) * a.kv_heads + kvh) * D;
    if (fresh != nullptr && key + 1 == a.keys)  // the step's new row (folded KvAppend)
      src = fresh + seq * a.new_stride + size_t(kvh) * D;
    uint8_t *dst = stages + stage * Shape::kStageBytes + (lane < 16 ? 0 : Shape::kTileBytes) +
                   row * Shape::kRowStride;
    bulk_g2s(dst, src, Shape::kRowBytes, &bars[stage], policy);
  };

  for (int s = 0; s < STAGES; ++s)
    if (begin + s < end)
      issue(begin + s, s);

  TileMath<D> math;
  uint32_t unit = 0xffffffffu;
  uint32_t t = begin;
  bool ok = true;
  for (; t < end; ++t) {
    const uint32_t j = t - begin;
    const int stage = j % STAGES;
    const uint32_t u = t / tpu;
    if (u != unit) {
      if (unit != 0xffffffffu)
        math.flush(a.records + record_index(pt, worker, unit, my_head) * a.record_floats, a.group,
                   lane);
      unit = u;
      const uint32_t seq = grouped ? u : u / a.kv_heads;
      const uint32_t kvh = grouped ? my_head : u % a.kv_heads;
      math.start(a.q + (size_t(seq) * a.kv_heads * a.group + kvh * a.group) * D, a.group, lane);
    }
    ok = __all_sync(0xffffffffu, mbar_wait(&bars[stage], (j / STAGES) & 1));
    if (!ok)
      break;
    const uint32_t kbase = smem_u32(stages + stage * Shape::kStageBytes);
    const uint32_t valid = min(uint32_t(kTileKeys), a.keys - (t % tpu) * kTileKeys);
    math.tile(kbase, kbase + Shape::kTileBytes, Shape::kRowStride, valid, a.scale_log2, lane);
    __syncwarp();  // every lane is done with this stage before it is refilled
    if (t + STAGES < end)
      issue(t + STAGES, stage);
  }

  if (ok) {
    math.flush(a.records + record_index(pt, worker, unit, my_head) * a.record_floats, a.group,
               lane);
    return;
  }
  // A wait gave up: let the copies already issued land (bounded) before the
  // shared memory is released, and write nothing.
  for (uint32_t r = t; r < min(end, t + STAGES); ++r) {
    const uint32_t j = r - begin;
    mbar_wait(&bars[j % STAGES], (j / STAGES) & 1);
  }
}

// ---------------------------------------------------------------------------
// partial_mma_cta: the same tile math with the CTA as the worker, for heads ==
// 1 (a unit is one (sequence, kv head)).  With warps as workers, a unit with
// few sequences or kv heads per GPU is split over dozens of warps and the
// merge then walks dozens of records; here the CTA's warps take the unit's
// tiles in turn (warp w: the CTA's tiles t0 + w, t0 + w + WARPS, ... of the
// unit), each with its own ring of copies, and at the end of every unit they
// combine their online-softmax states through shared memory into one record
// (max over the warps, sums and outputs rescaled by 2^(m_w - m)).  Every
// warp reaches every unit's barriers: a warp whose bounded wait gave up
// keeps taking part without computing, and the error word reports it.
template <int D, int WARPS, int STAGES>
struct MmaCtaShape {
  using Base = MmaShape<D, WARPS, STAGES>;
  static constexpr int kStatesOffset = WARPS * STAGES * Base::kStageBytes + WARPS * STAGES * 8;
  // + WARPS record-sized state slots (record_floats floats each), sized at launch.
  static size_t smem_bytes(uint32_t record_floats) {
    return size_t(kStatesOffset) + size_t(WARPS) * record_floats * sizeof(float);
  }
};

template <int D, int WARPS, int STAGES>
__global__ void __launch_bounds__(WARPS * 32, 1) partial_mma_cta(const Args a) {
  using Shape = MmaShape<D, WARPS, STAGES>;
  using CtaShape = MmaCtaShape<D, WARPS, STAGES>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t *stages = smem + warp * STAGES * Shape::kStageBytes;
  uint64_t *bars =
      reinterpret_cast<uint64_t *>(smem + WARPS * STAGES * Shape::kStageBytes) + warp * STAGES;
  float *states = reinterpret_cast<float *>(smem + CtaShape::kStatesOffset);

  const Partition pt = a.pt;  // heads == 1, workers are CTAs
  const uint32_t worker = blockIdx.x;
  const uint32_t total = pt.units * pt.tiles_per_unit;
  const uint32_t begin = min(total, worker * pt.tiles_per_worker);
  const uint32_t end = min(total, begin + pt.tiles_per_worker);
  // The warps take the range's tiles in turn: each warms its own first ones.
  for (uint32_t t = begin + warp; t < min(end, begin + pt.prefetch_tiles); t += WARPS)
    prefetch_head_rows<D>(a, t, lane);
  pdl_enter();  // before the first global read (prefetches aside)
  if (begin >= end)
    return;  // uniform over the CTA

  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s)
      mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  __syncwarp();

  const uint64_t policy = policy_evict_first();
  const uint32_t tpu = pt.tiles_per_unit;
  const __half *fresh = lane < 16 ? a.k_new : a.v_new;  // the step's new rows, if folded
  const uint32_t G = a.group, F = a.record_floats;
  const uint32_t u_first = begin / tpu, u_last = (end - 1) / tpu;

  // This warp's tiles, unit by unit: (unit u, tile t) with t running over
  // [max(begin, u*tpu) + warp, min(end, (u+1)*tpu)) in steps of WARPS.
  struct Cursor {
    uint32_t u, t;
  };
  auto settle = [&](Cursor &c) {  // move past units this warp has no tile left in
    while (c.u <= u_last && c.t >= min(end, (c.u + 1) * tpu)) {
      ++c.u;
      c.t = max(begin, c.u * tpu) + warp;
    }
  };
  auto step = [&](Cursor &c) {
    c.t += WARPS;
    settle(c);
  };
  auto issue = [&](uint32_t tile, int stage) {
    const uint32_t unit = tile / tpu, key0 = (tile % tpu) * kTileKeys;
    const uint32_t seq = unit / a.kv_heads, kvh = unit % a.kv_heads;
    const uint32_t valid = min(uint32_t(kTileKeys), a.keys - key0);
    if (lane == 0)
      mbar_arrive_expect_tx(&bars[stage], 2 * kTileKeys * Shape::kRowBytes);
    __syncwarp();
    const uint32_t row = lane & 15;
    const uint32_t key = key0 + min(row, valid - 1);
    const __half *src = (lane < 16 ? a.k : a.v) + seq * a.cache_stride +
                        (size_t(key) * a.kv_heads + kvh) * D;
    if (fresh != nullptr && key + 1 == a.keys)  // the step's new row (folded KvAppend)
      src = fresh + seq * a.new_stride + size_t(kvh) * D;
    uint8_t *dst = stages + stage * Shape::kStageBytes + (lane < 16 ? 0 : Shape::kTileBytes) +
                   row * Shape::kRowStride;
    bulk_g2s(dst, src, Shape::kRowBytes, &bars[stage], policy);
  };

  // The copy ring runs STAGES tiles ahead of the compute cursor.
  Cursor ahead{u_first, max(begin, u_first * tpu) + warp};
  settle(ahead);
  uint32_t issued = 0, done = 0;  // tiles of this warp issued / computed
  for (int s = 0; s < STAGES && ahead.u <= u_last; ++s) {
    issue(ahead.t, s);
    ++issued;
    step(ahead);
  }
  Cursor cur{u_first, max(begin, u_first * tpu) + warp};
  settle(cur);
  bool ok = true;
  TileMath<D> math;
  for (uint32_t u = u_first; u <= u_last; ++u) {
    const uint32_t seq = u / a.kv_heads, kvh = u % a.kv_heads;
    math.start(a.q + (size_t(seq) * a.kv_heads * G + kvh * G) * D, G, lane);
    while (ok && cur.u == u) {
      const int stage = done % STAGES;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[stage], (done / STAGES) & 1));
      if (!ok)
        break;
      const uint32_t kbase = smem_u32(stages + stage * Shape::kStageBytes);
      const uint32_t valid = min(uint32_t(kTileKeys), a.keys - (cur.t % tpu) * kTileKeys);
      math.tile(kbase, kbase + Shape::kTileBytes, Shape::kRowStride, valid, a.scale_log2, lane);
      __syncwarp();  // every lane is done with this stage before it is refilled
      ++done;
      step(cur);
      if (ahead.u <= u_last) {
        issue(ahead.t, stage);
        ++issued;
        step(ahead);
      }
    }
    // This warp's state for unit u (empty if it had no tile of u), then the
    // CTA's record: m = max m_w, l = sum l_w 2^(m_w - m), O = sum O_w 2^(m_w - m).
    math.flush(states + warp * F, G, lane);
    __syncthreads();
    float *rec = a.records + record_index(pt, worker, u, 0) * F;
    for (uint32_t i = threadIdx.x; i < G * (D + 1); i += WARPS * 32) {
      const uint32_t h = i < G ? i : (i - G) / D;
      float m = -INFINITY;
#pragma unroll
      for (int w = 0; w < WARPS; ++w)
        m = fmaxf(m, states[w * F + h]);
      float acc = 0.f;
      if (i < G) {
#pragma unroll
        for (int w = 0; w < WARPS; ++w)
          acc = fmaf(states[w * F + G + h], fast_exp2(states[w * F + h] - m), acc);
        rec[h] = m;
        rec[G + h] = acc;
      } else {
        const uint32_t d = (i - G) % D;
#pragma unroll
        for (int w = 0; w < WARPS; ++w)
          acc = fmaf(states[w * F + 2 * G + h * D + d], fast_exp2(states[w * F + h] - m), acc);
        rec[2 * G + h * D + d] = acc;
      }
    }
    __syncthreads();  // the state slots are reused by the next unit
  }
  if (!ok) {
    // A wait gave up: let the copies already issued land (bounded) before the
    // shared memory is released.
    for (uint32_t r = done; r < issued; ++r)
      mbar_wait(&bars[r % STAGES], (r / STAGES) & 1);
  }
}

// ---------------------------------------------------------------------------
// partial_simt: shapes outside the tensor-core kernels (any head_dim up to
// 512, any group).  One CTA per (unit, key split); warps take query heads.

constexpr int kSimtKeys = 4;  // keys per group in partial_simt
constexpr uint32_t kSimtMinKeys = 128;  // keys per split at least (bounds the records per unit)

__global__ void __launch_bounds__(128) partial_simt(const Args a) {
  constexpr int kMaxPerLane = 16;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Partition pt = a.pt;
  pdl_enter();
  const uint32_t worker = blockIdx.x;  // tiles_per_worker == 1
  const uint32_t unit = worker / pt.tiles_per_unit, split = worker % pt.tiles_per_unit;
  if (unit >= pt.units)
    return;
  const uint32_t chunk = (a.keys + pt.tiles_per_unit - 1) / pt.tiles_per_unit;
  const uint32_t k0 = split * chunk, k1 = min(a.keys, k0 + chunk);
  const uint32_t seq = unit / a.kv_heads, kvh = unit % a.kv_heads;
  const uint32_t D = a.head_dim, G = a.group;
  float *rec = a.records + record_index(pt, worker, unit) * a.record_floats;
  const __half *kbase = a.k + seq * a.cache_stride + size_t(kvh) * D;
  const __half *vbase = a.v + seq * a.cache_stride + size_t(kvh) * D;
  const size_t row = size_t(a.kv_heads) * D;

  for (uint32_t h = warp; h < G; h += blockDim.x / 32) {
    const __half *qrow = a.q + (size_t(seq) * a.kv_heads * G + kvh * G + h) * D;
    float qv[kMaxPerLane], o[kMaxPerLane];
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const uint32_t d = lane + 32 * i;
      qv[i] = d < D ? __half2float(qrow[d]) : 0.f;
      o[i] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    // Keys in groups of kSimtKeys: the group's K and V rows load together
    // and its dot products reduce side by side, so a group costs one round of
    // loads; the online softmax rescales once per group, and p is rounded to
    // fp16 before the P.V product as in the reference's decode.
    for (uint32_t key0 = k0; key0 < k1; key0 += kSimtKeys) {
      __half kv[kSimtKeys][kMaxPerLane], vv[kSimtKeys][kMaxPerLane];
#pragma unroll
      for (int j = 0; j < kSimtKeys; ++j) {
        const uint32_t key = min(key0 + j, k1 - 1);
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) {
          const uint32_t d = lane + 32 * i;
          kv[j][i] = d < D ? kbase[key * row + d] : __float2half(0.f);
          vv[j][i] = d < D ? vbase[key * row + d] : __float2half(0.f);
        }
      }
      float x[kSimtKeys];
#pragma unroll
      for (int j = 0; j < kSimtKeys; ++j) {
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i)
          dot = fmaf(qv[i], __half2float(kv[j][i]), dot);
        x[j] = dot;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (int j = 0; j < kSimtKeys; ++j)
          x[j] += __shfl_xor_sync(0xffffffffu, x[j], off);
      float n = m;
#pragma unroll
      for (int j = 0; j < kSimtKeys; ++j) {
        x[j] = key0 + j < k1 ? x[j] * a.scale_log2 : -INFINITY;
        n = fmaxf(n, x[j]);
      }
      const float r = fast_exp2(m - n);
      float p[kSimtKeys];
      l *= r;
#pragma unroll
      for (int j = 0; j < kSimtKeys; ++j) {
        p[j] = __half2float(__float2half_rn(fast_exp2(x[j] - n)));
        l += fast_exp2(x[j] - n);
      }
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i) {
        float acc = o[i] * r;
#pragma unroll
        for (int j = 0; j < kSimtKeys; ++j)
          acc = fmaf(p[j], __half2float(vv[j][i]), acc);
        o[i] = acc;
      }
      m = n;
    }
    if (lane == 0) {
      rec[h] = m;
      rec[G + h] = l;
    }
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const uint32_t d = lane + 32 * i;
      if (d < D)
        rec[2 * G + h * D + d] = o[i];
    }
  }
}

// ---------------------------------------------------------------------------
// Merge pass: one CTA per (sequence, kv head) and slice of head_dim, one warp
// per query head.  Lane i reads record i's max and sum once (records past 32
// fold in with a loop), the shuffled maximum gives every record's weight,
// and lane i's weight is broadcast by shuffle where the outputs are summed.
// head_dim is cut into gridDim.y slices so that few (sequence, kv head)
// units with many records (a GPU's shard of a few sequences or kv heads)
// still spread over many SMs.  Within a slice of F float4 columns, lanes
// form 32 / F groups that sum interleaved records (F < 32), or each lane
// owns F / 32 columns (F >= 32); loads go four records per round, and the
// groups' sums are combined by shuffles at the end.  Launched as a
// programmatic dependent of the partial pass: it may start while that grid
// drains and waits for it here.
constexpr int kMergeThreads = 128;
constexpr int kMergeMaxGroup = 64;
constexpr int kMergeMaxPerLane = 16;  // head_dim <= 512
constexpr int kMergeRound = 4;        // records per round of float4 loads
constexpr int kMergeSmemRecords = 512;  // records per unit whose weights are staged in smem
constexpr int kMergeHeld = 16;  // records per lane group held in registers by the one-round path
constexpr int kMergeAppendPerThread = 4;  // head_dim <= 512 over kMergeThreads threads

__global__ void __launch_bounds__(kMergeThreads) merge(const Args a) {
  launch_dependents();
  const Partition pt = a.pt;
  const uint32_t out_unit = blockIdx.x;  // seq * kv_heads + kvh
  const uint32_t seq = out_unit / a.kv_heads, kvh = out_unit % a.kv_heads;
  const bool grouped = pt.heads > 1;
  const uint32_t unit = grouped ? seq : out_unit, head = grouped ? kvh : 0u;
  const uint32_t G = a.group, D = a.head_dim;
  // This CTA's columns [d0, d1) of head_dim.
  const uint32_t slice = D / gridDim.y, d0 = blockIdx.y * slice, d1 = d0 + slice;
  // 32-bit partition arithmetic: the plan keeps the tile count within 32 bits
  // (the host rejects more), so (unit + 1) * tiles_per_unit and the first
  // tile of a worker that holds records both fit.
  const uint32_t tpu = pt.tiles_per_unit, tpw = pt.tiles_per_worker;
  const uint32_t w_lo = unit * tpu / tpw;
  const uint32_t w_hi = ((unit + 1) * tpu - 1) / tpw;
  const uint32_t n = w_hi - w_lo + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Record i of the unit is worker w_lo + i's.  Every worker after w_lo
  // starts inside this unit (w * tiles_per_worker > unit * tiles_per_unit),
  // so its record is slot 0 of its span: the records from i = 1 on are
  // evenly spaced, and only record 0 needs the general index (slot
  // unit - first_unit(w_lo)).
  const uint32_t slot0 = unit - w_lo * tpw / tpu;
  const float *rec0 =
      a.records + ((uint64_t(w_lo) * pt.max_span + slot0) * pt.heads + head) * a.record_floats;
  const float *rec1 = a.records + (uint64_t(w_lo) * pt.max_span * pt.heads + head) * a.record_floats;
  const size_t rstep = size_t(pt.max_span) * pt.heads * a.record_floats;
  auto record = [&](uint32_t i) { return i == 0 ? rec0 : rec1 + i * rstep; };
  // float4 path: every head's output row starts on a 16-byte boundary
  // (records are, and 2G and D are multiples of 4), the slice is whole
  // float4 columns and the fp16 output rows start on an 8-byte boundary.
  const bool vec = ((2 * G) & 3u) == 0 && (D & 3u) == 0 && (slice & 3u) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.out) & 7u) == 0;
  // Up to kMergeSmemRecords records per unit: the warp stages every record's
  // max and sum in shared memory with independent loads, then turns them into
  // weights there, so the output sums below read weights from shared memory
  // instead of chaining a global load per record.
  __shared__ float staged[kMergeThreads / 32][2][kMergeSmemRecords];
  const bool stage = n <= uint32_t(kMergeSmemRecords);
  // The slice's float4 columns, and the lane groups that sum interleaved
  // records (F a power of two below 32).
  const uint32_t F = (d1 - d0) / 4;
  const bool grouped_lanes = vec && F < 32 && (F & (F - 1)) == 0;
  const uint32_t R = grouped_lanes ? 32 / F : 1;
  const uint32_t g = grouped_lanes ? lane / F : 0, f = grouped_lanes ? lane % F : lane;
  const uint32_t c0 = d0 / 4;
  // Few records (at most 4 per lane, kMergeHeld per lane group): one round
  // of loads fetches every max, sum and output column the warp needs, so
  // the merge costs one trip to the partial pass's records in L2 instead of
  // one per dependent step.  Its per-lane addresses: lane l's headers are
  // records l + 32 s (hdr0 for s = 0, hdr1 + s * hstep after), lane group
  // g's output columns records g + R j (col0 for j = 0, col1 + j * jstep
  // after), the first `nj` of them valid.
  const bool one_round = grouped_lanes && n <= 128u && n <= R * uint32_t(kMergeHeld);
  // Addresses of records past the unit's last stay on record 0 (in bounds).
  const float *hdr1 = rec1 + size_t(lane) * rstep;
  const float *hdr0 = lane == 0 || uint32_t(lane) >= n ? rec0 : hdr1;
  const size_t hstep = 32 * rstep;
  const float *col1 = rec1 + size_t(g) * rstep + 2 * G + 4 * (c0 + f);
  const float *col0 = g == 0 || g >= n ? rec0 + 2 * G + 4 * (c0 + f) : col1;
  const size_t jstep = size_t(R) * rstep;
  const uint32_t nj = g < n ? (n - g + R - 1) / R : 0u;
  // Everything above depends only on the launch's arguments.  These operands
  // make the compiler finish it before the wait, while the partial pass
  // drains, instead of after it.
  // The folded KvAppend: this CTA's share is columns [d0, d1) of kv head
  // kvh of sequence seq's new K and V rows, loaded after the wait and stored
  // at the end (the load's latency hides under the merge).
  const bool append = a.k_new != nullptr || a.v_new != nullptr;
  const size_t new_at = seq * a.new_stride + size_t(kvh) * D;
  const size_t cache_at = seq * a.cache_stride + (size_t(a.keys - 1) * a.kv_heads + kvh) * D;
  asm volatile("" ::"l"(hdr0), "l"(hdr1), "l"(col0), "l"(col1), "r"(nj), "r"(n), "l"(rstep),
               "l"(new_at), "l"(cache_at));
  wait_primary();
  __half k_row[kMergeAppendPerThread], v_row[kMergeAppendPerThread];
#pragma unroll
  for (int r = 0; r < kMergeAppendPerThread; ++r) {
    const uint32_t d = d0 + threadIdx.x + r * kMergeThreads;
    k_row[r] = append && a.k_new && d < d1 ? a.k_new[new_at + d] : __half();
    v_row[r] = append && a.v_new && d < d1 ? a.v_new[new_at + d] : __half();
  }
  __half *out = a.out + (size_t(seq) * a.kv_heads * G + kvh * G) * D;
  for (uint32_t h = warp; one_round && h < G; h += kMergeThreads / 32) {
    float *sm_w = staged[warp][0];
    float mv[4], lv[4];
    float4 v[kMergeHeld];
#pragma unroll
    for (int s4 = 0; s4 < 4; ++s4) {
      const uint32_t i = lane + 32 * s4;
      const float *r = (s4 == 0 || i >= n ? hdr0 : hdr1 + s4 * hstep) + h;
      mv[s4] = i < n ? r[0] : -INFINITY;
      lv[s4] = i < n ? r[G] : 0.f;
    }
    const size_t hd = size_t(h) * D;
    // Only the lane group's nj records: the loops below stop there instead
    // of issuing the rest predicated off.
#pragma unroll
    for (int j = 0; j < kMergeHeld; ++j) {
      if (uint32_t(j) >= nj)
        break;
      const float *c = (j == 0 ? col0 : col1 + j * jstep) + hd;
      v[j] = *reinterpret_cast<const float4 *>(c);
    }
    float top = fmaxf(fmaxf(mv[0], mv[1]), fmaxf(mv[2], mv[3]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
      top = fmaxf(top, __shfl_xor_sync(0xffffffffu, top, off));
    float sum = 0.f;
#pragma unroll
    for (int s4 = 0; s4 < 4; ++s4) {
      const uint32_t i = lane + 32 * s4;
      if (i < n) {
        const float w = fast_exp2(mv[s4] - top);
        sm_w[i] = w;
        sum = fmaf(lv[s4], w, sum);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
      sum += __shfl_xor_sync(0xffffffffu, sum, off);
    __syncwarp();
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < kMergeHeld; ++j) {
      if (uint32_t(j) >= nj)
        break;
      const float w = sm_w[g + R * j];
      acc.x = fmaf(v[j].x, w, acc.x);
      acc.y = fmaf(v[j].y, w, acc.y);
      acc.z = fmaf(v[j].z, w, acc.z);
      acc.w = fmaf(v[j].w, w, acc.w);
    }
    for (uint32_t off = F; off < 32; off <<= 1) {
      acc.x += __shfl_xor_sync(0xffffffffu, acc.x, int(off));
      acc.y += __shfl_xor_sync(0xffffffffu, acc.y, int(off));
      acc.z += __shfl_xor_sync(0xffffffffu, acc.z, int(off));
      acc.w += __shfl_xor_sync(0xffffffffu, acc.w, int(off));
    }
    __syncwarp();  // the staged weights are rewritten for the warp's next head
    if (g == 0) {
      const float inv = 1.f / sum;
      *reinterpret_cast<uint2 *>(out + h * D + 4 * (c0 + f)) =
          make_uint2(pack_half2(acc.x * inv, acc.y * inv), pack_half2(acc.z * inv, acc.w * inv));
    }
  }
  for (uint32_t h = warp; !one_round && h < G; h += kMergeThreads / 32) {
    float *sm_w = staged[warp][0], *sm_l = staged[warp][1];
    float top = -INFINITY, sum = 0.f, w_own = 0.f;
    if (stage) {
#pragma unroll 4
      for (uint32_t i = lane; i < n; i += 32) {
        const float *r = record(i);
        const float m = r[h];
        sm_w[i] = m;
        sm_l[i] = r[G + h];
        top = fmaxf(top, m);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
        top = fmaxf(top, __shfl_xor_sync(0xffffffffu, top, off));
      for (uint32_t i = lane; i < n; i += 32) {
        const float w = fast_exp2(sm_w[i] - top);
        sm_w[i] = w;
        sum = fmaf(sm_l[i], w, sum);
      }
      __syncwarp();
    } else {
      float m_own = -INFINITY, l_own = 0.f;
      if (uint32_t(lane) < n) {
        const float *r = record(lane);
        m_own = r[h];
        l_own = r[G + h];
      }
      top = m_own;
      for (uint32_t i = lane + 32; i < n; i += 32)
        top = fmaxf(top, record(i)[h]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
        top = fmaxf(top, __shfl_xor_sync(0xffffffffu, top, off));
      w_own = uint32_t(lane) < n ? fast_exp2(m_own - top) : 0.f;
      sum = l_own * w_own;
      for (uint32_t i = lane + 32; i < n; i += 32) {
        const float *r = record(i);
        sum = fmaf(r[G + h], fast_exp2(r[h] - top), sum);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
      sum += __shfl_xor_sync(0xffffffffu, sum, off);
    // Record i's weight; every lane of the warp calls this (it shuffles).
    auto weight = [&](uint32_t i) {
      if (stage)
        return i < n ? sm_w[i] : 0.f;
      const float w = __shfl_sync(0xffffffffu, w_own, int(i & 31u));
      return i < 32 ? w : (i < n ? fast_exp2(record(i)[h] - top) : 0.f);
    };
    const float inv = 1.f / sum;
    if (vec) {
      float4 acc[kMergeMaxPerLane / 4];
#pragma unroll
      for (int k = 0; k < kMergeMaxPerLane / 4; ++k)
        acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (grouped_lanes) {
        // One float4 column per lane: eight records' loads per round.
        constexpr int kWide = 2 * kMergeRound;
        for (uint32_t i0 = 0; i0 < n; i0 += R * kWide) {
          float4 v[kWide];
          float w[kWide];
#pragma unroll
          for (int j = 0; j < kWide; ++j) {
            const uint32_t i = i0 + g + R * j;
            w[j] = weight(i);
            v[j] = i < n ? reinterpret_cast<const float4 *>(record(i) + 2 * G + h * D)[c0 + f]
                         : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int j = 0; j < kWide; ++j) {
            acc[0].x = fmaf(v[j].x, w[j], acc[0].x);
            acc[0].y = fmaf(v[j].y, w[j], acc[0].y);
            acc[0].z = fmaf(v[j].z, w[j], acc[0].z);
            acc[0].w = fmaf(v[j].w, w[j], acc[0].w);
          }
        }
      }
      for (uint32_t i0 = 0; !grouped_lanes && i0 < n; i0 += R * kMergeRound) {
        float4 v[kMergeRound][kMergeMaxPerLane / 4];
        float w[kMergeRound];
#pragma unroll
        for (int j = 0; j < kMergeRound; ++j) {
          const uint32_t i = i0 + g + R * j;
          w[j] = weight(i);
          const float4 *o =
              reinterpret_cast<const float4 *>(record(min(i, n - 1)) + 2 * G + h * D);
#pragma unroll
          for (int k = 0; k < kMergeMaxPerLane / 4; ++k) {
            const uint32_t c = f + 32 * k;
            v[j][k] = (i < n && c < F) ? o[c0 + c] : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
#pragma unroll
        for (int j = 0; j < kMergeRound; ++j)
#pragma unroll
          for (int k = 0; k < kMergeMaxPerLane / 4; ++k) {
            acc[k].x = fmaf(v[j][k].x, w[j], acc[k].x);
            acc[k].y = fmaf(v[j][k].y, w[j], acc[k].y);
            acc[k].z = fmaf(v[j][k].z, w[j], acc[k].z);
            acc[k].w = fmaf(v[j][k].w, w[j], acc[k].w);
          }
      }
      // Sum the record groups (lanes f, f + F, f + 2F, ...).
      for (uint32_t off = F; grouped_lanes && off < 32; off <<= 1) {
        acc[0].x += __shfl_xor_sync(0xffffffffu, acc[0].x, int(off));
        acc[0].y += __shfl_xor_sync(0xffffffffu, acc[0].y, int(off));
        acc[0].z += __shfl_xor_sync(0xffffffffu, acc[0].z, int(off));
        acc[0].w += __shfl_xor_sync(0xffffffffu, acc[0].w, int(off));
      }
      __syncwarp();  // the staged weights are rewritten for the warp's next head
      if (g == 0) {
#pragma unroll
        for (int k = 0; k < kMergeMaxPerLane / 4; ++k) {
          const uint32_t c = f + 32 * k;
          if (c < F)
            *reinterpret_cast<uint2 *>(out + h * D + 4 * (c0 + c)) =
                make_uint2(pack_half2(acc[k].x * inv, acc[k].y * inv),
                           pack_half2(acc[k].z * inv, acc[k].w * inv));
        }
      }
    } else {
      float acc[kMergeMaxPerLane];
#pragma unroll
      for (int k = 0; k < kMergeMaxPerLane; ++k)
        acc[k] = 0.f;
#pragma unroll 2
      for (uint32_t i = 0; i < n; ++i) {
        const float w = weight(i);
        const float *o = record(i) + 2 * G + h * D;
#pragma unroll
        for (int k = 0; k < kMergeMaxPerLane; ++k) {
          const uint32_t d = d0 + lane + 32 * k;
          if (d < d1)
            acc[k] = fmaf(o[d], w, acc[k]);
        }
      }
      __syncwarp();  // the staged weights are rewritten for the warp's next head
#pragma unroll
      for (int k = 0; k < kMergeMaxPerLane; ++k) {
        const uint32_t d = d0 + lane + 32 * k;
        if (d < d1)
          out[h * D + d] = __float2half_rn(acc[k] * inv);
      }
    }
  }
  if (append) {
#pragma unroll
    for (int r = 0; r < kMergeAppendPerThread; ++r) {
      const uint32_t d = d0 + threadIdx.x + r * kMergeThreads;
      if (d < d1) {
        if (a.k_new)
          const_cast<__half *>(a.k)[cache_at + d] = k_row[r];
        if (a.v_new)
          const_cast<__half *>(a.v)[cache_at + d] = v_row[r];
      }
    }
  }
}

}  // namespace decode
}  // namespace llmi
