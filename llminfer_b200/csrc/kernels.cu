// C ABI of the attention kernels (declared in include/llmi_cuda.h).
//
// All device code is compiled in this one translation unit so that the
// device error word is a single symbol.  Each entry point validates its
// arguments before launching anything, picks the kernel for the shape, and
// reports launch errors through the status / last-error convention.
#include "llmi_cuda.h"

#include <cstdlib>

#include "cache_append.cuh"
#include "common.cuh"
#include "delta_chunk_solve.cuh"
#include "delta_chunk_tc.cuh"
#include "delta_recurrent.cuh"
#include "gqa_decode.cuh"
#include "gqa_flash_simt.cuh"
#include "gqa_prefill_tc.cuh"
#include "gqa_prefill_tc2.cuh"
#include "producers.cuh"
#include "host/status.h"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <mutex>
#include <utility>
#include <vector>

using namespace llmi;

namespace {

constexpr float kLog2e = 1.4426950408889634f;

cudaStream_t as_stream(void *stream) { return static_cast<cudaStream_t>(stream); }

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Raises a kernel's dynamic shared-memory limit to at least `bytes` on the
// current device; the largest limit set so far is remembered per
// (kernel, device) so the driver call is made only when it grows.
int allow_smem(const void *kernel, size_t bytes, const DeviceInfo &dev) {
  struct Entry {
    const void *kernel;
    int device;
    size_t bytes;
  };
  static std::mutex mutex;
  static std::vector<Entry> granted;
  if (bytes > dev.max_smem_optin)
    return fail(LLMI_UNSUPPORTED, "kernel needs %zu B of shared memory, device allows %zu", bytes,
                dev.max_smem_optin);
  std::lock_guard<std::mutex> lock(mutex);
  Entry *entry = nullptr;
  for (auto &e : granted)
    if (e.kernel == kernel && e.device == dev.device)
      entry = &e;
  if (entry && entry->bytes >= bytes)
    return LLMI_OK;
  if (int s = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              int(bytes)),
                         "cudaFuncSetAttribute"))
    return s;
  if (entry)
    entry->bytes = bytes;
  else
    granted.push_back({kernel, dev.device, bytes});
  return LLMI_OK;
}

int launched(const char *kernel) {
  return check_cuda(cudaGetLastError(), kernel);
}

// Decode-path kernels launch as programmatic dependents unless
// LLMI_PROGRAMMATIC_LAUNCH=0 (read once per process); the kernels are the same
// either way.
bool programmatic_launch() {
  static const bool on = [] {
    const char *e = std::getenv("LLMI_PROGRAMMATIC_LAUNCH");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Launches a decode-path kernel as a programmatic dependent of the work before
// it on the stream (the kernel calls pdl_enter() at entry): its launch and CTA
// ramp overlap the previous kernel's tail.  Recorded into CUDA graphs as a
// programmatic edge.
template <typename... Params, typename... Actual>
int launch_dependent(const char *name, void (*kernel)(Params...), dim3 grid, dim3 block,
                     size_t smem, cudaStream_t stream, Actual &&...args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attr;
  config.numAttrs = programmatic_launch() ? 1 : 0;
  if (int e = check_cuda(cudaLaunchKernelEx(&config, kernel, std::forward<Actual>(args)...), name))
    return e;
  return launched(name);
}

int check_gqa(const llmi_gqa_params *p, unsigned batch, const void *q, const void *k,
              const void *v, size_t cache_stride, const void *out) {
  if (!p || !q || !k || !v || !out)
    return fail(LLMI_INVALID_ARGUMENT, "GQA: null parameter or tensor pointer");
  if (!batch || !p->tokens || !p->queryHeads || !p->kvHeads || !p->headDim)
    return fail(LLMI_INVALID_ARGUMENT, "GQA: batch, tokens, heads and head_dim must be positive");
  if (p->queryHeads % p->kvHeads)
    return fail(LLMI_INVALID_ARGUMENT, "GQA: %u query heads are not a multiple of %u kv heads",
                p->queryHeads, p->kvHeads);
  const uint64_t rows = uint64_t(p->past) + p->tokens;
  if (rows > UINT32_MAX)
    return fail(LLMI_INVALID_ARGUMENT, "GQA: past + tokens exceeds 32 bits");
  if (batch > 1 && cache_stride < rows * p->kvHeads * p->headDim)
    return fail(LLMI_INVALID_ARGUMENT,
                "GQA: cache stride %zu cannot hold %llu rows of %u x %u", cache_stride,
                (unsigned long long)rows, p->kvHeads, p->headDim);
  return LLMI_OK;
}

// ---- decode planning -------------------------------------------------------

struct DecodePlan {
  enum Kind { Rows256x4, Rows256x2, Rows128x8, Mma256, Mma128, Mma64, Simt } kind = Simt;
  bool cta_workers = false;  // Mma kinds with heads == 1: partial_mma_cta
  decode::Partition pt{};
  uint32_t record_floats = 0;
  uint32_t grid = 0, threads = 0;
  size_t smem = 0;
  size_t workspace = 0;
};

constexpr int kWarps256 = 4, kStages256 = 3;
constexpr int kWarps128 = 8, kStages128 = 3;
constexpr int kWarps64 = 8, kStages64 = 4;
// partial_mma_cta keeps one record-sized state slot per warp in shared
// memory beside the copy rings, so its rings are shorter for D 256 and 128.
constexpr int kCtaStages256 = 1, kCtaStages128 = 2, kCtaStages64 = 4;
// Warps per CTA of partial_mma_cta: for D 256 eight warps with one stage each
// keep as many bytes in flight as four with two, and twice the warps hide
// the latency of the tile math.
constexpr int kCtaWarps256 = 8, kCtaWarps128 = kWarps128, kCtaWarps64 = kWarps64;
constexpr int kRowStages = 3;
// Bytes of cache rows the CTA workers of the decode partial pass warm L2
// with, over the whole grid, before waiting for the kernel ahead of them
// (16 MB: about two tiles per warp at the shapes that use them, and well
// inside L2).  The whole-row kinds warm nothing: each CTA puts three 64 KB
// tiles in flight at once, and prefetches beside them only competed with
// those copies (a B=2, 16/4-head step took 1.5 us longer with them).
constexpr uint64_t kDecodePrefetchBytes = 16ull << 20;
// DeltaUpdate calls with at least this many tokens use the chunked kernel.
constexpr uint32_t kChunkedMinTokens = 16;

// Tiles per CTA worker to warm L2 with: at most 16 and at most
// kDecodePrefetchBytes over the grid.  `tile_bytes`: the K and V rows a
// worker reads for one tile.
uint32_t prefetch_tiles(const DecodePlan &plan, uint64_t tile_bytes) {
  const uint64_t round = std::max<uint64_t>(1, uint64_t(plan.grid) * tile_bytes);
  return uint32_t(std::min<uint64_t>({uint64_t(plan.pt.tiles_per_worker), 16ull,
                                      kDecodePrefetchBytes / round}));
}

// Picks the decode kernels and the work partition.  The tensor-core partial
// pass needs 16-byte aligned operands (bulk copies) and a supported shape;
// everything else takes the CUDA-core pass.
int plan_decode(const llmi_gqa_params &p, unsigned batch, bool aligned, const DeviceInfo &dev,
                DecodePlan &plan) {
  const uint32_t D = p.headDim, G = p.queryHeads / p.kvHeads;
  const uint32_t keys = p.past + 1;
  const uint32_t units = batch * p.kvHeads;
  plan.record_floats = decode::record_floats(G, D);
  const bool fits = G <= 8 && (D == 256 || D == 128 || D == 64);
  const bool rows = fits && aligned &&
                    ((D == 256 && (p.kvHeads == 4 || p.kvHeads == 2)) || (D == 128 && p.kvHeads == 8));
  // CTAs per SM: one for 2 KiB rows, two for the 1 KiB rows of 2 kv heads
  // (their CTAs have half the consumer warps and half the shared memory).
  uint32_t ctas_per_sm = 1;
  if (rows) {
    // Whole cache rows (every kv head of one key) per bulk copy; the CTA is
    // the worker.
    if (D == 256 && p.kvHeads == 4) {
      plan.kind = DecodePlan::Rows256x4;
      plan.threads = decode::RowShape<256, 4, kRowStages>::kThreads;
      plan.smem = decode::RowShape<256, 4, kRowStages>::kSmemBytes;
    } else if (D == 256) {
      plan.kind = DecodePlan::Rows256x2;
      plan.threads = decode::RowShape<256, 2, kRowStages>::kThreads;
      plan.smem = decode::RowShape<256, 2, kRowStages>::kSmemBytes;
      ctas_per_sm = 2;
    } else {
      plan.kind = DecodePlan::Rows128x8;
      plan.threads = decode::RowShape<128, 8, kRowStages>::kThreads;
      plan.smem = decode::RowShape<128, 8, kRowStages>::kSmemBytes;
    }
    const uint32_t tpu = (keys + decode::kTileKeys - 1) / decode::kTileKeys;
    const uint64_t tiles = uint64_t(batch) * tpu;
    if (tiles > UINT32_MAX)
      return fail(LLMI_UNSUPPORTED, "decode: %llu key tiles exceed 32 bits",
                  (unsigned long long)tiles);
    const uint64_t workers_max = uint64_t(dev.sm_count) * ctas_per_sm;
    const uint32_t tpw = uint32_t((tiles + workers_max - 1) / workers_max);
    plan.grid = uint32_t((tiles + tpw - 1) / tpw);
    plan.pt.units = batch;
    plan.pt.tiles_per_unit = tpu;
    plan.pt.tiles_per_worker = tpw;
    plan.pt.max_span = std::min<uint32_t>(batch, (tpw + tpu - 1) / tpu + 1);
    plan.pt.workers = plan.grid;
    plan.pt.heads = p.kvHeads;
  } else if (fits && aligned) {
    int warps, smem;
    if (D == 256) {
      plan.kind = DecodePlan::Mma256;
      warps = kWarps256;
      smem = decode::MmaShape<256, kWarps256, kStages256>::kSmemBytes;
    } else if (D == 128) {
      plan.kind = DecodePlan::Mma128;
      warps = kWarps128;
      smem = decode::MmaShape<128, kWarps128, kStages128>::kSmemBytes;
    } else {
      plan.kind = DecodePlan::Mma64;
      warps = kWarps64;
      smem = decode::MmaShape<64, kWarps64, kStages64>::kSmemBytes;
    }
    // When the kv heads match the warps of a CTA, the CTA is the worker and
    // its warps stream the same key rows of all kv heads (whole cache rows).
    // Otherwise the CTA is still the worker (partial_mma_cta): its warps take
    // a unit's tiles in turn and combine into one record, which keeps the
    // records per unit few when a GPU holds few sequences or kv heads.
    const bool grouped = p.kvHeads == uint32_t(warps);
    const uint32_t part_units = grouped ? batch : units;
    const uint32_t per_cta = 1u;
    plan.cta_workers = !grouped;
    if (!grouped) {
      const size_t floats = plan.record_floats;
      smem = int(D == 256   ? decode::MmaCtaShape<256, kCtaWarps256, kCtaStages256>::smem_bytes(floats)
                 : D == 128 ? decode::MmaCtaShape<128, kCtaWarps128, kCtaStages128>::smem_bytes(floats)
                            : decode::MmaCtaShape<64, kCtaWarps64, kCtaStages64>::smem_bytes(floats));
      warps = D == 256 ? kCtaWarps256 : D == 128 ? kCtaWarps128 : kCtaWarps64;
    }
    const uint32_t tpu = (keys + decode::kTileKeys - 1) / decode::kTileKeys;
    const uint64_t tiles = uint64_t(part_units) * tpu;
    if (tiles > UINT32_MAX)
      return fail(LLMI_UNSUPPORTED, "decode: %llu key tiles exceed 32 bits",
                  (unsigned long long)tiles);
    const uint64_t workers_max = uint64_t(dev.sm_count) * per_cta;
    const uint32_t tpw = uint32_t((tiles + workers_max - 1) / workers_max);
    const uint32_t busy = uint32_t((tiles + tpw - 1) / tpw);
    plan.grid = (busy + per_cta - 1) / per_cta;
    plan.threads = warps * 32;
    plan.smem = size_t(smem);
    plan.pt.units = part_units;
    plan.pt.tiles_per_unit = tpu;
    plan.pt.tiles_per_worker = tpw;
    plan.pt.max_span = std::min<uint32_t>(part_units, (tpw + tpu - 1) / tpu + 1);
    plan.pt.workers = plan.grid * per_cta;
    plan.pt.heads = grouped ? p.kvHeads : 1u;
    if (plan.cta_workers)
      plan.pt.prefetch_tiles = prefetch_tiles(plan, 2ull * decode::kTileKeys * D * 2);
  } else {
    if (D > 512)
      return fail(LLMI_UNSUPPORTED, "decode: head_dim %u above 512", D);
    plan.kind = DecodePlan::Simt;
    // Enough (unit, split) CTAs to fill the GPU, but at least kSimtMinKeys
    // keys per split, so that the merge walks few records per unit.
    const uint32_t want = (4u * dev.sm_count + units - 1) / units;
    const uint32_t splits =
        std::max(1u, std::min((keys + decode::kSimtMinKeys - 1) / decode::kSimtMinKeys, want));
    plan.pt.units = units;
    plan.pt.tiles_per_unit = splits;
    plan.pt.tiles_per_worker = 1;
    plan.pt.max_span = 1;
    plan.pt.workers = units * splits;
    plan.pt.heads = 1;
    plan.grid = plan.pt.workers;
    plan.threads = 128;
    plan.smem = 0;
  }
  if (G > uint32_t(decode::kMergeMaxGroup))
    return fail(LLMI_UNSUPPORTED, "decode: %u query heads per kv head (at most %d)", G,
                decode::kMergeMaxGroup);
  plan.workspace = size_t(plan.pt.workers) * plan.pt.max_span * plan.pt.heads *
                   plan.record_floats * sizeof(float);
  return LLMI_OK;
}

// ---- TMA tensor maps ----------------------------------------------------------

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library does not link libcuda directly.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult result;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &result) !=
            cudaSuccess ||
        result != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// 4-D fp16 tensor map with 128-byte swizzle and zero fill out of bounds.
// dims/box innermost first; strides in bytes for dims 1..3.
int encode_map_4d(CUtensorMap *map, const void *base, const uint64_t (&dims)[4],
                  const uint64_t (&strides)[3], const uint32_t (&box)[4]) {
  auto encode = tensor_map_encoder();
  if (!encode)
    return fail(LLMI_CUDA_ERROR, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t s[3] = {strides[0], strides[1], strides[2]};
  cuuint32_t b[4] = {box[0], box[1], box[2], box[3]};
  cuuint32_t e[4] = {1, 1, 1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void *>(base), d,
                            s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(LLMI_CUDA_ERROR, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return LLMI_OK;
}

// 3-D tensor map (no swizzle: row-major staging), zero fill out of bounds.
// dims/box innermost first; strides in bytes for dims 1..2.
int encode_map_3d(CUtensorMap *map, CUtensorMapDataType type, const void *base,
                  const uint64_t (&dims)[3], const uint64_t (&strides)[2],
                  const uint32_t (&box)[3],
                  CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
  auto encode = tensor_map_encoder();
  if (!encode)
    return fail(LLMI_CUDA_ERROR, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t s[2] = {strides[0], strides[1]};
  cuuint32_t b[3] = {box[0], box[1], box[2]};
  cuuint32_t e[3] = {1, 1, 1};
  const CUresult r = encode(map, type, 3, const_cast<void *>(base), d, s, b, e,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(LLMI_CUDA_ERROR, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return LLMI_OK;
}

// The tensor-core prefill runs on CTA pairs (cta_group::2 MMAs, half of
// each K/V tile per CTA): 1.3x the single-CTA kernel's rate at long
// prompts.  LLMI_PREFILL_CTA_PAIRS=0 selects the single-CTA kernel; the
// variable is read once per process.
bool prefill_on_pairs() {
  static const bool on = [] {
    const char *e = std::getenv("LLMI_PREFILL_CTA_PAIRS");
    return !(e && e[0] == '0');
  }();
  return on;
}

// The tensor-core prefill applies to head_dim 256 with a query group that
// divides the 128-row tile, 16-byte aligned operands and cache strides.
bool prefill_tc_fits(const llmi_gqa_params &p, unsigned batch, const void *q, const void *k,
                     const void *v, size_t cache_stride, const void *out) {
  const uint32_t G = p.queryHeads / p.kvHeads;
  return p.headDim == uint32_t(prefill_tc::kD) && G <= uint32_t(prefill_tc::kRows) &&
         prefill_tc::kRows % G == 0 && aligned16(q) && aligned16(k) && aligned16(v) &&
         aligned16(out) && (batch == 1 || cache_stride % 8 == 0) && batch <= 65535 &&
         p.kvHeads <= 65535;
}

// The prefill's tensor maps.  caches [batch][rows][Hkv][D] at sequence
// stride cache_stride: single CTAs stage K boxes of 64 dims x 1 head x 128
// keys and V boxes of 32 keys; each CTA of a pair stages K boxes of 64 keys
// and V boxes of 128 keys.  q [batch][tokens][Hq][D]: a box is the CTA's 128
// rows (G heads x 128/G tokens) x 64 dims, rows in (token, head) order.
int encode_prefill_maps(const llmi_gqa_params &p, unsigned batch, const uint16_t *q,
                        const uint16_t *k, const uint16_t *v, size_t cache_stride, bool pairs,
                        CUtensorMap &mq, CUtensorMap &mk, CUtensorMap &mv) {
  using namespace prefill_tc;
  const uint32_t G = p.queryHeads / p.kvHeads;
  const uint32_t rows = p.past + p.tokens;
  const uint64_t D = kD;
  {
    const uint64_t seq_bytes =
        batch > 1 ? uint64_t(cache_stride) * 2 : uint64_t(rows) * p.kvHeads * D * 2;
    const uint64_t dims[4] = {D, p.kvHeads, rows, batch};
    const uint64_t strides[3] = {D * 2, uint64_t(p.kvHeads) * D * 2, seq_bytes};
    const uint32_t kbox[4] = {64, 1, uint32_t(pairs ? prefill_tc2::kHalfKeys : kKeys), 1};
    const uint32_t vbox[4] = {64, 1, uint32_t(pairs ? prefill_tc2::kKeys : kVKeys), 1};
    if (int s = encode_map_4d(&mk, k, dims, strides, kbox))
      return s;
    if (int s = encode_map_4d(&mv, v, dims, strides, vbox))
      return s;
  }
  const uint64_t dims[4] = {D, p.queryHeads, p.tokens, batch};
  const uint64_t strides[3] = {D * 2, uint64_t(p.queryHeads) * D * 2,
                               uint64_t(p.tokens) * p.queryHeads * D * 2};
  const uint32_t box[4] = {64, G, uint32_t(kRows) / G, 1};
  return encode_map_4d(&mq, q, dims, strides, box);
}

// The prefill's three tensor maps for one call's operands.  Encoding them
// costs the host several microseconds per call, which dominates short
// prefills, so each thread keeps the maps of its last few distinct calls
// (same pointers, shape and cache stride: a serving loop or a replayed
// capture repeats them) and reuses them.
struct PrefillMaps {
  const void *q, *k, *v;
  int device;
  uint32_t tokens, past, query_heads, kv_heads;
  unsigned batch;
  size_t cache_stride;
  bool pairs;
  CUtensorMap mq, mk, mv;

  bool same(const PrefillMaps &o) const {
    return q == o.q && k == o.k && v == o.v && device == o.device && tokens == o.tokens &&
           past == o.past && query_heads == o.query_heads && kv_heads == o.kv_heads &&
           batch == o.batch && cache_stride == o.cache_stride && pairs == o.pairs;
  }
};

int launch_prefill_tc(const llmi_gqa_params &p, unsigned batch, const uint16_t *q,
                      const uint16_t *k, const uint16_t *v, size_t cache_stride, uint16_t *out,
                      const DeviceInfo &dev, cudaStream_t stream) {
  using namespace prefill_tc;
  const uint32_t G = p.queryHeads / p.kvHeads;
  const bool pairs = prefill_on_pairs();
  constexpr int kCached = 8;
  thread_local PrefillMaps cache[kCached];
  thread_local int cached = 0, next_slot = 0;
  PrefillMaps key{};
  key.q = q;
  key.k = k;
  key.v = v;
  key.device = dev.device;
  key.tokens = p.tokens;
  key.past = p.past;
  key.query_heads = p.queryHeads;
  key.kv_heads = p.kvHeads;
  key.batch = batch;
  key.cache_stride = batch > 1 ? cache_stride : 0;
  key.pairs = pairs;
  const PrefillMaps *hit = nullptr;
  for (int i = 0; i < cached && !hit; ++i)
    if (cache[i].same(key))
      hit = &cache[i];
  CUtensorMap mq, mk, mv;
  if (hit) {
    mq = hit->mq;
    mk = hit->mk;
    mv = hit->mv;
  } else {
    if (int s = encode_prefill_maps(p, batch, q, k, v, cache_stride, pairs, mq, mk, mv))
      return s;
    key.mq = mq;
    key.mk = mk;
    key.mv = mv;
    cache[next_slot] = key;
    next_slot = (next_slot + 1) % kCached;
    cached = std::min(cached + 1, kCached);
  }
  Args a;
  a.out = reinterpret_cast<__half *>(out);
  a.tokens = p.tokens;
  a.q_heads = p.queryHeads;
  a.kv_heads = p.kvHeads;
  a.group = G;
  a.past = p.past;
  a.tok_per_tile = kRows / G;
  a.tiles_per_head = (p.tokens + a.tok_per_tile - 1) / a.tok_per_tile;
  a.scale_log2 = kLog2e / std::sqrt(float(kD));
  if (pairs) {
    a.tiles_per_head += a.tiles_per_head & 1u;
    auto kernel = prefill_tc2::gqa_prefill_pair;
    if (int s = allow_smem(reinterpret_cast<const void *>(kernel), prefill_tc2::Smem::alloc, dev))
      return s;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.tiles_per_head, p.kvHeads, batch);
    cfg.blockDim = dim3(prefill_tc2::kThreads);
    cfg.dynamicSmemBytes = prefill_tc2::Smem::alloc;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (int s = check_cuda(cudaLaunchKernelEx(&cfg, kernel, mq, mk, mv, a), "cudaLaunchKernelEx"))
      return s;
    return launched("gqaFlashAttention (tensor cores, CTA pairs)");
  }
  if (int s = allow_smem(reinterpret_cast<const void *>(gqa_prefill_tcgen05), Smem::alloc, dev))
    return s;
  dim3 grid(a.tiles_per_head, p.kvHeads, batch);
  gqa_prefill_tcgen05<<<grid, kThreads, Smem::alloc, stream>>>(mq, mk, mv, a);
  return launched("gqaFlashAttention (tensor cores)");
}

template <int D, int HKV, int STAGES>
int launch_decode_rows(const DecodePlan &plan, const decode::Args &args, const DeviceInfo &dev,
                       cudaStream_t stream) {
  auto kernel = decode::partial_rows<D, HKV, STAGES>;
  if (int s = allow_smem(reinterpret_cast<const void *>(kernel), plan.smem, dev))
    return s;
  return launch_dependent("gqaScores (decode partial, row stream)", kernel, plan.grid,
                          plan.threads, plan.smem, stream, args);
}

template <int D, int WARPS, int STAGES, int CTA_WARPS, int CTA_STAGES>
int launch_decode_mma(const DecodePlan &plan, const decode::Args &args, const DeviceInfo &dev,
                      cudaStream_t stream) {
  if (plan.cta_workers) {
    auto kernel = decode::partial_mma_cta<D, CTA_WARPS, CTA_STAGES>;
    if (int s = allow_smem(reinterpret_cast<const void *>(kernel), plan.smem, dev))
      return s;
    return launch_dependent("gqaScores (decode partial, tensor cores, CTA workers)", kernel,
                            plan.grid, plan.threads, plan.smem, stream, args);
  }
  auto kernel = decode::partial_mma<D, WARPS, STAGES>;
  if (int s = allow_smem(reinterpret_cast<const void *>(kernel), plan.smem, dev))
    return s;
  return launch_dependent("gqaScores (decode partial, tensor cores)", kernel, plan.grid,
                          plan.threads, plan.smem, stream, args);
}

}  // namespace

// ---- cacheAppend -------------------------------------------------------------

extern "C" int llmi_cuda_cache_append(const llmi_cache_params *p, unsigned batch,
                                      const uint16_t *input, size_t input_stride,
                                      uint16_t *cache, size_t cache_stride, void *stream) {
  clear_error();
  if (!p || !input || !cache || !batch)
    return fail(LLMI_INVALID_ARGUMENT, "cacheAppend: null pointer or zero batch");
  if (p->count == 0)
    return LLMI_OK;
  if (batch > 1 && (input_stride < p->count || cache_stride < uint64_t(p->offset) + p->count))
    return fail(LLMI_INVALID_ARGUMENT, "cacheAppend: sequence strides overlap");
  AppendArgs a{input, cache, input_stride, cache_stride, p->count, p->offset, batch};
  const bool vec = p->count % 8 == 0 && p->offset % 8 == 0 && aligned16(input) &&
                   aligned16(cache) && (batch == 1 || (input_stride % 8 == 0 && cache_stride % 8 == 0));
  const uint64_t work = vec ? uint64_t(p->count / 8) * batch : uint64_t(p->count) * batch;
  const uint32_t grid = uint32_t(std::min<uint64_t>((work + 255) / 256, 4096));
  return launch_dependent("cacheAppend", vec ? cache_append_v8 : cache_append_scalar, grid, 256,
                          0, as_stream(stream), a);
}

// ---- gqaFlashAttention ------------------------------------------------------------

extern "C" int llmi_cuda_gqa_prefill(const llmi_gqa_params *p, unsigned batch,
                                     const uint16_t *q, const uint16_t *k_cache,
                                     const uint16_t *v_cache, size_t cache_stride,
                                     uint16_t *out, void *stream) {
  clear_error();
  if (int s = check_gqa(p, batch, q, k_cache, v_cache, cache_stride, out))
    return s;
  DeviceInfo dev;
  if (int s = current_device(dev))
    return s;
  if (prefill_tc_fits(*p, batch, q, k_cache, v_cache, cache_stride, out))
    return launch_prefill_tc(*p, batch, q, k_cache, v_cache, cache_stride, out, dev,
                             as_stream(stream));
  if (p->headDim > flash_simt::kMaxPerLane * 32)
    return fail(LLMI_UNSUPPORTED, "gqaFlashAttention: head_dim %u above 256", p->headDim);
  if (batch > 65535 || p->queryHeads > 65535)
    return fail(LLMI_UNSUPPORTED, "gqaFlashAttention: batch or heads above 65535");
  flash_simt::Args a;
  a.q = reinterpret_cast<const __half *>(q);
  a.k = reinterpret_cast<const __half *>(k_cache);
  a.v = reinterpret_cast<const __half *>(v_cache);
  a.cache_stride = cache_stride;
  a.out = reinterpret_cast<__half *>(out);
  a.tokens = p->tokens;
  a.q_heads = p->queryHeads;
  a.kv_heads = p->kvHeads;
  a.head_dim = p->headDim;
  a.past = p->past;
  a.group = p->queryHeads / p->kvHeads;
  a.scale_log2 = kLog2e / std::sqrt(float(p->headDim));
  const size_t smem = flash_simt::smem_bytes(p->headDim);
  if (int s = allow_smem(reinterpret_cast<const void *>(flash_simt::gqa_prefill_simt), smem, dev))
    return s;
  dim3 grid((p->tokens + flash_simt::kWarps - 1) / flash_simt::kWarps, p->queryHeads, batch);
  flash_simt::gqa_prefill_simt<<<grid, flash_simt::kWarps * 32, smem, as_stream(stream)>>>(a);
  return launched("gqaFlashAttention (CUDA cores)");
}

// ---- decode: gqaScores + gqaSoftmax ---------------------------------------------------

extern "C" size_t llmi_cuda_gqa_decode_workspace(const llmi_gqa_params *p, unsigned batch) {
  clear_error();
  if (!p || !batch || !p->queryHeads || !p->kvHeads || !p->headDim ||
      p->queryHeads % p->kvHeads) {
    fail(LLMI_INVALID_ARGUMENT, "decode workspace: invalid shape");
    return 0;
  }
  DeviceInfo dev;
  if (current_device(dev))
    return 0;
  // Operand alignment is not known yet: size for whichever pass runs.
  DecodePlan fast, simt;
  const int a = plan_decode(*p, batch, true, dev, fast);
  const int b = plan_decode(*p, batch, false, dev, simt);
  if (a && b)
    return 0;
  clear_error();
  return std::max(a ? 0 : fast.workspace, b ? 0 : simt.workspace);
}

namespace {

// A step's new K and V rows for the decode pass to append (each may be null).
struct NewRows {
  const uint16_t *k = nullptr, *v = nullptr;
  size_t stride = 0;  // halves between sequences
};

// gqaScores + gqaSoftmax, with the step's KvAppend folded in when `fresh`
// holds rows and the partial pass is a tensor-core one: that pass reads the
// new rows from `fresh` and the merge writes them into the caches.
// Otherwise the appends run first as their own launches.  Arguments checked.
int gqa_decode_run(const llmi_gqa_params *p, unsigned batch, const uint16_t *q,
                   const uint16_t *k_cache, const uint16_t *v_cache, size_t cache_stride,
                   uint16_t *out, void *workspace, size_t workspace_bytes, void *stream,
                   NewRows fresh, unsigned flags = 0) {
  if (!workspace)
    return fail(LLMI_INVALID_ARGUMENT, "decode: null workspace");
  DeviceInfo dev;
  if (int s = current_device(dev))
    return s;
  DecodePlan plan;
  const bool aligned = aligned16(q) && aligned16(k_cache) && aligned16(v_cache) &&
                       (batch == 1 || cache_stride % 8 == 0);
  if (int s = plan_decode(*p, batch, aligned, dev, plan))
    return s;
  if (workspace_bytes < plan.workspace)
    return fail(LLMI_WORKSPACE_TOO_SMALL, "decode: workspace of %zu B, %zu B needed",
                workspace_bytes, plan.workspace);
  if (!aligned16(workspace))
    return fail(LLMI_INVALID_ARGUMENT, "decode: workspace must be 16-byte aligned");
  if (fresh.k || fresh.v) {
    const bool fold = plan.kind != DecodePlan::Simt && (!fresh.k || aligned16(fresh.k)) &&
                      (!fresh.v || aligned16(fresh.v)) && (batch == 1 || fresh.stride % 8 == 0);
    if (!fold) {
      const unsigned row = p->kvHeads * p->headDim;
      llmi_cache_params c{row, p->past * row};
      const uint16_t *rows[2] = {fresh.k, fresh.v};
      const uint16_t *caches[2] = {k_cache, v_cache};
      for (int i = 0; i < 2; ++i)
        if (rows[i])
          if (int s = llmi_cuda_cache_append(&c, batch, rows[i], fresh.stride,
                                             const_cast<uint16_t *>(caches[i]), cache_stride,
                                             stream))
            return s;
      fresh = NewRows{};
    }
  }

  decode::Args a;
  a.q = reinterpret_cast<const __half *>(q);
  a.k = reinterpret_cast<const __half *>(k_cache);
  a.v = reinterpret_cast<const __half *>(v_cache);
  a.cache_stride = cache_stride;
  a.out = reinterpret_cast<__half *>(out);
  a.records = static_cast<float *>(workspace);
  a.pt = plan.pt;
  a.kv_heads = p->kvHeads;
  a.group = p->queryHeads / p->kvHeads;
  a.head_dim = p->headDim;
  a.keys = p->past + 1;
  a.record_floats = plan.record_floats;
  a.scale_log2 = kLog2e / std::sqrt(float(p->headDim));
  a.k_new = reinterpret_cast<const __half *>(fresh.k);
  a.v_new = reinterpret_cast<const __half *>(fresh.v);
  a.new_stride = fresh.stride;
  a.batch = batch;
  a.settled = (flags & LLMI_FLAG_SETTLED) ? 1u : 0u;
  cudaStream_t s = as_stream(stream);
  int status = LLMI_OK;
  switch (plan.kind) {
  case DecodePlan::Rows256x4:
    status = launch_decode_rows<256, 4, kRowStages>(plan, a, dev, s);
    break;
  case DecodePlan::Rows256x2:
    status = launch_decode_rows<256, 2, kRowStages>(plan, a, dev, s);
    break;
  case DecodePlan::Rows128x8:
    status = launch_decode_rows<128, 8, kRowStages>(plan, a, dev, s);
    break;
  case DecodePlan::Mma256:
    status = launch_decode_mma<256, kWarps256, kStages256, kCtaWarps256, kCtaStages256>(plan, a, dev, s);
    break;
  case DecodePlan::Mma128:
    status = launch_decode_mma<128, kWarps128, kStages128, kCtaWarps128, kCtaStages128>(plan, a, dev, s);
    break;
  case DecodePlan::Mma64:
    status = launch_decode_mma<64, kWarps64, kStages64, kCtaWarps64, kCtaStages64>(plan, a, dev, s);
    break;
  case DecodePlan::Simt:
    status = launch_dependent("gqaScores (decode partial, CUDA cores)", decode::partial_simt,
                              plan.grid, plan.threads, 0, s, a);
    break;
  }
  if (status)
    return status;
  // The merge may be scheduled while the partial grid drains; it waits for
  // it on the device.
  // head_dim slices per (sequence, kv head): enough merge CTAs for about two
  // per SM, each slice at least 16 columns and a whole number of float4s.
  const uint32_t units = batch * p->kvHeads;
  uint32_t slices = 1;
  while (uint64_t(units) * slices * 2 <= 2ull * uint64_t(dev.sm_count) &&
         p->headDim % (slices * 8) == 0 && p->headDim / (slices * 2) >= 16)
    slices *= 2;
  return launch_dependent("gqaSoftmax (decode merge)", decode::merge, dim3(units, slices),
                          dim3(decode::kMergeThreads), 0, s, a);
}

}  // namespace

extern "C" int llmi_cuda_gqa_decode(const llmi_gqa_params *p, unsigned batch, const uint16_t *q,
                                    const uint16_t *k_cache, const uint16_t *v_cache,
                                    size_t cache_stride, uint16_t *out, void *workspace,
                                    size_t workspace_bytes, void *stream) {
  clear_error();
  if (int s = check_gqa(p, batch, q, k_cache, v_cache, cache_stride, out))
    return s;
  if (p->tokens != 1)
    return fail(LLMI_UNSUPPORTED, "decode: %u tokens; the decode path takes one token (use prefill)",
                p->tokens);
  return gqa_decode_run(p, batch, q, k_cache, v_cache, cache_stride, out, workspace,
                        workspace_bytes, stream, NewRows{});
}

extern "C" int llmi_cuda_gqa_decode_append(const llmi_gqa_params *p, unsigned batch,
                                           const uint16_t *q, const uint16_t *k_new,
                                           const uint16_t *v_new, size_t new_stride,
                                           uint16_t *k_cache, uint16_t *v_cache,
                                           size_t cache_stride, uint16_t *out, void *workspace,
                                           size_t workspace_bytes, void *stream) {
  return llmi_cuda_gqa_decode_append_ex(p, batch, q, k_new, v_new, new_stride, k_cache, v_cache,
                                        cache_stride, out, workspace, workspace_bytes, stream, 0u);
}

extern "C" int llmi_cuda_gqa_decode_append_ex(const llmi_gqa_params *p, unsigned batch,
                                              const uint16_t *q, const uint16_t *k_new,
                                              const uint16_t *v_new, size_t new_stride,
                                              uint16_t *k_cache, uint16_t *v_cache,
                                              size_t cache_stride, uint16_t *out,
                                              void *workspace, size_t workspace_bytes,
                                              void *stream, unsigned flags) {
  clear_error();
  if (flags & ~LLMI_FLAG_SETTLED)
    return fail(LLMI_INVALID_ARGUMENT, "decode_append: unknown flags 0x%x", flags);
  if (int s = check_gqa(p, batch, q, k_cache, v_cache, cache_stride, out))
    return s;
  if (p->tokens != 1)
    return fail(LLMI_UNSUPPORTED, "decode_append: %u tokens; the decode path takes one token",
                p->tokens);
  const uint64_t row = uint64_t(p->kvHeads) * p->headDim;
  if (uint64_t(p->past) * row + row > UINT32_MAX)
    return fail(LLMI_UNSUPPORTED, "decode_append: cache offsets exceed 32 bits");
  if (batch > 1 && (k_new || v_new) && new_stride < row)
    return fail(LLMI_INVALID_ARGUMENT, "decode_append: new rows of sequences overlap");
  return gqa_decode_run(p, batch, q, k_cache, v_cache, cache_stride, out, workspace,
                        workspace_bytes, stream, NewRows{k_new, v_new, new_stride}, flags);
}

// ---- decode without a caller workspace ------------------------------------------------
//
// For callers that cannot allocate device memory themselves: an executor that
// hands out all device memory from its own fixed arena and forbids any other
// allocation, or a latency-critical decode loop that cannot absorb the
// device-wide synchronisation cudaMalloc may imply.  The scratch lives in
// this fixed array instead; every GPU that loads the library holds it until
// the process exits.

constexpr size_t kStaticDecodeScratchBytes = size_t(8) << 20;  // 8 MiB

static __device__ __align__(256) unsigned char g_static_decode_scratch[kStaticDecodeScratchBytes];

namespace {

// Device address of the static scratch on the current device.  The symbol's
// host-side name is not a device address, so it is looked up once per device
// with cudaGetSymbolAddress while that device is current, and cached.
int static_decode_scratch(const DeviceInfo &dev, void **address) {
  static std::mutex mutex;
  static void *cached[kMaxDevices] = {};
  std::lock_guard<std::mutex> lock(mutex);
  if (dev.device < 0 || dev.device >= kMaxDevices)
    return fail(LLMI_INVALID_ARGUMENT, "decode_noalloc: device %d outside [0, %d)", dev.device,
                kMaxDevices);
  if (!cached[dev.device]) {
    void *p = nullptr;
    if (int s = check_cuda(cudaGetSymbolAddress(&p, g_static_decode_scratch),
                           "cudaGetSymbolAddress(static decode scratch)"))
      return s;
    cached[dev.device] = p;
  }
  *address = cached[dev.device];
  return LLMI_OK;
}

}  // namespace

extern "C" int llmi_cuda_gqa_decode_noalloc(const llmi_gqa_params *p, unsigned batch,
                                            const uint16_t *q, const uint16_t *k_cache,
                                            const uint16_t *v_cache, size_t cache_stride,
                                            uint16_t *out, void *stream) {
  clear_error();
  if (int s = check_gqa(p, batch, q, k_cache, v_cache, cache_stride, out))
    return s;
  if (p->tokens != 1)
    return fail(LLMI_UNSUPPORTED, "decode_noalloc: %u tokens; decode takes one token", p->tokens);
  DeviceInfo dev;
  if (int s = current_device(dev))
    return s;
  const bool aligned = aligned16(q) && aligned16(k_cache) && aligned16(v_cache) &&
                       (batch == 1 || cache_stride % 8 == 0);
  DecodePlan plan;
  if (int s = plan_decode(*p, batch, aligned, dev, plan))
    return s;
  if (plan.workspace > kStaticDecodeScratchBytes)
    return fail(LLMI_WORKSPACE_TOO_SMALL,
                "decode_noalloc: this shape needs %zu B of scratch, the static scratch holds %zu B "
                "(call llmi_cuda_gqa_decode with a workspace instead)",
                plan.workspace, kStaticDecodeScratchBytes);
  void *scratch = nullptr;
  if (int s = static_decode_scratch(dev, &scratch))
    return s;
  return llmi_cuda_gqa_decode(p, batch, q, k_cache, v_cache, cache_stride, out, scratch,
                              kStaticDecodeScratchBytes, stream);
}

// ---- graphDeltaUpdate ----------------------------------------------------------------

namespace {

// The chunked tensor-core form applies (tokens >= kChunkedMinTokens, 128 x 128
// heads, 16-byte aligned operands).
bool delta_chunked(const llmi_delta_params *p, unsigned batch, const void *q, const void *k,
                   const void *v, const void *state, const void *out) {
  return p->tokens >= kChunkedMinTokens && p->keyDim == 128 && p->valueDim == 128 &&
         aligned16(q) && aligned16(k) && aligned16(v) && aligned16(state) && aligned16(out) &&
         batch <= 65535 && p->valueHeads <= 2147483647u && p->keyHeads <= 65535;
}

// Scratch of the chunk-parallel form: the Tu images of every (sequence,
// value head, chunk), then the fp16 k-row images of every (sequence, key
// head, chunk).
size_t delta_tu_bytes(const llmi_delta_params *p, unsigned batch) {
  const uint64_t chunks = (uint64_t(p->tokens) + delta_tc::C - 1) / delta_tc::C;
  return size_t(uint64_t(batch) * p->valueHeads * chunks * delta_tc::kTuBytes);
}

size_t delta_solved_bytes(const llmi_delta_params *p, unsigned batch) {
  const uint64_t chunks = (uint64_t(p->tokens) + delta_tc::C - 1) / delta_tc::C;
  return delta_tu_bytes(p, batch) +
         size_t(uint64_t(batch) * p->keyHeads * chunks * delta_tc::kKImageBytes);
}

int delta_update_impl(const llmi_delta_params *p, unsigned batch, const float *q, const float *k,
                      const uint16_t *v, const float *beta, const float *decay, float *state,
                      uint16_t *out, void *workspace, size_t workspace_bytes, bool with_ws,
                      void *stream, unsigned flags = 0);

}  // namespace

extern "C" size_t llmi_cuda_delta_update_workspace(const llmi_delta_params *p, unsigned batch) {
  clear_error();
  if (!p || !batch || !p->tokens || !p->keyHeads || !p->valueHeads) {
    fail(LLMI_INVALID_ARGUMENT, "DeltaUpdate workspace: null parameters or zero sizes");
    return 0;
  }
  // Alignment is the caller's; size as if the chunked form applies.
  if (p->tokens < kChunkedMinTokens || p->keyDim != 128 || p->valueDim != 128)
    return 0;
  return delta_solved_bytes(p, batch);
}

extern "C" int llmi_cuda_delta_update(const llmi_delta_params *p, unsigned batch, const float *q,
                                      const float *k, const uint16_t *v, const float *beta,
                                      const float *decay, float *state, uint16_t *out,
                                      void *stream) {
  return delta_update_impl(p, batch, q, k, v, beta, decay, state, out, nullptr, 0, false, stream);
}

extern "C" int llmi_cuda_delta_update_ws(const llmi_delta_params *p, unsigned batch,
                                         const float *q, const float *k, const uint16_t *v,
                                         const float *beta, const float *decay, float *state,
                                         uint16_t *out, void *workspace, size_t workspace_bytes,
                                         void *stream) {
  return delta_update_impl(p, batch, q, k, v, beta, decay, state, out, workspace,
                           workspace_bytes, true, stream);
}

extern "C" int llmi_cuda_delta_update_ws_ex(const llmi_delta_params *p, unsigned batch,
                                            const float *q, const float *k, const uint16_t *v,
                                            const float *beta, const float *decay, float *state,
                                            uint16_t *out, void *workspace,
                                            size_t workspace_bytes, void *stream,
                                            unsigned flags) {
  if (flags & ~LLMI_FLAG_SETTLED) {
    clear_error();
    return fail(LLMI_INVALID_ARGUMENT, "DeltaUpdate: unknown flags 0x%x", flags);
  }
  return delta_update_impl(p, batch, q, k, v, beta, decay, state, out, workspace,
                           workspace_bytes, true, stream, flags);
}

namespace {

int delta_update_impl(const llmi_delta_params *p, unsigned batch, const float *q, const float *k,
                      const uint16_t *v, const float *beta, const float *decay, float *state,
                      uint16_t *out, void *workspace, size_t workspace_bytes, bool with_ws,
                      void *stream, unsigned flags) {
  clear_error();
  if (!p || !q || !k || !v || !beta || !decay || !state || !out)
    return fail(LLMI_INVALID_ARGUMENT, "DeltaUpdate: null parameter or tensor pointer");
  if (!batch || !p->tokens || !p->keyHeads || !p->keyDim || !p->valueHeads || !p->valueDim)
    return fail(LLMI_INVALID_ARGUMENT, "DeltaUpdate: sizes must be positive");
  if (p->valueHeads % p->keyHeads)
    return fail(LLMI_INVALID_ARGUMENT, "DeltaUpdate: %u value heads are not a multiple of %u",
                p->valueHeads, p->keyHeads);
  delta::Args a;
  a.q = q;
  a.k = k;
  a.v = reinterpret_cast<const __half *>(v);
  a.beta = beta;
  a.decay = decay;
  a.state = state;
  a.out = reinterpret_cast<__half *>(out);
  a.batch = batch;
  a.tokens = p->tokens;
  a.key_heads = p->keyHeads;
  a.key_dim = p->keyDim;
  a.value_heads = p->valueHeads;
  a.value_dim = p->valueDim;
  a.group = p->valueHeads / p->keyHeads;
  a.settled = (flags & LLMI_FLAG_SETTLED) ? 1u : 0u;
  cudaStream_t s = as_stream(stream);
  // Multi-token calls: chunked form on tensor cores (dk = dv = 128).
  const bool chunked = delta_chunked(p, batch, q, k, v, state, out);
  if (chunked) {
    const bool presolve = with_ws;
    if (presolve) {
      const size_t need = delta_solved_bytes(p, batch);
      if (workspace_bytes < need || !workspace || !aligned16(workspace))
        return fail(LLMI_WORKSPACE_TOO_SMALL,
                    "DeltaUpdate: workspace of %zu B at %p; this shape needs %zu B, 16-byte "
                    "aligned (llmi_cuda_delta_update_workspace)",
                    workspace_bytes, workspace, need);
    }
    DeviceInfo dev;
    if (int e = current_device(dev))
      return e;
    // q, k fp32 [batch][tokens][keyHeads * 128]: a box is the 64 rows x 128
    // columns of one head's chunk.  v and out fp16 [batch][tokens][valueHeads * 128]:
    // v in two 128B-swizzled boxes of 64 columns (the MMA operand layout), out
    // written from a row-major tile.
    CUtensorMap mq, mk, mv, mo;
    const uint64_t kw = uint64_t(p->keyHeads) * 128, vw = uint64_t(p->valueHeads) * 128;
    const uint64_t T = p->tokens;
    const uint32_t C = delta_tc::C;
    {
      const uint64_t dims[3] = {kw, T, batch};
      const uint64_t strides[2] = {kw * 4, T * kw * 4};
      const uint32_t box[3] = {128, C, 1};
      if (int e = encode_map_3d(&mq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, q, dims, strides, box))
        return e;
      if (int e = encode_map_3d(&mk, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, k, dims, strides, box))
        return e;
    }
    {
      const uint64_t dims[3] = {vw, T, batch};
      const uint64_t strides[2] = {vw * 2, T * vw * 2};
      const uint32_t vbox[3] = {64, C, 1};
      if (int e = encode_map_3d(&mv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, v, dims, strides, vbox,
                                CU_TENSOR_MAP_SWIZZLE_128B))
        return e;
      const uint32_t obox[3] = {128, C, 1};
      if (int e = encode_map_3d(&mo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, out, dims, strides, obox))
        return e;
    }
    const size_t smem = delta_tc::Smem::total + 1024;
    const size_t smem_p = delta_tc::SmemP::total + 1024;
    dim3 grid(p->valueHeads, batch);
    if (presolve) {
      // Every chunk's triangular system at once, then the state recurrence.
      const size_t solve_smem = sizeof(delta_solve::Smem);
      if (int e = allow_smem(reinterpret_cast<const void *>(delta_solve::solve_pass), solve_smem,
                             dev))
        return e;
      if (int e = allow_smem(reinterpret_cast<const void *>(delta_tc::chunked_tc<true>), smem_p,
                             dev))
        return e;
      const uint32_t chunks = (p->tokens + delta_tc::C - 1) / delta_tc::C;
      uint8_t *solved = static_cast<uint8_t *>(workspace);
      uint8_t *kimages = solved + delta_tu_bytes(p, batch);
      delta_solve::solve_pass<<<dim3(chunks, p->keyHeads, batch), delta_solve::kThreads,
                                solve_smem, s>>>(a, solved, kimages);
      if (int e = launched("graphDeltaUpdate (chunk systems)"))
        return e;
      delta_tc::chunked_tc<true><<<grid, delta_tc::kThreadsPresolved, smem_p, s>>>(
          mq, mk, mv, mo, a, solved, kimages);
      return launched("graphDeltaUpdate (chunked, presolved, tcgen05)");
    }
    if (int e = allow_smem(reinterpret_cast<const void *>(delta_tc::chunked_tc<false>), smem, dev))
      return e;
    delta_tc::chunked_tc<false><<<grid, delta_tc::kThreads, smem, s>>>(mq, mk, mv, mo, a, nullptr,
                                                                      nullptr);
    return launched("graphDeltaUpdate (chunked, tcgen05)");
  }
  const bool fast = p->valueDim == 128 && (p->keyDim == 128 || p->keyDim == 64) &&
                    aligned16(state) && aligned16(v) && batch <= 65535 &&
                    p->valueHeads <= 2147483647u / 4;
  if (fast) {
    DeviceInfo dev;
    if (int e = current_device(dev))
      return e;
    // Fewer than four 128-column CTAs per SM: split the columns in four so
    // that the state streams through more CTAs at once.
    if (uint64_t(p->valueHeads) * batch < 4ull * uint64_t(dev.sm_count)) {
      const uint64_t ctas = uint64_t(p->valueHeads) * 4 * batch;
      const bool one_wave = ctas <= uint64_t(delta::kRecV32OneWave) * dev.sm_count;
      auto kernel = p->keyDim == 128
                        ? (one_wave ? delta::recurrent_v32<128, delta::kRecV32OneWave> : delta::recurrent_v32<128, delta::kRecV32Waves>)
                        : (one_wave ? delta::recurrent_v32<64, delta::kRecV32OneWave> : delta::recurrent_v32<64, delta::kRecV32Waves>);
      return launch_dependent("graphDeltaUpdate (recurrent, registers, 32-column blocks)", kernel,
                              dim3(p->valueHeads * 4, batch), delta::kRecWarps * 32, 0, s, a);
    }
    return launch_dependent("graphDeltaUpdate (recurrent, registers)",
                            p->keyDim == 128 ? delta::recurrent_v128<128> : delta::recurrent_v128<64>,
                            dim3(p->valueHeads, batch), delta::kRecWarps * 32, 0, s, a);
  }
  const uint64_t columns = uint64_t(batch) * p->valueHeads * p->valueDim;
  return launch_dependent("graphDeltaUpdate (recurrent, generic)", delta::recurrent_generic,
                          dim3(uint32_t((columns + 127) / 128)), 128, 0, s, a);
}

}  // namespace

// ---- device error word ---------------------------------------------------------------

namespace {
// Self-test of the failure path: waits on an mbarrier that nothing ever
// completes, gives up after `limit_ns` like every bounded wait of the
// kernels, and raises the error word.  It faults and hangs nothing.
__global__ void selftest_wait_timeout(unsigned long long limit_ns) {
  __shared__ uint64_t never;
  if (threadIdx.x != 0)
    return;
  mbar_init(&never, 1);
  fence_barrier_init();
  const uint64_t start = global_timer_ns();
  while (!mbar_try_wait(&never, 0)) {
    if (global_timer_ns() - start > limit_ns) {
      raise_error(kErrWaitTimeout);
      return;
    }
  }
}
}  // namespace

extern "C" int llmi_cuda_selftest_wait_timeout(unsigned limit_us, void *stream) {
  clear_error();
  if (!limit_us || limit_us > 1000000u)
    return fail(LLMI_INVALID_ARGUMENT, "selftest: limit %u us outside (0, 1 s]", limit_us);
  selftest_wait_timeout<<<1, 32, 0, as_stream(stream)>>>(uint64_t(limit_us) * 1000u);
  return launched("selftest_wait_timeout");
}

// ---- producers of the path's operands ---------------------------------------------

namespace {

unsigned grid_for(uint64_t work, unsigned per_block) {
  const uint64_t blocks = (work + per_block - 1) / per_block;
  return unsigned(blocks < 0x7fffffffull ? blocks : 0x7fffffffull);
}

int rope_common(const char *op, const llmi_rope_params *p, unsigned batch, const uint16_t *input,
                size_t input_stride, const float *weight, uint16_t *output, size_t output_stride,
                void *stream) {
  if (!p || !input || !output)
    return fail(LLMI_INVALID_ARGUMENT, "%s: null parameter or tensor pointer", op);
  if (!batch || !p->tokens || !p->heads || !p->headDim)
    return fail(LLMI_INVALID_ARGUMENT, "%s: sizes must be positive", op);
  if (p->headDim > unsigned(producers::kRopeMaxDim) || p->rotaryDim % 2 ||
      p->rotaryDim > p->headDim || p->rotaryDim > unsigned(producers::kRopeMaxRotary) ||
      p->headStride < p->headDim)
    return fail(LLMI_UNSUPPORTED, "%s: headDim %u, rotaryDim %u, headStride %u", op, p->headDim,
                p->rotaryDim, p->headStride);
  const uint64_t rows = uint64_t(p->tokens) * p->heads;
  if (batch > 1 && (input_stride < rows * p->headStride ||
                    output_stride < (uint64_t(p->outputStart) * p->heads + rows) * p->headDim))
    return fail(LLMI_INVALID_ARGUMENT, "%s: sequence strides overlap", op);
  producers::RopeArgs a;
  a.input = reinterpret_cast<const __half *>(input);
  a.input_stride = input_stride;
  a.weight = weight;
  a.output = reinterpret_cast<__half *>(output);
  a.output_stride = output_stride;
  a.batch = batch;
  a.tokens = p->tokens;
  a.heads = p->heads;
  a.head_dim = p->headDim;
  a.rotary_dim = p->rotaryDim;
  a.head_stride = p->headStride;
  a.past = p->past;
  a.output_start = p->outputStart;
  a.epsilon = p->epsilon;
  a.theta = p->theta;
  const bool vec = p->headDim % 8 == 0 && p->headStride % 8 == 0 && aligned16(input) &&
                   aligned16(output) && input_stride % 8 == 0 && output_stride % 8 == 0;
  const unsigned grid = grid_for(uint64_t(p->tokens) * batch, producers::kRopeWarps);
  cudaStream_t s = as_stream(stream);
  if (vec && p->headDim <= 256)
    producers::norm_rope<true, 1><<<grid, 32 * producers::kRopeWarps, 0, s>>>(a);
  else if (vec)
    producers::norm_rope<true, producers::kRopeMaxDim / 256>
        <<<grid, 32 * producers::kRopeWarps, 0, s>>>(a);
  else
    producers::norm_rope<false><<<grid, 32 * producers::kRopeWarps, 0, s>>>(a);
  return launched(op);
}

int conv_args(const char *op, const llmi_conv_params *p, unsigned batch, const uint16_t *input,
              size_t input_stride, const uint16_t *weight, uint16_t *history,
              size_t history_stride, producers::ConvArgs &a) {
  if (!p || !input || !weight || (!history && p->kernelSize > 1))
    return fail(LLMI_INVALID_ARGUMENT, "%s: null parameter or tensor pointer", op);
  if (!batch || !p->tokens || !p->channels || !p->kernelSize)
    return fail(LLMI_INVALID_ARGUMENT, "%s: sizes must be positive", op);
  const uint64_t hist = uint64_t(p->channels) * (p->kernelSize - 1);
  if (batch > 1 && (input_stride < uint64_t(p->tokens) * p->channels || history_stride < hist))
    return fail(LLMI_INVALID_ARGUMENT, "%s: sequence strides overlap", op);
  a.input = reinterpret_cast<const __half *>(input);
  a.input_stride = input_stride;
  a.weight = reinterpret_cast<const __half *>(weight);
  a.history = reinterpret_cast<const __half *>(history);
  a.history_stride = history_stride;
  a.batch = batch;
  a.tokens = p->tokens;
  a.channels = p->channels;
  a.kernel = p->kernelSize;
  a.apply_silu = p->applySilu != 0;
  return LLMI_OK;
}

// Runs after the step's outputs (stream order), which read the old history.
int advance_history(const producers::ConvArgs &a, uint16_t *history, cudaStream_t s) {
  if (a.kernel < 2)
    return LLMI_OK;
  const uint64_t n = uint64_t(a.batch) * a.channels;
  producers::conv_history<<<grid_for(n, 256), 256, 0, s>>>(a, reinterpret_cast<__half *>(history));
  return launched("causalConv (history)");
}

}  // namespace

extern "C" int llmi_cuda_norm_rope(const llmi_rope_params *p, unsigned batch,
                                   const uint16_t *input, size_t input_stride, const float *weight,
                                   uint16_t *output, size_t output_stride, void *stream) {
  clear_error();
  if (!weight)
    return fail(LLMI_INVALID_ARGUMENT, "normRope: null weight");
  return rope_common("normRope", p, batch, input, input_stride, weight, output, output_stride,
                     stream);
}

extern "C" int llmi_cuda_partial_rope(const llmi_rope_params *p, unsigned batch,
                                      const uint16_t *input, size_t input_stride,
                                      uint16_t *output, size_t output_stride, void *stream) {
  clear_error();
  return rope_common("partialRope", p, batch, input, input_stride, nullptr, output,
                     output_stride, stream);
}

extern "C" int llmi_cuda_causal_conv(const llmi_conv_params *p, unsigned batch,
                                     const uint16_t *input, size_t input_stride,
                                     const uint16_t *weight, uint16_t *history,
                                     size_t history_stride, uint16_t *output,
                                     size_t output_stride, void *stream) {
  clear_error();
  producers::ConvArgs a;
  if (int e = conv_args("causalConv", p, batch, input, input_stride, weight, history,
                        history_stride, a))
    return e;
  if (!output)
    return fail(LLMI_INVALID_ARGUMENT, "causalConv: null output");
  if (batch > 1 && output_stride < uint64_t(p->tokens) * p->channels)
    return fail(LLMI_INVALID_ARGUMENT, "causalConv: sequence strides overlap");
  cudaStream_t s = as_stream(stream);
  const uint64_t n = uint64_t(batch) * p->tokens * p->channels;
  producers::causal_conv<<<grid_for(n, 256), 256, 0, s>>>(a, reinterpret_cast<__half *>(output),
                                                          output_stride);
  if (int e = launched("causalConv"))
    return e;
  return advance_history(a, history, s);
}

extern "C" int llmi_cuda_l2_norm(const llmi_l2_params *p, const uint16_t *input, float *output,
                                 void *stream) {
  clear_error();
  if (!p || !input || !output)
    return fail(LLMI_INVALID_ARGUMENT, "l2NormF32: null parameter or tensor pointer");
  if (!p->rows || !p->width)
    return fail(LLMI_INVALID_ARGUMENT, "l2NormF32: sizes must be positive");
  producers::l2_norm<<<grid_for(p->rows, 8), 256, 0, as_stream(stream)>>>(
      reinterpret_cast<const __half *>(input), output, p->rows, p->width, p->epsilon, p->scale);
  return launched("l2NormF32");
}

extern "C" int llmi_cuda_delta_gates(const llmi_row_params *p, const uint16_t *a,
                                     const uint16_t *b, const float *aLog, const float *dtBias,
                                     float *beta, float *decay, void *stream) {
  clear_error();
  if (!p || !a || !b || !aLog || !dtBias || !beta || !decay)
    return fail(LLMI_INVALID_ARGUMENT, "deltaGates: null parameter or tensor pointer");
  if (!p->rows || !p->width)
    return fail(LLMI_INVALID_ARGUMENT, "deltaGates: sizes must be positive");
  const uint64_t n = uint64_t(p->rows) * p->width;
  producers::delta_gates<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(
      reinterpret_cast<const __half *>(a), reinterpret_cast<const __half *>(b), aLog, dtBias,
      beta, decay, n, p->width);
  return launched("deltaGates");
}

namespace {

// Fills the SiLU table (producers::g_silu_half) once per device before the
// first kernel that reads it.  The fill is waited for on the host, so every
// later call sees it whatever its stream; for that reason the first such call
// on a device cannot run under stream capture.
int ensure_silu_table(cudaStream_t s, const DeviceInfo &dev) {
  static std::mutex mutex;
  static bool ready[kMaxDevices] = {};
  std::lock_guard<std::mutex> lock(mutex);
  if (ready[dev.device])
    return LLMI_OK;
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  if (int e = check_cuda(cudaStreamIsCapturing(s, &capture), "cudaStreamIsCapturing"))
    return e;
  if (capture != cudaStreamCaptureStatusNone)
    return fail(LLMI_UNSUPPORTED,
                "deltaPrepare: the first call on a device fills the SiLU table and cannot be "
                "captured into a graph; make one call before capturing");
  producers::silu_table_init<<<256, 256, 0, s>>>();
  if (int e = launched("SiLU table"))
    return e;
  if (int e = check_cuda(cudaStreamSynchronize(s), "SiLU table"))
    return e;
  ready[dev.device] = true;
  return LLMI_OK;
}

}  // namespace

extern "C" int llmi_cuda_delta_prepare(const llmi_delta_prep_params *p, unsigned batch,
                                       const uint16_t *qkv, size_t qkv_stride,
                                       const uint16_t *conv_weight, uint16_t *history,
                                       size_t history_stride, float *q, float *k, uint16_t *v,
                                       void *stream) {
  clear_error();
  if (!p || !q || !k || !v)
    return fail(LLMI_INVALID_ARGUMENT, "deltaPrepare: null parameter or tensor pointer");
  if (!p->keyHeads || !p->keyDim || !p->valueHeads || !p->valueDim)
    return fail(LLMI_INVALID_ARGUMENT, "deltaPrepare: sizes must be positive");
  if (p->qkvWidth != 2 * p->keyHeads * p->keyDim + p->valueHeads * p->valueDim)
    return fail(LLMI_INVALID_ARGUMENT, "deltaPrepare: qkvWidth %u is not 2*%u*%u + %u*%u",
                p->qkvWidth, p->keyHeads, p->keyDim, p->valueHeads, p->valueDim);
  if (p->keyDim > 256 || p->valueDim > 256)
    return fail(LLMI_UNSUPPORTED, "deltaPrepare: keyDim %u / valueDim %u above 256", p->keyDim,
                p->valueDim);
  const llmi_conv_params cp{p->tokens, p->qkvWidth, p->kernelSize, 1};
  producers::PrepArgs a;
  if (int e = conv_args("deltaPrepare", &cp, batch, qkv, qkv_stride, conv_weight, history,
                        history_stride, a.conv))
    return e;
  a.key_heads = p->keyHeads;
  a.key_dim = p->keyDim;
  a.value_heads = p->valueHeads;
  a.value_dim = p->valueDim;
  a.epsilon = p->epsilon;
  a.q = q;
  a.k = k;
  a.v = reinterpret_cast<__half *>(v);
  cudaStream_t s = as_stream(stream);
  const unsigned heads = 2 * p->keyHeads + p->valueHeads;
  const bool tiled = p->keyDim == 128 && p->valueDim == 128 && p->kernelSize == 4 &&
                     aligned16(qkv) && aligned16(conv_weight) && aligned16(q) && aligned16(k) &&
                     aligned16(v) && (batch == 1 || qkv_stride % 8 == 0) && batch <= 65535;
  if (tiled) {
    DeviceInfo dev;
    if (int e = current_device(dev))
      return e;
    if (int e = ensure_silu_table(s, dev))
      return e;
    if (int e = allow_smem(reinterpret_cast<const void *>(producers::delta_prepare_resident),
                           producers::kPrepResidentSmem, dev))
      return e;
    const uint64_t tiles = (p->tokens + producers::kPrepTokens - 1) / producers::kPrepTokens;
    const uint64_t warps = uint64_t(batch) * tiles * heads;
    const uint64_t per_cta = producers::kPrepResidentThreads / 32;
    const unsigned grid = unsigned(std::min<uint64_t>(dev.sm_count, (warps + per_cta - 1) / per_cta));
    producers::delta_prepare_resident<<<grid, producers::kPrepResidentThreads,
                                        producers::kPrepResidentSmem, s>>>(a);
  } else {
    const uint64_t rows = uint64_t(batch) * p->tokens * heads;
    producers::delta_prepare<<<grid_for(rows, 8), 256, 0, s>>>(a);
  }
  if (int e = launched("deltaPrepare"))
    return e;
  return advance_history(a.conv, history, s);
}

extern "C" int llmi_cuda_poll_error(void *stream) {
  clear_error();
  if (int s = check_cuda(cudaStreamSynchronize(as_stream(stream)), "stream synchronize"))
    return s;
  unsigned word = 0;
  if (int s = check_cuda(cudaMemcpyFromSymbol(&word, g_error_word, sizeof word), "read error word"))
    return s;
  if (!word)
    return LLMI_OK;
  const unsigned zero = 0;
  if (int s = check_cuda(cudaMemcpyToSymbol(g_error_word, &zero, sizeof zero), "clear error word"))
    return s;
  return fail(LLMI_DEVICE_TIMEOUT, "device error word 0x%x:%s%s%s", word,
              (word & kErrWaitTimeout) ? " wait-timeout" : "",
              (word & kErrTmemAlloc) ? " tmem-alloc" : "",
              (word & kErrBadLaunch) ? " bad-launch" : "");
}
