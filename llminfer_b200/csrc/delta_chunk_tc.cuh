// Gated DeltaNet multi-token update on 5th-generation tensor cores (tcgen05
// MMA with TMEM accumulators, TMA-staged inputs), chunks of 64 tokens.
//
// Same result as the token-sequential graphDeltaUpdate
// (Graph.metal:146-170, Reference.metal:182-197) up to rounding, computed
// with the chunkwise (WY / UT) form of the gated delta rule (Yang, Kautz,
// Hatamizadeh, "Gated Delta Networks", 2024).  With S the [dk][dv] state at
// the start of a chunk, G_t the within-chunk cumulative log-decay
// (sum_{s<=t} log decay_s) and G_C that of the chunk's last token:
//   A[t][s] = beta_t (k_t . k_s) e^{G_t - G_s}       (s < t, else 0)
//   T       = (I + A)^-1                              (unit lower triangular)
//   W = T diag(beta e^G) K ;   U = T diag(beta) V
//   V'      = U - W S                                 (the chunk's deltas)
//   y_t     = e^{G_t} q_t^T S + sum_{s<=t} P[t][s] V'_s,
//             P[t][s] = (q_t . k_s) e^{G_t - G_s}
//   S      <- e^{G_C} S + sum_s k_s (e^{G_C - G_s} V'_s)^T
// Unrolling the per-token recurrence S_t = decay_t (I - beta_t k_t k_t^T)
// S_{t-1} + beta_t k_t v_t^T over a chunk gives exactly these terms.
//
// Every product is an M=128 tcgen05 MMA (fp16 operands from shared memory,
// fp32 accumulation in TMEM).  The value dimension sits on the M side (TMEM
// lanes) wherever a product involves the state, so the state lives in TMEM
// as S^T [dv][dk] - an fp32 accumulator that each chunk's update is added to
// in place - and every tile written back to shared memory is made of rows of
// one TMEM lane:
//   M1  D1[128 x 64]      = [K; Q] K^T        -> A (rows 0-63), Q K^T (64-127)
//   M2  Dw[128 x 64]      = K^T Tw^T = W^T,   Tw = T diag(beta e^G)
//   M3  Du[128 x 64]      = V^T Tu^T = U^T,   Tu = T diag(beta)
//   M4  Da[128 x 128]     = S^T [W; Q]^T      -> (W S)^T | (Q S)^T   (S^T fp16 in TMEM)
//   M5  Dy[128 x 64]      = V'^T P^T
//   M6  Ds[128 x 128]    += (V' e^{G_C - G})^T K   (Ds pre-scaled by e^{G_C})
// with V'^T = Du - Da[:, 0:64] and y^T = e^G Da[:, 64:128] + Dy formed by the
// epilogues.  The gates never touch K, Q or V: they scale the columns of T,
// the rows of V' and the epilogue, so K^T and V^T are read straight from the
// [K; Q] tile and from the 128B-swizzled TMA box of V as MN-major operands.
// T = (I + A)^-1 is built on the CUDA cores: the 16x16 diagonal blocks by
// forward substitution in fp32, the rest by blocked substitution on warp
// MMAs (each warp owns 8 columns of T, so no warp waits for another).
//
// One CTA owns one (sequence, value head) and walks its chunks in order, as
// two warpgroups that run a chunk apart:
//   warps 0-3  the chunk-local chain of chunk n: M1, A and P, the
//              triangular solve, M2/M3, W;
//   warps 4-7  the state chain of chunk n-1: M4 (under which warp 4 derives
//              chunk n+1's gates), V', M5/M6, y (through a shared-memory tile
//              and a TMA store) and the state; then the k rows (fp32,
//              TMA-staged a chunk ahead) and q rows of chunk n+1 into the
//              [K; Q] buffer M5/M6 just released, in fp16.
// The local chain is the longer one, so the conversions and the gates sit in
// the state chain, which would otherwise wait for the local one.
// [K; Q] and P are double-buffered; the groups hand buffers back and forth
// through mbarriers (MMA commits for "the MMAs reading it are done").  Each
// group's TMEM lanes are its threads (warp w % 4 owns lanes 32 (w % 4)..);
// one elected thread per group issues that group's MMAs.  Every wait is
// bounded: a wait that gives up raises the device error word and sets a CTA
// abort flag, both groups leave their loops at the next group barrier, drain
// their copies and MMAs (bounded) and free TMEM.  Requires key_dim ==
// value_dim == 128.
#pragma once

#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "delta_recurrent.cuh"
#include "tcgen05.cuh"

namespace llmi {
namespace delta_tc {

constexpr int C = 64;  // tokens per chunk
constexpr int DK = 128, DV = 128;
constexpr int kThreads = 256;
// The presolved form adds a third warpgroup (warps 8-11) for the chunk's
// inputs and outputs, so the state chain keeps only its own dependent steps.
constexpr int kThreadsPresolved = 384;
constexpr int kGroup = 128;            // threads per warpgroup
constexpr int kBarLocal = 1, kBarState = 2, kBarIO = 3;  // named barrier ids
constexpr uint32_t kTmemCols = 512;
// TMEM columns.  D1 and Dw share columns: D1 is read before M2 is issued.
constexpr uint32_t kColD1 = 0, kColW = 0, kColU = 64, kColA = 128, kColY = 256, kColS = 320;
constexpr uint32_t kColST = 448;  // S^T in fp16 (pairs of keys per column): the A operand of M4
constexpr int kLdA = 72;  // fp16 row stride of A (conflict-free ldmatrix)
constexpr int kLdT = 24;  // fp16 row stride of the diagonal-block inverses
constexpr int kGateSets = 4;

struct Gates {  // one chunk's gates in shared memory
  float g2[C];    // G_t in log2 units (G_t log2(e))
  float eg[C];    // e^{G_t}
  float ekg[C];   // e^{G_C - G_t}
  float bet[C];   // beta_t (0 past the last token)
  float ev[C];    // e^{G_e - G_t}, e the last token of t's 16-token block
  float egl[4];   // e^{G_C}
};

struct Smem {
  // [K; Q] fp16, K-major, two buffers: two 64-key blocks of 128 rows each
  // (K rows 0-63, Q rows 64-127).
  static constexpr int X = 0;
  // v fp16 [64 t][128 dv] as two TMA boxes [64 t][64 dv], 128B-swizzled.
  static constexpr int Vraw = X + 2 * 32768;
  static constexpr int Kst = Vraw + 16384;         // TMA staging of the next chunk's k rows, fp32 [64][128]
  static constexpr int WB = Kst + C * DK * 4;      // W fp16 [128 key][64 t], MN-major (B of M4)
  static constexpr int Vp = WB + 16384;            // V'^T fp16 [128 dv][64 t], K-major (A of M5)
  static constexpr int Ys = Vp;                    // y fp16 [64 t][128 dv] for the TMA store
  static constexpr int Vg = Vp + 16384;            // e^{G_C - G} V'^T (A of M6)
  static constexpr int P = Vg + 16384;             // 2 x fp16 [64 t][64 s], K-major (B of M5)
  static constexpr int Am = P + 2 * 8192;          // fp16 [64][kLdA]
  static constexpr int Ad = Am + C * kLdA * 2;     // fp32 [4 blocks][16 s][16 t] (column-major)
  static constexpr int Td = Ad + 4 * 16 * 16 * 4;  // fp16 [64][kLdT]
  static constexpr int Tw = Td + C * kLdT * 2;     // fp16 [64 t][64 s], K-major (B of M2)
  static constexpr int Tu = Tw + 8192;             // fp16 [64 t][64 s], K-major (B of M3)
  static constexpr int graw = Tu + 8192;           // fp32 decay[64], beta[64] (cp.async)
  static constexpr int gates = graw + 2 * C * 4;   // Gates[kGateSets], by chunk mod kGateSets
  static constexpr int bars = gates + kGateSets * int(sizeof(Gates));
  static constexpr int kBars = 19;
  static constexpr int tmem_slot = bars + kBars * 8;
  static constexpr int abort_flag = tmem_slot + 4;
  static constexpr int total = abort_flag + 12;
  static constexpr int YsP = 0;  // presolved form only
};
static_assert(Smem::Tw % 1024 == 0 && Smem::P % 1024 == 0, "operand tiles 1024-byte aligned");
static_assert(sizeof(Gates) % 16 == 0, "gate sets stay 16-byte aligned");
static_assert(Smem::total + 1024 <= 232448, "shared memory");

constexpr uint32_t kVBytes = C * DV * 2, kKBytes = C * DK * 4;
constexpr uint32_t kTuBytes = C * C * 2;      // one presolved Tu image
constexpr uint32_t kKImageBytes = C * DK * 2;  // one chunk's k rows, fp16, as the [K; Q] tile holds them

// Shared memory of the presolved form.  The k rows arrive in fp16 in the
// operand layout (bulk copies of the first pass's images), so there is no
// fp32 staging tile and no A / solve scratch; that room holds a third
// [K; Q] buffer (the IO group fills chunk n + 3 while chunks n .. n + 2 are
// in flight) and the y tile the IO group stores.
struct SmemP {
  static constexpr int X = 0;                      // 3 x [K; Q] (32 KB each)
  static constexpr int Vraw = X + 3 * 32768;
  static constexpr int WB = Vraw + 16384;
  static constexpr int Vp = WB + 16384;
  static constexpr int Vg = Vp + 16384;
  static constexpr int P = Vg + 16384;             // 3 x fp16 [64 t][64 s], one per [K; Q] buffer
  static constexpr int YsP = P + 3 * 8192;         // y fp16 [64 t][128 dv] for the TMA store
  static constexpr int Tw = YsP + 16384;
  static constexpr int Tu = Tw + 8192;
  static constexpr int graw = Tu + 8192;
  static constexpr int gates = graw + 2 * C * 4;
  static constexpr int bars = gates + kGateSets * int(sizeof(Gates));
  static constexpr int kBars = Smem::kBars;
  static constexpr int tmem_slot = bars + kBars * 8;
  static constexpr int abort_flag = tmem_slot + 4;
  static constexpr int total = abort_flag + 12;
  // Fused-form members the shared code names but this form never reaches.
  static constexpr int Kst = 0, Ys = 0, Am = 0, Ad = 0, Td = 0;
};
static_assert(SmemP::Tw % 1024 == 0 && SmemP::P % 1024 == 0 && SmemP::YsP % 1024 == 0 &&
                  SmemP::Vraw % 1024 == 0, "operand tiles 1024-byte aligned");
static_assert(SmemP::total + 1024 <= 232448, "shared memory (presolved)");

// A tile 16x16 of a row-major fp16 [m][k] array (ldmatrix, mma.m16n8k16 layout).
__device__ __forceinline__ void load_a(uint32_t (&f)[4], const __half *base, int ld, int m0, int k0,
                                       int lane) {
  ldmatrix_x4(f, smem_u32(base + (m0 + (lane & 15)) * ld + k0 + (lane >> 4) * 8));
}

__device__ __forceinline__ void st16(uint8_t *p, uint4 v) { *reinterpret_cast<uint4 *>(p) = v; }

__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  return make_uint4(pack_half2(v[0], v[1]), pack_half2(v[2], v[3]), pack_half2(v[4], v[5]),
                    pack_half2(v[6], v[7]));
}

__device__ __forceinline__ uint4 pack8(float4 a, float4 b) {
  return make_uint4(pack_half2(a.x, a.y), pack_half2(a.z, a.w), pack_half2(b.x, b.y),
                    pack_half2(b.z, b.w));
}

// 8 consecutive accumulator columns (fp32 bits) as 8 fp16.
__device__ __forceinline__ uint4 pack8_bits(const uint32_t *v) {
  return make_uint4(pack_half2(__uint_as_float(v[0]), __uint_as_float(v[1])),
                    pack_half2(__uint_as_float(v[2]), __uint_as_float(v[3])),
                    pack_half2(__uint_as_float(v[4]), __uint_as_float(v[5])),
                    pack_half2(__uint_as_float(v[6]), __uint_as_float(v[7])));
}

// 32 consecutive floats of a shared-memory array into registers.
__device__ __forceinline__ void load32(float (&d)[32], const float *p) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 v = reinterpret_cast<const float4 *>(p)[i];
    d[4 * i] = v.x;
    d[4 * i + 1] = v.y;
    d[4 * i + 2] = v.z;
    d[4 * i + 3] = v.w;
  }
}

// Grid (valueHeads, batch), kThreads threads, Smem::total + 1024 bytes.
// map_q / map_k: fp32 [batch][tokens][keyHeads * 128], box 128 x 64 x 1
// (used for L2 prefetches); map_v: fp16 [batch][tokens][valueHeads * 128],
// box 64 x 64 x 1, 128B swizzle; map_out: fp16 like v, box 128 x 64 x 1 (rows
// past the last token are neither read - zero fill - nor written).
//
// Presolved: the chunk-local systems were solved beforehand for every chunk
// at once (delta_chunk_solve.cuh); `solved` holds one 8 KB image of
// Tu = T diag(beta) per (sequence, value head, chunk), which arrives with the
// chunk's v boxes, and `kimages` one 16 KB image of the chunk's k rows in
// fp16 per (sequence, key head, chunk), copied straight into the [K; Q]
// buffer.  The local chain then skips A and the solve: warps 0-1 scale Tu's
// columns by e^{G_s} into Tw while warps 2-3 make P.  Grid as above,
// kThreadsPresolved threads, SmemP::total + 1024 bytes.
template <bool Presolved>
__global__ void __launch_bounds__(Presolved ? kThreadsPresolved : kThreads, 1)
    chunked_tc(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
               const __grid_constant__ CUtensorMap map_v,
               const __grid_constant__ CUtensorMap map_out, const delta::Args a,
               const uint8_t *__restrict__ solved, const uint8_t *__restrict__ kimages) {
  using Smem = std::conditional_t<Presolved, SmemP, delta_tc::Smem>;
  constexpr uint32_t kXBufs = Presolved ? 3 : 2;  // [K; Q] (and P) buffers
  extern __shared__ uint8_t smem_raw[];
  // Rounded up to 1024 bytes by an offset from the shared array itself, so
  // the compiler keeps every access through `smem` a shared-memory one (a
  // round trip through an integer address would make them generic).
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gt = tid & (kGroup - 1);  // thread within its group = its TMEM lane
  const uint32_t vh = blockIdx.x, seq = blockIdx.y;
  const uint32_t kh = vh / a.group;
  float *S = a.state + (size_t(seq) * a.value_heads + vh) * DK * DV;

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Smem::bars);
  uint64_t *bar_m1 = bars + 0;      // M1 done (local)
  uint64_t *bar_m23 = bars + 1;     // M2/M3 done (local)
  uint64_t *bar_v = bars + 2;       // v boxes landed (local)
  uint64_t *bar_ready = bars + 3;   // [2] chunk's W, [K; Q], P, U ready (local -> state)
  uint64_t *bar_m4 = bars + 5;      // M4 done (state)
  uint64_t *bar_wb = bars + 6;      // M4 done: W tile free (state -> local)
  uint64_t *bar_m56 = bars + 7;     // M5/M6 done (state)
  uint64_t *bar_xready = bars + 8;  // [kXBufs] [K; Q] and P buffers released by M5/M6 and the
                                    //     k and q rows of the buffer's next chunk written
                                    //     (state or IO -> local)
  uint64_t *bar_du = bars + 11;     // U read from TMEM (state -> local)
  uint64_t *bar_k = bars + 12;      // k rows staged (state or IO)
  uint64_t *bar_gates = bars + 13;  // [2 fused, 4 presolved] gates of a chunk (state or IO -> local)
  uint64_t *bar_m6 = bars + 17;     // presolved: M6 done (state)
  uint64_t *bar_yread = bars + 18;  // presolved: chunk's QS and Dy read from TMEM (IO -> state)
  // Chunk c's [K; Q] buffer, and its gates' barrier and parity: the presolved
  // form runs the groups up to three chunks apart, so its gates barriers are
  // four deep (no barrier can then be two phases ahead of a waiter).
  auto xbuf = [](uint32_t c) { return Presolved ? c % 3 : c & 1; };
  auto xready_parity = [](uint32_t c) { return Presolved ? (c / 3) & 1 : (c >> 1) & 1; };
  auto gate_bar = [&](uint32_t c) { return &bar_gates[Presolved ? c & 3 : c & 1]; };
  auto gate_parity = [](uint32_t c) { return Presolved ? (c >> 2) & 1 : (c >> 1) & 1; };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + Smem::tmem_slot);
  volatile uint32_t *abort = reinterpret_cast<volatile uint32_t *>(smem + Smem::abort_flag);
  float *graw = reinterpret_cast<float *>(smem + Smem::graw);
  Gates *gate_sets = reinterpret_cast<Gates *>(smem + Smem::gates);

  const uint32_t n_chunks = (a.tokens + C - 1) / C;

  if (tid == 0) {
    for (int i = 0; i < Smem::kBars; ++i)
      mbar_init(&bars[i], 1);
    *abort = 0u;
    fence_barrier_init();
    prefetch_map(&map_q);
    prefetch_map(&map_k);
    prefetch_map(&map_v);
    prefetch_map(&map_out);
  }
  if (warp == 1)
    tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tl = tmem + (uint32_t(32 * (warp & 3)) << 16);  // this warp's TMEM lane quarter

  auto issue_gates = [&](uint32_t chunk) {  // warp 4
    const uint32_t t0 = chunk * C;
    const int valid = int(min(uint32_t(C), a.tokens - t0));
    const size_t tok0 = size_t(seq) * a.tokens + t0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = lane + 32 * i, t = idx & (C - 1);
      const bool in = t < valid;
      const float *src =
          (idx < C ? a.decay : a.beta) + (tok0 + (in ? t : 0)) * a.value_heads + vh;
      cp_async4(graw + idx, src, in ? 4u : 0u);
    }
    cp_async_commit();
  };
  // Warp 4: gates of `chunk` from graw (G = inclusive cumsum of log(decay),
  // beta; pad tokens decay 1, beta 0), everything in log2 units.  A decay
  // of exactly 0 gets log2 -1e4: every factor 2^(G_t - G_s) across it is 0,
  // and G keeps full precision in the differences that stay.  (MUFU lg2 /
  // ex2: their relative error, ~2^-22, is far below the fp16 rounding of
  // the operands these factors scale.)
  auto gates = [&](uint32_t chunk) {
    Gates &gs = gate_sets[chunk % kGateSets];
    const int valid = int(min(uint32_t(C), a.tokens - chunk * C));
    cp_async_wait_all();
    __syncwarp();
    float la[2], bb[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int t = 2 * lane + i;
      const bool in = t < valid;
      const float d = graw[t];
      la[i] = in ? (d > 0.f ? fast_log2(d) : -1e4f) : 0.f;
      bb[i] = in ? graw[C + t] : 0.f;
    }
    const float pair = la[0] + la[1];
    float incl = pair;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off)
        incl += y;
    }
    const float gl = __shfl_sync(0xffffffffu, incl, 31);
    const float g[2] = {incl - pair + la[0], incl};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int t = 2 * lane + i;
      gs.g2[t] = g[i];
      gs.eg[t] = fast_exp2(g[i]);
      gs.ekg[t] = fast_exp2(gl - g[i]);
      gs.bet[t] = bb[i];
    }
    // The block ends: token 16 b + 15 is the second token of lane 8 b + 7.
    const float ge = __shfl_sync(0xffffffffu, incl, (lane & ~7) | 7);
#pragma unroll
    for (int i = 0; i < 2; ++i)
      gs.ev[2 * lane + i] = fast_exp2(ge - g[i]);
    if (lane == 0)
      gs.egl[0] = fast_exp2(gl);
    __syncwarp();
  };
  auto issue_k = [&](uint32_t chunk) {
    if constexpr (Presolved) {
      // The chunk's k rows in fp16, straight into its [K; Q] buffer (both
      // 64-key blocks); read by both value heads of the key head.
      mbar_arrive_expect_tx(bar_k, kKImageBytes);
      const uint8_t *src =
          kimages + ((size_t(seq) * a.key_heads + kh) * n_chunks + chunk) * kKImageBytes;
      uint8_t *xb = smem + Smem::X + xbuf(chunk) * 32768;
      bulk_g2s(xb, src, kKImageBytes / 2, bar_k, policy_evict_last());
      bulk_g2s(xb + 16384, src + kKImageBytes / 2, kKImageBytes / 2, bar_k, policy_evict_last());
    } else {
      mbar_arrive_expect_tx(bar_k, kKBytes);
      tma_load_3d(smem + Smem::Kst, &map_k, int(kh * DK), int(chunk * C), int(seq), bar_k);
    }
  };
  // Staged k rows of `chunk` (fp32) into rows 0-63 of its [K; Q] buffer
  // (fp16); every thread must have seen bar_k complete.
  auto convert_k = [&](uint32_t chunk) {
    uint8_t *Xb = smem + Smem::X + xbuf(chunk) * 32768;
    const float *kr = reinterpret_cast<const float *>(smem + Smem::Kst);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = gt + kGroup * i, t = idx >> 4, ch = idx & 15;
      const float4 *k4 = reinterpret_cast<const float4 *>(kr + t * DK + 8 * ch);
      st16(Xb + (ch >> 3) * 16384 + sw128_chunk(t, ch & 7), pack8(k4[0], k4[1]));
    }
    fence_proxy_async();
  };
  // q rows of `chunk` (fp32, global) into rows 64-127 of its [K; Q] buffer:
  // the loads, then the fp16 stores.
  auto load_q = [&](uint32_t chunk, float4 (&qr)[8][2]) {
    const uint32_t t0 = chunk * C;
    const int valid = int(min(uint32_t(C), a.tokens - t0));
    const size_t tok0 = size_t(seq) * a.tokens + t0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = gt + kGroup * i, t = idx >> 4, ch = idx & 15;
      if (t < valid) {
        const float4 *src = reinterpret_cast<const float4 *>(
            a.q + (tok0 + t) * size_t(a.key_heads) * DK + kh * DK + 8 * ch);
        qr[i][0] = __ldg(src);
        qr[i][1] = __ldg(src + 1);
      } else {
        qr[i][0] = qr[i][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  };
  auto store_q = [&](uint32_t chunk, const float4 (&qr)[8][2]) {
    uint8_t *Xb = smem + Smem::X + xbuf(chunk) * 32768;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = gt + kGroup * i, t = idx >> 4, ch = idx & 15;
      st16(Xb + (ch >> 3) * 16384 + sw128_chunk(C + t, ch & 7), pack8(qr[i][0], qr[i][1]));
    }
    fence_proxy_async();
  };
  if (warp < 4) {
    // ======================= local chain (warps 0-3) =======================
    const bool elected = gt == 0;
    // Parity of a phase issued but not yet seen complete (-1: none); drained
    // on the way out if the loop ends early.
    int m1_pending = -1, m23_pending = -1, v_pending = -1;
    auto issue_v = [&](uint32_t chunk) {
      mbar_arrive_expect_tx(bar_v, Presolved ? kVBytes + kTuBytes : kVBytes);
      const int t0 = int(chunk * C);
      tma_load_3d(smem + Smem::Vraw, &map_v, int(vh * DV), t0, int(seq), bar_v);
      tma_load_3d(smem + Smem::Vraw + 8192, &map_v, int(vh * DV + 64), t0, int(seq), bar_v);
      if (Presolved)
        bulk_g2s(smem + Smem::Tu,
                 solved + ((size_t(seq) * a.value_heads + vh) * n_chunks + chunk) * kTuBytes,
                 kTuBytes, bar_v, policy_evict_first());
    };
    if (elected) {
      issue_v(0);
      v_pending = 0;
    }

    for (uint32_t n = 0; n < n_chunks; ++n) {
      const int b = n & 1;
      const uint32_t xb = xbuf(n);
      Gates &gs = gate_sets[n % kGateSets];
      const uint32_t xs = sbase + Smem::X + xb * 32768;
      const bool more = n + 1 < n_chunks;

      // L1. [K; Q] buffer b holds chunk n's k and q rows (fp16, written by
      //     the state group once M5/M6 of chunk n - 2 released it).
      bool fail = !wait_or_abort(&bar_xready[xb], xready_parity(n), abort);
      if (named_sync_or(kBarLocal, kGroup, fail))
        break;

      // L2. M1: D1 = [K; Q] K^T.
      if (elected) {
        tc_fence_after();
        constexpr uint32_t id = idesc_f16(128, C, false);
#pragma unroll
        for (int k = 0; k < DK / 16; ++k) {
          const uint64_t d = desc_add(smem_desc(xs, 16, 1024), (k >> 2) * 16384 + (k & 3) * 32);
          mma_ss(tmem + kColD1, d, d, id, k > 0 ? 1u : 0u);
        }
        mma_commit(bar_m1);
        m1_pending = int(n & 1);
      }
      fail = !wait_or_abort(bar_m1, n & 1, abort) ||
             !wait_or_abort(gate_bar(n), gate_parity(n), abort);
      if (named_sync_or(kBarLocal, kGroup, fail))
        break;
      m1_pending = -1;
      tc_fence_after();

      // L3. A (fp16, and its diagonal blocks in fp32) from rows 0-63, P from
      //     rows 64-127.  Warp q reads accumulator rows 32q..32q+31: A rows
      //     (q < 2) or P rows (q >= 2) t = 32 (q % 2) + lane, so the column
      //     half h == q % 2 holds the row's diagonal blocks (exponentials per
      //     entry), h < q % 2 only whole 16-token blocks below the diagonal,
      //     whose factor splits as 2^(G_t - G_e) 2^(G_e - G_s) with e the
      //     block's last token (both <= 1; the second is the per-column ev),
      //     and h > q % 2 lies above the diagonal (A: never read; P: zeros).
      {
        __half *Am = reinterpret_cast<__half *>(smem + Smem::Am);
        float *Ad = reinterpret_cast<float *>(smem + Smem::Ad);
        uint8_t *Pb = smem + Smem::P + xb * 8192;
        const bool arow = warp < 2;
        const int hr = warp & 1;
        const int t = 32 * hr + lane;
        const float g_t = gs.g2[t], b_t = arow ? gs.bet[t] : 1.f;
        if (Presolved && arow) {
          // Tw = Tu diag(e^G): row t of the Tu image (loaded with the v
          // boxes), columns scaled, into the Tw tile (same swizzled layout).
          fail = !wait_or_abort(bar_v, n & 1, abort);
          if (!fail) {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const uint4 u = *reinterpret_cast<const uint4 *>(smem + Smem::Tu + sw128_chunk(t, c));
              const __half2 *h2 = reinterpret_cast<const __half2 *>(&u);
              float x[8];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(h2[e]);
                x[2 * e] = f.x * gs.eg[8 * c + 2 * e];
                x[2 * e + 1] = f.y * gs.eg[8 * c + 2 * e + 1];
              }
              st16(smem + Smem::Tw + sw128_chunk(t, c), pack8(x));
            }
            fence_proxy_async();
          }
        }
#pragma unroll 1
        for (int h = 0; h < 2 && !(Presolved && arow); ++h) {
          const int s0 = 32 * h;
          if (h > hr) {
            if (!arow) {
#pragma unroll
              for (int i = 0; i < 4; ++i)
                st16(Pb + sw128_chunk(t, 4 * h + i), make_uint4(0u, 0u, 0u, 0u));
            }
            continue;
          }
          uint32_t v[32];
          tmem_ld32(tl + kColD1 + s0, v);
          float f[32];
          if (h == hr) {
            float gsv[32];
            load32(gsv, gs.g2 + s0);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const bool keep = arow ? s0 + j < t : s0 + j <= t;
              f[j] = keep ? b_t * __uint_as_float(v[j]) * fast_exp2(g_t - gsv[j]) : 0.f;
            }
          } else {
            float evv[32];
            load32(evv, gs.ev + s0);
            const float u0 = b_t * fast_exp2(g_t - gs.g2[s0 + 15]);
            const float u1 = b_t * fast_exp2(g_t - gs.g2[s0 + 31]);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j)
              f[j] = __uint_as_float(v[j]) * (j < 16 ? u0 : u1) * evv[j];
          }
          if (arow) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              float x[8];
#pragma unroll
              for (int e = 0; e < 8; ++e)
                x[e] = f[8 * i + e];
              *reinterpret_cast<uint4 *>(Am + t * kLdA + s0 + 8 * i) = pack8(x);
            }
            // The diagonal block, column-major (Ad[block][s][t]) for the
            // substitution below.
            if (h == hr) {
              float *d = Ad + (t >> 4) * 256 + (t & 15);
              if (t & 16) {
#pragma unroll
                for (int j = 0; j < 16; ++j)
                  d[16 * j] = f[16 + j];
              } else {
#pragma unroll
                for (int j = 0; j < 16; ++j)
                  d[16 * j] = f[j];
              }
            }
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              float x[8];
#pragma unroll
              for (int e = 0; e < 8; ++e)
                x[e] = f[8 * i + e];
              st16(Pb + sw128_chunk(t, 4 * h + i), pack8(x));
            }
          }
        }
      }
      if constexpr (Presolved) {
        if (named_sync_or(kBarLocal, kGroup, fail))
          break;
        if (elected)
          v_pending = -1;
      } else {
      named_sync(kBarLocal, kGroup);

      // L4. T = (I + A)^-1.  Diagonal blocks by column-oriented forward
      //     substitution in fp32 (warp i = block i, lane = column): once
      //     x_j is final it updates every later row, so the dependent chain
      //     is 16 FMAs long ...
      {
        const float *Ad = reinterpret_cast<const float *>(smem + Smem::Ad);
        __half *Td = reinterpret_cast<__half *>(smem + Smem::Td);
        if (lane < 16) {
          const float4 *ab = reinterpret_cast<const float4 *>(Ad + warp * 256);
          float x[16];
#pragma unroll
          for (int r = 0; r < 16; ++r)
            x[r] = r == lane ? 1.f : 0.f;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float col[16];  // column j of the block: A[r][j], r = 0..15
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
            Td[(warp * 16 + r) * kLdT + lane] = __float2half_rn(x[r]);
        }
      }
      named_sync(kBarLocal, kGroup);
      // ... then block rows T_i = T_ii (I_i - sum_{k<i} A_ik T_k): warp w
      // owns the 16 columns of diagonal block w (zero above it).  T is
      // stored with its columns scaled: Tw = T diag(beta e^G), Tu = T diag(beta).
      {
        const __half *Am = reinterpret_cast<const __half *>(smem + Smem::Am);
        const __half *Td = reinterpret_cast<const __half *>(smem + Smem::Td);
        const int g = lane >> 2;
        float sw[2][2], su[2][2];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int c = 16 * warp + 8 * nt + 2 * (lane & 3) + e;
            su[nt][e] = gs.bet[c];
            sw[nt][e] = gs.bet[c] * gs.eg[c];
          }
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
                load_a(fa, Am, kLdA, 16 * i, 16 * kb, lane);
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
                  mma_f16_16816(acc[nt], fa, xb[kb][nt][0], xb[kb][nt][1]);
              }
            }
            uint32_t ft[4];
            load_a(ft, Td, kLdT, 16 * i, 0, lane);
            const int r0 = 16 * i + g;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
              const int c0 = 16 * warp + 8 * nt + 2 * (lane & 3);
              const uint32_t rb0 = movmatrix_trans(
                  pack_half2(float(r0 == c0) - acc[nt][0], float(r0 == c0 + 1) - acc[nt][1]));
              const uint32_t rb1 = movmatrix_trans(pack_half2(
                  float(r0 + 8 == c0) - acc[nt][2], float(r0 + 8 == c0 + 1) - acc[nt][3]));
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
            *reinterpret_cast<uint32_t *>(smem + Smem::Tw + o0) =
                pack_half2(x[nt][0] * sw[nt][0], x[nt][1] * sw[nt][1]);
            *reinterpret_cast<uint32_t *>(smem + Smem::Tw + o1) =
                pack_half2(x[nt][2] * sw[nt][0], x[nt][3] * sw[nt][1]);
            *reinterpret_cast<uint32_t *>(smem + Smem::Tu + o0) =
                pack_half2(x[nt][0] * su[nt][0], x[nt][1] * su[nt][1]);
            *reinterpret_cast<uint32_t *>(smem + Smem::Tu + o1) =
                pack_half2(x[nt][2] * su[nt][0], x[nt][3] * su[nt][1]);
          }
        }
      }
      fence_proxy_async();
      named_sync(kBarLocal, kGroup);
      }  // !Presolved

      // L5. M2, M3: W^T = K^T Tw^T (K^T read MN-major from the [K; Q] tile),
      //     U^T = V^T Tu^T (V^T from the swizzled TMA boxes), once the v boxes
      //     have landed and the state group has read the previous U.
      fail = false;
      if (elected) {
        fail = !wait_or_abort(bar_v, n & 1, abort);
        if (!fail)
          v_pending = -1;
        if (!fail && n >= 1)
          fail = !wait_or_abort(bar_du, (n - 1) & 1, abort);
        if (!fail) {
          tc_fence_after();
          constexpr uint32_t id = idesc_f16(128, C, false, true);
#pragma unroll
          for (int k = 0; k < C / 16; ++k) {
            mma_ss(tmem + kColW, desc_add(smem_desc(xs, 16384, 1024), k * 2048),
                   desc_add(smem_desc(sbase + Smem::Tw, 16, 1024), k * 32), id, k > 0 ? 1u : 0u);
            mma_ss(tmem + kColU, desc_add(smem_desc(sbase + Smem::Vraw, 8192, 1024), k * 2048),
                   desc_add(smem_desc(sbase + Smem::Tu, 16, 1024), k * 32), id, k > 0 ? 1u : 0u);
          }
          mma_commit(bar_m23);
          m23_pending = int(n & 1);
        }
      }
      if (named_sync_or(kBarLocal, kGroup, fail))
        break;
      fail = !wait_or_abort(bar_m23, n & 1, abort);
      if (named_sync_or(kBarLocal, kGroup, fail))
        break;
      m23_pending = -1;
      tc_fence_after();
      // L6. M3 has read the v boxes: load the next chunk's.  Then W (row =
      //     key, 64 tokens) into the W tile once M4 of chunk n - 1 is done.
      fail = false;
      if (elected) {
        if (more) {
          issue_v(n + 1);
          v_pending = int((n + 1) & 1);
        }
        if (n >= 1)
          fail = !wait_or_abort(bar_wb, (n - 1) & 1, abort);
      }
      if (named_sync_or(kBarLocal, kGroup, fail))
        break;
      {
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          uint32_t v[32];
          tmem_ld32(tl + kColW + 32 * h, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 4; ++i)
            st16(smem + Smem::WB + sw128_chunk(gt, 4 * h + i), pack8_bits(v + 8 * i));
        }
      }
      fence_proxy_async();
      tc_fence_before();
      named_sync(kBarLocal, kGroup);
      if (elected)
        mbar_arrive(&bar_ready[b]);
    }
    // Drain (bounded) what this group may still have in flight.
    if (elected) {
      if (m1_pending >= 0)
        mbar_wait(bar_m1, unsigned(m1_pending));
      if (m23_pending >= 0)
        mbar_wait(bar_m23, unsigned(m23_pending));
      if (v_pending >= 0)
        mbar_wait(bar_v, unsigned(v_pending));
    }
  } else if constexpr (!Presolved) {
    // ======================= state chain (warps 4-7) =======================
    const bool elected = gt == 0;
    const int dv = gt;  // this thread's value column (TMEM lane)
    int m4_pending = -1, m56_pending = -1, k_pending = -1;
    if (elected) {
      issue_k(0);
      k_pending = 0;
      if (n_chunks > 2)
        tma_prefetch_3d(&map_q, int(kh * DK), 2 * C, int(seq));
    }
    // Gates run two chunks ahead of the local chain: chunks 0 and 1 here,
    // chunk n + 2 while the state chain works on chunk n.
    if (warp == 4) {
      for (uint32_t c = 0; c < 2 && c < n_chunks; ++c) {
        issue_gates(c);
        gates(c);
        if (lane == 0)
          mbar_arrive(&bar_gates[c]);
      }
      if (n_chunks > 2)
        issue_gates(2);
    }
    named_sync(kBarState, kGroup);  // gates of chunk 0 visible to the group
    // Initial state: S^T into TMEM, in fp16 (M4's A operand) and in fp32 (the
    // accumulator M6 adds to), the latter already scaled by chunk 0's
    // e^{G_C}; the q rows of chunks 0 and 1.
    const float egl0 = gate_sets[0].egl[0];
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
      const int key0 = 32 * q4;
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j)
        v[j] = S[(key0 + j) * DV + dv];
      uint32_t st[32];
#pragma unroll
      for (int j = 0; j < 32; ++j)
        st[j] = __float_as_uint(v[j] * egl0);
      tmem_st32(tl + kColS + key0, st);
      uint32_t h[16];
#pragma unroll
      for (int j = 0; j < 16; ++j)
        h[j] = pack_half2(v[2 * j], v[2 * j + 1]);
      tmem_st16(tl + kColST + 16 * q4, h);
    }
    // The [K; Q] buffers of chunks 0 and 1 (a failed wait leaves them
    // unwritten: the local group then fails its own first wait).
    bool pro_fail = false;
    for (uint32_t c = 0; c < 2 && c < n_chunks; ++c) {
      float4 qr[8][2];
      load_q(c, qr);
      bool f = false;
      if (elected) {
        f = !wait_or_abort(bar_k, c & 1, abort);
        if (!f)
          k_pending = -1;
      }
      if (named_sync_or(kBarState, kGroup, f)) {
        pro_fail = true;
        break;
      }
      convert_k(c);
      store_q(c, qr);
      named_sync(kBarState, kGroup);
      if (elected && c + 1 < n_chunks) {
        issue_k(c + 1);
        k_pending = int((c + 1) & 1);
      }
    }
    tmem_wait_st();
    tc_fence_before();
    named_sync(kBarState, kGroup);
    if (elected && !pro_fail) {
      mbar_arrive(&bar_xready[0]);
      if (n_chunks > 1)
        mbar_arrive(&bar_xready[1]);
    }

    for (uint32_t n = 0; n < n_chunks; ++n) {
      const int b = n & 1;
      const uint32_t t0 = n * C;
      const bool last = n + 1 == n_chunks;
      const Gates &gs = gate_sets[n % kGateSets];
      const uint32_t xs = sbase + Smem::X + b * 32768;

      // S1. Chunk n's W, [K; Q], P and U are ready: M4 = S^T [W; Q]^T.
      //     (The fp32 state in TMEM is already scaled by e^{G_C} for M6.)
      bool fail = !wait_or_abort(&bar_ready[b], (n >> 1) & 1, abort);
      if (named_sync_or(kBarState, kGroup, fail))
        break;
      tc_fence_after();
      if (elected) {
        constexpr uint32_t id_w = idesc_f16(128, C, true);
        constexpr uint32_t id_q = idesc_f16(128, C, false);
#pragma unroll
        for (int k = 0; k < DK / 16; ++k) {
          const uint32_t as = tmem + kColST + k * 8;  // 16 keys = 8 columns of fp16 pairs
          mma_ts(tmem + kColA, as, desc_add(smem_desc(sbase + Smem::WB, 16384, 1024), k * 2048), id_w,
                 k > 0 ? 1u : 0u);
          mma_ts(tmem + kColA + C, as,
                 desc_add(smem_desc(xs, 16, 1024), (k >> 2) * 16384 + 8192 + (k & 3) * 32), id_q,
                 k > 0 ? 1u : 0u);
        }
        mma_commit(bar_m4);
        mma_commit(bar_wb);
        m4_pending = int(n & 1);
        if (n + 2 < n_chunks)  // q rows converted at the end of this chunk
          tma_prefetch_3d(&map_q, int(kh * DK), int(t0 + 2 * C), int(seq));
        bulk_wait_read();  // the previous output tile (Ys = Vp) has been read
      }
      // Gates of chunk n + 2, which the local group needs from its step L3.
      if (warp == 4 && n + 2 < n_chunks) {
        gates(n + 2);
        if (n + 3 < n_chunks)
          issue_gates(n + 3);
        if (lane == 0)
          mbar_arrive(&bar_gates[n & 1]);
      }

      // S2. V'^T = U^T - (W S)^T (row = value column, 64 tokens) into Vp,
      //     and scaled by e^{G_C - G_t} into Vg; then U may be overwritten.
      fail = !wait_or_abort(bar_m4, n & 1, abort);
      if (named_sync_or(kBarState, kGroup, fail))
        break;
      m4_pending = -1;
      tc_fence_after();
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        uint32_t u[32], w[32];
        tmem_ld32(tl + kColU + 32 * h, u);
        tmem_ld32(tl + kColA + 32 * h, w);
        float ek[32];
        load32(ek, gs.ekg + 32 * h);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float x[8], y[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            x[e] = __uint_as_float(u[8 * i + e]) - __uint_as_float(w[8 * i + e]);
            y[e] = x[e] * ek[8 * i + e];
          }
          st16(smem + Smem::Vp + sw128_chunk(dv, 4 * h + i), pack8(x));
          st16(smem + Smem::Vg + sw128_chunk(dv, 4 * h + i), pack8(y));
        }
      }
      fence_proxy_async();
      tc_fence_before();
      named_sync(kBarState, kGroup);
      // S3. M5: Dy = V'^T P^T;  M6: S^T += (e^{G_C - G} V')^T K.
      if (elected) {
        mbar_arrive(bar_du);
        tc_fence_after();
        constexpr uint32_t id5 = idesc_f16(128, C, false);
        constexpr uint32_t id6 = idesc_f16(128, 128, true);
#pragma unroll
        for (int k = 0; k < C / 16; ++k) {
          mma_ss(tmem + kColY, desc_add(smem_desc(sbase + Smem::Vp, 16, 1024), k * 32),
                 desc_add(smem_desc(sbase + Smem::P + b * 8192, 16, 1024), k * 32), id5, k > 0 ? 1u : 0u);
          mma_ss(tmem + kColS, desc_add(smem_desc(sbase + Smem::Vg, 16, 1024), k * 32),
                 desc_add(smem_desc(xs, 16384, 1024), k * 2048), id6, 1u);
        }
        mma_commit(bar_m56);
        m56_pending = int(n & 1);
      }

      // S4. y^T = e^G (Q S)^T + Dy into the output tile; fp16 S^T for the
      //     next chunk's M4 (or, after the last chunk, the state to memory).
      fail = !wait_or_abort(bar_m56, n & 1, abort);
      if (named_sync_or(kBarState, kGroup, fail))
        break;
      m56_pending = -1;
      tc_fence_after();
      // M5/M6 have released [K; Q] buffer b: start loading the q rows of
      // chunk n + 2 (stored below, after the outputs and the state).
      float4 qr[8][2];
      const bool q_next = n + 2 < n_chunks;
      if (q_next)
        load_q(n + 2, qr);
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        uint32_t ya[32], yd[32];
        tmem_ld32(tl + kColA + C + 32 * h, ya);
        tmem_ld32(tl + kColY + 32 * h, yd);
        float e[32];
        load32(e, gs.eg + 32 * h);
        tmem_wait_ld();
        __half *ys = reinterpret_cast<__half *>(smem + Smem::Ys) + dv;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          ys[(32 * h + j) * DV] =
              __float2half_rn(fmaf(e[j], __uint_as_float(ya[j]), __uint_as_float(yd[j])));
      }
      // The state after chunk n: fp16 for the next chunk's M4, and the fp32
      // accumulator scaled by the next chunk's e^{G_C} for its M6.
      const float egl_next = last ? 1.f : gate_sets[(n + 1) % kGateSets].egl[0];
#pragma unroll 1
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t v[32];
        tmem_ld32(tl + kColS + 32 * q4, v);
        tmem_wait_ld();
        if (!last) {
          uint32_t h[16];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            h[j] = pack_half2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
          tmem_st16(tl + kColST + 16 * q4, h);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            v[j] = __float_as_uint(__uint_as_float(v[j]) * egl_next);
          tmem_st32(tl + kColS + 32 * q4, v);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            S[(32 * q4 + j) * DV + dv] = __uint_as_float(v[j]);
        }
      }
      tmem_wait_st();
      fence_proxy_async();
      tc_fence_before();
      fail = false;
      if (elected && q_next) {  // k rows of chunk n + 2 staged
        fail = !wait_or_abort(bar_k, n & 1, abort);
        if (!fail)
          k_pending = -1;
      }
      if (named_sync_or(kBarState, kGroup, fail))
        break;
      if (elected) {
        tma_store_3d(&map_out, smem + Smem::Ys, int(vh * DV), int(t0), int(seq));
        bulk_commit();
      }
      if (q_next) {
        // Chunk n + 2's k and q rows into the buffer M5/M6 released; then
        // the staging tile takes the k rows of chunk n + 3.
        convert_k(n + 2);
        store_q(n + 2, qr);
        named_sync(kBarState, kGroup);
        if (elected) {
          if (n + 3 < n_chunks) {
            issue_k(n + 3);
            k_pending = int((n + 3) & 1);
          }
          mbar_arrive(&bar_xready[b]);
        }
      }
    }
    if (elected) {
      if (m4_pending >= 0)
        mbar_wait(bar_m4, unsigned(m4_pending));
      if (m56_pending >= 0)
        mbar_wait(bar_m56, unsigned(m56_pending));
      if (k_pending >= 0)
        mbar_wait(bar_k, unsigned(k_pending));
      bulk_wait();
    }
    if (warp == 4)
      cp_async_wait_all();
  } else if (warp < 8) {
    // ============== state chain, presolved form (warps 4-7) ===============
    // Only the steps each chunk's successor depends on: M4 (W half), V',
    // M6, the state copy.  M4's Q half and M5 ride along for the IO group.
    const bool elected = gt == 0;
    const int dv = gt;
    int m4_pending = -1, m6_pending = -1, m56_pending = -1;
    // Initial state: S^T into TMEM in fp16 (M4's A operand) and in fp32 (the
    // accumulator M6 adds to), the latter scaled by chunk 0's e^{G_C}, which
    // the IO group derives first.
    bool fail = elected && !wait_or_abort(gate_bar(0), gate_parity(0), abort);
    const bool pro_fail = named_sync_or(kBarState, kGroup, fail);
    if (!pro_fail) {
      const float egl0 = gate_sets[0].egl[0];
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const int key0 = 32 * q4;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j)
          v[j] = S[(key0 + j) * DV + dv];
        uint32_t st[32];
#pragma unroll
        for (int j = 0; j < 32; ++j)
          st[j] = __float_as_uint(v[j] * egl0);
        tmem_st32(tl + kColS + key0, st);
        uint32_t h[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
          h[j] = pack_half2(v[2 * j], v[2 * j + 1]);
        tmem_st16(tl + kColST + 16 * q4, h);
      }
      tmem_wait_st();
      tc_fence_before();
      named_sync(kBarState, kGroup);
    }
    for (uint32_t n = 0; n < n_chunks && !pro_fail; ++n) {
      const int b = n & 1;
      const bool last = n + 1 == n_chunks;
      const Gates &gs = gate_sets[n % kGateSets];
      const uint32_t xs = sbase + Smem::X + xbuf(n) * 32768;

      // P1. Chunk n's W, [K; Q], P and U are ready: M4's W half (S^T W^T),
      //     which V' needs, then its Q half (S^T Q^T) once the IO group has
      //     read chunk n - 1's QS from the same columns.
      fail = !wait_or_abort(&bar_ready[b], (n >> 1) & 1, abort);
      if (named_sync_or(kBarState, kGroup, fail))
        break;
      tc_fence_after();
      if (elected) {
        constexpr uint32_t id_w = idesc_f16(128, C, true);
        constexpr uint32_t id_q = idesc_f16(128, C, false);
#pragma unroll
        for (int k = 0; k < DK / 16; ++k)
          mma_ts(tmem + kColA, tmem + kColST + k * 8,
                 desc_add(smem_desc(sbase + Smem::WB, 16384, 1024), k * 2048), id_w, k > 0 ? 1u : 0u);
        mma_commit(bar_m4);
        mma_commit(bar_wb);
        m4_pending = int(n & 1);
        if (n >= 1)
          fail = !wait_or_abort(bar_yread, (n - 1) & 1, abort);
        if (!fail) {
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < DK / 16; ++k)
            mma_ts(tmem + kColA + C, tmem + kColST + k * 8,
                   desc_add(smem_desc(xs, 16, 1024), (k >> 2) * 16384 + 8192 + (k & 3) * 32), id_q,
                   k > 0 ? 1u : 0u);
        }
      }
      // P2. V'^T = U^T - (W S)^T into Vp, and scaled by e^{G_C - G_t} into Vg.
      fail = fail || !wait_or_abort(bar_m4, n & 1, abort);
      if (named_sync_or(kBarState, kGroup, fail))
        break;
      m4_pending = -1;
      tc_fence_after();
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        uint32_t u[32], w[32];
        tmem_ld32(tl + kColU + 32 * h, u);
        tmem_ld32(tl + kColA + 32 * h, w);
        float ek[32];
        load32(ek, gs.ekg + 32 * h);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float x[8], y[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            x[e] = __uint_as_float(u[8 * i + e]) - __uint_as_float(w[8 * i + e]);
            y[e] = x[e] * ek[8 * i + e];
          }
          st16(smem + Smem::Vp + sw128_chunk(dv, 4 * h + i), pack8(x));
          st16(smem + Smem::Vg + sw128_chunk(dv, 4 * h + i), pack8(y));
        }
      }
      fence_proxy_async();
      tc_fence_before();
      named_sync(kBarState, kGroup);
      // P3. M6: S^T += (e^{G_C - G} V')^T K first (the next chunk waits on
      //     it), then M5: Dy = V'^T P^T for the IO group.
      if (elected) {
        mbar_arrive(bar_du);
        tc_fence_after();
        constexpr uint32_t id5 = idesc_f16(128, C, false);
        constexpr uint32_t id6 = idesc_f16(128, 128, true);
#pragma unroll
        for (int k = 0; k < C / 16; ++k)
          mma_ss(tmem + kColS, desc_add(smem_desc(sbase + Smem::Vg, 16, 1024), k * 32),
                 desc_add(smem_desc(xs, 16384, 1024), k * 2048), id6, 1u);
        mma_commit(bar_m6);
#pragma unroll
        for (int k = 0; k < C / 16; ++k)
          mma_ss(tmem + kColY, desc_add(smem_desc(sbase + Smem::Vp, 16, 1024), k * 32),
                 desc_add(smem_desc(sbase + Smem::P + xbuf(n) * 8192, 16, 1024), k * 32), id5,
                 k > 0 ? 1u : 0u);
        mma_commit(bar_m56);
        m6_pending = m56_pending = int(n & 1);
      }
      // P4. The state after chunk n: fp16 for the next chunk's M4 and the
      //     fp32 accumulator scaled by the next chunk's e^{G_C} for its M6 (or,
      //     after the last chunk, the state to memory).
      fail = !wait_or_abort(bar_m6, n & 1, abort) ||
             (!last && !wait_or_abort(gate_bar(n + 1), gate_parity(n + 1), abort));
      if (named_sync_or(kBarState, kGroup, fail))
        break;
      m6_pending = -1;
      tc_fence_after();
      const float egl_next = last ? 1.f : gate_sets[(n + 1) % kGateSets].egl[0];
#pragma unroll 1
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t v[32];
        tmem_ld32(tl + kColS + 32 * q4, v);
        tmem_wait_ld();
        if (!last) {
          uint32_t h[16];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            h[j] = pack_half2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
          tmem_st16(tl + kColST + 16 * q4, h);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            v[j] = __float_as_uint(__uint_as_float(v[j]) * egl_next);
          tmem_st32(tl + kColS + 32 * q4, v);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            S[(32 * q4 + j) * DV + dv] = __uint_as_float(v[j]);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      named_sync(kBarState, kGroup);
    }
    if (elected) {
      if (m4_pending >= 0)
        mbar_wait(bar_m4, unsigned(m4_pending));
      if (m6_pending >= 0)
        mbar_wait(bar_m6, unsigned(m6_pending));
      if (m56_pending >= 0)
        mbar_wait(bar_m56, unsigned(m56_pending));
    }
  } else {
    // ================== IO group, presolved form (warps 8-11) ==================
    // The chunks' gates two ahead of the local chain; chunk n + 3's k rows
    // (bulk copy of their fp16 image) and q rows (converted) into the [K; Q]
    // buffer chunk n's MMAs release; y = e^G (Q S) + P V' from TMEM to
    // memory one chunk behind the state chain.
    const bool elected = gt == 0;
    const int dv = gt;
    int k_pending = -1;
    if (warp == 8) {
      for (uint32_t c = 0; c < 2 && c < n_chunks; ++c) {
        issue_gates(c);
        gates(c);
        if (lane == 0)
          mbar_arrive(gate_bar(c));
      }
      if (n_chunks > 2)
        issue_gates(2);
    }
    // [K; Q] buffers of chunks 0-2.
    bool pro_fail = false;
    for (uint32_t c = 0; c < kXBufs && c < n_chunks; ++c) {
      if (elected) {
        issue_k(c);
        k_pending = int(c & 1);
      }
      float4 qr[8][2];
      load_q(c, qr);
      bool f = false;
      if (elected) {
        f = !wait_or_abort(bar_k, c & 1, abort);
        if (!f)
          k_pending = -1;
      }
      if (named_sync_or(kBarIO, kGroup, f)) {
        pro_fail = true;
        break;
      }
      store_q(c, qr);
      named_sync(kBarIO, kGroup);
      if (elected)
        mbar_arrive(&bar_xready[xbuf(c)]);
    }
    for (uint32_t n = 0; n < n_chunks && !pro_fail; ++n) {
      const uint32_t t0 = n * C;
      const Gates &gs = gate_sets[n % kGateSets];
      // Q1. Gates of chunk n + 2 (they need only the decay and beta rows).
      if (warp == 8 && n + 2 < n_chunks) {
        gates(n + 2);
        if (n + 3 < n_chunks)
          issue_gates(n + 3);
        if (lane == 0)
          mbar_arrive(gate_bar(n + 2));
      }
      // Q2. Chunk n's M4 (Q half), M5 and M6 are done, which releases its
      //     [K; Q] buffer: chunk n + 3's k rows start to arrive in it.  The
      //     previous output tile has left shared memory.
      if (elected)
        bulk_wait_read();
      bool fail = !wait_or_abort(bar_m56, n & 1, abort);
      if (named_sync_or(kBarIO, kGroup, fail))
        break;
      tc_fence_after();
      const bool refill = n + kXBufs < n_chunks;
      if (elected && refill) {
        issue_k(n + kXBufs);
        k_pending = int((n + kXBufs) & 1);
        if (n + kXBufs + 1 < n_chunks)
          tma_prefetch_3d(&map_q, int(kh * DK), int(t0 + (kXBufs + 1) * C), int(seq));
      }
      // Q3. y^T = e^G (Q S)^T + Dy into the output tile, then to memory.
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        uint32_t ya[32], yd[32];
        tmem_ld32(tl + kColA + C + 32 * h, ya);
        tmem_ld32(tl + kColY + 32 * h, yd);
        float e[32];
        load32(e, gs.eg + 32 * h);
        tmem_wait_ld();
        __half *ys = reinterpret_cast<__half *>(smem + Smem::YsP) + dv;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          ys[(32 * h + j) * DV] =
              __float2half_rn(fmaf(e[j], __uint_as_float(ya[j]), __uint_as_float(yd[j])));
      }
      fence_proxy_async();
      tc_fence_before();
      named_sync(kBarIO, kGroup);
      if (elected) {
        mbar_arrive(bar_yread);
        tma_store_3d(&map_out, smem + Smem::YsP, int(vh * DV), int(t0), int(seq));
        bulk_commit();
      }
      // Q4. Chunk n + 3's q rows into the buffer; then it is ready.
      if (refill) {
        float4 qr[8][2];
        load_q(n + kXBufs, qr);
        fail = false;
        if (elected) {
          fail = !wait_or_abort(bar_k, (n + kXBufs) & 1, abort);
          if (!fail)
            k_pending = -1;
        }
        if (named_sync_or(kBarIO, kGroup, fail))
          break;
        store_q(n + kXBufs, qr);
        named_sync(kBarIO, kGroup);
        if (elected)
          mbar_arrive(&bar_xready[xbuf(n)]);
      }
    }
    if (elected) {
      if (k_pending >= 0)
        mbar_wait(bar_k, unsigned(k_pending));
      bulk_wait();
    }
    if (warp == 8)
      cp_async_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace delta_tc
}  // namespace llmi
