/*
 * llmi_cuda.h — C ABI of the B200 (sm_100a) attention backend for llminfer.
 *
 * These entry points replace, one for one, the Metal kernels that llminfer's
 * backend lowering dispatches for the attention ops of the Qwen3.5 hybrid
 * backbone (lib/Backend/Metal/MetalExecutionPlan.cpp:511-549 for
 * KvAppend/CausalGqa, :663-676 for DeltaUpdate).  The parameter structs keep
 * the field order and meaning of the reference's POD structs, so a CUDA
 * sibling of the lowering fills them exactly as the Metal lowering does.
 *
 * Conventions shared by every call:
 *  - All tensor pointers are DEVICE pointers owned by the caller (the
 *    executor); no call allocates, frees or retains them.  fp16 tensors are
 *    passed as uint16_t bit patterns (IEEE binary16).
 *  - `stream` is a cudaStream_t (NULL = the legacy default stream).  Calls are
 *    stream-ordered and do not synchronise; calls on different streams may run
 *    concurrently when they touch disjoint buffers.
 *  - The return value is an llmi_status.  On failure llmi_cuda_last_error()
 *    returns a message for the calling thread.  Argument errors are reported
 *    before anything is launched, so buffers are untouched (the reference's
 *    "failure before submit leaves the state untouched",
 *    lib/Backend/Metal/MetalExecutor.mm:285-287).
 *  - `batch` sequences are processed per call; sequence s of a tensor starts
 *    at element s * <stride> (cache strides are in elements).  Every sequence
 *    of a call shares the step shape (tokens, past), like one llminfer step.
 *  - There is no CPU fallback: shapes the CUDA kernels do not implement
 *    return LLMI_UNSUPPORTED.
 */
#ifndef LLMI_CUDA_H
#define LLMI_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  LLMI_OK = 0,
  LLMI_INVALID_ARGUMENT = 1,  /* rejected before launch; buffers untouched */
  LLMI_UNSUPPORTED = 2,       /* valid op, shape outside the CUDA kernels */
  LLMI_CUDA_ERROR = 3,        /* a CUDA runtime call failed */
  LLMI_DEVICE_TIMEOUT = 4,    /* a bounded device-side wait gave up */
  LLMI_WORKSPACE_TOO_SMALL = 5,
  LLMI_SESSION_INVALID = 6,   /* session poisoned by a failure after launch */
  LLMI_CAPACITY_EXCEEDED = 7  /* chunk does not fit capacity - past */
} llmi_status;

/* CacheParams (lib/Backend/Metal/Kernels/ReferenceParams.h:49-51):
 * `count` fp16 elements copied to element `offset` of each sequence's cache. */
typedef struct {
  unsigned count, offset;
} llmi_cache_params;

/* GqaParams (lib/Backend/Metal/Kernels/ReferenceParams.h:53-55). */
typedef struct {
  unsigned tokens, queryHeads, kvHeads, headDim, past;
} llmi_gqa_params;

/* GraphDeltaParams (lib/Backend/Metal/Kernels/GraphParams.h:50-52). */
typedef struct {
  unsigned tokens, keyHeads, keyDim, valueHeads, valueDim;
} llmi_delta_params;

/* Message of the calling thread's last failure ("" after success). */
const char *llmi_cuda_last_error(void);
/* Stable name of a status code, e.g. "LLMI_UNSUPPORTED". */
const char *llmi_cuda_status_name(int status);

/* cacheAppend (lib/Backend/Metal/Kernels/Reference.metal:295-301, lowered at
 * MetalExecutionPlan.cpp:516-522, once for keys and once for values):
 *   cache[s*cache_stride + p->offset + i] = input[s*input_stride + i]
 * for i < p->count and s < batch.  `input` rows are the step's new keys (or
 * values) [tokens][kvHeads][headDim]; offset = past*kvHeads*headDim. */
int llmi_cuda_cache_append(const llmi_cache_params *p, unsigned batch,
                           const uint16_t *input, size_t input_stride,
                           uint16_t *cache, size_t cache_stride, void *stream);

/* CausalGqa with tokens > 1: gqaFlashAttention
 * (lib/Backend/Metal/Kernels/FlashAttention.metal:1-83).
 *   q, out:  [batch][tokens][queryHeads][headDim] fp16, dense
 *   k_cache, v_cache: per sequence [capacity][kvHeads][headDim] fp16 at
 *            sequence stride cache_stride; rows [0, past+tokens) are read
 * Query token t attends to keys [0, past+t]; q head h reads kv head
 * h / (queryHeads/kvHeads); scores are scaled by 1/sqrt(headDim); softmax and
 * accumulation in fp32, output rounded to fp16.  Any tokens >= 1 is accepted. */
int llmi_cuda_gqa_prefill(const llmi_gqa_params *p, unsigned batch,
                          const uint16_t *q, const uint16_t *k_cache,
                          const uint16_t *v_cache, size_t cache_stride,
                          uint16_t *out, void *stream);

/* Bytes of device scratch llmi_cuda_gqa_decode needs for this shape on the
 * current device (0 on error; see llmi_cuda_last_error). */
size_t llmi_cuda_gqa_decode_workspace(const llmi_gqa_params *p, unsigned batch);

/* CausalGqa with tokens == 1: the reference's gqaScores / gqaSoftmax /
 * gqaValue dispatches (Reference.metal:303-323, Graph.metal:172-230,
 * lowered at MetalExecutionPlan.cpp:536-548), done as split-K flash decoding:
 * a partial-softmax pass over slices of the cache writes (max, sum, partial
 * output) records into `workspace`, and a merge pass combines them and writes
 * fp16 `out`.  Same layouts and semantics as llmi_cuda_gqa_prefill with
 * tokens == 1.  workspace_bytes must be at least
 * llmi_cuda_gqa_decode_workspace(p, batch). */
int llmi_cuda_gqa_decode(const llmi_gqa_params *p, unsigned batch,
                         const uint16_t *q, const uint16_t *k_cache,
                         const uint16_t *v_cache, size_t cache_stride,
                         uint16_t *out, void *workspace,
                         size_t workspace_bytes, void *stream);

/* KvAppend followed by CausalGqa with tokens == 1, in the decode's kernels: the
 * cacheAppend pair of the step's KvAppend (Reference.metal:295-301, lowered
 * at MetalExecutionPlan.cpp:516-522) and the decode above (:536-548), as the
 * reference's graph orders them (Graph.cpp:263-267).  Same result as
 *   llmi_cuda_cache_append(keys), llmi_cuda_cache_append(values),
 *   llmi_cuda_gqa_decode
 * with offset past*kvHeads*headDim and count kvHeads*headDim: after the call
 * row `past` of each sequence's caches holds k_new / v_new and `out` is the
 * decode over rows [0, past].  k_new, v_new: [batch][kvHeads][headDim] fp16
 * at sequence stride new_stride; either may be null when that cache row is
 * already written (e.g. keys written by llmi_cuda_norm_rope).  The partial
 * pass reads row `past` from k_new / v_new and the merge pass writes it into
 * the caches, which saves the two append launches of a decode step; shapes
 * that take the CUDA-core pass, and new rows that are not 16-byte aligned,
 * run the appends first as their own launches.  Workspace as
 * llmi_cuda_gqa_decode. */
int llmi_cuda_gqa_decode_append(const llmi_gqa_params *p, unsigned batch,
                                const uint16_t *q, const uint16_t *k_new,
                                const uint16_t *v_new, size_t new_stride,
                                uint16_t *k_cache, uint16_t *v_cache,
                                size_t cache_stride, uint16_t *out, void *workspace,
                                size_t workspace_bytes, void *stream);

/* Launch flag of the _ex entry points.  With it the caller guarantees that no
 * work that may still be running when the call's kernels start writes the
 * operands the call carries over from earlier steps: cache rows [0, past) of
 * a decode, the recurrent state of a DeltaNet update.  That holds when the
 * stream was synchronised after the last such write (a step-and-wait
 * executor, as the reference's MetalExecutor.mm:255-292), or when the write
 * belongs to an earlier CUDA graph launch on the stream.  It does not hold for
 * two calls on the same caches or state enqueued back to back.  The
 * decode-path kernels launch as programmatic dependents of the kernel ahead;
 * with the flag they read those operands before that kernel has finished.
 * The results are the same with and without it. */
#define LLMI_FLAG_SETTLED 1u

/* llmi_cuda_gqa_decode_append with launch flags (0 or LLMI_FLAG_SETTLED;
 * other bits are LLMI_INVALID_ARGUMENT).  The same lowering
 * (MetalExecutionPlan.cpp:516-548); the flag is the executor's knowledge of
 * its own step order. */
int llmi_cuda_gqa_decode_append_ex(const llmi_gqa_params *p, unsigned batch,
                                   const uint16_t *q, const uint16_t *k_new,
                                   const uint16_t *v_new, size_t new_stride,
                                   uint16_t *k_cache, uint16_t *v_cache,
                                   size_t cache_stride, uint16_t *out, void *workspace,
                                   size_t workspace_bytes, void *stream, unsigned flags);

/* Decode without a caller-provided workspace.  This entry point has no
 * counterpart in the reference.  It exists for callers that cannot allocate
 * device memory: an executor that hands out all device memory from its own
 * fixed arena and allows no other allocation, or a latency-critical decode
 * loop that cannot absorb the device-wide synchronisation cudaMalloc may
 * imply.  It computes exactly what llmi_cuda_gqa_decode computes, using as
 * scratch a fixed 8 MiB device array inside the library (held by every GPU
 * that loads the library until the process exits).  It allocates nothing and
 * frees nothing.
 *  - Shapes whose scratch would exceed 8 MiB are rejected with
 *    LLMI_WORKSPACE_TOO_SMALL before anything is launched; use
 *    llmi_cuda_gqa_decode for those.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress) with that device current; make that first call
 *    before any stream capture.
 *  - All calls share the one array, and it keeps the previous call's
 *    contents.  Nothing in it needs to start at zero: every record the merge
 *    pass reads is written earlier in the same call.
 *  - Calls that overlap on the GPU (for instance on two streams) race on the
 *    array; serialise them. */
int llmi_cuda_gqa_decode_noalloc(const llmi_gqa_params *p, unsigned batch,
                                 const uint16_t *q, const uint16_t *k_cache,
                                 const uint16_t *v_cache, size_t cache_stride,
                                 uint16_t *out, void *stream);

/* DeltaUpdate: graphDeltaUpdate (lib/Backend/Metal/Kernels/Graph.metal:146-170
 * with updateDeltaColumn, Reference.metal:182-197; operand contract
 * lib/GraphIR/Graph.cpp:226-246).  Per sequence:
 *   q, k:   [tokens][keyHeads*keyDim] fp32
 *   v:      [tokens][valueHeads*valueDim] fp16
 *   beta, decay: [tokens][valueHeads] fp32
 *   state:  [valueHeads][keyDim][valueDim] fp32, read and written in place
 *   out:    [tokens][valueHeads*valueDim] fp16
 * For each token: S = decay*S; pred = S^T k; delta = beta*(v - pred);
 * S += k delta^T; y = S^T q.  Value head vh uses key head
 * vh / (valueHeads/keyHeads).  Fewer than 16 tokens run the
 * register-resident recurrent kernel token by token; 16 or more (with
 * keyDim == valueDim == 128 and 16-byte aligned operands) run the chunked
 * (chunk 64) form on the tensor cores, equal up to rounding. */
int llmi_cuda_delta_update(const llmi_delta_params *p, unsigned batch,
                           const float *q, const float *k, const uint16_t *v,
                           const float *beta, const float *decay, float *state,
                           uint16_t *out, void *stream);

/* Bytes of device scratch llmi_cuda_delta_update_ws needs for this shape: 8 KB
 * per (sequence, value head, 64-token chunk) plus 16 KB per (sequence, key
 * head, chunk) when the call takes the chunked tensor-core form, else 0.  Same graphDeltaUpdate dispatch
 * (MetalExecutionPlan.cpp:663-676); the scratch is this backend's own. */
size_t llmi_cuda_delta_update_workspace(const llmi_delta_params *p, unsigned batch);

/* llmi_cuda_delta_update with caller scratch: for calls of 16 or more tokens
 * it solves every chunk's triangular system at once first (one CTA per
 * chunk and key head, all SMs busy) and keeps only the state recurrence
 * ordered over the chunks; same results up to rounding.  Shorter calls
 * ignore the workspace.  workspace_bytes must be at least
 * llmi_cuda_delta_update_workspace(p, batch), else LLMI_WORKSPACE_TOO_SMALL
 * before any launch. */
int llmi_cuda_delta_update_ws(const llmi_delta_params *p, unsigned batch,
                              const float *q, const float *k, const uint16_t *v,
                              const float *beta, const float *decay, float *state,
                              uint16_t *out, void *workspace, size_t workspace_bytes,
                              void *stream);

/* llmi_cuda_delta_update_ws with launch flags (0 or LLMI_FLAG_SETTLED; other
 * bits are LLMI_INVALID_ARGUMENT).  The same graphDeltaUpdate dispatch
 * (MetalExecutionPlan.cpp:663-676); the flag affects the recurrent form
 * (tokens < 16) only. */
int llmi_cuda_delta_update_ws_ex(const llmi_delta_params *p, unsigned batch,
                                 const float *q, const float *k, const uint16_t *v,
                                 const float *beta, const float *decay, float *state,
                                 uint16_t *out, void *workspace, size_t workspace_bytes,
                                 void *stream, unsigned flags);

/* ---- Producers of the path's operands -------------------------------------
 * The ops that turn the projections' outputs into the inputs of cacheAppend /
 * gqaFlashAttention and graphDeltaUpdate (Qwen35ModelBuilder.cpp:146-160 and
 * :187-192).  fp16 rounding points are the reference's, op by op; row sums
 * are warp trees, so fp32 results can differ from its serial order in the
 * last bits.  Argument errors are reported before any launch. */

/* RopeParams (lib/Backend/Metal/Kernels/ReferenceParams.h:44-47). */
typedef struct {
  unsigned tokens, heads, headDim, rotaryDim, headStride, past, outputStart;
  float epsilon, theta;
} llmi_rope_params;

/* ConvParams (lib/Backend/Metal/Kernels/ReferenceParams.h:32-34). */
typedef struct {
  unsigned tokens, channels, kernelSize, applySilu;
} llmi_conv_params;

/* L2Params (lib/Backend/Metal/Kernels/GraphParams.h:30-33). */
typedef struct {
  unsigned rows, width;
  float epsilon, scale;
} llmi_l2_params;

/* RowParams (lib/Backend/Metal/Kernels/ReferenceParams.h:23-26). */
typedef struct {
  unsigned rows, width;
  float epsilon;
} llmi_row_params;

/* DeltaParams (lib/Backend/Metal/Kernels/ReferenceParams.h:40-42), with the
 * conv kernel size and the L2Norm epsilon of the block. */
typedef struct {
  unsigned tokens, keyHeads, keyDim, valueHeads, valueDim, qkvWidth;
  unsigned kernelSize;
  float epsilon;
} llmi_delta_prep_params;

/* q/k RmsNorm + PartialRoPE, fused as normRope
 * (lib/Backend/Metal/Kernels/Reference.metal:271-293; = rmsNorm :105-117
 * then partialRope Graph.metal:111-129).  Per sequence s < batch, row r of
 * tokens*heads reads input + s*input_stride + r*headStride (headDim fp16;
 * headStride = 2*headDim for q sliced from q_proj's [q|gate] rows) and
 * writes output + s*output_stride + (outputStart*heads + r)*headDim: for
 * keys, pass the key cache and outputStart = past (the step's cacheAppend).
 * x = half(x * rsqrt(mean(x^2) + epsilon) * (1 + weight)), then pairs
 * (i, i + rotaryDim/2) rotate by (past + token) / theta^(2i/rotaryDim) with
 * fp16-rounded cos/sin.  headDim <= 1024, rotaryDim even, <= headDim and
 * <= 256. */
int llmi_cuda_norm_rope(const llmi_rope_params *p, unsigned batch, const uint16_t *input,
                        size_t input_stride, const float *weight, uint16_t *output,
                        size_t output_stride, void *stream);

/* PartialRoPE alone (lib/Backend/Metal/Kernels/Graph.metal:111-129, lowered
 * at MetalExecutionPlan.cpp:624-634): llmi_cuda_norm_rope without the norm;
 * epsilon is unused. */
int llmi_cuda_partial_rope(const llmi_rope_params *p, unsigned batch, const uint16_t *input,
                           size_t input_stride, uint16_t *output, size_t output_stride,
                           void *stream);

/* CausalConv1d (causalConv, lib/Backend/Metal/Kernels/Reference.metal:137-158,
 * lowered at MetalExecutionPlan.cpp:636-647 with applySilu 0).  Per
 * sequence: input/output [tokens][channels] fp16, weight [channels]
 * [kernelSize] fp16 (shared), history [channels][kernelSize-1] fp16 (the
 * ConvHistory state, read then advanced by the step).
 * out = half(sum_j w[j] x(t-K+1+j)), x before the step from the history;
 * with applySilu, half(silu(out)). */
int llmi_cuda_causal_conv(const llmi_conv_params *p, unsigned batch, const uint16_t *input,
                          size_t input_stride, const uint16_t *weight, uint16_t *history,
                          size_t history_stride, uint16_t *output, size_t output_stride,
                          void *stream);

/* L2Norm (l2NormF32, lib/Backend/Metal/Kernels/Graph.metal:96-109):
 * rows x width fp16 in, fp32 out, x * rsqrt(sum x^2 + epsilon) * scale. */
int llmi_cuda_l2_norm(const llmi_l2_params *p, const uint16_t *input, float *output,
                      void *stream);

/* DeltaGates (lib/Backend/Metal/Kernels/Graph.metal:131-144): a, b
 * [rows][width] fp16, aLog and dtBias [width] fp32 ->
 * beta = half(sigmoid(b)) and decay = exp(-exp(aLog) softplus(a + dtBias)),
 * [rows][width] fp32.  epsilon is unused. */
int llmi_cuda_delta_gates(const llmi_row_params *p, const uint16_t *a, const uint16_t *b,
                          const float *aLog, const float *dtBias, float *beta, float *decay,
                          void *stream);

/* The DeltaNet block's operands from its qkv projection, fused: CausalConv1d
 * with SiLU, the q/k/v Slices and the q and k L2Norms
 * (Qwen35ModelBuilder.cpp:146-157: q scaled by 1/sqrt(keyDim)).  Per
 * sequence: qkv [tokens][qkvWidth] fp16 in (qkvWidth = 2*keyHeads*keyDim +
 * valueHeads*valueDim), conv weight [qkvWidth][kernelSize] fp16, history as
 * for llmi_cuda_causal_conv; out q and k [tokens][keyHeads*keyDim] fp32 and
 * v [tokens][valueHeads*valueDim] fp16, the layouts llmi_cuda_delta_update
 * reads, packed over the batch.  keyDim, valueDim <= 256. */
int llmi_cuda_delta_prepare(const llmi_delta_prep_params *p, unsigned batch,
                            const uint16_t *qkv, size_t qkv_stride,
                            const uint16_t *conv_weight, uint16_t *history,
                            size_t history_stride, float *q, float *k, uint16_t *v,
                            void *stream);

/* Synchronises `stream`, then reads and clears the device error word that
 * kernels set when a bounded wait gives up.  Returns LLMI_OK,
 * LLMI_DEVICE_TIMEOUT or LLMI_CUDA_ERROR (for an asynchronous launch or
 * execution error).  The reference's equivalent check is the non-finite flag
 * read after each step (MetalExecutor.mm:180-187). */
int llmi_cuda_poll_error(void *stream);

/* Self-test of the failure path, for tests and health checks: launches on
 * `stream` one small kernel whose bounded wait on an mbarrier that nothing
 * completes gives up after limit_us (0 < limit_us <= 1e6) and raises the
 * device error word, exactly as a kernel's timed-out wait does.  The next
 * llmi_cuda_poll_error on that stream then returns LLMI_DEVICE_TIMEOUT.
 * Nothing faults or hangs. */
int llmi_cuda_selftest_wait_timeout(unsigned limit_us, void *stream);

/* ------------------------------------------------------------------------ */
/* Attention-stack session: the CUDA counterpart of MetalSession
 * (include/llminfer/Backend/Metal/MetalSession.h:28-44) reduced to the
 * attention ops.  It owns the per-layer state buffers (KV caches
 * [batch][capacity][kvHeads][headDim] fp16, recurrent states
 * [batch][valueHeads][keyDim][valueDim] fp32), keeps `past`, lowers each
 * step's ops to kernels with the reference's --plan names and runs them on
 * its stream. */

typedef struct llmi_session llmi_session;

enum { LLMI_LAYER_DELTANET = 0, LLMI_LAYER_GQA = 1 };

typedef struct {
  unsigned layers;
  const unsigned char *layer_kinds; /* layers entries of LLMI_LAYER_* */
  unsigned batch, capacity;
  unsigned queryHeads, kvHeads, headDim;            /* GQA layers */
  unsigned keyHeads, keyDim, valueHeads, valueDim;  /* DeltaNet layers */
} llmi_stack_config;

/* One layer's step operands (device pointers, dense, batch-major).
 *   GQA:      q f16 [B][T][Hq][D], k/v f16 [B][T][Hkv][D] (appended to the
 *             caches at rows [past, past+T)), out f16 [B][T][Hq][D]
 *   DeltaNet: q/k f32 [B][T][Hk*dk], v f16 [B][T][Hv*dv],
 *             beta/decay f32 [B][T][Hv], out f16 [B][T][Hv*dv] */
typedef struct {
  const void *q, *k, *v;
  const float *beta, *decay;
  void *out;
} llmi_layer_io;

enum {
  LLMI_STATE_KEYS = 0,
  LLMI_STATE_VALUES = 1,
  LLMI_STATE_RECURRENT = 2,
  LLMI_STATE_CONV_HISTORY = 3 /* DeltaNet layers, after set_producers */
};

/* Allocates and zeroes the states (MetalExecutor::initialize,
 * MetalExecutor.mm:56-94) on the current device; `stream` is borrowed. */
int llmi_cuda_session_open(const llmi_stack_config *config, void *stream,
                           llmi_session **session);
void llmi_cuda_session_close(llmi_session *session);

/* MetalSession::step (MetalExecutor.mm:255-292) for the attention ops: checks
 * 1 <= tokens <= capacity - past, lowers and launches every layer in order,
 * waits, checks the device error word, and advances past by tokens only on
 * success.  A failure after launch marks the session invalid until reset.
 * `io` has one entry per layer.  With trace_plan != 0 the dispatches are
 * recorded for llmi_cuda_session_plan. */
int llmi_cuda_session_step(llmi_session *session, unsigned tokens,
                           const llmi_layer_io *io, int trace_plan);

/* Like session_step but does not wait or poll: the work is only enqueued on
 * the session stream, and past advances when the launches were accepted.
 * For timed loops and CUDA-graph capture; follow with
 * llmi_cuda_session_sync before trusting the results.  A step enqueued right
 * after a synchronised one, or as the first step of a stream capture, passes
 * LLMI_FLAG_SETTLED to its decode-path calls; one enqueued behind an
 * unsynchronised step does not. */
int llmi_cuda_session_enqueue(llmi_session *session, unsigned tokens,
                              const llmi_layer_io *io);
/* Waits for the session stream and checks the device error word; on failure
 * the session becomes invalid. */
int llmi_cuda_session_sync(llmi_session *session);

/* Registers one cudaEvent_t per layer (count == layers; events == NULL with
 * count 0 clears them).  During step/enqueue the session records events[l]
 * on its stream right after the last launch of layer l, so a caller can
 * start a per-layer collective on another stream (cudaStreamWaitEvent) while
 * the following layers compute.  The events are borrowed, not destroyed. */
int llmi_cuda_session_set_layer_events(llmi_session *session,
                                       void *const *events, unsigned count);

/* Fault injection for tests: the next step or enqueue on this session also
 * launches llmi_cuda_selftest_wait_timeout(limit_us) after its kernels, so
 * its completion check reports LLMI_DEVICE_TIMEOUT and the session becomes
 * invalid, as after a real device-side failure (MetalExecutor.mm:285-287).
 * limit_us = 0 cancels a pending injection. */
int llmi_cuda_session_inject_fault(llmi_session *session, unsigned limit_us);

/* MetalSession::reset (MetalExecutor.mm:294-298): zero all states, past = 0,
 * clear the invalid mark. */
int llmi_cuda_session_reset(llmi_session *session);
uint64_t llmi_cuda_session_past(const llmi_session *session);
int llmi_cuda_session_is_invalid(const llmi_session *session);

/* Device pointer and size of one state buffer of `layer`
 * (which = LLMI_STATE_*).  Work that writes a buffer through this pointer
 * must be complete before the session's next step is issued (e.g. followed
 * by a stream synchronisation): after a synchronised step, and for the first
 * step of a stream capture, the session's decode-path calls pass
 * LLMI_FLAG_SETTLED. */
int llmi_cuda_session_state(llmi_session *session, unsigned layer,
                            unsigned which, void **pointer, size_t *bytes);

/* Copies `bytes` bytes between a state buffer of `layer` and caller device
 * memory, ordered on the session stream (read: state -> dst, write:
 * src -> state), then waits.  bytes must equal the state's size.  Used to
 * seed recurrent states and to inspect caches and states. */
int llmi_cuda_session_read_state(llmi_session *session, unsigned layer,
                                 unsigned which, void *dst, size_t bytes);
int llmi_cuda_session_write_state(llmi_session *session, unsigned layer,
                                  unsigned which, const void *src,
                                  size_t bytes);

/* Producers of the layers' operands inside the session: the KV-cache
 * producers and the DeltaNet input producers run ahead of the attention
 * ops.  Settings of Qwen3.5's q/k RmsNorm + PartialRoPE
 * (Qwen35ModelBuilder.cpp:187-191) and of the DeltaNet block's conv, L2Norm
 * and gates (Qwen35ModelBuilder.cpp:146-157). */
typedef struct {
  unsigned rotaryDim;  /* even, <= headDim and <= 256 */
  float ropeTheta, normEpsilon;
  unsigned convKernel; /* 1..8 */
  float l2Epsilon;
} llmi_producer_config;

/* Enables llmi_cuda_session_step_projections: keeps the settings and
 * allocates one ConvHistory state per DeltaNet layer ([batch][W][convKernel-1]
 * fp16, W = 2*keyHeads*keyDim + valueHeads*valueDim), zeroed now and by every
 * reset.  Once per session. */
int llmi_cuda_session_set_producers(llmi_session *session,
                                    const llmi_producer_config *config);

/* One layer's projection outputs and weights (device pointers, dense,
 * batch-major), the inputs of llmi_cuda_session_step_projections:
 *   GQA:      qg f16 [B][T][Hq][2D] (q_proj's [q | gate] rows; q is read,
 *             gate is left to the caller), k, v f16 [B][T][Hkv][D],
 *             qNorm, kNorm f32 [D] (RmsNorm weights, applied as 1 + w),
 *             out f16 [B][T][Hq][D]
 *   DeltaNet: qkv f16 [B][T][W], a, b f16 [B][T][Hv], convWeight f16 [W][K],
 *             aLog, dtBias f32 [Hv], out f16 [B][T][Hv*dv] */
typedef struct {
  const void *qg, *k, *v;
  const float *qNorm, *kNorm;
  const void *qkv, *a, *b, *convWeight;
  const float *aLog, *dtBias;
  void *out;
} llmi_layer_projections;

/* llmi_cuda_session_step from the projections: per GQA layer normRope of q
 * (into session scratch), normRope of k straight into the key cache at row
 * past (the keys' cacheAppend), cacheAppend of v, then the attention; per
 * DeltaNet layer deltaPrepare (conv + SiLU over the layer's ConvHistory, the
 * slices, the q/k L2Norms) and deltaGates into session scratch, then
 * graphDeltaUpdate.  Same checks, wait and failure rules as session_step;
 * the scratch grows to the largest step seen (so the first step of a size
 * may allocate).  The traced plan lists the producer dispatches too. */
int llmi_cuda_session_step_projections(llmi_session *session, unsigned tokens,
                                       const llmi_layer_projections *io,
                                       int trace_plan);

/* The last traced step's dispatches as JSON lines
 * {"op_index":i,"kernel":"...","layer":l} — the records llmi-run --plan prints
 * (tools/run/Main.cpp:244-255).  Copies at most len-1 bytes plus a NUL and
 * returns the full length. */
size_t llmi_cuda_session_plan(const llmi_session *session, char *buffer,
                              size_t len);

/* Host-only lowering of one step (no GPU needed): JSON with the step, each
 * op's kind, layer, state effects and logical cost (the `llmi graph --json`
 * fields of tools/modelconverter/GraphCommand.cpp:82-146 for these ops), and
 * the dispatches the CUDA backend would launch.  Returns the full length
 * (0 on error, with *status set). */
size_t llmi_cuda_describe_step(const llmi_stack_config *config,
                               unsigned tokens, uint64_t past, char *buffer,
                               size_t len, int *status);

#ifdef __cplusplus
}
#endif

#endif
