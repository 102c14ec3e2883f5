// Attention-stack session: the CUDA counterpart of MetalSession /
// MetalExecutor (lib/Backend/Metal/MetalExecutor.mm) restricted to the
// attention ops.  It owns the state buffers, keeps `past`, lowers every step
// through AttentionGraph + lower() and launches the kernels of the C ABI on
// its stream.  Semantics kept from the reference:
//   - open allocates one buffer per state slot and zeroes it
//     (MetalExecutor::initialize, MetalExecutor.mm:56-94);
//   - step rejects an empty chunk or one that exceeds capacity - past before
//     touching anything (MetalExecutor.mm:261-265);
//   - a failure after work was launched marks the session invalid until
//     reset (MetalExecutor.mm:259-260, 285-287);
//   - past advances only on success (MetalExecutor.mm:289);
//   - reset zeroes every state and sets past = 0 (MetalExecutor.mm:294-298);
//   - calls on one session must be serialised (MetalSession.h:40).
// Every sequence of the batch has its own slice of each state buffer, in the
// reference's per-sequence layout.
#include "attention_graph.h"
#include "status.h"

#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

using namespace llmi;
using namespace llmi::host;

struct llmi_session {
  StackConfig config;
  cudaStream_t stream = nullptr;
  int device = 0;
  // Per layer; null where the layer has no such state.
  std::vector<void *> keys, values, recurrent;
  size_t cacheBytes = 0, recurrentBytes = 0;  // whole batch, per buffer
  void *workspace = nullptr;
  size_t workspaceBytes = 0;
  uint64_t past = 0;
  bool invalid = false;
  // Whether this session's earlier steps are complete before the next step's
  // kernels can start, so that its decode-path calls may pass
  // LLMI_FLAG_SETTLED for the caches and states they carry over: yes after a
  // synchronising step or sync; no after an eagerly enqueued step; under
  // stream capture, yes for the first step of a capture (a graph launch runs
  // after all earlier work on its stream), no for later ones.
  bool inFlight = false;
  unsigned long long lastCaptureId = 0;
  std::string plan;
  std::vector<cudaEvent_t> layerEvents;  // borrowed; recorded after each layer
  unsigned injectFaultUs = 0;             // > 0: the next step also runs the wait self-test
  // Producers (llmi_cuda_session_set_producers): their settings, the
  // ConvHistory state of each DeltaNet layer and a scratch arena for the
  // producers' outputs, shared by the layers (they run in order on one
  // stream).
  bool producers = false;
  llmi_producer_config prod{};
  std::vector<void *> convHistory;
  size_t historyBytes = 0;
  void *scratch = nullptr;
  size_t scratchBytes = 0;

  ~llmi_session() {
    for (auto *list : {&keys, &values, &recurrent, &convHistory})
      for (void *p : *list)
        if (p)
          cudaFree(p);
    if (workspace)
      cudaFree(workspace);
    if (scratch)
      cudaFree(scratch);
  }
};

namespace {

int zero_states(llmi_session &s) {
  for (size_t l = 0; l < s.config.kinds.size(); ++l) {
    if (s.keys[l]) {
      if (int e = check_cuda(cudaMemsetAsync(s.keys[l], 0, s.cacheBytes, s.stream), "zero keys"))
        return e;
      if (int e = check_cuda(cudaMemsetAsync(s.values[l], 0, s.cacheBytes, s.stream),
                             "zero values"))
        return e;
    }
    if (s.recurrent[l])
      if (int e = check_cuda(cudaMemsetAsync(s.recurrent[l], 0, s.recurrentBytes, s.stream),
                             "zero recurrent state"))
        return e;
    if (l < s.convHistory.size() && s.convHistory[l])
      if (int e = check_cuda(cudaMemsetAsync(s.convHistory[l], 0, s.historyBytes, s.stream),
                             "zero conv history"))
        return e;
  }
  return check_cuda(cudaStreamSynchronize(s.stream), "zero states");
}

int ensure_workspace(llmi_session &s, size_t bytes) {
  if (bytes <= s.workspaceBytes)
    return LLMI_OK;
  if (s.workspace) {
    if (int e = check_cuda(cudaStreamSynchronize(s.stream), "workspace resize"))
      return e;
    cudaFree(s.workspace);
    s.workspace = nullptr;
    s.workspaceBytes = 0;
  }
  if (int e = check_cuda(cudaMalloc(&s.workspace, bytes), "allocate decode workspace"))
    return e;
  s.workspaceBytes = bytes;
  return LLMI_OK;
}

int check_io(const llmi_session &s, const llmi_layer_io *io) {
  if (!io)
    return fail(LLMI_INVALID_ARGUMENT, "step: null layer operand table");
  for (size_t l = 0; l < s.config.kinds.size(); ++l) {
    const llmi_layer_io &x = io[l];
    const bool delta = s.config.kinds[l] == LLMI_LAYER_DELTANET;
    if (!x.q || !x.k || !x.v || !x.out || (delta && (!x.beta || !x.decay)))
      return fail(LLMI_INVALID_ARGUMENT, "step: layer %zu is missing an operand", l);
  }
  return LLMI_OK;
}

int check_projections(const llmi_session &s, const llmi_layer_projections *io) {
  if (!s.producers)
    return fail(LLMI_INVALID_ARGUMENT,
                "step_projections: the session has no producer settings (set_producers)");
  if (!io)
    return fail(LLMI_INVALID_ARGUMENT, "step_projections: null layer operand table");
  for (size_t l = 0; l < s.config.kinds.size(); ++l) {
    const llmi_layer_projections &x = io[l];
    const bool ok = s.config.kinds[l] == LLMI_LAYER_GQA
                        ? x.qg && x.k && x.v && x.qNorm && x.kNorm && x.out
                        : x.qkv && x.a && x.b && x.convWeight && x.aLog && x.dtBias && x.out;
    if (!ok)
      return fail(LLMI_INVALID_ARGUMENT, "step_projections: layer %zu is missing an operand", l);
  }
  return LLMI_OK;
}

// Offsets of the producers' outputs in the scratch arena for a step of
// `tokens` (256-byte aligned): GQA layers use q, DeltaNet layers q..decay.
struct ScratchLayout {
  size_t q = 0, k = 0, v = 0, beta = 0, decay = 0, bytes = 0;
  ScratchLayout(const StackConfig &c, unsigned tokens) {
    const size_t rows = size_t(c.batch) * tokens;
    auto up = [](size_t n) { return (n + 255) & ~size_t(255); };
    const size_t gqa = up(rows * c.queryHeads * c.headDim * 2);
    k = up(rows * c.keyHeads * c.keyDim * 4);
    v = 2 * k;
    beta = v + up(rows * c.valueHeads * c.valueDim * 2);
    decay = beta + up(rows * c.valueHeads * 4);
    const size_t delta = decay + up(rows * c.valueHeads * 4);
    bytes = std::max(c.hasGqa() ? gqa : 0, c.hasDelta() ? delta : 0);
  }
};

int ensure_scratch(llmi_session &s, size_t bytes) {
  if (bytes <= s.scratchBytes)
    return LLMI_OK;
  if (s.scratch) {
    if (int e = check_cuda(cudaStreamSynchronize(s.stream), "scratch resize"))
      return e;
    cudaFree(s.scratch);
    s.scratch = nullptr;
    s.scratchBytes = 0;
  }
  if (int e = check_cuda(cudaMalloc(&s.scratch, bytes), "allocate producer scratch"))
    return e;
  s.scratchBytes = bytes;
  return LLMI_OK;
}

// Lowers and launches one step.  `launchedAny` reports whether any kernel
// may have been enqueued (the reference's "submitted").  With `proj`, each
// layer's producers run first (into the scratch arena, and for keys straight
// into the cache) and the layer's attention operands are their outputs.
int run_step(llmi_session &s, unsigned tokens, const llmi_layer_io *io, bool trace,
             bool &launchedAny, const llmi_layer_projections *proj = nullptr) {
  launchedAny = false;
  AttentionGraph graph;
  if (int e = AttentionGraph::build(s.config, {tokens, s.past, s.config.capacity}, graph))
    return e;
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  unsigned long long captureId = 0;
  if (int e = check_cuda(cudaStreamGetCaptureInfo(s.stream, &capture, &captureId),
                         "cudaStreamGetCaptureInfo"))
    return e;
  const bool capturing = capture == cudaStreamCaptureStatusActive;
  // Each layer's caches and state are written once per step, by its own op,
  // so within a step nothing ahead of an op writes what it carries over.
  const unsigned flags =
      (capturing ? captureId != s.lastCaptureId : !s.inFlight) ? LLMI_FLAG_SETTLED : 0u;
  struct Mark {
    llmi_session &s;
    bool capturing;
    unsigned long long id;
    const bool &launched;
    ~Mark() {
      if (!launched)
        return;
      if (capturing)
        s.lastCaptureId = id;
      else
        s.inFlight = true;
    }
  } mark{s, capturing, captureId, launchedAny};
  const StackConfig &c = s.config;
  const unsigned B = c.batch;
  std::vector<llmi_layer_io> produced;
  ScratchLayout layout(c, tokens);
  if (proj) {
    if (int e = check_projections(s, proj))
      return e;
    if (int e = ensure_scratch(s, layout.bytes))
      return e;
    produced.assign(c.kinds.size(), llmi_layer_io{});
    io = produced.data();
  } else if (int e = check_io(s, io)) {
    return e;
  }
  if (tokens == 1 && c.hasGqa()) {
    llmi_gqa_params g{1, c.queryHeads, c.kvHeads, c.headDim, unsigned(s.past)};
    const size_t need = llmi_cuda_gqa_decode_workspace(&g, B);
    if (!need)
      return fail(LLMI_CUDA_ERROR, "decode workspace: %s", last_error());
    if (int e = ensure_workspace(s, need))
      return e;
  }
  // Multi-token DeltaNet steps solve every chunk's system first, into the
  // same workspace (a step has either a decode or a chunked DeltaUpdate
  // need, never both); it grows to the longest prefill step seen.
  if (tokens > 1 && c.hasDelta()) {
    llmi_delta_params d{tokens, c.keyHeads, c.keyDim, c.valueHeads, c.valueDim};
    if (const size_t need = llmi_cuda_delta_update_workspace(&d, B))
      if (int e = ensure_workspace(s, need))
        return e;
  }
  const size_t cacheStride = size_t(c.capacity) * c.kvHeads * c.headDim;
  const auto dispatches = lower(graph);
  size_t next = 0;  // first dispatch of the current op
  const auto &ops = graph.ops();
  auto record = [&](size_t opIndex, const char *kernel, uint32_t layer) {
    char line[160];
    std::snprintf(line, sizeof line, "{\"op_index\":%zu,\"kernel\":\"%s\",\"layer\":%u}\n",
                  opIndex, kernel, layer);
    s.plan += line;
  };
  // The producers of layer l from its projections (step_projections).
  auto produce = [&](uint32_t l, size_t opIndex) -> int {
    const llmi_layer_projections &p = proj[l];
    llmi_layer_io &x = produced[l];
    uint8_t *base = static_cast<uint8_t *>(s.scratch);
    x.out = p.out;
    launchedAny = true;
    if (c.kinds[l] == LLMI_LAYER_GQA) {
      uint16_t *q = reinterpret_cast<uint16_t *>(base + layout.q);
      const llmi_rope_params rq{tokens, c.queryHeads, c.headDim, s.prod.rotaryDim,
                                2 * c.headDim, unsigned(s.past), 0u, s.prod.normEpsilon,
                                s.prod.ropeTheta};
      if (int e = llmi_cuda_norm_rope(&rq, B, static_cast<const uint16_t *>(p.qg),
                                      size_t(tokens) * c.queryHeads * 2 * c.headDim, p.qNorm, q,
                                      size_t(tokens) * c.queryHeads * c.headDim, s.stream))
        return e;
      // Keys go straight into the cache at row past: the keys' cacheAppend.
      const llmi_rope_params rk{tokens, c.kvHeads, c.headDim, s.prod.rotaryDim, c.headDim,
                                unsigned(s.past), unsigned(s.past), s.prod.normEpsilon,
                                s.prod.ropeTheta};
      if (int e = llmi_cuda_norm_rope(&rk, B, static_cast<const uint16_t *>(p.k),
                                      size_t(tokens) * c.kvHeads * c.headDim, p.kNorm,
                                      static_cast<uint16_t *>(s.keys[l]), cacheStride, s.stream))
        return e;
      x.q = q;
      x.v = p.v;
      if (trace) {
        record(opIndex, "normRope", l);
        record(opIndex, "normRope", l);
      }
    } else {
      const unsigned W = 2 * c.keyHeads * c.keyDim + c.valueHeads * c.valueDim;
      float *q = reinterpret_cast<float *>(base + layout.q);
      float *k = reinterpret_cast<float *>(base + layout.k);
      uint16_t *v = reinterpret_cast<uint16_t *>(base + layout.v);
      float *beta = reinterpret_cast<float *>(base + layout.beta);
      float *decay = reinterpret_cast<float *>(base + layout.decay);
      const llmi_delta_prep_params dp{tokens, c.keyHeads, c.keyDim, c.valueHeads, c.valueDim,
                                      W, s.prod.convKernel, s.prod.l2Epsilon};
      if (int e = llmi_cuda_delta_prepare(&dp, B, static_cast<const uint16_t *>(p.qkv),
                                          size_t(tokens) * W,
                                          static_cast<const uint16_t *>(p.convWeight),
                                          static_cast<uint16_t *>(s.convHistory[l]),
                                          size_t(W) * (s.prod.convKernel - 1), q, k, v, s.stream))
        return e;
      const llmi_row_params rp{B * tokens, c.valueHeads, 0.f};
      if (int e = llmi_cuda_delta_gates(&rp, static_cast<const uint16_t *>(p.a),
                                        static_cast<const uint16_t *>(p.b), p.aLog, p.dtBias,
                                        beta, decay, s.stream))
        return e;
      x.q = q;
      x.k = k;
      x.v = v;
      x.beta = beta;
      x.decay = decay;
      if (trace) {
        record(opIndex, "deltaPrepare", l);
        record(opIndex, "deltaGates", l);
      }
    }
    return LLMI_OK;
  };
  // A decode step's KvAppend rows, held for the layer's CausalGqa, which
  // appends them in its own partial pass (llmi_cuda_gqa_decode_append).
  const uint16_t *foldK = nullptr, *foldV = nullptr;
  for (size_t i = 0; i < ops.size(); ++i) {
    const Op &op = ops[i];
    if (proj && (i == 0 || ops[i - 1].layer != op.layer))
      if (int e = produce(op.layer, next < dispatches.size() ? dispatches[next].opIndex : i))
        return e;
    const llmi_layer_io &x = io[op.layer];
    int e = LLMI_OK;
    size_t count = 1;
    size_t skip = 0;  // leading dispatches of the op that the producers already did
    // One NVTX range per op (no-op unless a profiler is attached), named
    // like its first --plan dispatch.
    struct Range {
      explicit Range(const char *name) { nvtxRangePushA(name); }
      ~Range() { nvtxRangePop(); }
    } range(next < dispatches.size() ? dispatches[next].kernel : "op");
    switch (op.kind) {
    case OpKind::KvAppend: {
      const unsigned row = c.kvHeads * c.headDim;
      llmi_cache_params p{tokens * row, unsigned(s.past) * row};
      const size_t inStride = size_t(tokens) * row;
      launchedAny = true;
      if (proj)
        skip = 1;  // normRope wrote the keys
      count = 2;
      if (tokens == 1 && i + 1 < ops.size() && ops[i + 1].kind == OpKind::CausalGqa &&
          ops[i + 1].layer == op.layer) {
        foldK = proj ? nullptr : static_cast<const uint16_t *>(x.k);
        foldV = static_cast<const uint16_t *>(x.v);
        break;
      }
      if (!proj)
        e = llmi_cuda_cache_append(&p, B, static_cast<const uint16_t *>(x.k), inStride,
                                   static_cast<uint16_t *>(s.keys[op.layer]), cacheStride,
                                   s.stream);
      if (!e)
        e = llmi_cuda_cache_append(&p, B, static_cast<const uint16_t *>(x.v), inStride,
                                   static_cast<uint16_t *>(s.values[op.layer]), cacheStride,
                                   s.stream);
      break;
    }
    case OpKind::CausalGqa: {
      llmi_gqa_params p{tokens, c.queryHeads, c.kvHeads, c.headDim, unsigned(s.past)};
      launchedAny = true;
      if (tokens > 1) {
        e = llmi_cuda_gqa_prefill(&p, B, static_cast<const uint16_t *>(x.q),
                                  static_cast<const uint16_t *>(s.keys[op.layer]),
                                  static_cast<const uint16_t *>(s.values[op.layer]), cacheStride,
                                  static_cast<uint16_t *>(x.out), s.stream);
      } else if (foldK || foldV) {
        e = llmi_cuda_gqa_decode_append_ex(
            &p, B, static_cast<const uint16_t *>(x.q), foldK, foldV,
            size_t(c.kvHeads) * c.headDim, static_cast<uint16_t *>(s.keys[op.layer]),
            static_cast<uint16_t *>(s.values[op.layer]), cacheStride,
            static_cast<uint16_t *>(x.out), s.workspace, s.workspaceBytes, s.stream, flags);
        foldK = foldV = nullptr;
        count = 2;
      } else {
        e = llmi_cuda_gqa_decode(&p, B, static_cast<const uint16_t *>(x.q),
                                 static_cast<const uint16_t *>(s.keys[op.layer]),
                                 static_cast<const uint16_t *>(s.values[op.layer]), cacheStride,
                                 static_cast<uint16_t *>(x.out), s.workspace, s.workspaceBytes,
                                 s.stream);
        count = 2;
      }
      break;
    }
    case OpKind::DeltaUpdate: {
      llmi_delta_params p{tokens, c.keyHeads, c.keyDim, c.valueHeads, c.valueDim};
      launchedAny = true;
      e = llmi_cuda_delta_update_ws_ex(&p, B, static_cast<const float *>(x.q),
                                       static_cast<const float *>(x.k),
                                       static_cast<const uint16_t *>(x.v), x.beta, x.decay,
                                       static_cast<float *>(s.recurrent[op.layer]),
                                       static_cast<uint16_t *>(x.out), s.workspace,
                                       s.workspaceBytes, s.stream, flags);
      break;
    }
    }
    if (e)
      return e;
    if (!s.layerEvents.empty() && (i + 1 == ops.size() || ops[i + 1].layer != op.layer))
      if (int st = check_cuda(cudaEventRecord(s.layerEvents[op.layer], s.stream),
                              "record layer event"))
        return st;
    if (trace)
      for (size_t d = next + skip; d < next + count && d < dispatches.size(); ++d)
        record(dispatches[d].opIndex, dispatches[d].kernel, dispatches[d].layer);
    next += count;
  }
  if (s.injectFaultUs) {
    launchedAny = true;
    const unsigned limit = s.injectFaultUs;
    s.injectFaultUs = 0;
    if (int e = llmi_cuda_selftest_wait_timeout(limit, s.stream))
      return e;
  }
  return LLMI_OK;
}

}  // namespace

extern "C" int llmi_cuda_session_open(const llmi_stack_config *config, void *stream,
                                      llmi_session **session) {
  clear_error();
  if (!session)
    return fail(LLMI_INVALID_ARGUMENT, "session_open: null output pointer");
  *session = nullptr;
  StackConfig c;
  if (int e = StackConfig::from(config, c))
    return e;
  auto *s = new llmi_session;
  s->config = c;
  s->stream = static_cast<cudaStream_t>(stream);
  if (int e = check_cuda(cudaGetDevice(&s->device), "cudaGetDevice")) {
    delete s;
    return e;
  }
  const size_t layers = c.kinds.size();
  s->keys.assign(layers, nullptr);
  s->values.assign(layers, nullptr);
  s->recurrent.assign(layers, nullptr);
  s->cacheBytes = size_t(c.batch) * c.capacity * c.kvHeads * c.headDim * 2;
  s->recurrentBytes = size_t(c.batch) * c.valueHeads * c.keyDim * c.valueDim * 4;
  for (size_t l = 0; l < layers; ++l) {
    int e = LLMI_OK;
    if (c.kinds[l] == LLMI_LAYER_GQA) {
      e = check_cuda(cudaMalloc(&s->keys[l], s->cacheBytes), "allocate key cache");
      if (!e)
        e = check_cuda(cudaMalloc(&s->values[l], s->cacheBytes), "allocate value cache");
    } else {
      e = check_cuda(cudaMalloc(&s->recurrent[l], s->recurrentBytes), "allocate recurrent state");
    }
    if (e) {
      delete s;
      return e;
    }
  }
  // The decode workspace is sized once, for the largest need over every
  // `past` the session can reach (the split changes every 16 keys), so no
  // step allocates: steps can be captured into CUDA graphs.
  if (c.hasGqa()) {
    std::vector<uint64_t> pasts;
    for (uint64_t past = 0; past < c.capacity; past += 16)
      pasts.push_back(past);
    pasts.push_back(c.capacity - 1);
    size_t need = 0;
    for (const uint64_t past : pasts) {
      llmi_gqa_params g{1, c.queryHeads, c.kvHeads, c.headDim, unsigned(past)};
      const size_t bytes = llmi_cuda_gqa_decode_workspace(&g, c.batch);
      if (!bytes) {
        delete s;
        return fail(LLMI_CUDA_ERROR, "decode workspace: %s", last_error());
      }
      need = std::max(need, bytes);
    }
    if (int e = ensure_workspace(*s, need)) {
      delete s;
      return e;
    }
  }
  if (int e = zero_states(*s)) {
    delete s;
    return e;
  }
  *session = s;
  return LLMI_OK;
}

extern "C" void llmi_cuda_session_close(llmi_session *session) {
  if (session)
    cudaStreamSynchronize(session->stream);
  delete session;
}

namespace {

// session_step and session_step_projections: launch, wait, check the device
// error word; past advances only on success, and a failure after launch
// invalidates the session.
int step_and_wait(llmi_session *s, unsigned tokens, const llmi_layer_io *io,
                  const llmi_layer_projections *proj, int trace_plan) {
  clear_error();
  if (!s)
    return fail(LLMI_INVALID_ARGUMENT, "step: null session");
  if (s->invalid)
    return fail(LLMI_SESSION_INVALID, "CUDA session is invalid after a failed GPU step");
  if (trace_plan)
    s->plan.clear();
  bool launchedAny = false;
  int e = run_step(*s, tokens, io, trace_plan != 0, launchedAny, proj);
  if (!e && launchedAny)
    e = llmi_cuda_poll_error(s->stream);
  if (e) {
    s->invalid = launchedAny;
    return e;
  }
  s->inFlight = false;  // poll_error synchronised the stream
  s->past += tokens;
  return LLMI_OK;
}

}  // namespace

extern "C" int llmi_cuda_session_step(llmi_session *s, unsigned tokens, const llmi_layer_io *io,
                                      int trace_plan) {
  return step_and_wait(s, tokens, io, nullptr, trace_plan);
}

extern "C" int llmi_cuda_session_step_projections(llmi_session *s, unsigned tokens,
                                                  const llmi_layer_projections *io,
                                                  int trace_plan) {
  if (!io) {
    clear_error();
    return fail(LLMI_INVALID_ARGUMENT, "step_projections: null layer operand table");
  }
  return step_and_wait(s, tokens, nullptr, io, trace_plan);
}

extern "C" int llmi_cuda_session_set_producers(llmi_session *s, const llmi_producer_config *p) {
  clear_error();
  if (!s || !p)
    return fail(LLMI_INVALID_ARGUMENT, "set_producers: null session or settings");
  if (s->producers)
    return fail(LLMI_INVALID_ARGUMENT, "set_producers: already set for this session");
  const StackConfig &c = s->config;
  if (c.hasGqa() && (p->rotaryDim % 2 || p->rotaryDim > c.headDim || p->rotaryDim > 256 ||
                     c.headDim > 1024))
    return fail(LLMI_UNSUPPORTED,
                "set_producers: rotaryDim %u (even, <= headDim %u and <= 256; headDim <= 1024)",
                p->rotaryDim, c.headDim);
  if (c.hasDelta() && (p->convKernel < 2 || p->convKernel > 8 || c.keyDim > 256 ||
                       c.valueDim > 256))
    return fail(LLMI_UNSUPPORTED,
                "set_producers: convKernel %u (2..8) with keyDim %u / valueDim %u (<= 256)",
                p->convKernel, c.keyDim, c.valueDim);
  const size_t W = 2 * size_t(c.keyHeads) * c.keyDim + size_t(c.valueHeads) * c.valueDim;
  s->convHistory.assign(c.kinds.size(), nullptr);
  s->historyBytes = size_t(c.batch) * W * (p->convKernel - 1) * 2;
  for (size_t l = 0; l < c.kinds.size(); ++l) {
    if (c.kinds[l] != LLMI_LAYER_DELTANET)
      continue;
    if (int e = check_cuda(cudaMalloc(&s->convHistory[l], s->historyBytes),
                           "allocate conv history"))
      return e;
    if (int e = check_cuda(cudaMemsetAsync(s->convHistory[l], 0, s->historyBytes, s->stream),
                           "zero conv history"))
      return e;
  }
  if (int e = check_cuda(cudaStreamSynchronize(s->stream), "zero conv history"))
    return e;
  s->prod = *p;
  s->producers = true;
  return LLMI_OK;
}

extern "C" int llmi_cuda_session_enqueue(llmi_session *s, unsigned tokens,
                                         const llmi_layer_io *io) {
  clear_error();
  if (!s)
    return fail(LLMI_INVALID_ARGUMENT, "enqueue: null session");
  if (s->invalid)
    return fail(LLMI_SESSION_INVALID, "CUDA session is invalid after a failed GPU step");
  bool launchedAny = false;
  if (int e = run_step(*s, tokens, io, false, launchedAny)) {
    s->invalid = launchedAny;
    return e;
  }
  s->past += tokens;
  return LLMI_OK;
}

extern "C" int llmi_cuda_session_sync(llmi_session *s) {
  clear_error();
  if (!s)
    return fail(LLMI_INVALID_ARGUMENT, "sync: null session");
  if (int e = llmi_cuda_poll_error(s->stream)) {
    s->invalid = true;
    return e;
  }
  s->inFlight = false;
  return LLMI_OK;
}

extern "C" int llmi_cuda_session_set_layer_events(llmi_session *s, void *const *events,
                                                  unsigned count) {
  clear_error();
  if (!s)
    return fail(LLMI_INVALID_ARGUMENT, "set_layer_events: null session");
  if (count == 0 && !events) {
    s->layerEvents.clear();
    return LLMI_OK;
  }
  if (!events || count != s->config.kinds.size())
    return fail(LLMI_INVALID_ARGUMENT, "set_layer_events: %u events for %zu layers", count,
                s->config.kinds.size());
  std::vector<cudaEvent_t> list(count);
  for (unsigned l = 0; l < count; ++l) {
    if (!events[l])
      return fail(LLMI_INVALID_ARGUMENT, "set_layer_events: event %u is null", l);
    list[l] = static_cast<cudaEvent_t>(events[l]);
  }
  s->layerEvents = std::move(list);
  return LLMI_OK;
}

extern "C" int llmi_cuda_session_inject_fault(llmi_session *s, unsigned limit_us) {
  clear_error();
  if (!s)
    return fail(LLMI_INVALID_ARGUMENT, "inject_fault: null session");
  if (limit_us > 1000000u)
    return fail(LLMI_INVALID_ARGUMENT, "inject_fault: limit %u us above 1 s", limit_us);
  s->injectFaultUs = limit_us;
  return LLMI_OK;
}

extern "C" int llmi_cuda_session_reset(llmi_session *s) {
  clear_error();
  if (!s)
    return fail(LLMI_INVALID_ARGUMENT, "reset: null session");
  if (int e = zero_states(*s))
    return e;
  s->inFlight = false;  // zero_states synchronised the stream
  s->past = 0;
  s->invalid = false;
  s->plan.clear();
  return LLMI_OK;
}

extern "C" uint64_t llmi_cuda_session_past(const llmi_session *s) { return s ? s->past : 0; }

extern "C" int llmi_cuda_session_is_invalid(const llmi_session *s) { return s ? s->invalid : 1; }

extern "C" int llmi_cuda_session_state(llmi_session *s, unsigned layer, unsigned which,
                                       void **pointer, size_t *bytes) {
  clear_error();
  if (!s || !pointer || !bytes || layer >= s->config.kinds.size())
    return fail(LLMI_INVALID_ARGUMENT, "session_state: bad session, layer or output");
  void *p = nullptr;
  size_t n = 0;
  if (which == LLMI_STATE_KEYS) {
    p = s->keys[layer];
    n = s->cacheBytes;
  } else if (which == LLMI_STATE_VALUES) {
    p = s->values[layer];
    n = s->cacheBytes;
  } else if (which == LLMI_STATE_RECURRENT) {
    p = s->recurrent[layer];
    n = s->recurrentBytes;
  } else if (which == LLMI_STATE_CONV_HISTORY && layer < s->convHistory.size()) {
    p = s->convHistory[layer];
    n = s->historyBytes;
  }
  if (!p)
    return fail(LLMI_INVALID_ARGUMENT, "session_state: layer %u has no such state", layer);
  *pointer = p;
  *bytes = n;
  return LLMI_OK;
}

namespace {
int copy_state(llmi_session *s, unsigned layer, unsigned which, void *dst, const void *src,
               size_t bytes, bool toState) {
  void *p = nullptr;
  size_t n = 0;
  if (int e = llmi_cuda_session_state(s, layer, which, &p, &n))
    return e;
  if (bytes != n)
    return fail(LLMI_INVALID_ARGUMENT, "state copy of %zu bytes, the state holds %zu", bytes, n);
  if (!(toState ? src : dst))
    return fail(LLMI_INVALID_ARGUMENT, "state copy: null device pointer");
  const cudaError_t e = toState ? cudaMemcpyAsync(p, src, n, cudaMemcpyDeviceToDevice, s->stream)
                                : cudaMemcpyAsync(dst, p, n, cudaMemcpyDeviceToDevice, s->stream);
  if (int st = check_cuda(e, "state copy"))
    return st;
  return check_cuda(cudaStreamSynchronize(s->stream), "state copy");
}
}  // namespace

extern "C" int llmi_cuda_session_read_state(llmi_session *s, unsigned layer, unsigned which,
                                            void *dst, size_t bytes) {
  clear_error();
  return copy_state(s, layer, which, dst, nullptr, bytes, false);
}

extern "C" int llmi_cuda_session_write_state(llmi_session *s, unsigned layer, unsigned which,
                                             const void *src, size_t bytes) {
  clear_error();
  return copy_state(s, layer, which, nullptr, src, bytes, true);
}

extern "C" size_t llmi_cuda_session_plan(const llmi_session *s, char *buffer, size_t len) {
  if (!s)
    return 0;
  if (buffer && len) {
    const size_t n = std::min(len - 1, s->plan.size());
    std::memcpy(buffer, s->plan.data(), n);
    buffer[n] = '\0';
  }
  return s->plan.size();
}

extern "C" size_t llmi_cuda_describe_step(const llmi_stack_config *config, unsigned tokens,
                                          uint64_t past, char *buffer, size_t len, int *status) {
  clear_error();
  int dummy;
  int &st = status ? *status : dummy;
  StackConfig c;
  if ((st = StackConfig::from(config, c)))
    return 0;
  AttentionGraph graph;
  if ((st = AttentionGraph::build(c, {tokens, past, c.capacity}, graph)))
    return 0;
  const std::string json = describe(graph, c);
  if (buffer && len) {
    const size_t n = std::min(len - 1, json.size());
    std::memcpy(buffer, json.data(), n);
    buffer[n] = '\0';
  }
  st = LLMI_OK;
  return json.size();
}
