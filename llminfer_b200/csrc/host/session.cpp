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
  std::string plan;
  std::vector<cudaEvent_t> layerEvents;  // borrowed; recorded after each layer
  unsigned injectFaultUs = 0;             // > 0: the next step also runs the wait self-test

  ~llmi_session() {
    for (auto *list : {&keys, &values, &recurrent})
      for (void *p : *list)
        if (p)
          cudaFree(p);
    if (workspace)
      cudaFree(workspace);
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

// Lowers and launches one step.  `launchedAny` reports whether any kernel
// may have been enqueued (the reference's "submitted").
int run_step(llmi_session &s, unsigned tokens, const llmi_layer_io *io, bool trace,
             bool &launchedAny) {
  launchedAny = false;
  AttentionGraph graph;
  if (int e = AttentionGraph::build(s.config, {tokens, s.past, s.config.capacity}, graph))
    return e;
  if (int e = check_io(s, io))
    return e;
  const StackConfig &c = s.config;
  const unsigned B = c.batch;
  if (tokens == 1 && c.hasGqa()) {
    llmi_gqa_params g{1, c.queryHeads, c.kvHeads, c.headDim, unsigned(s.past)};
    const size_t need = llmi_cuda_gqa_decode_workspace(&g, B);
    if (!need)
      return fail(LLMI_CUDA_ERROR, "decode workspace: %s", last_error());
    if (int e = ensure_workspace(s, need))
      return e;
  }
  const size_t cacheStride = size_t(c.capacity) * c.kvHeads * c.headDim;
  const auto dispatches = lower(graph);
  size_t next = 0;  // first dispatch of the current op
  const auto &ops = graph.ops();
  for (size_t i = 0; i < ops.size(); ++i) {
    const Op &op = ops[i];
    const llmi_layer_io &x = io[op.layer];
    int e = LLMI_OK;
    size_t count = 1;
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
      e = llmi_cuda_cache_append(&p, B, static_cast<const uint16_t *>(x.k), inStride,
                                 static_cast<uint16_t *>(s.keys[op.layer]), cacheStride, s.stream);
      if (!e)
        e = llmi_cuda_cache_append(&p, B, static_cast<const uint16_t *>(x.v), inStride,
                                   static_cast<uint16_t *>(s.values[op.layer]), cacheStride,
                                   s.stream);
      count = 2;
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
      e = llmi_cuda_delta_update(&p, B, static_cast<const float *>(x.q),
                                 static_cast<const float *>(x.k),
                                 static_cast<const uint16_t *>(x.v), x.beta, x.decay,
                                 static_cast<float *>(s.recurrent[op.layer]),
                                 static_cast<uint16_t *>(x.out), s.stream);
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
      for (size_t d = next; d < next + count && d < dispatches.size(); ++d) {
        char line[160];
        std::snprintf(line, sizeof line, "{\"op_index\":%zu,\"kernel\":\"%s\",\"layer\":%u}\n",
                      dispatches[d].opIndex, dispatches[d].kernel, dispatches[d].layer);
        s.plan += line;
      }
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

extern "C" int llmi_cuda_session_step(llmi_session *s, unsigned tokens, const llmi_layer_io *io,
                                      int trace_plan) {
  clear_error();
  if (!s)
    return fail(LLMI_INVALID_ARGUMENT, "step: null session");
  if (s->invalid)
    return fail(LLMI_SESSION_INVALID, "CUDA session is invalid after a failed GPU step");
  if (trace_plan)
    s->plan.clear();
  bool launchedAny = false;
  int e = run_step(*s, tokens, io, trace_plan != 0, launchedAny);
  if (!e && launchedAny)
    e = llmi_cuda_poll_error(s->stream);
  if (e) {
    s->invalid = launchedAny;
    return e;
  }
  s->past += tokens;
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
