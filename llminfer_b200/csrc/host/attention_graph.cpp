#include "attention_graph.h"

#include "status.h"

#include <cstdarg>
#include <cstdio>

namespace llmi {
namespace host {

const char *name(OpKind kind) {
  switch (kind) {
  case OpKind::KvAppend: return "KvAppend";
  case OpKind::CausalGqa: return "CausalGqa";
  case OpKind::DeltaUpdate: return "DeltaUpdate";
  }
  return "?";
}

const char *name(StateKind kind) {
  switch (kind) {
  case StateKind::KeyCache: return "KeyCache";
  case StateKind::ValueCache: return "ValueCache";
  case StateKind::DeltaRecurrent: return "DeltaRecurrent";
  }
  return "?";
}

const char *name(Access access) {
  switch (access) {
  case Access::Read: return "Read";
  case Access::Write: return "Write";
  case Access::ReadWrite: return "ReadWrite";
  }
  return "?";
}

int StackConfig::from(const llmi_stack_config *c, StackConfig &out) {
  if (!c || !c->layers || !c->layer_kinds)
    return fail(LLMI_INVALID_ARGUMENT, "stack config: no layers");
  out = StackConfig{};
  out.kinds.assign(c->layer_kinds, c->layer_kinds + c->layers);
  out.batch = c->batch;
  out.capacity = c->capacity;
  out.queryHeads = c->queryHeads;
  out.kvHeads = c->kvHeads;
  out.headDim = c->headDim;
  out.keyHeads = c->keyHeads;
  out.keyDim = c->keyDim;
  out.valueHeads = c->valueHeads;
  out.valueDim = c->valueDim;
  if (!out.batch || !out.capacity)
    return fail(LLMI_INVALID_ARGUMENT, "stack config: batch and capacity must be positive");
  for (unsigned char kind : out.kinds)
    if (kind != LLMI_LAYER_DELTANET && kind != LLMI_LAYER_GQA)
      return fail(LLMI_INVALID_ARGUMENT, "stack config: unknown layer kind %u", unsigned(kind));
  if (out.hasGqa() && (!out.queryHeads || !out.kvHeads || !out.headDim ||
                       out.queryHeads % out.kvHeads))
    return fail(LLMI_INVALID_ARGUMENT, "stack config: invalid GQA head shape");
  if (out.hasDelta() && (!out.keyHeads || !out.keyDim || !out.valueHeads || !out.valueDim ||
                         out.valueHeads % out.keyHeads))
    return fail(LLMI_INVALID_ARGUMENT, "stack config: invalid DeltaNet head shape");
  return LLMI_OK;
}

bool StackConfig::hasGqa() const {
  for (unsigned char k : kinds)
    if (k == LLMI_LAYER_GQA)
      return true;
  return false;
}

bool StackConfig::hasDelta() const {
  for (unsigned char k : kinds)
    if (k == LLMI_LAYER_DELTANET)
      return true;
  return false;
}

int AttentionGraph::addState(StateKind kind, uint32_t layer, uint64_t a, uint64_t b, uint64_t c,
                             unsigned elementBytes, uint32_t &id) {
  if (!a || !b || !c)
    return fail(LLMI_INVALID_ARGUMENT, "Invalid graph state type");
  if (kind != StateKind::DeltaRecurrent && a != step_.capacity)
    return fail(LLMI_INVALID_ARGUMENT, "Invalid graph state type: a KV cache has capacity rows");
  for (const auto &slot : states_)
    if (slot.kind == kind && slot.layer == layer)
      return fail(LLMI_INVALID_ARGUMENT, "Duplicate state slot in layer");
  id = uint32_t(states_.size());
  states_.push_back(StateSlot{kind, layer, {a, b, c}, elementBytes, 0});
  return LLMI_OK;
}

int AttentionGraph::kvAppend(uint32_t layer, uint32_t keys, uint32_t values, const StackConfig &c) {
  StateSlot &k = states_[keys], &v = states_[values];
  if (k.version != 0 || v.version != 0)
    return fail(LLMI_INVALID_ARGUMENT, "KvAppend: KV cache is already appended");
  const uint64_t T = step_.tokens, row = uint64_t(c.kvHeads) * c.headDim;
  Op op{OpKind::KvAppend, layer, keys, values, {}, {}};
  op.effects.push_back({keys, Access::Write, step_.past, T, 0, 1});
  op.effects.push_back({values, Access::Write, step_.past, T, 0, 1});
  // Operands: new keys and values [T, Hkv, D] f16; effects write T rows each.
  op.cost.readBytes = 2 * T * row * 2;
  op.cost.writeBytes = 2 * T * row * 2;
  k.version = v.version = 1;
  ops_.push_back(std::move(op));
  return LLMI_OK;
}

int AttentionGraph::causalGqa(uint32_t layer, uint32_t keys, uint32_t values, const StackConfig &c) {
  const StateSlot &k = states_[keys], &v = states_[values];
  if (k.version != 1 || v.version != 1)
    return fail(LLMI_INVALID_ARGUMENT, "CausalGqa: Attention requires the appended KV version");
  const uint64_t T = step_.tokens, P = step_.past;
  const uint64_t visible = P + T, row = uint64_t(c.kvHeads) * c.headDim;
  Op op{OpKind::CausalGqa, layer, keys, values, {}, {}};
  op.effects.push_back({keys, Access::Read, 0, visible, 1, 1});
  op.effects.push_back({values, Access::Read, 0, visible, 1, 1});
  const uint64_t pairs = T * P + T * (T + 1) / 2;
  const uint64_t qBytes = T * c.queryHeads * c.headDim * 2;
  op.cost.fpMacs = 2 * uint64_t(c.queryHeads) * pairs * c.headDim;
  op.cost.readBytes = qBytes + 2 * visible * row * 2;
  op.cost.writeBytes = qBytes;
  ops_.push_back(std::move(op));
  return LLMI_OK;
}

int AttentionGraph::deltaUpdate(uint32_t layer, uint32_t state, const StackConfig &c) {
  StateSlot &s = states_[state];
  if (s.version != 0)
    return fail(LLMI_INVALID_ARGUMENT,
                "DeltaUpdate: Expected an unwritten recurrent state in this layer");
  const uint64_t T = step_.tokens;
  const uint64_t keyWidth = uint64_t(c.keyHeads) * c.keyDim;
  const uint64_t valueWidth = uint64_t(c.valueHeads) * c.valueDim;
  const uint64_t stateBytes = uint64_t(c.valueHeads) * c.keyDim * c.valueDim * 4;
  Op op{OpKind::DeltaUpdate, layer, state, state, {}, {}};
  op.effects.push_back({state, Access::ReadWrite, 0, c.valueHeads, 0, 1});
  op.cost.fpMacs = 3 * T * uint64_t(c.valueHeads) * c.keyDim * c.valueDim;
  // q, k f32; v f16; beta, decay f32; state read.
  op.cost.readBytes = 2 * T * keyWidth * 4 + T * valueWidth * 2 + 2 * T * c.valueHeads * 4 +
                      stateBytes;
  op.cost.writeBytes = T * valueWidth * 2 + stateBytes;
  s.version = 1;
  ops_.push_back(std::move(op));
  return LLMI_OK;
}

int AttentionGraph::build(const StackConfig &config, StepShape step, AttentionGraph &out) {
  out = AttentionGraph{};
  if (!step.tokens || step.past > step.capacity || step.tokens > step.capacity - step.past)
    return fail(LLMI_CAPACITY_EXCEEDED,
                "Invalid graph step: expected 0 < tokens <= capacity - past (tokens %llu, past "
                "%llu, capacity %llu)",
                (unsigned long long)step.tokens, (unsigned long long)step.past,
                (unsigned long long)step.capacity);
  out.step_ = step;
  for (uint32_t layer = 0; layer < config.kinds.size(); ++layer) {
    if (config.kinds[layer] == LLMI_LAYER_GQA) {
      uint32_t keys, values;
      if (int s = out.addState(StateKind::KeyCache, layer, step.capacity, config.kvHeads,
                               config.headDim, 2, keys))
        return s;
      if (int s = out.addState(StateKind::ValueCache, layer, step.capacity, config.kvHeads,
                               config.headDim, 2, values))
        return s;
      if (int s = out.kvAppend(layer, keys, values, config))
        return s;
      if (int s = out.causalGqa(layer, keys, values, config))
        return s;
    } else {
      uint32_t state;
      if (int s = out.addState(StateKind::DeltaRecurrent, layer, config.valueHeads, config.keyDim,
                               config.valueDim, 4, state))
        return s;
      if (int s = out.deltaUpdate(layer, state, config))
        return s;
    }
  }
  return LLMI_OK;
}

std::vector<Dispatch> lower(const AttentionGraph &graph) {
  std::vector<Dispatch> out;
  const auto &ops = graph.ops();
  for (size_t i = 0; i < ops.size(); ++i) {
    const Op &op = ops[i];
    switch (op.kind) {
    case OpKind::KvAppend:
      out.push_back({"cacheAppend", i, op.layer});
      out.push_back({"cacheAppend", i, op.layer});
      break;
    case OpKind::CausalGqa:
      if (graph.step().tokens > 1) {
        out.push_back({"gqaFlashAttention", i, op.layer});
      } else {
        out.push_back({"gqaScores", i, op.layer});
        out.push_back({"gqaSoftmax", i, op.layer});
      }
      break;
    case OpKind::DeltaUpdate:
      out.push_back({"graphDeltaUpdate", i, op.layer});
      break;
    }
  }
  return out;
}

namespace {
void appendf(std::string &s, const char *format, ...) __attribute__((format(printf, 2, 3)));
void appendf(std::string &s, const char *format, ...) {
  char buffer[512];
  va_list args;
  va_start(args, format);
  std::vsnprintf(buffer, sizeof buffer, format, args);
  va_end(args);
  s += buffer;
}
}  // namespace

std::string describe(const AttentionGraph &graph, const StackConfig &config) {
  std::string s;
  const StepShape &st = graph.step();
  appendf(s, "{\"step\":{\"tokens\":%llu,\"past\":%llu,\"capacity\":%llu},\"batch\":%u,",
          (unsigned long long)st.tokens, (unsigned long long)st.past,
          (unsigned long long)st.capacity, config.batch);
  s += "\"states\":[";
  for (size_t i = 0; i < graph.states().size(); ++i) {
    const StateSlot &slot = graph.states()[i];
    appendf(s, "%s{\"kind\":\"%s\",\"layer\":%u,\"shape\":[%llu,%llu,%llu],\"element\":\"%s\"}",
            i ? "," : "", name(slot.kind), slot.layer, (unsigned long long)slot.shape[0],
            (unsigned long long)slot.shape[1], (unsigned long long)slot.shape[2],
            slot.elementBytes == 2 ? "F16" : "F32");
  }
  s += "],\"ops\":[";
  for (size_t i = 0; i < graph.ops().size(); ++i) {
    const Op &op = graph.ops()[i];
    appendf(s, "%s{\"index\":%zu,\"kind\":\"%s\",\"layer\":%u,\"effects\":[", i ? "," : "", i,
            name(op.kind), op.layer);
    for (size_t e = 0; e < op.effects.size(); ++e) {
      const Effect &ef = op.effects[e];
      appendf(s,
              "%s{\"state\":%u,\"access\":\"%s\",\"begin\":%llu,\"length\":%llu,"
              "\"version_before\":%u,\"version_after\":%u}",
              e ? "," : "", ef.state, name(ef.access), (unsigned long long)ef.begin,
              (unsigned long long)ef.length, ef.versionBefore, ef.versionAfter);
    }
    appendf(s,
            "],\"cost\":{\"fp_macs\":%llu,\"logical_read_bytes\":%llu,"
            "\"logical_write_bytes\":%llu}}",
            (unsigned long long)op.cost.fpMacs, (unsigned long long)op.cost.readBytes,
            (unsigned long long)op.cost.writeBytes);
  }
  s += "],\"dispatches\":[";
  const auto dispatches = lower(graph);
  for (size_t i = 0; i < dispatches.size(); ++i)
    appendf(s, "%s{\"op_index\":%zu,\"kernel\":\"%s\",\"layer\":%u}", i ? "," : "",
            dispatches[i].opIndex, dispatches[i].kernel, dispatches[i].layer);
  s += "]}";
  return s;
}

}  // namespace host
}  // namespace llmi
