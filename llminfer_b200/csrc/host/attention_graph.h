// The attention ops of one step of the Qwen3.5 hybrid stack, with the
// operand contracts, state effects and logical cost that llminfer's GraphIR
// assigns them.  This is the part of the reference's typed SSA graph the CUDA
// backend consumes:
//   - KvAppend / CausalGqa verification and effects:
//     lib/GraphIR/Graph.cpp:248-279 (append writes rows [past, past+tokens)
//     of both caches, version 0 -> 1; attention needs version 1 and reads
//     rows [0, past+tokens));
//   - DeltaUpdate verification: lib/GraphIR/Graph.cpp:226-246 (recurrent
//     state [Hv, dk, dv] f32, read-write over [0, Hv), version 0 -> 1);
//   - state slot rules: lib/GraphIR/Graph.cpp:423-443 (KV caches have
//     capacity rows);
//   - cost: lib/GraphIR/Cost.cpp:85-93 (logical traffic of operands, outputs
//     and state effects) and :180-201 (MACs).
// Only these three op kinds exist here; projections, norms and the rest of
// the model graph are outside the attention path.
#pragma once

#include "llmi_cuda.h"

#include <cstdint>
#include <string>
#include <vector>

namespace llmi {
namespace host {

enum class OpKind { KvAppend, CausalGqa, DeltaUpdate };
enum class StateKind { KeyCache, ValueCache, DeltaRecurrent };
enum class Access { Read, Write, ReadWrite };

const char *name(OpKind kind);
const char *name(StateKind kind);
const char *name(Access access);

struct StepShape {
  uint64_t tokens, past, capacity;
};

// The attention-stack shape (llmi_stack_config as owned C++ values).
struct StackConfig {
  std::vector<unsigned char> kinds;  // LLMI_LAYER_* per layer
  unsigned batch = 0, capacity = 0;
  unsigned queryHeads = 0, kvHeads = 0, headDim = 0;
  unsigned keyHeads = 0, keyDim = 0, valueHeads = 0, valueDim = 0;

  static int from(const llmi_stack_config *c, StackConfig &out);
  bool hasGqa() const;
  bool hasDelta() const;
};

struct StateSlot {
  StateKind kind;
  uint32_t layer;
  uint64_t shape[3];   // per sequence (the reference layout)
  unsigned elementBytes;
  unsigned version = 0;
  uint64_t rowElements() const { return shape[1] * shape[2]; }
  uint64_t bytes() const { return shape[0] * shape[1] * shape[2] * elementBytes; }
};

struct Effect {
  uint32_t state;
  Access access;
  uint64_t begin, length;  // interval along axis 0
  unsigned versionBefore, versionAfter;
};

// Logical work of one op for ONE sequence (the reference graph is batch 1);
// multiply by the batch for a batched step.
struct Cost {
  uint64_t fpMacs = 0, readBytes = 0, writeBytes = 0;
};

struct Op {
  OpKind kind;
  uint32_t layer;
  uint32_t stateA = 0, stateB = 0;  // keys/values, or the recurrent state
  std::vector<Effect> effects;
  Cost cost;
};

// Builds and verifies the ops of one step: per GQA layer KvAppend then
// CausalGqa, per DeltaNet layer DeltaUpdate, in layer order (the order
// Qwen35ModelBuilder emits them, lib/Models/Qwen35/Qwen35ModelBuilder.cpp:
// 159-162 and 192-193).
class AttentionGraph {
public:
  static int build(const StackConfig &config, StepShape step, AttentionGraph &out);

  const StepShape &step() const { return step_; }
  const std::vector<StateSlot> &states() const { return states_; }
  const std::vector<Op> &ops() const { return ops_; }

private:
  int addState(StateKind kind, uint32_t layer, uint64_t a, uint64_t b, uint64_t c,
               unsigned elementBytes, uint32_t &id);
  int kvAppend(uint32_t layer, uint32_t keys, uint32_t values, const StackConfig &c);
  int causalGqa(uint32_t layer, uint32_t keys, uint32_t values, const StackConfig &c);
  int deltaUpdate(uint32_t layer, uint32_t state, const StackConfig &c);

  StepShape step_{};
  std::vector<StateSlot> states_;
  std::vector<Op> ops_;
};

// One kernel launch reported by --plan.
struct Dispatch {
  const char *kernel;
  size_t opIndex;
  uint32_t layer;
};

// The CUDA lowering of the attention ops (the counterpart of
// Lowering::attention and the DeltaUpdate case of Lowering::lower,
// lib/Backend/Metal/MetalExecutionPlan.cpp:511-549 and :663-676):
//   KvAppend    -> cacheAppend (keys), cacheAppend (values)
//   CausalGqa   -> tokens > 1: gqaFlashAttention
//                  tokens == 1: gqaScores (split-K partial softmax and P.V)
//                               gqaSoftmax (log-sum-exp merge, fp16 output;
//                               also does the reference gqaValue's job)
//   DeltaUpdate -> graphDeltaUpdate
std::vector<Dispatch> lower(const AttentionGraph &graph);

// JSON description of a step: step shape, states, ops with effects and
// per-sequence costs, and the dispatches.
std::string describe(const AttentionGraph &graph, const StackConfig &config);

}  // namespace host
}  // namespace llmi
