// C entry points over the reference's own portable C++ — TEST INFRASTRUCTURE.
//
// oracle/Makefile compiles this file together with the reference's
// lib/GraphIR/Graph.cpp, lib/GraphIR/Cost.cpp and
// lib/ModelFormat/Quantization.cpp, straight from the reference tree, into
// oracle/_ref/libllmi_ref.so.  Tests use it to pin (1) the oracle's fp16
// conversion against llminfer::floatToHalf / halfToFloat and (2) the CUDA
// host's op verifier and cost model against ir::Graph::append and
// ir::estimateCost, for the three ops on the attention path.
#include "llminfer/GraphIR/Cost.h"
#include "llminfer/ModelFormat/Quantization.h"

#include <cstdint>

using namespace llminfer;
using namespace llminfer::ir;

extern "C" uint16_t ref_float_to_half(float value) { return floatToHalf(value); }
extern "C" float ref_half_to_float(uint16_t bits) { return halfToFloat(bits); }

// Field order of the record written by ref_attention_costs.
enum RefField {
  KvWriteBytes,
  KvEffectBegin,
  KvEffectLength,
  KvVersionBefore,
  KvVersionAfter,
  GqaReadBytes,
  GqaWriteBytes,
  GqaFpMacs,
  GqaEffectBegin,
  GqaEffectLength,
  GqaVersionBefore,
  GqaVersionAfter,
  DeltaReadBytes,
  DeltaWriteBytes,
  DeltaFpMacs,
  FieldCount
};

extern "C" int ref_field_count() { return FieldCount; }

// Builds one GQA layer (KvAppend then CausalGqa) and one DeltaNet layer
// (DeltaUpdate) for the step {tokens, past, capacity} through the reference's
// GraphIR verifier and prices them with its cost model.  Returns 0 on
// success, 1 when the reference rejects the graph (the record is untouched).
extern "C" int ref_attention_costs(uint64_t tokens, uint64_t past,
                                   uint64_t capacity, uint64_t queryHeads,
                                   uint64_t kvHeads, uint64_t headDim,
                                   uint64_t keyHeads, uint64_t keyDim,
                                   uint64_t valueHeads, uint64_t valueDim,
                                   uint64_t *record) {
  auto graph = Graph::create({tokens, past, capacity});
  if (!graph)
    return 1;
  auto q = graph->addInput({ElementType::F16, {tokens, queryHeads, headDim}});
  auto k = graph->addInput({ElementType::F16, {tokens, kvHeads, headDim}});
  auto v = graph->addInput({ElementType::F16, {tokens, kvHeads, headDim}});
  auto keys = graph->addState(StateKind::KeyCache, 0,
                              {ElementType::F16, {capacity, kvHeads, headDim}});
  auto values = graph->addState(
      StateKind::ValueCache, 0, {ElementType::F16, {capacity, kvHeads, headDim}});
  if (!q || !k || !v || !keys || !values)
    return 1;
  KvAttr slots{*keys, *values};
  if (!graph->append(OpKind::KvAppend, {*k, *v}, slots, 0))
    return 1;
  if (!graph->append(OpKind::CausalGqa, {*q}, slots, 0))
    return 1;

  auto dq = graph->addInput({ElementType::F32, {tokens, keyHeads * keyDim}});
  auto dk = graph->addInput({ElementType::F32, {tokens, keyHeads * keyDim}});
  auto dv = graph->addInput({ElementType::F16, {tokens, valueHeads * valueDim}});
  auto beta = graph->addInput({ElementType::F32, {tokens, valueHeads}});
  auto decay = graph->addInput({ElementType::F32, {tokens, valueHeads}});
  auto state = graph->addState(StateKind::DeltaRecurrent, 1,
                               {ElementType::F32, {valueHeads, keyDim, valueDim}});
  if (!dq || !dk || !dv || !beta || !decay || !state)
    return 1;
  if (!graph->append(OpKind::DeltaUpdate, {*dq, *dk, *dv, *beta, *decay},
                     StateAttr{*state}, 1))
    return 1;

  auto cost = estimateCost(*graph);
  if (!cost)
    return 1;
  const auto &ops = graph->getOps();
  const auto &kv = ops[0].effects.front();
  const auto &gqa = ops[1].effects.front();
  record[KvWriteBytes] = cost->perOp[0].logicalWriteBytes;
  record[KvEffectBegin] = kv.begin;
  record[KvEffectLength] = kv.length;
  record[KvVersionBefore] = kv.versionBefore;
  record[KvVersionAfter] = kv.versionAfter;
  record[GqaReadBytes] = cost->perOp[1].logicalReadBytes;
  record[GqaWriteBytes] = cost->perOp[1].logicalWriteBytes;
  record[GqaFpMacs] = cost->perOp[1].fpMacs;
  record[GqaEffectBegin] = gqa.begin;
  record[GqaEffectLength] = gqa.length;
  record[GqaVersionBefore] = gqa.versionBefore;
  record[GqaVersionAfter] = gqa.versionAfter;
  record[DeltaReadBytes] = cost->perOp[2].logicalReadBytes;
  record[DeltaWriteBytes] = cost->perOp[2].logicalWriteBytes;
  record[DeltaFpMacs] = cost->perOp[2].fpMacs;
  return 0;
}
