// Reference-side integration check of the CUDA attention backend — TEST
// INFRASTRUCTURE.
//
// Built by tests/boundary/Makefile against the reference's own GraphIR
// (include/llminfer/GraphIR, lib/GraphIR/Graph.cpp and Cost.cpp compiled from
// the reference tree), this repository's include/llmi_cuda.h and the CPU
// oracle (oracle/oracle.c); linked against llminfer_b200/_lib/libllmi_cuda.so.
//
// It is the CUDA sibling of the reference's Lowering::attention
// (lib/Backend/Metal/MetalExecutionPlan.cpp:511-549) and of its DeltaUpdate
// case (:663-676), written over the reference's ir::Graph exactly as a
// CudaExecutionPlan would be:
//   1. builds reference graphs (KvAppend -> CausalGqa, DeltaUpdate) for
//      prefill (T > 1) and decode (T = 1) steps; the reference verifier
//      (Graph.cpp:226-279) must accept them;
//   2. lowers every op to the C ABI, filling CacheParams / GqaParams /
//      GraphDeltaParams from the graph's shapes where the Metal lowering does;
//   3. checks the dispatch names against the reference lowering's rules, and
//      the ops' state effects and costs (reference ir::estimateCost) against
//      this backend's own llmi_cuda_describe_step;
//   4. with --run (needs a CUDA device): executes the lowered calls on device
//      buffers and checks the outputs and the updated state against the CPU
//      oracle at the acceptance bar (max-abs <= 1e-2, rel-L2 <= 2e-3).
// Prints one line per checked step and "boundary: ok" at the end; exits
// non-zero on the first mismatch.
#include "llminfer/GraphIR/Cost.h"
#include "llmi_cuda.h"

#include "oracle.h"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <string>
#include <vector>

using namespace llminfer;
using namespace llminfer::ir;

namespace {

[[noreturn]] void die(const std::string &what) {
  std::fprintf(stderr, "boundary: FAIL: %s\n", what.c_str());
  std::exit(1);
}

void expect(bool ok, const std::string &what) {
  if (!ok)
    die(what);
}

// ---- the step's graph, built through the reference's GraphIR ---------------------

struct Shapes {
  uint64_t queryHeads, kvHeads, headDim;                 // GQA layer
  uint64_t keyHeads, keyDim, valueHeads, valueDim;       // DeltaNet layer
};

struct StepGraph {
  Graph graph;
  ValueId q, k, v, gqaOut;
  ValueId dq, dk, dv, beta, decay, deltaOut;
  StateId keys, values, recurrent;
};

template <class T> T take(Result<T> r, const char *what) {
  if (!r)
    die(std::string(what) + ": " + r.getError().getMessage());
  return std::move(*r);
}

StepGraph build_graph(StepShape step, const Shapes &s) {
  auto g = take(Graph::create(step), "Graph::create");
  const uint64_t T = step.tokens, cap = step.capacity;
  ValueId q = take(g.addInput({ElementType::F16, {T, s.queryHeads, s.headDim}}), "q");
  ValueId k = take(g.addInput({ElementType::F16, {T, s.kvHeads, s.headDim}}), "k");
  ValueId v = take(g.addInput({ElementType::F16, {T, s.kvHeads, s.headDim}}), "v");
  StateId keys = take(g.addState(StateKind::KeyCache, 0, {ElementType::F16, {cap, s.kvHeads, s.headDim}}),
                      "keys");
  StateId values = take(
      g.addState(StateKind::ValueCache, 0, {ElementType::F16, {cap, s.kvHeads, s.headDim}}), "values");
  take(g.append(OpKind::KvAppend, {k, v}, KvAttr{keys, values}, 0), "KvAppend");
  Values gqa = take(g.append(OpKind::CausalGqa, {q}, KvAttr{keys, values}, 0), "CausalGqa");

  const uint64_t kw = s.keyHeads * s.keyDim, vw = s.valueHeads * s.valueDim;
  ValueId dq = take(g.addInput({ElementType::F32, {T, kw}}), "dq");
  ValueId dk = take(g.addInput({ElementType::F32, {T, kw}}), "dk");
  ValueId dv = take(g.addInput({ElementType::F16, {T, vw}}), "dv");
  ValueId beta = take(g.addInput({ElementType::F32, {T, s.valueHeads}}), "beta");
  ValueId decay = take(g.addInput({ElementType::F32, {T, s.valueHeads}}), "decay");
  StateId rec = take(g.addState(StateKind::DeltaRecurrent, 1,
                                {ElementType::F32, {s.valueHeads, s.keyDim, s.valueDim}}),
                     "recurrent");
  Values delta = take(g.append(OpKind::DeltaUpdate, {dq, dk, dv, beta, decay}, StateAttr{rec}, 1),
                      "DeltaUpdate");
  return StepGraph{std::move(g), q, k, v, gqa[0], dq, dk, dv, beta, decay, delta[0], keys, values, rec};
}

// ---- the lowering --------------------------------------------------------------

// Device (or, when only recording, placeholder) addresses of the graph's
// values and states, batch 1.
struct Buffers {
  std::vector<void *> value;  // by ValueId.index
  std::vector<void *> state;  // by StateId.index
  void *decode_scratch = nullptr;
  size_t decode_scratch_bytes = 0;
  void *delta_scratch = nullptr;
  size_t delta_scratch_bytes = 0;
};

// One lowered dispatch: its --plan name and the C-ABI call that performs it.
struct Dispatch {
  std::string plan;
  std::function<int()> call;
};

// Fills the reference parameter structs from the graph as
// MetalExecutionPlan.cpp does and binds each op to the C ABI.
std::vector<Dispatch> lower(const StepGraph &sg, Buffers &buf, void *stream) {
  const Graph &g = sg.graph;
  const StepShape step = g.getStep();
  std::vector<Dispatch> out;
  for (const Operation &op : g.getOps()) {
    switch (op.kind) {
    case OpKind::KvAppend: {  // :516-522, two dispatches, keys then values
      const auto &attr = *std::get_if<KvAttr>(&op.attributes);
      const auto &cache = g.getStates()[attr.keys.index].type.shape;
      const unsigned heads = unsigned(cache[1]), headDim = unsigned(cache[2]);
      const auto &in = g.getValues()[op.inputs[0].index].type.shape;
      const unsigned width = unsigned(in[0] * in[1] * in[2]);
      const llmi_cache_params params{width, unsigned(step.past * heads * headDim)};
      const size_t stride = size_t(step.capacity) * heads * headDim;
      for (int i = 0; i < 2; ++i) {
        const void *rows = buf.value[op.inputs[i].index];
        void *cache_buf = buf.state[(i == 0 ? attr.keys : attr.values).index];
        out.push_back({"cacheAppend", [=] {
                         return llmi_cuda_cache_append(&params, 1, static_cast<const uint16_t *>(rows),
                                                       width, static_cast<uint16_t *>(cache_buf),
                                                       stride, stream);
                       }});
      }
      break;
    }
    case OpKind::CausalGqa: {  // :525-548
      const auto &attr = *std::get_if<KvAttr>(&op.attributes);
      const auto &cache = g.getStates()[attr.keys.index].type.shape;
      const auto &query = g.getValues()[op.inputs[0].index].type.shape;
      const llmi_gqa_params params{unsigned(step.tokens), unsigned(query[1]), unsigned(cache[1]),
                                   unsigned(cache[2]), unsigned(step.past)};
      const size_t stride = size_t(step.capacity) * cache[1] * cache[2];
      const auto *q = static_cast<const uint16_t *>(buf.value[op.inputs[0].index]);
      const auto *kc = static_cast<const uint16_t *>(buf.state[attr.keys.index]);
      const auto *vc = static_cast<const uint16_t *>(buf.state[attr.values.index]);
      auto *o = static_cast<uint16_t *>(buf.value[op.outputs[0].index]);
      if (step.tokens > 1) {
        out.push_back({"gqaFlashAttention", [=] {
                         return llmi_cuda_gqa_prefill(&params, 1, q, kc, vc, stride, o, stream);
                       }});
      } else {
        // Split-K decode: the partial pass and the merge (which also does
        // gqaValue's rescale-and-sum) under the reference's first two names.
        Buffers *b = &buf;
        out.push_back({"gqaScores", [=] {
                         return llmi_cuda_gqa_decode(&params, 1, q, kc, vc, stride, o,
                                                     b->decode_scratch, b->decode_scratch_bytes,
                                                     stream);
                       }});
        out.push_back({"gqaSoftmax", [] { return 0; }});  // same call as above
      }
      break;
    }
    case OpKind::DeltaUpdate: {  // :663-676
      const StateId slot = std::get_if<StateAttr>(&op.attributes)->state;
      const auto &dims = g.getStates()[slot.index].type.shape;
      const unsigned keyDim = unsigned(dims[1]);
      const auto &qshape = g.getValues()[op.inputs[0].index].type.shape;
      const llmi_delta_params params{unsigned(step.tokens), unsigned(qshape[1] / keyDim), keyDim,
                                     unsigned(dims[0]), unsigned(dims[2])};
      const auto *q = static_cast<const float *>(buf.value[op.inputs[0].index]);
      const auto *k = static_cast<const float *>(buf.value[op.inputs[1].index]);
      const auto *v = static_cast<const uint16_t *>(buf.value[op.inputs[2].index]);
      const auto *beta = static_cast<const float *>(buf.value[op.inputs[3].index]);
      const auto *decay = static_cast<const float *>(buf.value[op.inputs[4].index]);
      auto *state = static_cast<float *>(buf.state[slot.index]);
      auto *o = static_cast<uint16_t *>(buf.value[op.outputs[0].index]);
      Buffers *b = &buf;
      out.push_back({"graphDeltaUpdate", [=] {
                       return llmi_cuda_delta_update_ws(&params, 1, q, k, v, beta, decay, state, o,
                                                        b->delta_scratch, b->delta_scratch_bytes,
                                                        stream);
                     }});
      break;
    }
    default:
      die(std::string("unexpected op ") + std::string(getName(op.kind)));
    }
  }
  return out;
}

// The names the reference's lowering emits for these ops on a device with
// flash attention (MetalExecutionPlan.cpp:516-548, :667-675): flash iff the
// step has more than one token (head dims of the configs qualify), else the
// three-dispatch decode; this backend folds gqaValue into gqaSoftmax.
std::vector<std::string> reference_names(const Graph &g) {
  std::vector<std::string> names;
  for (const Operation &op : g.getOps()) {
    if (op.kind == OpKind::KvAppend) {
      names.push_back("cacheAppend");
      names.push_back("cacheAppend");
    } else if (op.kind == OpKind::CausalGqa) {
      if (g.getStep().tokens > 1) {
        names.push_back("gqaFlashAttention");
      } else {
        names.push_back("gqaScores");
        names.push_back("gqaSoftmax");
      }
    } else if (op.kind == OpKind::DeltaUpdate) {
      names.push_back("graphDeltaUpdate");
    }
  }
  return names;
}

// ---- checks against this backend's own step description --------------------------

uint64_t json_u64(const std::string &js, size_t from, const char *key) {
  const std::string k = std::string("\"") + key + "\":";
  size_t at = js.find(k, from);
  expect(at != std::string::npos, std::string("describe_step: no ") + key);
  return std::strtoull(js.c_str() + at + k.size(), nullptr, 10);
}

void check_effects_and_costs(const StepGraph &sg, const Shapes &s) {
  const Graph &g = sg.graph;
  const StepShape step = g.getStep();
  const unsigned char kinds[2] = {LLMI_LAYER_GQA, LLMI_LAYER_DELTANET};
  llmi_stack_config cfg{2, kinds, 1, unsigned(step.capacity), unsigned(s.queryHeads),
                        unsigned(s.kvHeads), unsigned(s.headDim), unsigned(s.keyHeads),
                        unsigned(s.keyDim), unsigned(s.valueHeads), unsigned(s.valueDim)};
  int status = 0;
  std::string js(llmi_cuda_describe_step(&cfg, unsigned(step.tokens), step.past, nullptr, 0, &status),
                 '\0');
  expect(!js.empty() && status == 0, "describe_step failed");
  llmi_cuda_describe_step(&cfg, unsigned(step.tokens), step.past, js.data(), js.size() + 1, &status);
  auto cost = take(estimateCost(g), "estimateCost");
  size_t at = js.find("\"ops\":");
  const auto &ops = g.getOps();
  for (size_t i = 0; i < ops.size(); ++i) {
    at = js.find("\"index\":" + std::to_string(i), at);
    expect(at != std::string::npos, "describe_step: op missing");
    const std::string kind = "\"kind\":\"" + std::string(getName(ops[i].kind)) + "\"";
    expect(js.compare(js.find("\"kind\"", at), kind.size(), kind) == 0,
           "op kind differs from the reference graph: " + kind);
    size_t e = js.find("\"effects\"", at);
    for (const StateEffect &eff : ops[i].effects) {
      e = js.find("{\"state\"", e + 1);
      expect(e != std::string::npos, "describe_step: effect missing");
      expect(json_u64(js, e, "begin") == eff.begin && json_u64(js, e, "length") == eff.length &&
                 json_u64(js, e, "version_before") == eff.versionBefore &&
                 json_u64(js, e, "version_after") == eff.versionAfter,
             "state effect differs from Graph.cpp's for op " + std::to_string(i));
    }
    expect(json_u64(js, at, "fp_macs") == cost.perOp[i].fpMacs &&
               json_u64(js, at, "logical_read_bytes") == cost.perOp[i].logicalReadBytes &&
               json_u64(js, at, "logical_write_bytes") == cost.perOp[i].logicalWriteBytes,
           "cost differs from the reference cost model for op " + std::to_string(i));
  }
  // This backend's plan for the step is the lowering's.
  std::vector<std::string> planned;
  for (size_t p = js.find("\"dispatches\""); (p = js.find("\"kernel\":\"", p)) != std::string::npos;) {
    p += 10;
    planned.push_back(js.substr(p, js.find('"', p) - p));
  }
  expect(planned == reference_names(g), "describe_step's dispatches differ from the reference names");
}

// ---- execution against the oracle (--run) ------------------------------------

struct Rng {  // SplitMix64 -> Box-Muller, seeded per tensor
  uint64_t s;
  uint64_t next() {
    uint64_t z = (s += 0x9e3779b97f4a7c15ull);
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
  }
  float normal() {
    const double u1 = (double(next() >> 11) + 0.5) / 9007199254740992.0;
    const double u2 = double(next() >> 11) / 9007199254740992.0;
    return float(std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
  }
};

std::vector<uint16_t> half_normal(size_t n, uint64_t seed) {
  Rng r{seed};
  std::vector<uint16_t> h(n);
  for (auto &x : h)
    x = oracle_f32_to_f16(r.normal());
  return h;
}

void *upload(const void *host, size_t bytes) {
  void *d = nullptr;
  expect(cudaMalloc(&d, bytes) == cudaSuccess, "cudaMalloc");
  expect(cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice) == cudaSuccess, "H2D");
  return d;
}

template <class T> std::vector<T> download(const void *dev, size_t n) {
  std::vector<T> h(n);
  expect(cudaMemcpy(h.data(), dev, n * sizeof(T), cudaMemcpyDeviceToHost) == cudaSuccess, "D2H");
  return h;
}

void within_bar(const std::vector<double> &got, const std::vector<double> &want,
                const std::string &what) {
  double max_abs = 0, num = 0, den = 0;
  for (size_t i = 0; i < got.size(); ++i) {
    expect(std::isfinite(got[i]), what + ": unwritten or non-finite output");
    const double d = got[i] - want[i];
    max_abs = std::fmax(max_abs, std::fabs(d));
    num += d * d;
    den += want[i] * want[i];
  }
  const double rel = std::sqrt(num / std::fmax(den, 1e-300));
  std::printf("  %s: max-abs %.3e rel-L2 %.3e\n", what.c_str(), max_abs, rel);
  expect(max_abs <= 1e-2 && rel <= 2e-3, what + " outside the bar");
}

void run_step(const StepGraph &sg, const Shapes &s, uint64_t seed) {
  const Graph &g = sg.graph;
  const StepShape st = g.getStep();
  const uint64_t T = st.tokens, P = st.past, cap = st.capacity;
  const size_t row = s.kvHeads * s.headDim, kw = s.keyHeads * s.keyDim,
               vw = s.valueHeads * s.valueDim;
  // Host inputs: caches with rows [0, past) filled, the step's rows, DeltaNet
  // operands as the benchmark configs draw them.
  std::vector<uint16_t> kcache(cap * row, 0), vcache(cap * row, 0);
  auto kpast = half_normal(P * row, seed + 1), vpast = half_normal(P * row, seed + 2);
  std::copy(kpast.begin(), kpast.end(), kcache.begin());
  std::copy(vpast.begin(), vpast.end(), vcache.begin());
  auto q = half_normal(T * s.queryHeads * s.headDim, seed + 3);
  auto knew = half_normal(T * row, seed + 4), vnew = half_normal(T * row, seed + 5);
  Rng r{seed + 6};
  std::vector<float> dq(T * kw), dk(T * kw), beta(T * s.valueHeads), decay(T * s.valueHeads);
  for (auto *x : {&dq, &dk})
    for (auto &e : *x)
      e = r.normal();
  for (uint64_t t = 0; t < T * s.keyHeads; ++t)  // L2 rows; q also * 1/sqrt(dk)
    for (auto *x : {&dq, &dk}) {
      double n2 = 0;
      for (uint64_t i = 0; i < s.keyDim; ++i)
        n2 += double((*x)[t * s.keyDim + i]) * (*x)[t * s.keyDim + i];
      const double f = (x == &dq ? 1.0 / std::sqrt(double(s.keyDim)) : 1.0) / std::sqrt(n2 + 1e-6);
      for (uint64_t i = 0; i < s.keyDim; ++i)
        (*x)[t * s.keyDim + i] = float((*x)[t * s.keyDim + i] * f);
    }
  for (auto &b : beta)
    b = oracle_f16_to_f32(oracle_f32_to_f16(1.f / (1.f + std::exp(-r.normal()))));
  for (auto &d : decay)
    d = std::exp(-std::log1p(std::exp(r.normal())));
  auto dv = half_normal(T * vw, seed + 7);
  std::vector<float> state(s.valueHeads * s.keyDim * s.valueDim);
  for (auto &x : state)
    x = 0.02f * r.normal();

  Buffers buf;
  buf.value.assign(g.getValues().size(), nullptr);
  buf.state.assign(g.getStates().size(), nullptr);
  buf.value[sg.q.index] = upload(q.data(), q.size() * 2);
  buf.value[sg.k.index] = upload(knew.data(), knew.size() * 2);
  buf.value[sg.v.index] = upload(vnew.data(), vnew.size() * 2);
  buf.value[sg.gqaOut.index] = upload(std::vector<uint16_t>(q.size(), 0x7e00).data(), q.size() * 2);
  buf.value[sg.dq.index] = upload(dq.data(), dq.size() * 4);
  buf.value[sg.dk.index] = upload(dk.data(), dk.size() * 4);
  buf.value[sg.dv.index] = upload(dv.data(), dv.size() * 2);
  buf.value[sg.beta.index] = upload(beta.data(), beta.size() * 4);
  buf.value[sg.decay.index] = upload(decay.data(), decay.size() * 4);
  buf.value[sg.deltaOut.index] = upload(std::vector<uint16_t>(dv.size(), 0x7e00).data(), dv.size() * 2);
  buf.state[sg.keys.index] = upload(kcache.data(), kcache.size() * 2);
  buf.state[sg.values.index] = upload(vcache.data(), vcache.size() * 2);
  buf.state[sg.recurrent.index] = upload(state.data(), state.size() * 4);
  const llmi_gqa_params gp{unsigned(T), unsigned(s.queryHeads), unsigned(s.kvHeads),
                           unsigned(s.headDim), unsigned(P)};
  const llmi_delta_params dp{unsigned(T), unsigned(s.keyHeads), unsigned(s.keyDim),
                             unsigned(s.valueHeads), unsigned(s.valueDim)};
  buf.decode_scratch_bytes = T == 1 ? llmi_cuda_gqa_decode_workspace(&gp, 1) : 0;
  buf.delta_scratch_bytes = llmi_cuda_delta_update_workspace(&dp, 1);
  if (buf.decode_scratch_bytes)
    expect(cudaMalloc(&buf.decode_scratch, buf.decode_scratch_bytes) == cudaSuccess, "scratch");
  if (buf.delta_scratch_bytes)
    expect(cudaMalloc(&buf.delta_scratch, buf.delta_scratch_bytes) == cudaSuccess, "scratch");

  for (Dispatch &d : lower(sg, buf, nullptr))
    if (int status = d.call())
      die(d.plan + ": " + llmi_cuda_status_name(status) + ": " + llmi_cuda_last_error());
  expect(llmi_cuda_poll_error(nullptr) == 0, std::string("device error: ") + llmi_cuda_last_error());

  // Oracle: cacheAppend on the host copies, the dense fp64 check, the
  // token-sequential DeltaNet.
  std::copy(knew.begin(), knew.end(), kcache.begin() + P * row);
  std::copy(vnew.begin(), vnew.end(), vcache.begin() + P * row);
  auto got_k = download<uint16_t>(buf.state[sg.keys.index], kcache.size());
  expect(std::memcmp(got_k.data(), kcache.data(), kcache.size() * 2) == 0,
         "cacheAppend: key cache differs from the appended rows");
  oracle_gqa_params op{unsigned(T), unsigned(s.queryHeads), unsigned(s.kvHeads),
                       unsigned(s.headDim), unsigned(P)};
  std::vector<double> want(q.size());
  oracle_gqa_dense(&op, 1, q.data(), q.size(), kcache.data(), vcache.data(), kcache.size(),
                   want.data(), 0);
  std::vector<double> got;
  for (uint16_t h : download<uint16_t>(buf.value[sg.gqaOut.index], q.size()))
    got.push_back(oracle_f16_to_f32(h));
  within_bar(got, want, T > 1 ? "gqaFlashAttention" : "gqaScores/gqaSoftmax");

  oracle_delta_params odp{unsigned(T), unsigned(s.keyHeads), unsigned(s.keyDim),
                          unsigned(s.valueHeads), unsigned(s.valueDim)};
  std::vector<uint16_t> want_out(dv.size());
  std::vector<float> want_state = state;
  oracle_delta_update(&odp, 1, dq.data(), dk.data(), dv.data(), beta.data(), decay.data(),
                      want_state.data(), want_out.data(), 0);
  got.clear();
  want.clear();
  for (uint16_t h : download<uint16_t>(buf.value[sg.deltaOut.index], dv.size()))
    got.push_back(oracle_f16_to_f32(h));
  for (uint16_t h : want_out)
    want.push_back(oracle_f16_to_f32(h));
  within_bar(got, want, "graphDeltaUpdate output");
  got.clear();
  want.clear();
  for (float x : download<float>(buf.state[sg.recurrent.index], state.size()))
    got.push_back(x);
  for (float x : want_state)
    want.push_back(x);
  within_bar(got, want, "graphDeltaUpdate state");

  for (void *p : buf.value)
    cudaFree(p);
  for (void *p : buf.state)
    cudaFree(p);
  cudaFree(buf.decode_scratch);
  cudaFree(buf.delta_scratch);
}

}  // namespace

int main(int argc, char **argv) {
  const bool run = argc > 1 && std::strcmp(argv[1], "--run") == 0;
  // The configs' head shapes (Qwen3.5-4B attention and DeltaNet layers),
  // prefill and decode steps, short enough for the oracle.
  const Shapes s{16, 4, 256, 16, 128, 32, 128};
  const StepShape steps[] = {{128, 0, 128}, {37, 60, 256}, {1, 4096, 8192}, {1, 0, 16}, {200, 0, 256}};
  uint64_t seed = 179531;
  for (const StepShape &step : steps) {
    StepGraph sg = build_graph(step, s);
    Buffers placeholders;
    placeholders.value.assign(sg.graph.getValues().size(), nullptr);
    placeholders.state.assign(sg.graph.getStates().size(), nullptr);
    std::vector<std::string> names;
    for (const Dispatch &d : lower(sg, placeholders, nullptr))
      names.push_back(d.plan);
    expect(names == reference_names(sg.graph), "lowered dispatch names differ from the reference's");
    check_effects_and_costs(sg, s);
    std::printf("step tokens=%llu past=%llu capacity=%llu: graph verified, %zu dispatches",
                (unsigned long long)step.tokens, (unsigned long long)step.past,
                (unsigned long long)step.capacity, names.size());
    for (const auto &n : names)
      std::printf(" %s", n.c_str());
    std::printf("; effects and costs match\n");
    if (run)
      run_step(sg, s, seed++);
  }
  std::printf("boundary: ok%s\n", run ? " (executed on the GPU)" : "");
  return 0;
}
