// ref_harness.cpp — drives the REFERENCE implementation (its own headers,
// compiled from the reference tree by oracle/build.py) on arrays handed
// over from Python, so the oracle restatement and the CPU baseline can be
// checked against the reference itself.
//
// TEST INFRASTRUCTURE ONLY (oracle side). Networks are built through the
// reference's LayerBuilder extension point (include/plastix/layers.hpp:48-51)
// and stepped with the reference's unmodified Network::Do* loops. The only
// change to the reference sources is made by the build recipe: the fixed
// allocator capacities of include/plastix/plastix.hpp:82 become the two
// functions below, so the BASELINE-size networks fit.
#include <cstddef>
#include <cstdint>

static std::size_t g_unit_cap = 4096;
static std::size_t g_conn_cap = 4096 * 4;
std::size_t plx_ref_unit_capacity() { return g_unit_cap; }
std::size_t plx_ref_conn_capacity() { return g_conn_cap; }

#include <plastix/plastix.hpp>

#include "structural_policies.hpp"

#include <algorithm>
#include <cstring>
#include <memory>
#include <span>
#include <thread>
#include <vector>

namespace {

struct TraceTag {};

float g_decay = 0.9f;
float g_rate = 1e-3f;

// The single-layer sweep workload's rule: trace decay + Hebbian product.
struct HebbianTraceConn {
  static void UpdateIncomingConnection(auto &U, size_t DstId, size_t SrcId,
                                       auto &C, size_t ConnId, auto &) {
    float &E = plastix::GetField<TraceTag>(C, ConnId);
    E = g_decay * E +
        plastix::GetActivation(U, SrcId) * plastix::GetActivation(U, DstId);
    plastix::GetWeight(C, ConnId) += g_rate * E;
  }
  static void UpdateOutgoingConnection(auto &, size_t, size_t, auto &, size_t,
                                       auto &) {}
};

struct SweepTraits : plastix::DefaultNetworkTraits<> {
  using UpdateConn = HebbianTraceConn;
  using ExtraConnFields =
      plastix::ConnFieldList<plastix::alloc::SOAField<plastix::WeightTag, float>,
                             plastix::alloc::SOAField<TraceTag, float>>;
  static constexpr plastix::Propagation Model = plastix::Propagation::Pipeline;
};
using SweepNet = plastix::Network<SweepTraits>;

// Builds one layer of `num_dst` units fed by an explicit connection list
// (ToId values are absolute unit ids).
struct EdgeListLayer {
  size_t NumDst;
  const uint32_t *From;
  const uint32_t *To;
  const float *W;
  const float *Trace;
  uint64_t N;
  uint32_t ToOffset;  // subtracted from To (shards renumber their rows)

  template <typename UA, typename CA>
  plastix::UnitRange operator()(UA &U, CA &C, plastix::UnitRange Prev) const {
    uint16_t NewLevel = plastix::GetLevel(U, Prev.Begin) + 1;
    plastix::UnitRange Units = U.AllocateMany(NumDst);
    for (auto Id : Units.Ids()) plastix::GetLevel(U, Id) = NewLevel;
    for (uint64_t I = 0; I < N; ++I) {
      auto Id = C.Allocate();
      plastix::GetField<plastix::ToIdTag>(C, Id) = To[I] - ToOffset;
      plastix::GetField<plastix::FromIdTag>(C, Id) = From[I];
      plastix::GetField<plastix::SrcLevelTag>(C, Id) = 0;
      plastix::GetWeight(C, Id) = W[I];
      if constexpr (requires { plastix::GetField<TraceTag>(C, Id); })
        plastix::GetField<TraceTag>(C, Id) = Trace ? Trace[I] : 0.0f;
    }
    return Units;
  }
};

struct SweepShard {
  std::unique_ptr<SweepNet> Net;
  size_t NumSrc;
};

// A Topological network with default traits (their constructor runs
// SortConnectionsByLevel, hence RecomputeLevels, plastix.hpp:91-93).
using TopoNet = plastix::Network<plastix::DefaultNetworkTraits<>>;

// Allocates `NumNew` non-input units and an explicit connection list over all
// units (any FromId/ToId below the unit count, Dead flags optional).
struct GraphLayer {
  size_t NumNew;
  const uint32_t *From;
  const uint32_t *To;
  const uint8_t *Dead;
  uint64_t N;

  template <typename UA, typename CA>
  plastix::UnitRange operator()(UA &U, CA &C, plastix::UnitRange) const {
    plastix::UnitRange Units = U.AllocateMany(NumNew);
    for (uint64_t I = 0; I < N; ++I) {
      auto Id = C.Allocate();
      plastix::GetField<plastix::ToIdTag>(C, Id) = To[I];
      plastix::GetField<plastix::FromIdTag>(C, Id) = From[I];
      plastix::GetField<plastix::SrcLevelTag>(C, Id) = 0;
      plastix::GetField<plastix::DeadTag>(C, Id) = Dead ? Dead[I] != 0 : false;
      plastix::GetWeight(C, Id) = 0.0f;
    }
    return Units;
  }
};

}  // namespace


// Structural parity run: a Topological network n_in -> FC h1 -> FC h2
// (weights RandomUniformWeight(seed, -0.3, 0.3), seed + 1 for the second
// layer) with the policies of
// structural_policies.hpp, `steps` DoStep calls on the given inputs
// (steps x n_in). Outputs the per-step outputs (steps x h2), the final
// connections in storage order (capacity `cap`), every unit's Level and
// Activation.
template <class Tr>
static int structural_run(uint32_t n_in, uint32_t h1, uint32_t h2, uint32_t seed, int steps,
                          const float *inputs, uint64_t cap, float *outputs, uint32_t *from,
                          uint32_t *to, uint8_t *dead, uint16_t *src_level, float *w,
                          uint64_t *n_conn, uint16_t *level, float *act, uint64_t *n_units) {
  using Net = plastix::Network<Tr>;
  g_unit_cap = n_in + h1 + h2 + 1;
  g_conn_cap = cap + 1;
  Net N(n_in, plastix::FullyConnected{h1, plastix::RandomUniformWeight{seed, -0.3f, 0.3f}},
        plastix::FullyConnected{h2, plastix::RandomUniformWeight{seed + 1, -0.3f, 0.3f}});
  for (int S = 0; S < steps; ++S) {
    N.DoStep(std::span<const float>(inputs + (size_t)S * n_in, n_in));
    auto out = N.GetOutput();
    for (uint32_t I = 0; I < h2; ++I) outputs[(size_t)S * h2 + I] = out[I];
  }
  auto &CA = N.GetConnAlloc();
  auto &UA = N.GetUnitAlloc();
  if (CA.Size() > cap) return -1;
  for (size_t C = 0; C < CA.Size(); ++C) {
    from[C] = plastix::GetField<plastix::FromIdTag>(CA, C);
    to[C] = plastix::GetField<plastix::ToIdTag>(CA, C);
    dead[C] = plastix::GetField<plastix::DeadTag>(CA, C) ? 1 : 0;
    src_level[C] = plastix::GetField<plastix::SrcLevelTag>(CA, C);
    w[C] = plastix::GetWeight(CA, C);
  }
  *n_conn = CA.Size();
  for (size_t I = 0; I < UA.Size(); ++I) {
    level[I] = plastix::GetLevel(UA, I);
    act[I] = plastix::GetActivation(UA, I);
  }
  *n_units = UA.Size();
  return 0;
}

extern "C" {

const char *ref_version() { return plastix::version(); }

// Runs `sweeps` DoStep calls of the single-layer workload. Connections must be
// given in the order the reference should hold them. Outputs: final weights,
// traces and the destination activations.
int ref_sweep_run(uint64_t n_src, uint64_t n_dst, uint64_t n_conn,
                  const uint32_t *from, const uint32_t *to, const float *w0,
                  const float *trace0, const float *act_in, int sweeps,
                  float decay, float rate, float *w_out, float *trace_out,
                  float *act_out) {
  g_decay = decay;
  g_rate = rate;
  g_unit_cap = n_src + n_dst + 1;
  g_conn_cap = n_conn + 1;
  SweepNet Net(n_src, EdgeListLayer{n_dst, from, to, w0, trace0, n_conn, 0});
  for (int S = 0; S < sweeps; ++S)
    Net.DoStep(std::span<const float>(act_in, n_src));
  auto &CA = Net.GetConnAlloc();
  auto &UA = Net.GetUnitAlloc();
  if (CA.Size() != n_conn) return -1;
  for (uint64_t C = 0; C < n_conn; ++C) {
    w_out[C] = plastix::GetWeight(CA, C);
    trace_out[C] = plastix::GetField<TraceTag>(CA, C);
  }
  for (uint64_t I = 0; I < n_dst; ++I)
    act_out[I] = plastix::GetActivation(UA, n_src + I);
  return 0;
}

// CPU baseline: `n_threads` independent reference networks, each owning a
// contiguous range of destination rows (the connections are dst-sorted, so a
// shard is a contiguous connection range). Returns an opaque handle.
void *ref_sweep_shards_create(uint64_t n_src, uint64_t n_dst, uint64_t n_conn,
                              const uint32_t *from, const uint32_t *to,
                              const float *w0, int n_threads, float decay,
                              float rate) {
  g_decay = decay;
  g_rate = rate;
  auto *Shards = new std::vector<SweepShard>();
  uint64_t Begin = 0;
  for (int T = 0; T < n_threads; ++T) {
    uint64_t RowEnd = n_dst * (uint64_t)(T + 1) / (uint64_t)n_threads;
    uint32_t RowBegin = (uint32_t)(n_dst * (uint64_t)T / (uint64_t)n_threads);
    uint64_t End = Begin;
    while (End < n_conn && to[End] < n_src + RowEnd) ++End;
    g_unit_cap = n_src + (RowEnd - RowBegin) + 1;
    g_conn_cap = (End - Begin) + 1;
    SweepShard Sh;
    Sh.NumSrc = n_src;
    Sh.Net = std::make_unique<SweepNet>(
        n_src, EdgeListLayer{RowEnd - RowBegin, from + Begin, to + Begin,
                             w0 + Begin, nullptr, End - Begin, RowBegin});
    Shards->push_back(std::move(Sh));
    Begin = End;
  }
  return Shards;
}

// One DoStep on every shard, shards in parallel threads.
void ref_sweep_shards_step(void *handle, const float *act_in) {
  auto *Shards = static_cast<std::vector<SweepShard> *>(handle);
  std::vector<std::thread> Threads;
  for (auto &Sh : *Shards)
    Threads.emplace_back([&Sh, act_in] {
      Sh.Net->DoStep(std::span<const float>(act_in, Sh.NumSrc));
    });
  for (auto &T : Threads) T.join();
}

// The reference allocators never unmap their arenas (alloc.hpp has no
// destructor); the shards are released but their arenas stay mapped.
void ref_sweep_shards_destroy(void *handle) {
  delete static_cast<std::vector<SweepShard> *>(handle);
}

int ref_structural_run(int variant, uint32_t n_in, uint32_t h1, uint32_t h2, uint32_t seed,
                       int steps, const float *inputs, uint64_t cap, float *outputs,
                       uint32_t *from, uint32_t *to, uint8_t *dead, uint16_t *src_level, float *w,
                       uint64_t *n_conn, uint16_t *level, float *act, uint64_t *n_units) {
  using namespace structural_test;
  if (variant == 0)
    return structural_run<SmallTraits>(n_in, h1, h2, seed, steps, inputs, cap, outputs,
                                                from, to, dead, src_level, w, n_conn, level, act,
                                                n_units);
  return structural_run<MediumTraits>(n_in, h1, h2, seed, steps, inputs, cap, outputs,
                                                from, to, dead, src_level, w, n_conn, level, act,
                                                n_units);
}

// Unit levels and the level sort through the reference's own constructor:
// n_input input units, n_units - n_input more, the given connections. Outputs
// every unit's Level and the connections (FromId, ToId, SrcLevel, Dead) in the
// order SortConnectionsByLevel left them.
int ref_levels_run(uint64_t n_units, uint64_t n_input, uint64_t n_conn, const uint32_t *from,
                   const uint32_t *to, const uint8_t *dead, uint16_t *level_out,
                   uint32_t *from_out, uint32_t *to_out, uint16_t *src_level_out,
                   uint8_t *dead_out) {
  if (n_input > n_units) return -2;
  g_unit_cap = n_units + 1;
  g_conn_cap = n_conn + 1;
  TopoNet Net(n_input, GraphLayer{n_units - n_input, from, to, dead, n_conn});
  auto &CA = Net.GetConnAlloc();
  auto &UA = Net.GetUnitAlloc();
  if (CA.Size() != n_conn || UA.Size() != n_units) return -1;
  for (uint64_t I = 0; I < n_units; ++I) level_out[I] = plastix::GetLevel(UA, I);
  for (uint64_t C = 0; C < n_conn; ++C) {
    from_out[C] = plastix::GetField<plastix::FromIdTag>(CA, C);
    to_out[C] = plastix::GetField<plastix::ToIdTag>(CA, C);
    src_level_out[C] = plastix::GetField<plastix::SrcLevelTag>(CA, C);
    dead_out[C] = plastix::GetField<plastix::DeadTag>(CA, C) ? 1 : 0;
  }
  return 0;
}

}  // extern "C"

// ---- The reference's SwiftTD example (examples/swifttd/swifttd.cpp), -----
// compiled unchanged in this translation unit with its main() renamed, so its
// own traits (SwiftTDTraits, Gamma = 1.0 as that file sets it) drive the
// reference Network here.
#define main plx_ref_swifttd_example_main
#include "swifttd.cpp"
#undef main

// Runs `steps` DoStep calls of the example's network (n features -> 1 value
// unit, FullyConnected with SwiftTDConnInit{alpha_init}). features: steps x n
// row-major; rewards: steps. Outputs: the ten connection fields (10 x n, in
// the example's ExtraConnFields order) and V after every step.
extern "C" int ref_swifttd_example_run(uint64_t n, const float *features,
                                       const float *rewards, int steps,
                                       float alpha_init, float *fields_out,
                                       float *v_out) {
  g_unit_cap = n + 2;
  g_conn_cap = n + 1;
  using FC = plastix::FullyConnected<SwiftTDConnInit>;
  ImprintingLearner Net(n, FC{1, SwiftTDConnInit{alpha_init}});
  for (int S = 0; S < steps; ++S) {
    const float R[1] = {rewards[S]};
    Net.DoStep(std::span<const float>(features + (uint64_t)S * n, n),
               std::span<const float>(R, 1));
    v_out[S] = Net.GetOutput()[0];
  }
  auto &CA = Net.GetConnAlloc();
  if (CA.Size() != n) return -1;
  for (uint64_t I = 0; I < n; ++I) {
    fields_out[0 * n + I] = plastix::GetWeight(CA, I);
    fields_out[1 * n + I] = plastix::GetField<ZTag>(CA, I);
    fields_out[2 * n + I] = plastix::GetField<ZDeltaTag>(CA, I);
    fields_out[3 * n + I] = plastix::GetField<DeltaWTag>(CA, I);
    fields_out[4 * n + I] = plastix::GetField<HTag>(CA, I);
    fields_out[5 * n + I] = plastix::GetField<HOldTag>(CA, I);
    fields_out[6 * n + I] = plastix::GetField<HTempTag>(CA, I);
    fields_out[7 * n + I] = plastix::GetField<ZBarTag>(CA, I);
    fields_out[8 * n + I] = plastix::GetField<PTag>(CA, I);
    fields_out[9 * n + I] = plastix::GetField<BetaTag>(CA, I);
  }
  return 0;
}
