// plastix/traits.hpp -- the policy / traits API (the reference's
// include/plastix/traits.hpp): propagation models, the policy concepts, the
// default and no-op policies, the losses, DefaultNetworkTraits and the
// NetworkTraits concept. Policies are structs of static member functions
// taking `auto &` accessors, ids and the global state; on the B200 they are
// called from kernels, so each member function carries PLASTIX_HD
// (__host__ __device__ under nvcc, nothing otherwise).
//
// Execution knobs a traits struct may add (all optional):
//   static constexpr bool ReadOnlyGlobalState
//       true: no hook writes the global state, so every pass runs in
//       parallel on the device. Default: true when GlobalState is an empty
//       type, false otherwise -- hooks that may accumulate into the globals
//       (SwiftTD's reductions, the imprinting learner's flags) then run in
//       one device thread in the reference's order, which keeps its
//       sequential semantics exactly.
//   static constexpr bool SequentialConnectionUpdate
//       overrides the above for DoUpdateConnectionState only.
//   static constexpr bool DeviceStructure
//       true: DoPruneUnits' predicate and DoAddConnections' proposal
//       predicates run on the device (in parallel, or in one thread with
//       SequentialStructure). Default false: these structural decisions run
//       on the host over the network's coherent host copy, in the
//       reference's order, so predicates may use host-only facilities
//       (host random engines, streams, static data members); proposals are
//       still sorted and deduplicated on the device. AddUnit always runs on
//       the host (unit growth is host-orchestrated).
//   static constexpr bool SequentialStructure
//       with DeviceStructure: run the structural predicates in one thread.
#pragma once

#include <cmath>
#include <concepts>
#include <cstddef>
#include <cstdint>
#include <limits>
#include <optional>
#include <span>

#include "plastix/conn.hpp"
#include "plastix/layers.hpp"
#include "plastix/unit_state.hpp"

namespace plastix {

enum class Propagation { Topological, Pipeline };

// ---------------------------------------------------------------------------
// Policy concepts (checked against the host allocators, as the reference's)
// ---------------------------------------------------------------------------
template <typename P, typename UnitAlloc, typename ConnAlloc, typename Global>
concept PassPolicy =
    std::default_initializable<typename P::Accumulator> &&
    requires(UnitAlloc &U, size_t A, size_t B, ConnAlloc &C, size_t ConnId, Global &G,
             typename P::Accumulator AccA, typename P::Accumulator AccB) {
      typename P::Accumulator;
      { P::Map(U, A, B, C, ConnId, G) } -> std::convertible_to<typename P::Accumulator>;
      { P::Combine(AccA, AccB) } -> std::convertible_to<typename P::Accumulator>;
      { P::Apply(U, A, G, AccA) } -> std::same_as<void>;
    };

template <typename P, typename UnitAlloc, typename Global>
concept UpdateUnitPolicy = requires(UnitAlloc &U, size_t Id, Global &G) {
  { P::Update(U, Id, G) } -> std::same_as<void>;
};

template <typename P, typename UnitAlloc, typename ConnAlloc, typename Global>
concept UpdateConnPolicy =
    requires(UnitAlloc &U, size_t DstId, size_t SrcId, ConnAlloc &C, size_t ConnId, Global &G) {
      { P::UpdateIncomingConnection(U, DstId, SrcId, C, ConnId, G) } -> std::same_as<void>;
      { P::UpdateOutgoingConnection(U, SrcId, DstId, C, ConnId, G) } -> std::same_as<void>;
    };

template <typename P, typename UnitAlloc, typename Global>
concept PruneUnitPolicy = requires(UnitAlloc &U, size_t Id, Global &G) {
  { P::ShouldPrune(U, Id, G) } -> std::convertible_to<bool>;
};

template <typename P, typename UnitAlloc, typename ConnAlloc, typename Global>
concept PruneConnPolicy =
    requires(UnitAlloc &U, size_t DstId, size_t SrcId, ConnAlloc &C, size_t ConnId, Global &G) {
      { P::ShouldPrune(U, DstId, SrcId, C, ConnId, G) } -> std::convertible_to<bool>;
    };

template <typename P, typename UnitAlloc, typename Global>
concept AddUnitPolicy = requires(UnitAlloc &U, size_t ParentId, size_t NewId, Global &G) {
  { P::AddUnit(U, ParentId, G) } -> std::same_as<std::optional<int16_t>>;
  { P::InitUnit(U, NewId, ParentId, G) } -> std::same_as<void>;
};

template <typename P, typename UnitAlloc, typename ConnAlloc, typename Global>
concept AddConnPolicy = requires(UnitAlloc &U, size_t SelfId, size_t CandidateId, ConnAlloc &C,
                                 size_t ConnId, Global &G) {
  { P::ShouldAddIncomingConnection(U, SelfId, CandidateId, G) } -> std::convertible_to<bool>;
  { P::ShouldAddOutgoingConnection(U, SelfId, CandidateId, G) } -> std::convertible_to<bool>;
  { P::InitConnection(U, SelfId, CandidateId, C, ConnId, G) } -> std::same_as<void>;
};

template <typename P, typename Global>
concept ResetGlobalStatePolicy = requires(Global &G) {
  { P::Reset(G) } -> std::same_as<void>;
};

template <typename P, typename UnitAlloc, typename Global>
concept LossPolicy = requires(UnitAlloc &U, UnitRange R, std::span<const float> T, Global &G) {
  { P::CalculateLoss(U, R, T, G) } -> std::same_as<void>;
};

// ---------------------------------------------------------------------------
// Default and no-op policies
// ---------------------------------------------------------------------------
struct DefaultForwardPass {
  using Accumulator = float;
  PLASTIX_HD static float Map(auto &U, size_t, size_t SrcId, auto &C, size_t ConnId, auto &) {
    return GetWeight(C, ConnId) * GetActivation(U, SrcId);
  }
  PLASTIX_HD static float Combine(float A, float B) { return A + B; }
  PLASTIX_HD static void Apply(auto &U, size_t Id, auto &, float Accumulated) {
    GetActivation(U, Id) = Accumulated;
  }
};

// The No* policies satisfy their concepts; the Network detects them and
// skips the whole step.
struct NoBackwardPass {
  using Accumulator = float;
  PLASTIX_HD static float Map(auto &, size_t, size_t, auto &, size_t, auto &) { return 0.0f; }
  PLASTIX_HD static float Combine(float A, float B) { return A + B; }
  PLASTIX_HD static void Apply(auto &, size_t, auto &, float) {}
};
struct NoUpdateUnit {
  PLASTIX_HD static void Update(auto &, size_t, auto &) {}
};
struct NoUpdateConn {
  PLASTIX_HD static void UpdateIncomingConnection(auto &, size_t, size_t, auto &, size_t, auto &) {}
  PLASTIX_HD static void UpdateOutgoingConnection(auto &, size_t, size_t, auto &, size_t, auto &) {}
};
struct NoPruneUnit {
  PLASTIX_HD static bool ShouldPrune(auto &, size_t, auto &) { return false; }
};
struct NoPruneConn {
  PLASTIX_HD static bool ShouldPrune(auto &, size_t, size_t, auto &, size_t, auto &) {
    return false;
  }
};
struct NoAddUnit {
  static std::optional<int16_t> AddUnit(auto &, size_t, auto &) { return std::nullopt; }
  static void InitUnit(auto &, size_t, size_t, auto &) {}
};
struct NoAddConn {
  PLASTIX_HD static bool ShouldAddIncomingConnection(auto &, size_t, size_t, auto &) {
    return false;
  }
  PLASTIX_HD static bool ShouldAddOutgoingConnection(auto &, size_t, size_t, auto &) {
    return false;
  }
  PLASTIX_HD static void InitConnection(auto &, size_t, size_t, auto &, size_t, auto &) {}
};
struct NoResetGlobalState {
  PLASTIX_HD static void Reset(auto &) {}
};

// A Hebbian connection rule with a decaying eligibility trace (an addition;
// the reference ships no plasticity rule): per live connection, with pre =
// Activation[Src] and post = Activation[Dst] after the forward pass,
//   trace' = Decay * trace + pre * post,   weight' = weight + Rate * trace'
// (each product and sum rounded separately). Needs WeightTag and TraceTag
// among the connection fields. A single Pipeline layer whose traits use
// DefaultForwardPass with this rule (and no other hook) steps through one
// fused device sweep per DoStep.
template <float Decay, float Rate> struct HebbianTraceUpdate {
  static constexpr float kDecay = Decay, kRate = Rate;
  PLASTIX_HD static void UpdateIncomingConnection(auto &U, size_t DstId, size_t SrcId, auto &C,
                                                  size_t ConnId, auto &) {
    float &E = GetField<TraceTag>(C, ConnId);
    E = Decay * E + GetActivation(U, SrcId) * GetActivation(U, DstId);
    GetWeight(C, ConnId) += Rate * E;
  }
  PLASTIX_HD static void UpdateOutgoingConnection(auto &, size_t, size_t, auto &, size_t, auto &) {}
};

// Losses stage dL/dActivation of each output unit into its BackwardAcc.
struct NoLoss {
  PLASTIX_HD static void CalculateLoss(auto &, UnitRange, std::span<const float>, auto &) {}
};

// L = 0.5 * sum (pred - target)^2;  dL/dpred = pred - target.
struct MSELoss {
  PLASTIX_HD static void CalculateLoss(auto &U, UnitRange Outputs, std::span<const float> Targets,
                                       auto &) {
    size_t I = 0;
    for (size_t Id = Outputs.Begin; Id < Outputs.End; ++Id) {
      const float Pred = GetActivation(U, Id);
      GetBackwardAcc(U, Id) = Pred - Targets[I++];
    }
  }
};

// L = sqrt(mean (pred - target)^2);  dL/dpred = (pred - target) / (N (L + 1e-8)).
struct RMSLoss {
  PLASTIX_HD static void CalculateLoss(auto &U, UnitRange Outputs, std::span<const float> Targets,
                                       auto &) {
    float SumSq = 0.0f;
    size_t I = 0;
    for (size_t Id = Outputs.Begin; Id < Outputs.End; ++Id) {
      const float Diff = GetActivation(U, Id) - Targets[I++];
      SumSq += Diff * Diff;
    }
    const float N = static_cast<float>(Outputs.Size());
    const float Rms = std::sqrt(SumSq / N);
    const float Denom = N * (Rms + 1e-8f);
    I = 0;
    for (size_t Id = Outputs.Begin; Id < Outputs.End; ++Id) {
      const float Pred = GetActivation(U, Id);
      GetBackwardAcc(U, Id) = (Pred - Targets[I++]) / Denom;
    }
  }
};

// Softmax of the outputs against a target distribution;
// dL/dpred_i = softmax(pred)_i - target_i.
struct SoftmaxCrossEntropyLoss {
  PLASTIX_HD static void CalculateLoss(auto &U, UnitRange Outputs, std::span<const float> Targets,
                                       auto &) {
    float Max = -std::numeric_limits<float>::infinity();
    for (size_t Id = Outputs.Begin; Id < Outputs.End; ++Id) {
      const float P = GetActivation(U, Id);
      if (P > Max) Max = P;
    }
    float Sum = 0.0f;
    for (size_t Id = Outputs.Begin; Id < Outputs.End; ++Id)
      Sum += std::exp(GetActivation(U, Id) - Max);
    size_t I = 0;
    for (size_t Id = Outputs.Begin; Id < Outputs.End; ++Id) {
      const float Soft = std::exp(GetActivation(U, Id) - Max) / Sum;
      GetBackwardAcc(U, Id) = Soft - Targets[I++];
    }
  }
};

struct EmptyGlobalState {};

// ---------------------------------------------------------------------------
// Default traits: inherit and override individual policies
// ---------------------------------------------------------------------------
template <typename Global = EmptyGlobalState> struct DefaultNetworkTraits {
  using GlobalState = Global;
  using ForwardPass = DefaultForwardPass;
  using BackwardPass = NoBackwardPass;
  using Loss = NoLoss;
  using UpdateUnit = NoUpdateUnit;
  using UpdateConn = NoUpdateConn;
  using PruneUnit = NoPruneUnit;
  using PruneConn = NoPruneConn;
  using AddUnit = NoAddUnit;
  using AddConn = NoAddConn;
  using ResetGlobal = NoResetGlobalState;
  using ExtraUnitFields = UnitFieldList<>;
  using ExtraConnFields = ConnFieldList<alloc::SOAField<WeightTag, float>>;
  static constexpr uint16_t Neighbourhood = 1;
  static constexpr Propagation Model = Propagation::Topological;
};

template <typename T>
using UnitAllocFor = MakeUnitAllocatorFrom<typename T::ForwardPass::Accumulator,
                                           typename T::BackwardPass::Accumulator,
                                           typename T::ExtraUnitFields>;
template <typename T> using ConnAllocFor = MakeConnAllocatorFrom<typename T::ExtraConnFields>;

template <typename T>
concept NetworkTraits =
    requires {
      typename T::GlobalState;
      typename T::ForwardPass;
      typename T::ForwardPass::Accumulator;
      typename T::BackwardPass;
      typename T::BackwardPass::Accumulator;
      typename T::Loss;
      typename T::UpdateUnit;
      typename T::UpdateConn;
      typename T::PruneUnit;
      typename T::PruneConn;
      typename T::AddUnit;
      typename T::AddConn;
      typename T::ResetGlobal;
      typename T::ExtraUnitFields;
      typename T::ExtraConnFields;
      { T::Neighbourhood } -> std::convertible_to<uint16_t>;
      { T::Model } -> std::convertible_to<Propagation>;
    } &&
    PassPolicy<typename T::ForwardPass, UnitAllocFor<T>, ConnAllocFor<T>, typename T::GlobalState> &&
    PassPolicy<typename T::BackwardPass, UnitAllocFor<T>, ConnAllocFor<T>,
               typename T::GlobalState> &&
    LossPolicy<typename T::Loss, UnitAllocFor<T>, typename T::GlobalState> &&
    UpdateUnitPolicy<typename T::UpdateUnit, UnitAllocFor<T>, typename T::GlobalState> &&
    UpdateConnPolicy<typename T::UpdateConn, UnitAllocFor<T>, ConnAllocFor<T>,
                     typename T::GlobalState> &&
    PruneUnitPolicy<typename T::PruneUnit, UnitAllocFor<T>, typename T::GlobalState> &&
    PruneConnPolicy<typename T::PruneConn, UnitAllocFor<T>, ConnAllocFor<T>,
                    typename T::GlobalState> &&
    AddUnitPolicy<typename T::AddUnit, UnitAllocFor<T>, typename T::GlobalState> &&
    AddConnPolicy<typename T::AddConn, UnitAllocFor<T>, ConnAllocFor<T>, typename T::GlobalState> &&
    ResetGlobalStatePolicy<typename T::ResetGlobal, typename T::GlobalState>;

}  // namespace plastix
