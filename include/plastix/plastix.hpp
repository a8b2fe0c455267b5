// plastix/plastix.hpp -- the Plastix network API (Network<Traits>, SoA field
// accessors, traits, layer builders) on the B200: the same names and policy
// signatures as the reference header library (include/plastix/*.hpp of
// DhanrajHira/plastix), with the state in device memory and every Do* step a
// kernel that calls the user's policies on the GPU.
//
// Differences a user sees:
//   * Policy functions run on the device, so they carry PLASTIX_HD
//     (__host__ __device__ under nvcc, nothing otherwise):
//       struct MyMap { PLASTIX_HD static float Map(auto &U, ...) {...} };
//     The translation unit is compiled by nvcc (-std=c++20
//     --expt-relaxed-constexpr -arch=sm_100a).
//   * DoForwardPass / DoBackwardPass fold each unit's connections in the
//     reference's order (Pipeline: connection index order, backward in
//     descending order; Topological: by level, then index), one thread per
//     unit, so Map/Combine/Apply see the same sequence of values.
//   * DoUpdateConnectionState runs UpdateIncomingConnection over all
//     connections in parallel, then UpdateOutgoingConnection. Policies that
//     mutate the global state from those hooks (a reduction into a global, as
//     SwiftTD does) set `static constexpr bool SequentialConnectionUpdate =
//     true` in their traits to keep the reference's sequential semantics.
//   * Structural policies (PruneUnit/PruneConn/AddUnit/AddConn) are not
//     supported here; structural change runs through the C ABI (compaction,
//     radix re-sort, regrowth).
//   * No fixed capacity: networks of any size that fit the GPU.
//   * GetUnitAlloc()/GetConnAlloc() return host copies (downloaded on call;
//     edits made through them are uploaded before the next Do* call).
//     GetGlobals() (an addition) returns the global state.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <random>
#include <ranges>
#include <span>
#include <stdexcept>
#include <string>
#include <tuple>
#include <type_traits>
#include <utility>
#include <vector>

#if defined(__CUDACC__)
#define PLASTIX_HD __host__ __device__
#else
#define PLASTIX_HD
#endif

namespace plastix {

inline const char *version() { return "0.1.0"; }

inline void cuda_check(cudaError_t e, const char *what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// ---------------------------------------------------------------------------
// Structure-of-arrays storage
// ---------------------------------------------------------------------------
namespace alloc {

template <typename Tag, typename T> struct SOAField {
  using tag = Tag;
  using type = T;
};

template <typename Tag, typename... Fs> struct FieldIndex;
template <typename Tag, typename F, typename... Fs> struct FieldIndex<Tag, F, Fs...> {
  static constexpr size_t value =
      std::is_same_v<Tag, typename F::tag> ? 0 : 1 + FieldIndex<Tag, Fs...>::value;
};
template <typename Tag> struct FieldIndex<Tag> {
  static constexpr size_t value = 0;  // not found: index == number of fields
};

// Pointers to one array per field; what device code (and host code on a host
// copy) reads and writes through Get<Tag>(Id).
template <typename... Fs> struct SOAView {
  void *ptr[sizeof...(Fs) > 0 ? sizeof...(Fs) : 1];
  size_t size;

  template <typename Tag> PLASTIX_HD auto &Get(size_t Id) const {
    constexpr size_t I = FieldIndex<Tag, Fs...>::value;
    static_assert(I < sizeof...(Fs), "no such field");
    using T = typename std::tuple_element_t<I, std::tuple<Fs...>>::type;
    return static_cast<T *>(ptr[I])[Id];
  }
  PLASTIX_HD size_t Size() const { return size; }
};

// Host storage of the same fields (construction, host copies): one vector
// per field, addressed by field position.
template <typename Entity, typename... Fs> class SOAAllocator {
 public:
  using View = SOAView<Fs...>;
  static constexpr size_t NumFields = sizeof...(Fs);

  size_t Allocate() {
    push(std::index_sequence_for<Fs...>{});
    return n_++;
  }
  std::pair<size_t, size_t> AllocateMany(size_t Count) {
    const size_t B = n_;
    for (size_t I = 0; I < Count; ++I) Allocate();
    return {B, n_};
  }
  size_t Size() const { return n_; }
  template <typename Tag> auto &Get(size_t Id) {
    return std::get<FieldIndex<Tag, Fs...>::value>(store_)[Id];
  }
  template <typename Tag> const auto &Get(size_t Id) const {
    return std::get<FieldIndex<Tag, Fs...>::value>(store_)[Id];
  }
  template <typename Tag> auto *GetArrayFor() {
    return std::get<FieldIndex<Tag, Fs...>::value>(store_).data();
  }
  void *field_data(size_t I) { return data_ptr(I, std::index_sequence_for<Fs...>{}); }
  static constexpr size_t field_bytes(size_t I) {
    constexpr size_t B[] = {sizeof(typename Fs::type)...};
    return B[I];
  }
  // dst[i] = src[perm[i]] for every field (SOAAllocator::Gather semantics).
  void Gather(const std::vector<size_t> &Perm) { gather(Perm, std::index_sequence_for<Fs...>{}); }

 private:
  template <size_t... Is> void push(std::index_sequence<Is...>) {
    (std::get<Is>(store_).emplace_back(), ...);
  }
  template <size_t... Is> void *data_ptr(size_t I, std::index_sequence<Is...>) {
    void *p = nullptr;
    ((I == Is ? (p = static_cast<void *>(std::get<Is>(store_).data()), 0) : 0), ...);
    return p;
  }
  template <size_t... Is> void gather(const std::vector<size_t> &Perm, std::index_sequence<Is...>) {
    (gather_one(std::get<Is>(store_), Perm), ...);
  }
  template <typename V> static void gather_one(V &v, const std::vector<size_t> &Perm) {
    V out(Perm.size());
    for (size_t i = 0; i < Perm.size(); ++i) out[i] = v[Perm[i]];
    v.swap(out);
  }

  std::tuple<std::vector<typename Fs::type>...> store_;
  size_t n_ = 0;
};

}  // namespace alloc

// ---------------------------------------------------------------------------
// Unit and connection schemas, accessors
// ---------------------------------------------------------------------------
struct UnitState {};
struct ConnectionState {};
struct ActivationTag {};
struct ForwardAccTag {};
struct BackwardAccTag {};
struct PrunedTag {};
struct LevelTag {};
struct FromIdTag {};
struct ToIdTag {};
struct DeadTag {};
struct SrcLevelTag {};
struct WeightTag {};

// Accessors work on the device views and on the host allocators (host-only
// Get): the execution-space check is lifted for these templates, each
// instantiation is only ever called where its Get exists.
#if defined(__CUDACC__)
#define PLASTIX_NO_EXEC_CHECK _Pragma("nv_exec_check_disable")
#else
#define PLASTIX_NO_EXEC_CHECK
#endif
PLASTIX_NO_EXEC_CHECK
template <typename Tag> PLASTIX_HD constexpr auto &GetField(auto &Alloc, size_t Id) {
  return Alloc.template Get<Tag>(Id);
}
PLASTIX_NO_EXEC_CHECK
PLASTIX_HD constexpr auto &GetWeight(auto &Alloc, size_t Id) {
  return GetField<WeightTag>(Alloc, Id);
}
PLASTIX_NO_EXEC_CHECK
PLASTIX_HD constexpr auto &GetActivation(auto &Alloc, size_t Id) {
  return GetField<ActivationTag>(Alloc, Id);
}
PLASTIX_NO_EXEC_CHECK
PLASTIX_HD constexpr auto &GetForwardAcc(auto &Alloc, size_t Id) {
  return GetField<ForwardAccTag>(Alloc, Id);
}
PLASTIX_NO_EXEC_CHECK
PLASTIX_HD constexpr auto &GetBackwardAcc(auto &Alloc, size_t Id) {
  return GetField<BackwardAccTag>(Alloc, Id);
}
PLASTIX_NO_EXEC_CHECK
PLASTIX_HD constexpr auto &GetLevel(auto &Alloc, size_t Id) {
  return GetField<LevelTag>(Alloc, Id);
}

template <typename... Fields> struct UnitFieldList {};
template <typename... Fields> struct ConnFieldList {};

// ---------------------------------------------------------------------------
// Traits
// ---------------------------------------------------------------------------
enum class Propagation { Topological, Pipeline };

struct UnitRange {
  size_t Begin = 0;
  size_t End = 0;
  UnitRange() = default;
  PLASTIX_HD UnitRange(size_t B, size_t E) : Begin(B), End(E) {}
  UnitRange(std::pair<size_t, size_t> P) : Begin(P.first), End(P.second) {}
  PLASTIX_HD size_t Size() const { return End - Begin; }
  auto Ids() const { return std::views::iota(Begin, End); }
};

struct EmptyGlobalState {};

struct DefaultForwardPass {
  using Accumulator = float;
  PLASTIX_HD static float Map(auto &U, size_t, size_t SrcId, auto &C, size_t ConnId, auto &) {
    return GetWeight(C, ConnId) * GetActivation(U, SrcId);
  }
  PLASTIX_HD static float Combine(float A, float B) { return A + B; }
  PLASTIX_HD static void Apply(auto &U, size_t Id, auto &, float Acc) {
    GetActivation(U, Id) = Acc;
  }
};
struct NoBackwardPass {
  using Accumulator = float;
};
struct NoLoss {};
struct NoUpdateUnit {};
struct NoUpdateConn {};
struct NoPruneUnit {};
struct NoPruneConn {};
struct NoAddUnit {};
struct NoAddConn {};
struct NoResetGlobalState {};

// Mean squared error: BackwardAcc of each output = prediction - target.
struct MSELoss {
  PLASTIX_HD static void CalculateLoss(auto &U, UnitRange Outputs, std::span<const float> Targets,
                                       auto &) {
    size_t I = 0;
    for (size_t Id = Outputs.Begin; Id < Outputs.End; ++Id)
      GetBackwardAcc(U, Id) = GetActivation(U, Id) - Targets[I++];
  }
};

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

// ---------------------------------------------------------------------------
// Layer builders (host side, at construction)
// ---------------------------------------------------------------------------
struct NoUnitInit {
  void operator()(auto &, auto) const {}
};
struct NoConnInit {
  void operator()(auto &, auto) const {}
};

struct RandomUniformWeight {
  RandomUniformWeight(uint32_t Seed = 0, float Min = -1.0f, float Max = 1.0f)
      : Rng(Seed), Dist(Min, Max) {}
  void operator()(auto &CA, auto Id) const { GetWeight(CA, Id) = Dist(Rng); }

 private:
  mutable std::mt19937 Rng;
  mutable std::uniform_real_distribution<float> Dist;
};

// NumUnits new units one level above the previous layer, each fed by every
// unit of the previous layer (destination-major connection order).
template <typename ConnInit = NoConnInit, typename UnitInit = NoUnitInit> struct FullyConnected {
  size_t NumUnits;
  ConnInit InitConn = {};
  UnitInit InitUnit = {};

  template <typename UA, typename CA> UnitRange operator()(UA &U, CA &C, UnitRange Prev) const {
    const uint16_t Lvl = GetLevel(U, Prev.Begin) + 1;
    UnitRange Units = U.AllocateMany(NumUnits);
    for (size_t Id = Units.Begin; Id < Units.End; ++Id) {
      GetLevel(U, Id) = Lvl;
      InitUnit(U, Id);
    }
    const uint16_t SrcLvl = GetLevel(U, Prev.Begin);
    for (size_t Dst = Units.Begin; Dst < Units.End; ++Dst)
      for (size_t Src = Prev.Begin; Src < Prev.End; ++Src) {
        const size_t Id = C.Allocate();
        GetField<ToIdTag>(C, Id) = static_cast<uint32_t>(Dst);
        GetField<FromIdTag>(C, Id) = static_cast<uint32_t>(Src);
        GetField<SrcLevelTag>(C, Id) = SrcLvl;
        InitConn(C, Id);
      }
    return Units;
  }
};
template <typename CI> FullyConnected(size_t, CI) -> FullyConnected<CI, NoUnitInit>;
template <typename CI, typename UI>
FullyConnected(size_t, CI, UI) -> FullyConnected<CI, UI>;

// ---------------------------------------------------------------------------
// Device kernels (templated on the traits; instantiated in the user's TU)
// ---------------------------------------------------------------------------
namespace detail {

template <class Entity, class FwdAcc, class BwdAcc, class... Extra>
using UnitAllocT = alloc::SOAAllocator<Entity, alloc::SOAField<ActivationTag, float>,
                                       alloc::SOAField<ForwardAccTag, FwdAcc>,
                                       alloc::SOAField<BackwardAccTag, BwdAcc>,
                                       alloc::SOAField<PrunedTag, uint8_t>,
                                       alloc::SOAField<LevelTag, uint16_t>, Extra...>;
template <class Entity, class... Extra>
using ConnAllocT = alloc::SOAAllocator<Entity, alloc::SOAField<FromIdTag, uint32_t>,
                                       alloc::SOAField<ToIdTag, uint32_t>,
                                       alloc::SOAField<DeadTag, uint8_t>,
                                       alloc::SOAField<SrcLevelTag, uint16_t>, Extra...>;

template <class Fwd, class Bwd, class L> struct UnitAllocFromList;
template <class Fwd, class Bwd, class... E> struct UnitAllocFromList<Fwd, Bwd, UnitFieldList<E...>> {
  using type = UnitAllocT<UnitState, Fwd, Bwd, E...>;
};
template <class L> struct ConnAllocFromList;
template <class... E> struct ConnAllocFromList<ConnFieldList<E...>> {
  using type = ConnAllocT<ConnectionState, E...>;
};

template <class T> struct SequentialUpdate {
  static constexpr bool value = false;
};
template <class T>
  requires requires { T::SequentialConnectionUpdate; }
struct SequentialUpdate<T> {
  static constexpr bool value = T::SequentialConnectionUpdate;
};

inline unsigned blocks(size_t n) { return (unsigned)std::max<size_t>(1, (n + 255) / 256); }

// Forward accumulation: unit I (in [lo, hi), optionally only level `lvl`)
// folds its incoming connections in the stored order.
template <class Tr, class UV, class CV, class G>
__global__ void k_fwd_acc(UV U, CV C, G *g, const uint32_t *in_ptr, const uint32_t *in_conn,
                          size_t lo, size_t hi, int lvl) {
  using FP = typename Tr::ForwardPass;
  const size_t I = lo + blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (I >= hi) return;
  if (lvl >= 0 && GetLevel(U, I) != lvl) return;
  auto acc = GetForwardAcc(U, I);
  for (uint32_t k = in_ptr[I]; k < in_ptr[I + 1]; ++k) {
    const uint32_t c = in_conn[k];
    if (GetField<DeadTag>(C, c)) continue;
    acc = FP::Combine(acc, FP::Map(U, I, GetField<FromIdTag>(C, c), C, c, *g));
  }
  GetForwardAcc(U, I) = acc;
}

template <class Tr, class UV, class G>
__global__ void k_fwd_apply(UV U, G *g, size_t lo, size_t hi, int lvl) {
  using FP = typename Tr::ForwardPass;
  using Acc = typename FP::Accumulator;
  const size_t I = lo + blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (I >= hi) return;
  if (lvl >= 0 && GetLevel(U, I) != lvl) return;
  FP::Apply(U, I, *g, GetForwardAcc(U, I));
  GetForwardAcc(U, I) = Acc{};
}

// Backward accumulation: unit I folds its outgoing connections, descending
// index order (Pipeline) or ascending (Topological), starting from its current
// BackwardAcc (which a loss may have set).
template <class Tr, class UV, class CV, class G>
__global__ void k_bwd_acc(UV U, CV C, G *g, const uint32_t *out_ptr, const uint32_t *out_conn,
                          size_t n, int lvl, bool descending) {
  using BP = typename Tr::BackwardPass;
  const size_t I = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (I >= n) return;
  if (lvl >= 0 && GetLevel(U, I) != lvl) return;
  auto acc = GetBackwardAcc(U, I);
  const uint32_t b = out_ptr[I], e = out_ptr[I + 1];
  for (uint32_t j = 0; j < e - b; ++j) {
    const uint32_t c = out_conn[descending ? e - 1 - j : b + j];
    if (GetField<DeadTag>(C, c)) continue;
    acc = BP::Combine(acc, BP::Map(U, I, GetField<ToIdTag>(C, c), C, c, *g));
  }
  GetBackwardAcc(U, I) = acc;
}

template <class Tr, class UV, class G>
__global__ void k_bwd_apply(UV U, G *g, size_t lo, size_t hi, int lvl) {
  using BP = typename Tr::BackwardPass;
  using Acc = typename BP::Accumulator;
  const size_t I = lo + blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (I >= hi) return;
  if (lvl >= 0 && GetLevel(U, I) != lvl) return;
  BP::Apply(U, I, *g, GetBackwardAcc(U, I));
  GetBackwardAcc(U, I) = Acc{};
}

template <class Tr, class UV, class G>
__global__ void k_loss(UV U, G *g, UnitRange out, const float *t, size_t nt) {
  Tr::Loss::CalculateLoss(U, out, std::span<const float>(t, nt), *g);
}

template <class Tr, class UV, class G> __global__ void k_update_unit(UV U, G *g, size_t n) {
  const size_t I = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (I < n) Tr::UpdateUnit::Update(U, I, *g);
}

// Per-connection update: parallel over connections, or one thread in index
// order when the traits ask for sequential semantics.
template <class Tr, bool Incoming, class UV, class CV, class G>
__global__ void k_update_conn(UV U, CV C, G *g, size_t n, bool sequential) {
  using UP = typename Tr::UpdateConn;
  const size_t first = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t step = sequential ? 1 : (size_t)gridDim.x * blockDim.x;
  if (sequential && first != 0) return;
  for (size_t c = first; c < n; c += step) {
    if (GetField<DeadTag>(C, c)) continue;
    const size_t to = GetField<ToIdTag>(C, c), from = GetField<FromIdTag>(C, c);
    if constexpr (Incoming) UP::UpdateIncomingConnection(U, to, from, C, c, *g);
    else UP::UpdateOutgoingConnection(U, from, to, C, c, *g);
  }
}

template <class Tr, class G> __global__ void k_reset(G *g) { Tr::ResetGlobal::Reset(*g); }

}  // namespace detail

// ---------------------------------------------------------------------------
// Network
// ---------------------------------------------------------------------------
template <typename Traits> class Network {
 public:
  using GlobalState = typename Traits::GlobalState;
  using FP = typename Traits::ForwardPass;
  using BP = typename Traits::BackwardPass;
  using UnitAllocator = typename detail::UnitAllocFromList<
      typename FP::Accumulator, typename BP::Accumulator, typename Traits::ExtraUnitFields>::type;
  using ConnAllocator = typename detail::ConnAllocFromList<typename Traits::ExtraConnFields>::type;
  using UView = typename UnitAllocator::View;
  using CView = typename ConnAllocator::View;

  static_assert(std::is_same_v<typename Traits::PruneUnit, NoPruneUnit> &&
                    std::is_same_v<typename Traits::PruneConn, NoPruneConn> &&
                    std::is_same_v<typename Traits::AddUnit, NoAddUnit> &&
                    std::is_same_v<typename Traits::AddConn, NoAddConn>,
                "structural policies run through the C ABI on this path");
  static_assert(std::is_trivially_copyable_v<GlobalState>, "global state is copied to the GPU");

  template <typename... Builders>
    requires(sizeof...(Builders) > 0)
  Network(size_t InputDim, Builders... Layers) : Network(InputDim, NoUnitInit{}, Layers...) {}

  template <typename InputInit, typename... Builders>
    requires(std::is_invocable_v<InputInit, UnitAllocator &, size_t> && sizeof...(Builders) > 0)
  Network(size_t InputDim, InputInit Init, Builders... Layers) : NumInput(InputDim) {
    for (size_t I = 0; I < InputDim; ++I) Init(UA, UA.Allocate());
    UnitRange Prev{0, InputDim};
    ((Prev = Layers(UA, CA, Prev)), ...);
    OutputRange = Prev;
    if constexpr (Traits::Model == Propagation::Topological) SortByLevel();
    BuildIndex();
    Upload();
  }

  Network(size_t InputDim, size_t OutputDim = 1) : Network(InputDim, FullyConnected<>{OutputDim}) {}

  ~Network() { Release(); }
  Network(const Network &) = delete;
  Network &operator=(const Network &) = delete;

  size_t GetStep() const { return Step; }

  void DoForwardPass(std::span<const float> Inputs) {
    SyncToDevice();
    if (NumInput)
      cuda_check(cudaMemcpyAsync(d_uf[0], Inputs.data(), NumInput * sizeof(float),
                                 cudaMemcpyHostToDevice, Stream),
                 "inputs");
    const size_t n = UA.Size();
    if constexpr (Traits::Model == Propagation::Topological) {
      for (int L = 1; L <= NumLevels; ++L) {
        detail::k_fwd_acc<Traits><<<detail::blocks(n), 256, 0, Stream>>>(
            UV(), CV(), d_g, d_in_ptr, d_in_conn, NumInput, n, L);
        detail::k_fwd_apply<Traits><<<detail::blocks(n), 256, 0, Stream>>>(UV(), d_g, NumInput, n, L);
      }
    } else {
      detail::k_fwd_acc<Traits><<<detail::blocks(n), 256, 0, Stream>>>(UV(), CV(), d_g, d_in_ptr,
                                                                        d_in_conn, NumInput, n, -1);
      detail::k_fwd_apply<Traits><<<detail::blocks(n), 256, 0, Stream>>>(UV(), d_g, NumInput, n, -1);
    }
    cuda_check(cudaGetLastError(), "forward pass");
    ++Step;
  }

  void DoCalculateLoss(std::span<const float> Targets) {
    if constexpr (!std::is_same_v<typename Traits::Loss, NoLoss>) {
      if (Targets.empty()) return;
      SyncToDevice();
      if (Targets.size() > TargetCap) {
        if (d_targets) cudaFree(d_targets);
        cuda_check(cudaMalloc(&d_targets, Targets.size() * sizeof(float)), "targets");
        TargetCap = Targets.size();
      }
      cuda_check(cudaMemcpyAsync(d_targets, Targets.data(), Targets.size() * sizeof(float),
                                 cudaMemcpyHostToDevice, Stream),
                 "targets");
      detail::k_loss<Traits><<<1, 1, 0, Stream>>>(UV(), d_g, OutputRange, d_targets,
                                                  Targets.size());
      cuda_check(cudaGetLastError(), "loss");
    }
  }

  void DoBackwardPass() {
    if constexpr (!std::is_same_v<BP, NoBackwardPass>) {
      SyncToDevice();
      const size_t n = UA.Size();
      if constexpr (Traits::Model == Propagation::Topological) {
        for (int L = NumLevels; L >= 1; --L) {
          detail::k_bwd_acc<Traits><<<detail::blocks(n), 256, 0, Stream>>>(
              UV(), CV(), d_g, d_out_ptr, d_out_conn, n, L, false);
          detail::k_bwd_apply<Traits><<<detail::blocks(n), 256, 0, Stream>>>(UV(), d_g, 0, n, L);
        }
      } else {
        detail::k_bwd_acc<Traits><<<detail::blocks(n), 256, 0, Stream>>>(
            UV(), CV(), d_g, d_out_ptr, d_out_conn, n, -1, true);
        detail::k_bwd_apply<Traits><<<detail::blocks(n), 256, 0, Stream>>>(UV(), d_g, 0, n, -1);
      }
      cuda_check(cudaGetLastError(), "backward pass");
    }
  }

  void DoResetGlobalState() {
    if constexpr (!std::is_same_v<typename Traits::ResetGlobal, NoResetGlobalState>) {
      SyncToDevice();
      detail::k_reset<Traits><<<1, 1, 0, Stream>>>(d_g);
      cuda_check(cudaGetLastError(), "reset");
    }
  }

  void DoUpdateUnitState() {
    if constexpr (!std::is_same_v<typename Traits::UpdateUnit, NoUpdateUnit>) {
      SyncToDevice();
      detail::k_update_unit<Traits><<<detail::blocks(UA.Size()), 256, 0, Stream>>>(UV(), d_g,
                                                                                  UA.Size());
      cuda_check(cudaGetLastError(), "unit update");
    }
  }

  void DoUpdateConnectionState() {
    if constexpr (!std::is_same_v<typename Traits::UpdateConn, NoUpdateConn>) {
      SyncToDevice();
      constexpr bool seq = detail::SequentialUpdate<Traits>::value;
      const size_t n = CA.Size();
      const unsigned grid = seq ? 1 : std::min<unsigned>(detail::blocks(n), 4096);
      detail::k_update_conn<Traits, true><<<grid, 256, 0, Stream>>>(UV(), CV(), d_g, n, seq);
      detail::k_update_conn<Traits, false><<<grid, 256, 0, Stream>>>(UV(), CV(), d_g, n, seq);
      cuda_check(cudaGetLastError(), "connection update");
    }
  }

  void DoPruneUnits() {}
  void DoPruneConnections() {}
  void DoAddUnits() {}
  void DoAddConnections() {}

  void DoStep(std::span<const float> Inputs, std::span<const float> Targets = {}) {
    DoForwardPass(Inputs);
    DoCalculateLoss(Targets);
    DoBackwardPass();
    DoUpdateUnitState();
    DoUpdateConnectionState();
    DoPruneUnits();
    DoPruneConnections();
    DoAddUnits();
    DoAddConnections();
    DoResetGlobalState();
  }

  // Activations of the output units (waits for the device).
  std::span<const float> GetOutput() {
    Output.resize(OutputRange.Size());
    cuda_check(cudaMemcpyAsync(Output.data(), static_cast<float *>(d_uf[0]) + OutputRange.Begin,
                               Output.size() * sizeof(float), cudaMemcpyDeviceToHost, Stream),
               "output");
    cuda_check(cudaStreamSynchronize(Stream), "output");
    return {Output.data(), Output.size()};
  }

  // Host copies: downloaded unless the host copy already holds edits not yet
  // uploaded (no Do* call since the last access); edits are uploaded before
  // the next Do* call.
  UnitAllocator &GetUnitAlloc() {
    if (!UnitDirty) Download(UA, d_uf);
    UnitDirty = true;
    return UA;
  }
  ConnAllocator &GetConnAlloc() {
    if (!ConnDirty) Download(CA, d_cf);
    ConnDirty = true;
    return CA;
  }
  GlobalState GetGlobals() {
    GlobalState g;
    cuda_check(cudaMemcpyAsync(&g, d_g, sizeof(g), cudaMemcpyDeviceToHost, Stream), "globals");
    cuda_check(cudaStreamSynchronize(Stream), "globals");
    return g;
  }
  void SetGlobals(const GlobalState &g) {
    cuda_check(cudaMemcpyAsync(d_g, &g, sizeof(g), cudaMemcpyHostToDevice, Stream), "globals");
    cuda_check(cudaStreamSynchronize(Stream), "globals");
  }
  void SetStream(cudaStream_t s) { Stream = s; }
  UnitRange GetOutputRange() const { return OutputRange; }

 private:
  UView UV() const {
    UView v{};
    for (size_t i = 0; i < UnitAllocator::NumFields; ++i) v.ptr[i] = d_uf[i];
    v.size = UA.Size();
    return v;
  }
  CView CV() const {
    CView v{};
    for (size_t i = 0; i < ConnAllocator::NumFields; ++i) v.ptr[i] = d_cf[i];
    v.size = CA.Size();
    return v;
  }

  // Stable reorder of the connections by source level (the Topological
  // processing order), as the reference does at construction.
  void SortByLevel() {
    std::vector<size_t> perm(CA.Size());
    for (size_t i = 0; i < perm.size(); ++i) perm[i] = i;
    std::stable_sort(perm.begin(), perm.end(), [&](size_t a, size_t b) {
      return CA.template Get<SrcLevelTag>(a) < CA.template Get<SrcLevelTag>(b);
    });
    CA.Gather(perm);
  }

  // Incoming connection lists per destination (stored order) and outgoing per
  // source (ascending index), as CSR arrays on the device.
  void BuildIndex() {
    const size_t n = UA.Size(), m = CA.Size();
    NumLevels = 0;
    for (size_t i = 0; i < n; ++i)
      NumLevels = std::max<int>(NumLevels, (int)UA.template Get<LevelTag>(i));
    std::vector<uint32_t> in_ptr(n + 1, 0), out_ptr(n + 1, 0), in_conn(m), out_conn(m);
    for (size_t c = 0; c < m; ++c) {
      ++in_ptr[CA.template Get<ToIdTag>(c) + 1];
      ++out_ptr[CA.template Get<FromIdTag>(c) + 1];
    }
    for (size_t i = 0; i < n; ++i) {
      in_ptr[i + 1] += in_ptr[i];
      out_ptr[i + 1] += out_ptr[i];
    }
    std::vector<uint32_t> fi(in_ptr.begin(), in_ptr.end() - 1), fo(out_ptr.begin(), out_ptr.end() - 1);
    for (size_t c = 0; c < m; ++c) {
      in_conn[fi[CA.template Get<ToIdTag>(c)]++] = (uint32_t)c;
      out_conn[fo[CA.template Get<FromIdTag>(c)]++] = (uint32_t)c;
    }
    auto up = [&](uint32_t *&d, const std::vector<uint32_t> &h) {
      cuda_check(cudaMalloc(&d, std::max<size_t>(1, h.size()) * 4), "index");
      if (!h.empty())
        cuda_check(cudaMemcpy(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice), "index");
    };
    up(d_in_ptr, in_ptr);
    up(d_out_ptr, out_ptr);
    up(d_in_conn, in_conn);
    up(d_out_conn, out_conn);
  }

  template <class A> void UploadAlloc(A &a, std::vector<void *> &d, bool alloc) {
    if (alloc) d.assign(A::NumFields, nullptr);
    for (size_t i = 0; i < A::NumFields; ++i) {
      const size_t bytes = std::max<size_t>(1, a.Size()) * A::field_bytes(i);
      if (alloc) cuda_check(cudaMalloc(&d[i], bytes), "field");
      if (a.Size())
        cuda_check(cudaMemcpy(d[i], a.field_data(i), a.Size() * A::field_bytes(i),
                              cudaMemcpyHostToDevice),
                   "field upload");
    }
  }
  template <class A> void Download(A &a, std::vector<void *> &d) {
    cuda_check(cudaStreamSynchronize(Stream), "download");
    for (size_t i = 0; i < A::NumFields; ++i)
      if (a.Size())
        cuda_check(cudaMemcpy(a.field_data(i), d[i], a.Size() * A::field_bytes(i),
                              cudaMemcpyDeviceToHost),
                   "field download");
  }
  void Upload() {
    UploadAlloc(UA, d_uf, true);
    UploadAlloc(CA, d_cf, true);
    cuda_check(cudaMalloc(&d_g, sizeof(GlobalState) > 0 ? sizeof(GlobalState) : 1), "globals");
    GlobalState g{};
    cuda_check(cudaMemcpy(d_g, &g, sizeof(GlobalState), cudaMemcpyHostToDevice), "globals");
  }
  void SyncToDevice() {
    if (UnitDirty) {
      UploadAlloc(UA, d_uf, false);
      UnitDirty = false;
    }
    if (ConnDirty) {
      UploadAlloc(CA, d_cf, false);
      ConnDirty = false;
    }
  }
  void Release() {
    for (void *p : d_uf) cudaFree(p);
    for (void *p : d_cf) cudaFree(p);
    for (void *p : {(void *)d_g, (void *)d_in_ptr, (void *)d_out_ptr, (void *)d_in_conn,
                    (void *)d_out_conn, (void *)d_targets})
      if (p) cudaFree(p);
  }

  size_t NumInput;
  UnitRange OutputRange;
  UnitAllocator UA;
  ConnAllocator CA;
  int NumLevels = 0;
  size_t Step = 0;
  std::vector<void *> d_uf, d_cf;
  GlobalState *d_g = nullptr;
  uint32_t *d_in_ptr = nullptr, *d_out_ptr = nullptr, *d_in_conn = nullptr, *d_out_conn = nullptr;
  float *d_targets = nullptr;
  size_t TargetCap = 0;
  bool UnitDirty = false, ConnDirty = false;
  cudaStream_t Stream = nullptr;
  std::vector<float> Output;
};

}  // namespace plastix
