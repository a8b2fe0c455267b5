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
//   * Structural policies: PruneUnit and PruneConn run per unit / per
//     connection on the device; AddConn's proposals are enumerated on the
//     device in the reference's order (level window, unit pairs, the four
//     checks), then sorted, de-duplicated and committed through the C ABI
//     (libplastix_b200: link with -lplastix_b200), and Topological networks
//     re-sort by source level on the device (RecomputeLevels included), as
//     the reference's constructor and DoStep do. The predicates run in
//     parallel, so they must not change the global state -- traits with
//     `static constexpr bool SequentialStructure = true` run them in one
//     thread in the reference's order instead. AddUnit is not supported.
//   * Topological passes follow the reference level by level: level L folds
//     the connections whose SrcLevel is L - 1 into their targets' forward
//     accumulators (one thread per unit, stored order), then applies the
//     units of level L.
//   * No fixed capacity: networks of any size that fit the GPU.
//   * GetUnitAlloc()/GetConnAlloc() return host copies (downloaded on call;
//     edits made through them are uploaded before the next Do* call).
//     GetGlobals()/SetGlobals() and Save(path)/Load(path) (checkpoints of
//     every field plus the global state) are additions.
#pragma once

#include <cuda_runtime.h>
#include <plastix_b200.h>

#include <cub/block/block_scan.cuh>
#include <cub/device/device_scan.cuh>

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <cstdio>
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
  // Sets the number of entities (new ones value-initialised).
  void Resize(size_t N) {
    resize(N, std::index_sequence_for<Fs...>{});
    n_ = N;
  }
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
  template <size_t... Is> void resize(size_t N, std::index_sequence<Is...>) {
    (std::get<Is>(store_).resize(N), ...);
  }
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

// Traits flag for structural policies that mutate the global state (an RNG
// drawn inside a predicate): prune, proposal and commit hooks then run in one
// thread, in the reference's order.
template <class T> struct SequentialStructure {
  static constexpr bool value = false;
};
template <class T>
  requires requires { T::SequentialStructure; }
struct SequentialStructure<T> {
  static constexpr bool value = T::SequentialStructure;
};

// Topological forward accumulation of level L (plastix.hpp:111-119 of the
// reference): every unit folds, in stored order, those incoming connections
// whose SrcLevel is L - 1 -- whatever the unit's own level. Connections are
// kept sorted by SrcLevel, so each unit's incoming list is too; `cur` is the
// unit's position in it, advanced level by level.
template <class Tr, class UV, class CV, class G>
__global__ void k_fwd_acc_level(UV U, CV C, G *g, const uint32_t *in_ptr, const uint32_t *in_conn,
                                uint32_t *cur, size_t n, int L) {
  using FP = typename Tr::ForwardPass;
  const size_t I = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (I >= n) return;
  uint32_t k = cur[I];
  const uint32_t e = in_ptr[I + 1];
  if (k >= e) return;
  const uint16_t want = (uint16_t)(L - 1);
  auto acc = GetForwardAcc(U, I);
  bool any = false;
  for (; k < e; ++k) {
    const uint32_t c = in_conn[k];
    const uint16_t sl = GetField<SrcLevelTag>(C, c);
    if (sl > want) break;
    if (sl != want || GetField<DeadTag>(C, c)) continue;
    acc = FP::Combine(acc, FP::Map(U, I, GetField<FromIdTag>(C, c), C, c, *g));
    any = true;
  }
  cur[I] = k;
  if (any) GetForwardAcc(U, I) = acc;
}

// DoPruneUnits (reference plastix.hpp:257-267): Pruned = ShouldPrune.
template <class Tr, class UV, class G> __global__ void k_prune_units(UV U, G *g, size_t n, bool seq) {
  const size_t first = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t step = seq ? 1 : (size_t)gridDim.x * blockDim.x;
  if (seq && first != 0) return;
  for (size_t I = first; I < n; I += step)
    GetField<PrunedTag>(U, I) = Tr::PruneUnit::ShouldPrune(U, I, *g) ? 1 : 0;
}

// DoPruneConnections (reference plastix.hpp:269-299): a live connection dies
// when either endpoint was pruned or the connection policy says so.
template <class Tr, class UV, class CV, class G>
__global__ void k_prune_conns(UV U, CV C, G *g, size_t m, bool seq) {
  constexpr bool HasUnit = !std::is_same_v<typename Tr::PruneUnit, NoPruneUnit>;
  constexpr bool HasConn = !std::is_same_v<typename Tr::PruneConn, NoPruneConn>;
  const size_t first = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t step = seq ? 1 : (size_t)gridDim.x * blockDim.x;
  if (seq && first != 0) return;
  for (size_t c = first; c < m; c += step) {
    if (GetField<DeadTag>(C, c)) continue;
    const size_t to = GetField<ToIdTag>(C, c), from = GetField<FromIdTag>(C, c);
    bool rm = false;
    if constexpr (HasUnit) rm = GetField<PrunedTag>(U, to) || GetField<PrunedTag>(U, from);
    if constexpr (HasConn)
      if (!rm) rm = Tr::PruneConn::ShouldPrune(U, to, from, C, c, *g);
    if (rm) GetField<DeadTag>(C, c) = 1;
  }
}

// One level pair of DoAddConnections' window (reference plastix.hpp:363-389):
// units UnitsByLevel[a0, a0+na) x UnitsByLevel[b0, b0+nb), slots numbered
// from `first` in the reference's enumeration order.
struct LevelPair {
  uint64_t first;
  uint32_t a0, na, b0, nb, same;
};
constexpr int kPropItems = 4;                      // slots per thread
constexpr uint64_t kPropChunk = 256 * kPropItems;  // slots per block and chunk

PLASTIX_HD inline uint64_t compact_edge(size_t from, size_t to) {  // CompactEdge::Bits
  return (uint64_t)(uint32_t)from | ((uint64_t)(uint32_t)to << 32);
}

__device__ inline uint32_t find_pair(const LevelPair *p, uint32_t n, uint64_t s) {
  uint32_t lo = 0, hi = n;
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) / 2;
    if (p[mid].first <= s) lo = mid;
    else hi = mid;
  }
  return lo;
}

// The proposals of one slot (unit pair), in the reference's order of checks.
template <class Tr, class UV, class G>
__device__ uint32_t propose_slot(UV &U, G *g, const LevelPair *pairs, uint32_t np,
                                 const uint32_t *ubl, uint64_t s, uint64_t *out) {
  using AC = typename Tr::AddConn;
  const LevelPair P = pairs[find_pair(pairs, np, s)];
  const uint64_t r = s - P.first;
  const size_t A = ubl[P.a0 + r / P.nb], B = ubl[P.b0 + r % P.nb];
  if (A == B) return 0;
  uint32_t k = 0;
  if (AC::ShouldAddIncomingConnection(U, A, B, *g)) out[k++] = compact_edge(B, A);
  if (AC::ShouldAddOutgoingConnection(U, A, B, *g)) out[k++] = compact_edge(A, B);
  if (!P.same) {
    if (AC::ShouldAddIncomingConnection(U, B, A, *g)) out[k++] = compact_edge(A, B);
    if (AC::ShouldAddOutgoingConnection(U, B, A, *g)) out[k++] = compact_edge(B, A);
  }
  return k;
}

// Parallel proposal enumeration in two passes over chunks of slots: COUNT
// writes each chunk's number of proposals; WRITE puts them at the chunk's
// offset in slot order, dropping those at index >= cap (the reference stops
// proposing at its capacity). The predicates are evaluated in both passes.
template <class Tr, bool WRITE, class UV, class G>
__global__ void __launch_bounds__(256)
    k_propose(UV U, G *g, const LevelPair *pairs, uint32_t np, const uint32_t *ubl, uint64_t total,
              uint64_t n_chunks, uint64_t *chunk_counts, const uint64_t *chunk_off, uint64_t cap,
              uint64_t *props) {
  using BS = cub::BlockScan<uint32_t, 256>;
  __shared__ typename BS::TempStorage tmp;
  for (uint64_t ch = blockIdx.x; ch < n_chunks; ch += gridDim.x) {
    uint64_t bits[4 * kPropItems];
    uint32_t cnt = 0;
    const uint64_t s0 = ch * kPropChunk + (uint64_t)threadIdx.x * kPropItems;
    for (int it = 0; it < kPropItems; ++it) {
      const uint64_t s = s0 + it;
      if (s >= total) break;
      cnt += propose_slot<Tr>(U, g, pairs, np, ubl, s, bits + cnt);
    }
    uint32_t off, agg;
    BS(tmp).ExclusiveSum(cnt, off, agg);
    if constexpr (!WRITE) {
      if (threadIdx.x == 0) chunk_counts[ch] = agg;
    } else {
      const uint64_t base = chunk_off[ch] + off;
      for (uint32_t k = 0; k < cnt; ++k)
        if (base + k < cap) props[base + k] = bits[k];
    }
    __syncthreads();
  }
}

// The same enumeration in one thread, stopping at the capacity exactly as the
// reference does (a predicate is not called once the list is full).
template <class Tr, class UV, class G>
__global__ void k_propose_seq(UV U, G *g, const LevelPair *pairs, uint32_t np, const uint32_t *ubl,
                              uint64_t cap, uint64_t *props, uint64_t *count) {
  using AC = typename Tr::AddConn;
  uint64_t n = 0;
  for (uint32_t p = 0; p < np; ++p) {
    const LevelPair P = pairs[p];
    for (uint32_t ai = 0; ai < P.na; ++ai) {
      const size_t A = ubl[P.a0 + ai];
      for (uint32_t bi = 0; bi < P.nb; ++bi) {
        const size_t B = ubl[P.b0 + bi];
        if (A == B) continue;
        if (n < cap && AC::ShouldAddIncomingConnection(U, A, B, *g)) props[n++] = compact_edge(B, A);
        if (n < cap && AC::ShouldAddOutgoingConnection(U, A, B, *g)) props[n++] = compact_edge(A, B);
        if (!P.same) {
          if (n < cap && AC::ShouldAddIncomingConnection(U, B, A, *g))
            props[n++] = compact_edge(A, B);
          if (n < cap && AC::ShouldAddOutgoingConnection(U, B, A, *g))
            props[n++] = compact_edge(B, A);
        }
      }
    }
  }
  *count = n;
}

// Commit of the unique proposals (reference plastix.hpp:421-431): connection
// m0 + i gets FromId, ToId and SrcLevel = Level[FromId] (the other fields
// were zeroed), then InitConnection.
template <class Tr, class UV, class CV, class G>
__global__ void k_commit_conns(UV U, CV C, G *g, const uint64_t *edges, size_t k, size_t m0,
                               bool seq) {
  const size_t first = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t step = seq ? 1 : (size_t)gridDim.x * blockDim.x;
  if (seq && first != 0) return;
  for (size_t i = first; i < k; i += step) {
    const uint64_t b = edges[i];
    const size_t c = m0 + i, F = (uint32_t)b, T = (uint32_t)(b >> 32);
    GetField<FromIdTag>(C, c) = (uint32_t)F;
    GetField<ToIdTag>(C, c) = (uint32_t)T;
    GetField<SrcLevelTag>(C, c) = GetLevel(U, F);
    Tr::AddConn::InitConnection(U, F, T, C, c, *g);
  }
}

__global__ inline void k_widen_u16(const uint16_t *in, size_t n, uint32_t *out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = in[i];
}

__global__ inline void k_level_hist(const uint16_t *level, size_t n, uint32_t *hist) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    atomicAdd(hist + level[i], 1u);
}

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

  static_assert(std::is_same_v<typename Traits::AddUnit, NoAddUnit>,
                "AddUnit policies are not supported on the device");
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
    cuda_check(cudaGetDevice(&Device), "device");
    Upload();
    // As the reference's constructor: Topological networks recompute the
    // unit levels and sort the connections by source level.
    if constexpr (Traits::Model == Propagation::Topological) SortConnectionsByLevel();
    RebuildIndex();
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
      if (NeedsResort) SortConnectionsByLevel();
      if (IndexStale) RebuildIndex();
      if (n)
        cuda_check(cudaMemcpyAsync(d_cursor, d_in_ptr, n * sizeof(uint32_t),
                                   cudaMemcpyDeviceToDevice, Stream),
                   "cursor");
      for (int L = 1; L <= NumLevels; ++L) {
        detail::k_fwd_acc_level<Traits><<<detail::blocks(n), 256, 0, Stream>>>(
            UV(), CV(), d_g, d_in_ptr, d_in_conn, d_cursor, n, L);
        detail::k_fwd_apply<Traits><<<detail::blocks(n), 256, 0, Stream>>>(UV(), d_g, NumInput, n, L);
      }
    } else {
      if (IndexStale) RebuildIndex();
      detail::k_fwd_acc<Traits><<<detail::blocks(n), 256, 0, Stream>>>(UV(), CV(), d_g, d_in_ptr,
                                                                        d_in_conn, 0, n, -1);
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
      if (IndexStale) RebuildIndex();
      const size_t n = UA.Size();
      if constexpr (Traits::Model == Propagation::Topological) {
        for (int L = NumLevels; L >= 1; --L) {
          detail::k_bwd_acc<Traits><<<detail::blocks(n), 256, 0, Stream>>>(
              UV(), CV(), d_g, d_out_ptr, d_out_conn, n, L, false);
          detail::k_bwd_apply<Traits><<<detail::blocks(n), 256, 0, Stream>>>(UV(), d_g, NumInput,
                                                                             n, L);
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

  void DoPruneUnits() {
    if constexpr (!std::is_same_v<typename Traits::PruneUnit, NoPruneUnit>) {
      SyncToDevice();
      const size_t n = UA.Size();
      detail::k_prune_units<Traits><<<kSeq ? 1 : detail::blocks(n), 256, 0, Stream>>>(UV(), d_g, n,
                                                                                     kSeq);
      cuda_check(cudaGetLastError(), "prune units");
    }
  }

  void DoPruneConnections() {
    if constexpr (!std::is_same_v<typename Traits::PruneUnit, NoPruneUnit> ||
                  !std::is_same_v<typename Traits::PruneConn, NoPruneConn>) {
      SyncToDevice();
      const size_t m = CA.Size();
      const unsigned grid = kSeq ? 1 : std::min<unsigned>(detail::blocks(m), 4096);
      detail::k_prune_conns<Traits><<<grid, 256, 0, Stream>>>(UV(), CV(), d_g, m, kSeq);
      cuda_check(cudaGetLastError(), "prune connections");
    }
  }

  void DoAddUnits() {}

  // DoAddConnections (reference plastix.hpp:320-435): units bucketed by level
  // (phase 0), the level-pair window enumerated on the device in the
  // reference's order (phase 1), sort + unique commit (phases 2-3) through the
  // C ABI, new connections appended and initialised by InitConnection.
  void DoAddConnections() {
    if constexpr (!std::is_same_v<typename Traits::AddConn, NoAddConn>) {
      SyncToDevice();
      const size_t n = UA.Size();
      if (n == 0) return;
      plx_ctx *ctx = PlxCtx();
      // phase 0: units by level (stable by id), level offsets
      uint32_t *hist = Buf<uint32_t>(0, 65536);
      cuda_check(cudaMemsetAsync(hist, 0, 65536 * sizeof(uint32_t), Stream), "histogram");
      detail::k_level_hist<<<detail::blocks(n), 256, 0, Stream>>>(LevelPtr(), n, hist);
      std::vector<uint32_t> h(65536);
      cuda_check(cudaMemcpyAsync(h.data(), hist, h.size() * 4, cudaMemcpyDeviceToHost, Stream),
                 "histogram");
      cuda_check(cudaStreamSynchronize(Stream), "histogram");
      uint32_t highest = 0;
      for (uint32_t L = 0; L < 65536; ++L)
        if (h[L]) highest = L;
      std::vector<uint32_t> off(highest + 2, 0);
      for (uint32_t L = 0; L <= highest; ++L) off[L + 1] = off[L] + h[L];
      uint32_t *keys = Buf<uint32_t>(1, n), *keys_out = Buf<uint32_t>(2, n);
      uint32_t *ubl = Buf<uint32_t>(3, n);
      detail::k_widen_u16<<<detail::blocks(n), 256, 0, Stream>>>(LevelPtr(), n, keys);
      RadixSort(n, keys, keys_out, ubl, 16);
      // phase 1: the level pairs of the window, in the reference's order
      std::vector<detail::LevelPair> pairs;
      uint64_t total = 0;
      auto add = [&](uint32_t La, uint32_t Lb) {
        const uint32_t na = off[La + 1] - off[La], nb = off[Lb + 1] - off[Lb];
        if (!na || !nb) return;
        pairs.push_back({total, off[La], na, off[Lb], nb, La == Lb ? 1u : 0u});
        total += (uint64_t)na * nb;
      };
      constexpr uint32_t N = Traits::Neighbourhood;
      const uint32_t init_right = std::min<uint32_t>(N, highest);
      for (uint32_t La = 0; La <= init_right; ++La)
        for (uint32_t Lb = La; Lb <= init_right; ++Lb) add(La, Lb);
      for (uint32_t R = N + 1; R <= highest; ++R)
        for (uint32_t W = R - N; W <= R; ++W) add(W, R);
      if (total == 0) return;
      auto *d_pairs = Buf<detail::LevelPair>(4, pairs.size());
      cuda_check(cudaMemcpyAsync(d_pairs, pairs.data(), pairs.size() * sizeof(detail::LevelPair),
                                 cudaMemcpyHostToDevice, Stream),
                 "level pairs");
      const uint32_t np = (uint32_t)pairs.size();
      uint64_t n_props = 0;
      uint64_t *props = nullptr;
      if constexpr (kSeq) {
        const uint64_t cap = std::min<uint64_t>(ProposalCap, 4 * total);
        props = Buf<uint64_t>(5, cap);
        uint64_t *cnt = Buf<uint64_t>(6, 1);
        detail::k_propose_seq<Traits><<<1, 1, 0, Stream>>>(UV(), d_g, d_pairs, np, ubl, cap, props,
                                                           cnt);
        cuda_check(cudaMemcpyAsync(&n_props, cnt, 8, cudaMemcpyDeviceToHost, Stream), "count");
        cuda_check(cudaStreamSynchronize(Stream), "proposals");
      } else {
        const uint64_t n_chunks = (total + detail::kPropChunk - 1) / detail::kPropChunk;
        uint64_t *counts = Buf<uint64_t>(6, n_chunks + 1), *coff = Buf<uint64_t>(7, n_chunks + 1);
        const unsigned grid = (unsigned)std::min<uint64_t>(n_chunks, 8192);
        detail::k_propose<Traits, false><<<grid, 256, 0, Stream>>>(
            UV(), d_g, d_pairs, np, ubl, total, n_chunks, counts, nullptr, 0, nullptr);
        cuda_check(cudaMemsetAsync(counts + n_chunks, 0, 8, Stream), "counts");
        size_t tb = 0;
        cuda_check(cub::DeviceScan::ExclusiveSum(nullptr, tb, counts, coff, n_chunks + 1, Stream),
                   "scan");
        void *tmp = Buf<uint8_t>(8, tb);
        cuda_check(cub::DeviceScan::ExclusiveSum(tmp, tb, counts, coff, n_chunks + 1, Stream),
                   "scan");
        cuda_check(cudaMemcpyAsync(&n_props, coff + n_chunks, 8, cudaMemcpyDeviceToHost, Stream),
                   "count");
        cuda_check(cudaStreamSynchronize(Stream), "proposals");
        n_props = std::min<uint64_t>(n_props, ProposalCap);
        if (n_props == 0) return;
        props = Buf<uint64_t>(5, n_props);
        detail::k_propose<Traits, true><<<grid, 256, 0, Stream>>>(
            UV(), d_g, d_pairs, np, ubl, total, n_chunks, nullptr, coff, n_props, props);
      }
      cuda_check(cudaGetLastError(), "proposals");
      if (n_props == 0) return;
      // phases 2-3: sorted unique proposals, committed in that order
      uint64_t *uniq = Buf<uint64_t>(9, n_props), *ucnt = Buf<uint64_t>(10, 1);
      const size_t sb = plx_sort_unique_u64_scratch_bytes(n_props);
      plx_check(plx_sort_unique_u64(ctx, n_props, props, uniq, ucnt, Buf<uint8_t>(11, sb), sb),
                "plx_sort_unique_u64");
      uint64_t k = 0;
      cuda_check(cudaMemcpyAsync(&k, ucnt, 8, cudaMemcpyDeviceToHost, Stream), "unique");
      cuda_check(cudaStreamSynchronize(Stream), "unique");
      if (k == 0) return;
      const size_t m0 = CA.Size();
      GrowConnections(k);
      detail::k_commit_conns<Traits><<<kSeq ? 1 : detail::blocks(k), 256, 0, Stream>>>(
          UV(), CV(), d_g, uniq, k, m0, kSeq);
      cuda_check(cudaGetLastError(), "commit");
      NeedsResort = Traits::Model == Propagation::Topological;
      IndexStale = true;
    }
  }

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
    if constexpr (Traits::Model == Propagation::Topological)
      if (NeedsResort) SortConnectionsByLevel();
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
  void SetStream(cudaStream_t s) {
    Stream = s;
    if (Ctx) plx_check(plx_ctx_set_stream(Ctx, s), "plx_ctx_set_stream");
  }
  // Upper bound on one DoAddConnections' proposal list (the reference's is its
  // connection capacity): proposals past it are not made.
  void SetProposalCapacity(uint64_t n) { ProposalCap = n; }
  UnitRange GetOutputRange() const { return OutputRange; }
  int GetNumLevels() const { return NumLevels; }

  // Checkpoint: a header (counts, output range, step, level state, field
  // sizes, global-state size), every unit and connection field, the global
  // state. Load replaces this network's state with the file's; the traits
  // (field schema and global state) must be the ones that wrote it.
  void Save(const std::string &Path) {
    SyncToDevice();
    Download(UA, d_uf);
    Download(CA, d_cf);
    const GlobalState G = GetGlobals();
    CheckpointHeader H = Header();
    FILE *F = std::fopen(Path.c_str(), "wb");
    if (!F) throw std::runtime_error("cannot write " + Path);
    bool ok = std::fwrite(&H, sizeof(H), 1, F) == 1;
    ok = ok && WriteFieldSizes<UnitAllocator>(F) && WriteFieldSizes<ConnAllocator>(F);
    for (size_t i = 0; ok && i < UnitAllocator::NumFields; ++i)
      ok = WriteAll(F, UA.field_data(i), UA.Size() * UnitAllocator::field_bytes(i));
    for (size_t i = 0; ok && i < ConnAllocator::NumFields; ++i)
      ok = WriteAll(F, CA.field_data(i), CA.Size() * ConnAllocator::field_bytes(i));
    ok = ok && WriteAll(F, &G, sizeof(G));
    ok = (std::fclose(F) == 0) && ok;
    if (!ok) throw std::runtime_error("short write to " + Path);
  }

  void Load(const std::string &Path) {
    FILE *F = std::fopen(Path.c_str(), "rb");
    if (!F) throw std::runtime_error("cannot read " + Path);
    auto fail = [&](const char *why) {
      std::fclose(F);
      throw std::runtime_error(Path + ": " + why);
    };
    CheckpointHeader H{}, Want = Header();
    if (std::fread(&H, sizeof(H), 1, F) != 1) fail("truncated header");
    if (std::memcmp(H.Magic, Want.Magic, sizeof(H.Magic)) != 0) fail("not a checkpoint");
    if (H.UnitFields != Want.UnitFields || H.ConnFields != Want.ConnFields ||
        H.GlobalBytes != Want.GlobalBytes)
      fail("field schema or global state differs from these traits");
    if (!CheckFieldSizes<UnitAllocator>(F) || !CheckFieldSizes<ConnAllocator>(F))
      fail("field sizes differ from these traits");
    cuda_check(cudaStreamSynchronize(Stream), "load");
    UA.Resize(H.Units);
    CA.Resize(H.Conns);
    for (size_t i = 0; i < UnitAllocator::NumFields; ++i)
      if (!ReadAll(F, UA.field_data(i), UA.Size() * UnitAllocator::field_bytes(i)))
        fail("truncated unit field");
    for (size_t i = 0; i < ConnAllocator::NumFields; ++i)
      if (!ReadAll(F, CA.field_data(i), CA.Size() * ConnAllocator::field_bytes(i)))
        fail("truncated connection field");
    GlobalState G{};
    if (!ReadAll(F, &G, sizeof(G))) fail("truncated global state");
    std::fclose(F);
    for (void *p : d_uf) cudaFree(p);
    for (void *p : d_cf) cudaFree(p);
    UploadAlloc(UA, d_uf, true);
    UploadAlloc(CA, d_cf, true);
    SetGlobals(G);
    NumInput = H.NumInput;
    OutputRange = UnitRange(H.OutBegin, H.OutEnd);
    Step = H.Step;
    NumLevels = H.NumLevels;
    NeedsResort = (H.Flags & 1u) != 0;
    UnitDirty = ConnDirty = false;
    RebuildIndex();
  }

 private:
  static constexpr bool kSeq = detail::SequentialStructure<Traits>::value;

  struct CheckpointHeader {
    char Magic[8];
    uint64_t NumInput, Step, Units, Conns, OutBegin, OutEnd;
    int32_t NumLevels;
    uint32_t Flags;  // bit 0: a level re-sort is pending
    uint32_t UnitFields, ConnFields, GlobalBytes, Reserved;
  };
  CheckpointHeader Header() const {
    CheckpointHeader H{};
    std::memcpy(H.Magic, "PLXCKPT1", 8);
    H.NumInput = NumInput;
    H.Step = Step;
    H.Units = UA.Size();
    H.Conns = CA.Size();
    H.OutBegin = OutputRange.Begin;
    H.OutEnd = OutputRange.End;
    H.NumLevels = NumLevels;
    H.Flags = NeedsResort ? 1u : 0u;
    H.UnitFields = (uint32_t)UnitAllocator::NumFields;
    H.ConnFields = (uint32_t)ConnAllocator::NumFields;
    H.GlobalBytes = (uint32_t)sizeof(GlobalState);
    return H;
  }
  static bool WriteAll(FILE *F, const void *P, size_t N) {
    return N == 0 || std::fwrite(P, 1, N, F) == N;
  }
  static bool ReadAll(FILE *F, void *P, size_t N) { return N == 0 || std::fread(P, 1, N, F) == N; }
  template <class A> static bool WriteFieldSizes(FILE *F) {
    for (size_t i = 0; i < A::NumFields; ++i) {
      const uint32_t b = (uint32_t)A::field_bytes(i);
      if (std::fwrite(&b, 4, 1, F) != 1) return false;
    }
    return true;
  }
  template <class A> static bool CheckFieldSizes(FILE *F) {
    for (size_t i = 0; i < A::NumFields; ++i) {
      uint32_t b = 0;
      if (std::fread(&b, 4, 1, F) != 1 || b != A::field_bytes(i)) return false;
    }
    return true;
  }

  static void plx_check(int rc, const char *what) {
    if (rc) throw std::runtime_error(std::string(what) + ": " + plx_last_error());
  }
  plx_ctx *PlxCtx() {
    if (!Ctx) plx_check(plx_ctx_create(Device, Stream, &Ctx), "plx_ctx_create");
    return Ctx;
  }
  // Grow-only device scratch buffer `slot` of at least `count` elements.
  template <class T> T *Buf(int slot, size_t count) {
    const size_t bytes = std::max<size_t>(count, 1) * sizeof(T);
    if (ScratchBytes[slot] < bytes) {
      cuda_check(cudaStreamSynchronize(Stream), "scratch");
      if (Scratch[slot]) cudaFree(Scratch[slot]);
      cuda_check(cudaMalloc(&Scratch[slot], bytes), "scratch");
      ScratchBytes[slot] = bytes;
    }
    return static_cast<T *>(Scratch[slot]);
  }
  void RadixSort(size_t n, const uint32_t *keys, uint32_t *keys_out, uint32_t *perm, uint32_t bits) {
    const size_t sb = plx_radix_sort_scratch_bytes(n);
    plx_check(plx_radix_sort_u32(PlxCtx(), n, keys, keys_out, perm, 0, bits, Buf<uint8_t>(12, sb),
                                 sb),
              "plx_radix_sort_u32");
  }
  static uint32_t BitsFor(size_t n) {
    uint32_t b = 1;
    while (b < 32 && (size_t(1) << b) < n) ++b;
    return b;
  }

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
  // Field positions of the core schema (detail::UnitAllocT / ConnAllocT).
  uint16_t *LevelPtr() const { return static_cast<uint16_t *>(d_uf[4]); }
  uint32_t *FromPtr() const { return static_cast<uint32_t *>(d_cf[0]); }
  uint32_t *ToPtr() const { return static_cast<uint32_t *>(d_cf[1]); }
  uint8_t *DeadPtr() const { return static_cast<uint8_t *>(d_cf[2]); }
  uint16_t *SrcLevelPtr() const { return static_cast<uint16_t *>(d_cf[3]); }

  // SortConnectionsByLevel (reference plastix.hpp:539-579) on the device:
  // RecomputeLevels, SrcLevel = Level[FromId], stable radix sort on the
  // 16-bit key, Gather of every connection field; NumLevels = highest
  // SrcLevel + 1.
  void SortConnectionsByLevel() {
    SyncToDevice();
    const size_t n = UA.Size(), m = CA.Size();
    plx_ctx *ctx = PlxCtx();
    const size_t lb = plx_recompute_levels_scratch_bytes(n, m);
    plx_check(plx_recompute_levels(ctx, (uint32_t)n, (uint32_t)NumInput, m, FromPtr(), ToPtr(),
                                   DeadPtr(), LevelPtr(), nullptr, Buf<uint8_t>(13, lb), lb),
              "plx_recompute_levels");
    NeedsResort = false;
    if (m == 0) {
      NumLevels = 0;
      return;
    }
    plx_check(plx_src_levels(ctx, m, FromPtr(), LevelPtr(), (uint32_t)n, SrcLevelPtr()),
              "plx_src_levels");
    uint32_t *keys = Buf<uint32_t>(1, m), *keys_out = Buf<uint32_t>(2, m);
    uint32_t *perm = Buf<uint32_t>(3, m);
    detail::k_widen_u16<<<detail::blocks(m), 256, 0, Stream>>>(SrcLevelPtr(), m, keys);
    RadixSort(m, keys, keys_out, perm, 16);
    std::vector<plx_field> f(ConnAllocator::NumFields);
    std::vector<void *> fresh(ConnAllocator::NumFields);
    for (size_t i = 0; i < ConnAllocator::NumFields; ++i) {
      const size_t fb = ConnAllocator::field_bytes(i);
      if (fb != 1 && fb != 2 && fb != 4 && fb != 8)
        throw std::runtime_error("connection fields must be 1, 2, 4 or 8 bytes to be re-sorted");
      cuda_check(cudaMalloc(&fresh[i], std::max<size_t>(1, m) * fb), "field");
      f[i] = plx_field{d_cf[i], fresh[i], (uint32_t)fb, 0};
    }
    plx_check(plx_gather(ctx, m, perm, f.data(), (uint32_t)f.size()), "plx_gather");
    uint32_t last = 0;
    cuda_check(cudaMemcpyAsync(&last, keys_out + m - 1, 4, cudaMemcpyDeviceToHost, Stream),
               "levels");
    cuda_check(cudaStreamSynchronize(Stream), "levels");
    for (size_t i = 0; i < ConnAllocator::NumFields; ++i) {
      cudaFree(d_cf[i]);
      d_cf[i] = fresh[i];
    }
    NumLevels = (int)(last & 0xFFFFu) + 1;
    IndexStale = true;
  }

  // Incoming connection lists per destination (stored order) and outgoing per
  // source (ascending index), as CSR arrays on the device: stable radix sorts
  // of ToId and FromId, row offsets from the sorted keys.
  void RebuildIndex() {
    const size_t n = UA.Size(), m = CA.Size();
    for (uint32_t *p : {d_in_ptr, d_out_ptr, d_in_conn, d_out_conn, d_cursor})
      if (p) cudaFree(p);
    cuda_check(cudaMalloc(&d_in_ptr, (n + 1) * 4), "index");
    cuda_check(cudaMalloc(&d_out_ptr, (n + 1) * 4), "index");
    cuda_check(cudaMalloc(&d_in_conn, std::max<size_t>(1, m) * 4), "index");
    cuda_check(cudaMalloc(&d_out_conn, std::max<size_t>(1, m) * 4), "index");
    cuda_check(cudaMalloc(&d_cursor, std::max<size_t>(1, n) * 4), "index");
    IndexStale = false;
    if (m == 0) {
      cuda_check(cudaMemsetAsync(d_in_ptr, 0, (n + 1) * 4, Stream), "index");
      cuda_check(cudaMemsetAsync(d_out_ptr, 0, (n + 1) * 4, Stream), "index");
      return;
    }
    plx_ctx *ctx = PlxCtx();
    uint32_t *keys_out = Buf<uint32_t>(2, m);
    const uint32_t bits = BitsFor(n);
    RadixSort(m, ToPtr(), keys_out, d_in_conn, bits);
    plx_check(plx_csr_row_ptr(ctx, keys_out, m, 0, (uint32_t)n, d_in_ptr), "plx_csr_row_ptr");
    RadixSort(m, FromPtr(), keys_out, d_out_conn, bits);
    plx_check(plx_csr_row_ptr(ctx, keys_out, m, 0, (uint32_t)n, d_out_ptr), "plx_csr_row_ptr");
  }

  // Appends k zeroed connections (device arrays and the host copy's size).
  void GrowConnections(size_t k) {
    const size_t m = CA.Size();
    for (size_t i = 0; i < ConnAllocator::NumFields; ++i) {
      const size_t fb = ConnAllocator::field_bytes(i);
      void *p = nullptr;
      cuda_check(cudaMalloc(&p, (m + k) * fb), "field");
      if (m)
        cuda_check(cudaMemcpyAsync(p, d_cf[i], m * fb, cudaMemcpyDeviceToDevice, Stream), "field");
      cuda_check(cudaMemsetAsync(static_cast<char *>(p) + m * fb, 0, k * fb, Stream), "field");
      cuda_check(cudaStreamSynchronize(Stream), "field");
      cudaFree(d_cf[i]);
      d_cf[i] = p;
    }
    for (size_t i = 0; i < k; ++i) CA.Allocate();
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
    if (Stream) cudaStreamSynchronize(Stream);
    else cudaDeviceSynchronize();
    for (void *p : d_uf) cudaFree(p);
    for (void *p : d_cf) cudaFree(p);
    for (void *p : {(void *)d_g, (void *)d_in_ptr, (void *)d_out_ptr, (void *)d_in_conn,
                    (void *)d_out_conn, (void *)d_cursor, (void *)d_targets})
      if (p) cudaFree(p);
    for (void *p : Scratch)
      if (p) cudaFree(p);
    if (Ctx) plx_ctx_destroy(Ctx);
  }

  size_t NumInput;
  UnitRange OutputRange;
  UnitAllocator UA;
  ConnAllocator CA;
  int NumLevels = 0;
  size_t Step = 0;
  int Device = 0;
  std::vector<void *> d_uf, d_cf;
  GlobalState *d_g = nullptr;
  uint32_t *d_in_ptr = nullptr, *d_out_ptr = nullptr, *d_in_conn = nullptr, *d_out_conn = nullptr;
  uint32_t *d_cursor = nullptr;
  float *d_targets = nullptr;
  size_t TargetCap = 0;
  bool UnitDirty = false, ConnDirty = false;
  bool NeedsResort = false, IndexStale = true;
  uint64_t ProposalCap = uint64_t(1) << 26;
  cudaStream_t Stream = nullptr;
  plx_ctx *Ctx = nullptr;
  void *Scratch[16] = {};
  size_t ScratchBytes[16] = {};
  std::vector<float> Output;
};

}  // namespace plastix
