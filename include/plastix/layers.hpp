// plastix/layers.hpp -- unit ranges and layer builders (the reference's
// include/plastix/layers.hpp). Builders run on the host at construction,
// writing the host copies of the allocators; FullyConnected emits the
// destination-major connection order (for each new unit, one connection
// from every unit of the previous layer) that the sweeps rely on.
#pragma once

#include <concepts>
#include <cstddef>
#include <cstdint>
#include <random>
#include <ranges>
#include <utility>

#include "plastix/conn.hpp"
#include "plastix/unit_state.hpp"

namespace plastix {

struct UnitRange {
  size_t Begin;
  size_t End;
  UnitRange() = default;
  PLASTIX_HD UnitRange(size_t B, size_t E) : Begin(B), End(E) {}
  UnitRange(std::pair<size_t, size_t> P) : Begin(P.first), End(P.second) {}
  PLASTIX_HD size_t Size() const { return End - Begin; }
  auto Ids() const { return std::views::iota(Begin, End); }
};

template <typename B, typename UA, typename CA>
concept LayerBuilder = requires(B Builder, UA &U, CA &C, UnitRange R) {
  { Builder(U, C, R) } -> std::same_as<UnitRange>;
};

struct NoUnitInit {
  void operator()(auto &, auto) const {}
};
struct NoConnInit {
  void operator()(auto &, auto) const {}
};

// Weights drawn U(Min, Max) from a std::mt19937 seeded with Seed, one draw
// per connection in allocation order (the stream the reference's examples
// are pinned to).
struct RandomUniformWeight {
  RandomUniformWeight(uint32_t Seed = 0, float Min = -1.0f, float Max = 1.0f)
      : Rng(Seed), Dist(Min, Max) {}
  void operator()(auto &CA, auto Id) const { GetWeight(CA, Id) = Dist(Rng); }

 private:
  mutable std::mt19937 Rng;
  mutable std::uniform_real_distribution<float> Dist;
};

template <typename ConnInit = NoConnInit, typename UnitInit = NoUnitInit> struct FullyConnected {
  size_t NumUnits;
  ConnInit InitConn = {};
  UnitInit InitUnit = {};

  template <typename UA, typename CA> UnitRange operator()(UA &U, CA &C, UnitRange Prev) const {
    const uint16_t SrcLvl = GetLevel(U, Prev.Begin);
    const UnitRange Units = U.AllocateMany(NumUnits);
    for (size_t Id = Units.Begin; Id < Units.End; ++Id) {
      GetLevel(U, Id) = static_cast<uint16_t>(SrcLvl + 1);
      InitUnit(U, Id);
    }
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
template <typename CI, typename UI> FullyConnected(size_t, CI, UI) -> FullyConnected<CI, UI>;

}  // namespace plastix
