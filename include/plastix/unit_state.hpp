// plastix/unit_state.hpp -- the unit schema (the reference's
// include/plastix/unit_state.hpp): the core fields every unit allocator has
// (Activation f32, ForwardAcc, BackwardAcc of the passes' accumulator types,
// Pruned bool, Level u16, in that order), their accessors, and the allocator
// aliases built from a UnitFieldList of extra fields.
#pragma once

#include <cstdint>

#include "plastix/alloc.hpp"

namespace plastix {

struct UnitState {};
using UnitStateId = alloc::AllocId<UnitState>;

struct ActivationTag {};
struct ForwardAccTag {};
struct BackwardAccTag {};
struct PrunedTag {};
struct LevelTag {};

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

template <typename FwdAcc, typename BwdAcc, typename... ExtraFields>
using MakeUnitAllocator =
    alloc::SOAAllocator<UnitState, alloc::SOAField<ActivationTag, float>,
                        alloc::SOAField<ForwardAccTag, FwdAcc>,
                        alloc::SOAField<BackwardAccTag, BwdAcc>, alloc::SOAField<PrunedTag, bool>,
                        alloc::SOAField<LevelTag, uint16_t>, ExtraFields...>;

template <typename FwdAcc, typename BwdAcc, typename FL> struct MakeUnitAllocatorFromList;
template <typename FwdAcc, typename BwdAcc, typename... Extra>
struct MakeUnitAllocatorFromList<FwdAcc, BwdAcc, UnitFieldList<Extra...>> {
  using type = MakeUnitAllocator<FwdAcc, BwdAcc, Extra...>;
};
template <typename FwdAcc, typename BwdAcc, typename FL>
using MakeUnitAllocatorFrom = typename MakeUnitAllocatorFromList<FwdAcc, BwdAcc, FL>::type;

using UnitStateAllocator = MakeUnitAllocator<float, float>;

// Positions of the core fields in every unit allocator.
namespace core {
inline constexpr size_t kActivation = 0, kForwardAcc = 1, kBackwardAcc = 2, kPruned = 3,
                        kLevel = 4;
}

}  // namespace plastix
