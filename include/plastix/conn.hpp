// plastix/conn.hpp -- the connection schema (the reference's
// include/plastix/conn.hpp): the core fields every connection allocator has
// (FromId u32, ToId u32, Dead bool, SrcLevel u16, in that order), the common
// Weight tag, and the allocator aliases built from a ConnFieldList of extra
// fields.
#pragma once

#include <cstdint>

#include "plastix/alloc.hpp"

namespace plastix {

struct ConnectionState {};
using ConnStateId = alloc::AllocId<ConnectionState>;

struct FromIdTag {};
struct ToIdTag {};
struct DeadTag {};
struct SrcLevelTag {};
struct WeightTag {};
// The eligibility trace of HebbianTraceUpdate (traits.hpp); not a core field.
struct TraceTag {};

PLASTIX_NO_EXEC_CHECK
PLASTIX_HD constexpr auto &GetWeight(auto &Alloc, size_t Id) {
  return GetField<WeightTag>(Alloc, Id);
}

template <typename... Fields> struct ConnFieldList {};

template <typename... ExtraFields>
using MakeConnAllocator =
    alloc::SOAAllocator<ConnectionState, alloc::SOAField<FromIdTag, uint32_t>,
                        alloc::SOAField<ToIdTag, uint32_t>, alloc::SOAField<DeadTag, bool>,
                        alloc::SOAField<SrcLevelTag, uint16_t>, ExtraFields...>;

template <typename FL> struct MakeConnAllocatorFromList;
template <typename... Extra> struct MakeConnAllocatorFromList<ConnFieldList<Extra...>> {
  using type = MakeConnAllocator<Extra...>;
};
template <typename FL> using MakeConnAllocatorFrom = typename MakeConnAllocatorFromList<FL>::type;

using ConnStateAllocator = MakeConnAllocator<alloc::SOAField<WeightTag, float>>;

// Positions of the core fields in every connection allocator.
namespace core {
inline constexpr size_t kFromId = 0, kToId = 1, kDead = 2, kSrcLevel = 3;
}

}  // namespace plastix
