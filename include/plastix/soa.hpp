// plastix/soa.hpp -- code generation for structure-of-arrays entity types,
// the reference's include/plastix/soa.hpp interface: a schema written once as
//
//   SOA_TYPE(Name)  FIELD(Field, Type) ...  SOA_END()
//
// is expanded by including this header (deliberately without an include
// guard) in one of three modes, selected by defining exactly one macro before
// the include (the header consumes it):
//
//   PLASTIX_SOA_MODE_TAGS    struct Name {}; using NameId = AllocId<Name>;
//                            and an empty tag struct FieldTag per field;
//   PLASTIX_SOA_MODE_ALLOC   using NameAllocator =
//                                SOAAllocator<Name, SOAField<FieldTag, Type>...>;
//   PLASTIX_SOA_MODE_HANDLE  struct NameHandle, a thin id wrapper convertible
//                            to and from NameId, with Type &GetField(NameAllocator&)
//                            per field.
//
// The generated names and shapes are the reference's, so schemas written for
// it compile unchanged; the allocator behind them is plastix/alloc.hpp.
#include "plastix/alloc.hpp"

#undef SOA_TYPE
#undef FIELD
#undef SOA_END

#if defined(PLASTIX_SOA_MODE_TAGS)
#undef PLASTIX_SOA_MODE_TAGS

#define SOA_TYPE(Name)                                                                  \
  struct Name {};                                                                       \
  using Name##Id = ::plastix::alloc::AllocId<Name>;
#define FIELD(Name, Type) \
  struct Name##Tag {};
#define SOA_END()

#elif defined(PLASTIX_SOA_MODE_ALLOC)
#undef PLASTIX_SOA_MODE_ALLOC

#define SOA_TYPE(Name) using Name##Allocator = ::plastix::alloc::SOAAllocator<Name
#define FIELD(Name, Type) , ::plastix::alloc::SOAField<Name##Tag, Type>
#define SOA_END() >;

#elif defined(PLASTIX_SOA_MODE_HANDLE)
#undef PLASTIX_SOA_MODE_HANDLE

#define SOA_TYPE(Name)                                                                  \
  struct Name##Handle {                                                                 \
    using Alloc_ = Name##Allocator;                                                     \
    ::plastix::alloc::AllocId<Name> Id;                                                 \
    Name##Handle(::plastix::alloc::AllocId<Name> I) : Id(I) {}                          \
    operator ::plastix::alloc::AllocId<Name>() const { return Id; }
#define FIELD(Name, Type) \
  Type &Get##Name(Alloc_ &A) { return A.template Get<Name##Tag>(Id); }
#define SOA_END() \
  };

#endif
