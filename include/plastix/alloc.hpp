// plastix/alloc.hpp -- structure-of-arrays storage (the reference's
// include/plastix/alloc.hpp API: SOAField, SOAAllocator, GetField).
//
// SOAAllocator keeps one contiguous host array per field, with the
// reference's semantics: a fixed capacity given at construction, Allocate /
// AllocateMany returning size_t(-1) when it is exhausted, value-initialised
// new entities, Get<Tag>(Id), GetArrayFor<Tag>(), PermutationScratch() and
// Gather(N) (dst[i] = src[perm[i]] for i < N into the second copy of every
// field, then the two copies swap, alloc.hpp:145-156 of the reference).
//
// Differences a user sees:
//   * Arrays grow on demand (up to the capacity) instead of being mapped at
//     construction, so a reference obtained from Get() is valid until the
//     next Allocate/AllocateMany, like an element of a std::vector.
//   * An allocator that belongs to a device Network is a coherent host
//     mirror of the device copy: reading a field the device has changed
//     downloads it first, and a field touched through a non-const Get or
//     GetArrayFor is uploaded before the Network's next device step.
//     Standalone allocators are plain host storage.
//   * SOAView is the device-side accessor: the same Get<Tag>(Id) surface over
//     device pointers, which is what policies receive inside kernels.
#pragma once

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <new>
#include <tuple>
#include <type_traits>
#include <utility>

#if defined(__CUDACC__)
#define PLASTIX_HD __host__ __device__
// Accessor templates serve device views (device code) and host allocators
// (host code); the execution-space check is lifted for them because each
// instantiation is only ever called where its Get exists.
#define PLASTIX_NO_EXEC_CHECK _Pragma("nv_exec_check_disable")
#else
#define PLASTIX_HD
#define PLASTIX_NO_EXEC_CHECK
#endif

namespace plastix {
namespace alloc {

template <typename T> using AllocId = size_t;

template <typename FieldTag, typename T> struct SOAField {
  static_assert(std::is_class_v<FieldTag> && std::is_empty_v<FieldTag>,
                "a field tag is an empty marker type; the stored type is the second argument");
  using Tag = FieldTag;
  using Type = T;
};

// Position of Tag among the fields (== number of fields when absent).
template <typename Tag, typename... Fs> struct FieldIndex;
template <typename Tag, typename F, typename... Fs> struct FieldIndex<Tag, F, Fs...> {
  static constexpr size_t value =
      std::is_same_v<Tag, typename F::Tag> ? 0 : 1 + FieldIndex<Tag, Fs...>::value;
};
template <typename Tag> struct FieldIndex<Tag> {
  static constexpr size_t value = 0;
};

template <size_t I, typename... Fs>
using FieldType = typename std::tuple_element_t<I, std::tuple<Fs...>>::Type;

// Device-side accessor: one pointer per field (device memory), the count.
template <typename... Fs> struct SOAView {
  void *ptr[sizeof...(Fs) > 0 ? sizeof...(Fs) : 1];
  size_t size;

  template <typename Tag> PLASTIX_HD auto &Get(size_t Id) const {
    constexpr size_t I = FieldIndex<Tag, Fs...>::value;
    static_assert(I < sizeof...(Fs), "no such field");
    return static_cast<FieldType<I, Fs...> *>(ptr[I])[Id];
  }
  PLASTIX_HD auto &Get(size_t Id) const
    requires(sizeof...(Fs) == 1)
  {
    return static_cast<FieldType<0, Fs...> *>(ptr[0])[Id];
  }
  template <typename Tag> PLASTIX_HD auto *GetArrayFor() const {
    constexpr size_t I = FieldIndex<Tag, Fs...>::value;
    static_assert(I < sizeof...(Fs), "no such field");
    return static_cast<FieldType<I, Fs...> *>(ptr[I]);
  }
  PLASTIX_HD size_t Size() const { return size; }
};

// Hooks through which a device Network keeps an allocator coherent:
// `fetch(owner, field)` downloads one field into the host array.
struct MirrorLink {
  void (*fetch)(void *owner, size_t field) = nullptr;
  void *owner = nullptr;
};

namespace detail {
// Contiguous, value-initialised, growable array (no std::vector<bool>).
template <typename T> class Column {
 public:
  Column() = default;
  Column(const Column &) = delete;
  Column &operator=(const Column &) = delete;
  ~Column() { std::free(data_); }
  T *data() { return data_; }
  const T *data() const { return data_; }
  size_t size() const { return size_; }
  // Grows to n entities; new ones are value-initialised.
  void resize(size_t n) {
    if (n > cap_) {
      size_t c = std::max<size_t>(cap_ ? cap_ : 16, 16);
      while (c < n) c *= 2;
      T *p = static_cast<T *>(std::malloc(c * sizeof(T)));
      if (!p) throw std::bad_alloc();
      if (size_) std::memcpy(static_cast<void *>(p), data_, size_ * sizeof(T));
      std::free(data_);
      data_ = p;
      cap_ = c;
    }
    for (size_t i = size_; i < n; ++i) ::new (static_cast<void *>(data_ + i)) T();
    size_ = n;
  }
  void swap(Column &o) {
    std::swap(data_, o.data_);
    std::swap(size_, o.size_);
    std::swap(cap_, o.cap_);
  }

 private:
  T *data_ = nullptr;
  size_t size_ = 0, cap_ = 0;
};
}  // namespace detail

template <typename T, typename... Fields> class SOAAllocator {
  static_assert((std::is_trivially_copyable_v<typename Fields::Type> && ...),
                "fields are copied between host and device byte for byte");
  static_assert(sizeof...(Fields) <= 64, "at most 64 fields");

 public:
  using Entity = T;
  using View = SOAView<Fields...>;
  static constexpr size_t NumFields = sizeof...(Fields);
  template <size_t I> using FieldTypeAt = FieldType<I, Fields...>;

  explicit SOAAllocator(size_t NumElements) : Capacity(NumElements) {}
  SOAAllocator(const SOAAllocator &) = delete;
  SOAAllocator &operator=(const SOAAllocator &) = delete;

  template <typename FieldTag> constexpr static size_t IndexOf() {
    return FieldIndex<FieldTag, Fields...>::value;
  }

  AllocId<T> Allocate() {
    if (Count >= Capacity) return static_cast<size_t>(-1);
    Grow(Count + 1);
    return Count++;
  }

  std::pair<size_t, size_t> AllocateMany(size_t N) {
    if (N > Capacity || Count > Capacity - N)
      return {static_cast<size_t>(-1), static_cast<size_t>(-1)};
    const size_t Begin = Count;
    Grow(Count + N);
    Count += N;
    return {Begin, Begin + N};
  }

  template <typename FieldTag> auto &Get(AllocId<T> Id) {
    constexpr size_t I = IndexOf<FieldTag>();
    static_assert(I < NumFields, "no such field");
    Touch(I);
    return std::get<I>(Front).data()[Id];
  }
  template <typename FieldTag> const auto &Get(AllocId<T> Id) const {
    constexpr size_t I = IndexOf<FieldTag>();
    static_assert(I < NumFields, "no such field");
    Fresh(I);
    return std::get<I>(Front).data()[Id];
  }
  auto &Get(AllocId<T> Id)
    requires(sizeof...(Fields) == 1)
  {
    Touch(0);
    return std::get<0>(Front).data()[Id];
  }
  const auto &Get(AllocId<T> Id) const
    requires(sizeof...(Fields) == 1)
  {
    Fresh(0);
    return std::get<0>(Front).data()[Id];
  }

  template <typename FieldTag> auto *GetArrayFor() {
    constexpr size_t I = IndexOf<FieldTag>();
    static_assert(I < NumFields, "no such field");
    Touch(I);
    return std::get<I>(Front).data();
  }
  template <typename FieldTag> const auto *GetArrayFor() const {
    constexpr size_t I = IndexOf<FieldTag>();
    static_assert(I < NumFields, "no such field");
    Fresh(I);
    return std::get<I>(Front).data();
  }

  size_t Size() const { return Count; }
  size_t GetCapacity() const { return Capacity; }

  // Scratch for Gather: at least Size() entries (all of the capacity for
  // capacities up to 2^20, as the reference's arena).
  size_t *PermutationScratch() {
    const size_t want = Capacity <= (size_t(1) << 20) ? Capacity : Count;
    if (Perm.size() < want) Perm.resize(want);
    return Perm.data();
  }

  // dst[i] = src[perm[i]] for i < N (perm from PermutationScratch) into the
  // second copy of every field, then the two copies swap.
  void Gather(size_t N) {
    FetchAll();
    gather(N, std::index_sequence_for<Fields...>{});
    MarkAllDirty();
  }

  // ---- raw access for the device mirror (no coherence hooks) --------------
  void *field_data(size_t I) { return data_ptr(I, std::index_sequence_for<Fields...>{}); }
  static constexpr size_t field_bytes(size_t I) {
    constexpr size_t B[] = {sizeof(typename Fields::Type)...};
    return B[I];
  }
  // Sets the number of entities (new ones value-initialised); the capacity
  // grows with it if needed.
  void Resize(size_t N) {
    Capacity = std::max(Capacity, N);
    Grow(N);
    Count = N;
  }
  void SetCapacity(size_t N) { Capacity = std::max(N, Count); }
  void Link(MirrorLink L) { Mirror = L; }
  uint64_t StaleMask() const { return Stale; }
  uint64_t DirtyMask() const { return Dirty; }
  void MarkStale(uint64_t Mask) { Stale |= Mask; }
  void ClearStale(size_t I) { Stale &= ~(uint64_t(1) << I); }
  void ClearAllStale() { Stale = 0; }
  void ClearDirty() { Dirty = 0; }
  void MarkAllDirty() { Dirty |= AllFields(); }
  static constexpr uint64_t AllFields() {
    return NumFields >= 64 ? ~uint64_t(0) : (uint64_t(1) << NumFields) - 1;
  }
  // Downloads every stale field (a host pass over the whole allocator).
  void FetchAll() const {
    for (size_t I = 0; I < NumFields; ++I) Fresh(I);
  }

 private:
  void Fresh(size_t I) const {
    if ((Stale >> I) & 1u) {
      if (Mirror.fetch) Mirror.fetch(Mirror.owner, I);
      Stale &= ~(uint64_t(1) << I);
    }
  }
  void Touch(size_t I) {
    Fresh(I);
    Dirty |= uint64_t(1) << I;
  }
  void Grow(size_t N) {
    std::apply([N](auto &...C) { (C.resize(N), ...); }, Front);
    if (HasBack) std::apply([N](auto &...C) { (C.resize(N), ...); }, Back);
  }
  template <size_t... Is> void *data_ptr(size_t I, std::index_sequence<Is...>) {
    void *p = nullptr;
    ((I == Is ? (p = static_cast<void *>(std::get<Is>(Front).data()), 0) : 0), ...);
    return p;
  }
  template <size_t... Is> void gather(size_t N, std::index_sequence<Is...>) {
    if (!HasBack) {
      HasBack = true;
      std::apply([this](auto &...C) { (C.resize(Count), ...); }, Back);
    }
    const size_t *P = PermutationScratch();
    ((gather_one(std::get<Is>(Front), std::get<Is>(Back), P, N)), ...);
    ((std::get<Is>(Front).swap(std::get<Is>(Back))), ...);
  }
  template <typename Col> static void gather_one(Col &Src, Col &Dst, const size_t *P, size_t N) {
    if (Dst.size() < N) Dst.resize(N);
    for (size_t I = 0; I < N; ++I) Dst.data()[I] = Src.data()[P[I]];
  }

  std::tuple<detail::Column<typename Fields::Type>...> Front, Back;
  detail::Column<size_t> Perm;
  size_t Count = 0;
  size_t Capacity;
  bool HasBack = false;
  MirrorLink Mirror;
  mutable uint64_t Stale = 0;
  uint64_t Dirty = 0;
};

}  // namespace alloc

// Alloc.template Get<Tag>(Id), on a host allocator or a device view.
PLASTIX_NO_EXEC_CHECK
template <typename Tag> PLASTIX_HD constexpr auto &GetField(auto &Alloc, size_t Id) {
  return Alloc.template Get<Tag>(Id);
}

}  // namespace plastix
