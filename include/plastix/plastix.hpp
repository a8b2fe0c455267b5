// plastix/plastix.hpp -- the Plastix network API (Network<Traits>) on the
// B200: the reference header library's names, policy signatures and step
// order (include/plastix/*.hpp of DhanrajHira/plastix), with the state in
// device memory and every Do* step run by kernels that call the user's
// policies on the GPU. The sub-headers (alloc.hpp, soa.hpp, conn.hpp,
// unit_state.hpp, layers.hpp, traits.hpp) are the reference's too.
//
// Differences a user sees:
//   * Policy member functions run on the device, so they carry PLASTIX_HD
//     (__host__ __device__ under nvcc, nothing otherwise):
//       struct MyMap { PLASTIX_HD static float Map(auto &U, ...) {...} };
//     The translation unit is compiled by nvcc (-std=c++20
//     --expt-relaxed-constexpr, sm_100a) and linked with -lplastix_b200.
//   * Passes fold each unit's connections in the reference's order
//     (Pipeline: connection index order, backward in descending order;
//     Topological: level by level, index order within a level), so every
//     Map/Combine/Apply sees the same sequence of values. Units run in
//     parallel; traits whose global state may be written by the hooks (see
//     ReadOnlyGlobalState in traits.hpp) run every hook that receives it in
//     one device thread, in the reference's order.
//   * Pipeline networks whose connections are stored destination-major (as
//     FullyConnected builds them) take a warp-tiled forward accumulation:
//     Map on consecutive connections per lane (coalesced reads of the
//     connection fields), each unit's values still combined strictly in
//     connection order.
//   * GetUnitAlloc()/GetConnAlloc() return the network's host copies, kept
//     coherent with the device: a field the device has changed is downloaded
//     when the host reads it, and fields the host touched are uploaded before
//     the next Do* step. References obtained from them stay valid across
//     steps, as with the reference.
//   * AddUnit runs on the host (unit growth is host-orchestrated); the new
//     units are uploaded before the next device step. Structural decisions
//     (PruneUnit, AddConn's predicates) run on the host copy by default and
//     on the device with `DeviceStructure` (traits.hpp); proposals are sorted
//     and deduplicated on the device either way, and Topological networks
//     recompute levels and re-sort connections on the device.
//   * No fixed capacity: networks of any size that fit the GPU.
//   * Additions: GetGlobals()/SetGlobals(), Save(path)/Load(path)
//     (checkpoints of every field and the global state), SetStream(),
//     SetProposalCapacity().
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
#include <optional>
#include <random>
#include <span>
#include <stdexcept>
#include <string>
#include <tuple>
#include <type_traits>
#include <utility>
#include <vector>

#include "plastix/alloc.hpp"
#include "plastix/conn.hpp"
#include "plastix/layers.hpp"
#include "plastix/traits.hpp"
#include "plastix/unit_state.hpp"

namespace plastix {

inline const char *version() { return "0.1.0"; }

inline void cuda_check(cudaError_t e, const char *what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Highest unit level + 1 (AddUnit clamps new levels to [1, MaxLevels - 1]).
static constexpr uint16_t MaxLevels = 1024;

struct LevelRange {
  uint32_t Begin;
  uint32_t End;
};

// A proposed connection packed as From | To << 32 (sorted and deduplicated
// by these bits in DoAddConnections).
struct CompactEdge {
  uint64_t Bits;
  PLASTIX_HD CompactEdge() : Bits(0) {}
  PLASTIX_HD CompactEdge(uint32_t From, uint32_t To)
      : Bits(static_cast<uint64_t>(From) | (static_cast<uint64_t>(To) << 32)) {}
  PLASTIX_HD uint32_t From() const { return static_cast<uint32_t>(Bits); }
  PLASTIX_HD uint32_t To() const { return static_cast<uint32_t>(Bits >> 32); }
};

// ---------------------------------------------------------------------------
// Device kernels (templated on the traits; instantiated in the user's TU)
// ---------------------------------------------------------------------------
namespace detail {

template <class T> constexpr bool read_only_globals() {
  if constexpr (requires { T::ReadOnlyGlobalState; }) return T::ReadOnlyGlobalState;
  else return std::is_empty_v<typename T::GlobalState>;
}
template <class T> constexpr bool sequential_conn_update() {
  if constexpr (requires { T::SequentialConnectionUpdate; }) return T::SequentialConnectionUpdate;
  else return !read_only_globals<T>();
}
template <class T> constexpr bool device_structure() {
  if constexpr (requires { T::DeviceStructure; }) return T::DeviceStructure;
  else return false;
}
template <class T> constexpr bool sequential_structure() {
  if constexpr (requires { T::SequentialStructure; }) return T::SequentialStructure;
  else return !read_only_globals<T>();
}

inline unsigned blocks(size_t n) { return (unsigned)std::max<size_t>(1, (n + 255) / 256); }

// ---- passes, one thread per unit ------------------------------------------

// Pipeline forward accumulation: unit I folds its incoming connections in
// index order (in_conn lists them per destination, ascending).
template <class Tr, class UV, class CV, class G>
__device__ __forceinline__ void fwd_acc_unit(UV &U, CV &C, G *g, const uint32_t *in_ptr,
                                             const uint32_t *in_conn, size_t I) {
  using FP = typename Tr::ForwardPass;
  auto acc = GetForwardAcc(U, I);
  for (uint32_t k = in_ptr[I]; k < in_ptr[I + 1]; ++k) {
    const uint32_t c = in_conn[k];
    if (GetField<DeadTag>(C, c)) continue;
    acc = FP::Combine(acc, FP::Map(U, I, GetField<FromIdTag>(C, c), C, c, *g));
  }
  GetForwardAcc(U, I) = acc;
}
template <class Tr, class UV, class CV, class G>
__global__ void k_fwd_acc(UV U, CV C, G *g, const uint32_t *in_ptr, const uint32_t *in_conn,
                          size_t n) {
  const size_t I = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (I < n) fwd_acc_unit<Tr>(U, C, g, in_ptr, in_conn, I);
}

// Pipeline forward accumulation for connections stored destination-major
// (ToId non-decreasing, as FullyConnected and destination-sorted builders
// emit them): units in blocks of 32, one lane per unit; the block's
// connections are evaluated 32 at a time with Map -- consecutive connections
// on consecutive lanes, so connection fields are read coalesced --, staged in
// shared memory, and each lane folds its unit's staged values with Combine
// strictly in connection order (the same sequence as k_fwd_acc).
constexpr uint32_t kTileChunk = 256;  // connections per staged chunk
constexpr uint32_t kTileWarps = 8;
template <class Tr, class UV, class CV, class G>
__global__ void __launch_bounds__(kTileWarps * 32)
    k_fwd_acc_tiled(UV U, CV C, G *g, const uint32_t *in_ptr, size_t n) {
  using FP = typename Tr::ForwardPass;
  using Acc = typename FP::Accumulator;
  __shared__ __align__(16) unsigned char raw[kTileWarps][kTileChunk * sizeof(Acc)];
  __shared__ bool live[kTileWarps][kTileChunk];
  const uint32_t lane = threadIdx.x & 31u, w = threadIdx.x >> 5;
  Acc *stage = reinterpret_cast<Acc *>(raw[w]);
  for (size_t r0 = ((size_t)blockIdx.x * kTileWarps + w) * 32; r0 < n;
       r0 += (size_t)gridDim.x * kTileWarps * 32) {
    const size_t r = r0 + lane;
    const size_t r_end = r0 + 32 < n ? r0 + 32 : n;
    const uint32_t rs = r < n ? in_ptr[r] : 0u, re = r < n ? in_ptr[r + 1] : 0u;
    const uint32_t c_lo = in_ptr[r0], c_hi = in_ptr[r_end];
    Acc acc = r < n ? GetForwardAcc(U, r) : Acc{};
    for (uint32_t c0 = c_lo; c0 < c_hi; c0 += kTileChunk) {
      const uint32_t cn = c_hi - c0 < kTileChunk ? c_hi - c0 : kTileChunk;
      for (uint32_t j = lane; j < cn; j += 32) {
        const size_t c = (size_t)c0 + j;
        const bool ok = !GetField<DeadTag>(C, c);
        live[w][j] = ok;
        if (ok) stage[j] = FP::Map(U, GetField<ToIdTag>(C, c), GetField<FromIdTag>(C, c), C, c, *g);
      }
      __syncwarp();
      const uint32_t lo = rs > c0 ? rs : c0, hi = re < c0 + cn ? re : c0 + cn;
      for (uint32_t c = lo; c < hi; ++c)
        if (live[w][c - c0]) acc = FP::Combine(acc, stage[c - c0]);
      __syncwarp();
    }
    if (r < n) GetForwardAcc(U, r) = acc;
  }
}

// Topological forward accumulation of level L (reference plastix.hpp:111-119):
// every unit folds, in stored order, those incoming connections whose
// SrcLevel is L - 1. Connections are sorted by SrcLevel, so each unit's
// incoming list is too; `cur` is the unit's position in it.
template <class Tr, class UV, class CV, class G>
__device__ __forceinline__ void fwd_acc_level_unit(UV &U, CV &C, G *g, const uint32_t *in_ptr,
                                                   const uint32_t *in_conn, uint32_t *cur,
                                                   size_t I, int L) {
  using FP = typename Tr::ForwardPass;
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
template <class Tr, class UV, class CV, class G>
__global__ void k_fwd_acc_level(UV U, CV C, G *g, const uint32_t *in_ptr, const uint32_t *in_conn,
                                uint32_t *cur, size_t n, int L) {
  const size_t I = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (I < n) fwd_acc_level_unit<Tr>(U, C, g, in_ptr, in_conn, cur, I, L);
}

// Apply of the units in [lo, hi) (only those at level `lvl` when lvl >= 0),
// then the accumulator is reset. With `mse` (the targets of the output units
// [out_lo, out_hi)), MSELoss runs in the same thread right after an output
// unit's Apply: BackwardAcc = pred - target (traits.hpp MSELoss, the
// reference's DoCalculateLoss after DoForwardPass -- an output unit's
// activation is final once its Apply has run).
template <class Tr, class UV, class G>
__device__ __forceinline__ void fwd_apply_unit(UV &U, G *g, size_t I, int lvl, const float *mse,
                                               size_t out_lo, size_t out_hi) {
  using FP = typename Tr::ForwardPass;
  using Acc = typename FP::Accumulator;
  if (lvl >= 0 && GetLevel(U, I) != lvl) return;
  FP::Apply(U, I, *g, GetForwardAcc(U, I));
  GetForwardAcc(U, I) = Acc{};
  if (mse && I >= out_lo && I < out_hi) GetBackwardAcc(U, I) = GetActivation(U, I) - mse[I - out_lo];
}
template <class Tr, class UV, class G>
__global__ void k_fwd_apply(UV U, G *g, size_t lo, size_t hi, int lvl, const float *mse,
                            size_t out_lo, size_t out_hi) {
  const size_t I = lo + blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (I < hi) fwd_apply_unit<Tr>(U, g, I, lvl, mse, out_lo, out_hi);
}

// MSELoss over the output units, one thread per unit (the loss is
// elementwise, so this equals the reference's loop bit for bit).
template <class UV>
__global__ void k_loss_mse(UV U, size_t out_lo, size_t out_n, const float *t) {
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < out_n) GetBackwardAcc(U, out_lo + i) = GetActivation(U, out_lo + i) - t[i];
}

// Backward accumulation: unit I folds its outgoing connections into its
// BackwardAcc -- descending index order (Pipeline, plastix.hpp:193), or, for
// Topological level L, ascending over those whose SrcLevel is L
// (plastix.hpp:170-181).
template <class Tr, class UV, class CV, class G>
__device__ __forceinline__ void bwd_acc_unit(UV &U, CV &C, G *g, const uint32_t *out_ptr,
                                             const uint32_t *out_conn, size_t I, int L) {
  using BP = typename Tr::BackwardPass;
  const uint32_t b = out_ptr[I], e = out_ptr[I + 1];
  if (b == e) return;
  auto acc = GetBackwardAcc(U, I);
  for (uint32_t j = 0; j < e - b; ++j) {
    const uint32_t c = out_conn[L < 0 ? e - 1 - j : b + j];
    if (GetField<DeadTag>(C, c)) continue;
    if (L >= 0 && GetField<SrcLevelTag>(C, c) != (uint16_t)L) continue;
    acc = BP::Combine(acc, BP::Map(U, I, GetField<ToIdTag>(C, c), C, c, *g));
  }
  GetBackwardAcc(U, I) = acc;
}
template <class Tr, class UV, class CV, class G>
__global__ void k_bwd_acc(UV U, CV C, G *g, const uint32_t *out_ptr, const uint32_t *out_conn,
                          size_t n, int L) {
  const size_t I = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (I < n) bwd_acc_unit<Tr>(U, C, g, out_ptr, out_conn, I, L);
}

template <class Tr, class UV, class G>
__device__ __forceinline__ void bwd_apply_unit(UV &U, G *g, size_t I, int lvl) {
  using BP = typename Tr::BackwardPass;
  using Acc = typename BP::Accumulator;
  if (lvl >= 0 && GetLevel(U, I) != lvl) return;
  BP::Apply(U, I, *g, GetBackwardAcc(U, I));
  GetBackwardAcc(U, I) = Acc{};
}
template <class Tr, class UV, class G>
__global__ void k_bwd_apply(UV U, G *g, size_t lo, size_t hi, int lvl) {
  const size_t I = lo + blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (I < hi) bwd_apply_unit<Tr>(U, g, I, lvl);
}

// ---- passes in one thread: the reference's loops verbatim in order ---------
// (hooks that may write the global state). `ranges[L]` is the first
// connection whose SrcLevel is >= L (Topological, after the level sort).
template <class Tr, class UV, class CV, class G>
__global__ void k_fwd_seq(UV U, CV C, G *g, size_t n_input, size_t n, size_t m,
                          const uint32_t *ranges, int levels, bool topo) {
  using FP = typename Tr::ForwardPass;
  using Acc = typename FP::Accumulator;
  auto fold = [&](size_t c) {
    if (GetField<DeadTag>(C, c)) return;
    const size_t To = GetField<ToIdTag>(C, c), From = GetField<FromIdTag>(C, c);
    auto &A = GetForwardAcc(U, To);
    A = FP::Combine(A, FP::Map(U, To, From, C, c, *g));
  };
  if (topo) {
    for (int L = 1; L <= levels; ++L) {
      for (size_t c = ranges[L - 1]; c < ranges[L]; ++c) fold(c);
      for (size_t I = n_input; I < n; ++I)
        if (GetLevel(U, I) == L) {
          FP::Apply(U, I, *g, GetForwardAcc(U, I));
          GetForwardAcc(U, I) = Acc{};
        }
    }
  } else {
    for (size_t c = 0; c < m; ++c) fold(c);
    for (size_t I = n_input; I < n; ++I) {
      FP::Apply(U, I, *g, GetForwardAcc(U, I));
      GetForwardAcc(U, I) = Acc{};
    }
  }
}

template <class Tr, class UV, class CV, class G>
__global__ void k_bwd_seq(UV U, CV C, G *g, size_t n_input, size_t n, size_t m,
                          const uint32_t *ranges, int levels, bool topo) {
  using BP = typename Tr::BackwardPass;
  using Acc = typename BP::Accumulator;
  auto fold = [&](size_t c) {
    if (GetField<DeadTag>(C, c)) return;
    const size_t To = GetField<ToIdTag>(C, c), From = GetField<FromIdTag>(C, c);
    auto &A = GetBackwardAcc(U, From);
    A = BP::Combine(A, BP::Map(U, From, To, C, c, *g));
  };
  if (topo) {
    for (int L = levels; L >= 1; --L) {
      for (size_t c = ranges[L]; c < ranges[L + 1]; ++c) fold(c);
      for (size_t I = n_input; I < n; ++I)
        if (GetLevel(U, I) == L) {
          BP::Apply(U, I, *g, GetBackwardAcc(U, I));
          GetBackwardAcc(U, I) = Acc{};
        }
    }
  } else {
    for (size_t c = m; c-- > 0;) fold(c);
    for (size_t I = 0; I < n; ++I) {
      BP::Apply(U, I, *g, GetBackwardAcc(U, I));
      GetBackwardAcc(U, I) = Acc{};
    }
  }
}

template <class Tr, class UV, class G>
__global__ void k_loss(UV U, G *g, UnitRange out, const float *t, size_t nt) {
  Tr::Loss::CalculateLoss(U, out, std::span<const float>(t, nt), *g);
}

template <class Tr, class UV, class G>
__global__ void k_update_unit(UV U, G *g, size_t n, bool seq) {
  const size_t first = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t step = seq ? 1 : (size_t)gridDim.x * blockDim.x;
  if (seq && first != 0) return;
  for (size_t I = first; I < n; I += step) Tr::UpdateUnit::Update(U, I, *g);
}

// Per-connection update: parallel over connections, or one thread in index
// order for sequential semantics.
template <class Tr, bool Incoming, class UV, class CV, class G>
__device__ __forceinline__ void update_conn_one(UV &U, CV &C, G *g, size_t c) {
  using UP = typename Tr::UpdateConn;
  if (GetField<DeadTag>(C, c)) return;
  const size_t to = GetField<ToIdTag>(C, c), from = GetField<FromIdTag>(C, c);
  if constexpr (Incoming) UP::UpdateIncomingConnection(U, to, from, C, c, *g);
  else UP::UpdateOutgoingConnection(U, from, to, C, c, *g);
}
template <class Tr, bool Incoming, class UV, class CV, class G>
__global__ void k_update_conn(UV U, CV C, G *g, size_t n, bool sequential) {
  const size_t first = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t step = sequential ? 1 : (size_t)gridDim.x * blockDim.x;
  if (sequential && first != 0) return;
  for (size_t c = first; c < n; c += step) update_conn_one<Tr, Incoming>(U, C, g, c);
}

template <class Tr, class G> __global__ void k_reset(G *g) { Tr::ResetGlobal::Reset(*g); }

// ---- a whole DoStep in one CTA (small networks) ------------------------------
// For networks of a few thousand units and connections every pass is a
// handful of microseconds of launch latency and almost no work; one CTA runs
// the passes of DoStep in the order and with the per-unit / per-connection
// functions of the kernels above, a barrier where those are separate launches.
constexpr unsigned kSmallThreads = 512;
constexpr size_t kSmallUnits = 4096, kSmallConns = size_t(1) << 16;

struct SmallStepArgs {
  const uint32_t *in_ptr, *in_conn, *out_ptr, *out_conn;
  uint32_t *cur;
  size_t n_input, n, m;
  int levels;
  const float *mse;     // targets when MSELoss runs in the forward Apply
  const float *loss_t;  // targets of a separate loss pass
  size_t n_t;
  int loss_kind;        // 0 none, 1 MSELoss per output, 2 the loss policy in one thread
  UnitRange out;
};

template <class Tr, class UV, class CV, class G>
__global__ void __launch_bounds__(kSmallThreads) k_step_small(UV U, CV C, G *g, SmallStepArgs a) {
  constexpr bool topo = Tr::Model == Propagation::Topological;
  const size_t t0 = threadIdx.x, bs = blockDim.x;
  // DoForwardPass
  if constexpr (topo) {
    for (size_t I = t0; I < a.n; I += bs) a.cur[I] = a.in_ptr[I];
    __syncthreads();
    for (int L = 1; L <= a.levels; ++L) {
      for (size_t I = t0; I < a.n; I += bs)
        fwd_acc_level_unit<Tr>(U, C, g, a.in_ptr, a.in_conn, a.cur, I, L);
      __syncthreads();
      for (size_t I = a.n_input + t0; I < a.n; I += bs)
        fwd_apply_unit<Tr>(U, g, I, L, a.mse, a.out.Begin, a.out.End);
      __syncthreads();
    }
  } else {
    for (size_t I = t0; I < a.n; I += bs) fwd_acc_unit<Tr>(U, C, g, a.in_ptr, a.in_conn, I);
    __syncthreads();
    for (size_t I = a.n_input + t0; I < a.n; I += bs)
      fwd_apply_unit<Tr>(U, g, I, -1, a.mse, a.out.Begin, a.out.End);
    __syncthreads();
  }
  // DoCalculateLoss
  if (a.loss_kind == 1) {
    for (size_t i = t0; i < a.out.Size(); i += bs)
      GetBackwardAcc(U, a.out.Begin + i) = GetActivation(U, a.out.Begin + i) - a.loss_t[i];
  } else if (a.loss_kind == 2) {
    if constexpr (!std::is_same_v<typename Tr::Loss, NoLoss>)
      if (t0 == 0) Tr::Loss::CalculateLoss(U, a.out, std::span<const float>(a.loss_t, a.n_t), *g);
  }
  __syncthreads();
  // DoBackwardPass
  if constexpr (!std::is_same_v<typename Tr::BackwardPass, NoBackwardPass>) {
    if constexpr (topo) {
      for (int L = a.levels; L >= 1; --L) {
        for (size_t I = t0; I < a.n; I += bs)
          bwd_acc_unit<Tr>(U, C, g, a.out_ptr, a.out_conn, I, L);
        __syncthreads();
        for (size_t I = a.n_input + t0; I < a.n; I += bs) bwd_apply_unit<Tr>(U, g, I, L);
        __syncthreads();
      }
    } else {
      for (size_t I = t0; I < a.n; I += bs) bwd_acc_unit<Tr>(U, C, g, a.out_ptr, a.out_conn, I, -1);
      __syncthreads();
      for (size_t I = t0; I < a.n; I += bs) bwd_apply_unit<Tr>(U, g, I, -1);
      __syncthreads();
    }
  }
  // DoUpdateUnitState
  if constexpr (!std::is_same_v<typename Tr::UpdateUnit, NoUpdateUnit>) {
    for (size_t I = t0; I < a.n; I += bs) Tr::UpdateUnit::Update(U, I, *g);
    __syncthreads();
  }
  // DoUpdateConnectionState
  if constexpr (!std::is_same_v<typename Tr::UpdateConn, NoUpdateConn>) {
    for (size_t c = t0; c < a.m; c += bs) update_conn_one<Tr, true>(U, C, g, c);
    __syncthreads();
    for (size_t c = t0; c < a.m; c += bs) update_conn_one<Tr, false>(U, C, g, c);
    __syncthreads();
  }
  // DoResetGlobalState
  if constexpr (!std::is_same_v<typename Tr::ResetGlobal, NoResetGlobalState>)
    if (t0 == 0) Tr::ResetGlobal::Reset(*g);
}

// ---- structure --------------------------------------------------------------

// DoPruneUnits (reference plastix.hpp:257-267): Pruned = ShouldPrune.
template <class Tr, class UV, class G> __global__ void k_prune_units(UV U, G *g, size_t n, bool seq) {
  const size_t first = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t step = seq ? 1 : (size_t)gridDim.x * blockDim.x;
  if (seq && first != 0) return;
  for (size_t I = first; I < n; I += step)
    GetField<PrunedTag>(U, I) = Tr::PruneUnit::ShouldPrune(U, I, *g) ? true : false;
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
    if (rm) GetField<DeadTag>(C, c) = true;
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
  if (AC::ShouldAddIncomingConnection(U, A, B, *g)) out[k++] = CompactEdge(B, A).Bits;
  if (AC::ShouldAddOutgoingConnection(U, A, B, *g)) out[k++] = CompactEdge(A, B).Bits;
  if (!P.same) {
    if (AC::ShouldAddIncomingConnection(U, B, A, *g)) out[k++] = CompactEdge(A, B).Bits;
    if (AC::ShouldAddOutgoingConnection(U, B, A, *g)) out[k++] = CompactEdge(B, A).Bits;
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
        if (n < cap && AC::ShouldAddIncomingConnection(U, A, B, *g))
          props[n++] = CompactEdge(B, A).Bits;
        if (n < cap && AC::ShouldAddOutgoingConnection(U, A, B, *g))
          props[n++] = CompactEdge(A, B).Bits;
        if (!P.same) {
          if (n < cap && AC::ShouldAddIncomingConnection(U, B, A, *g))
            props[n++] = CompactEdge(A, B).Bits;
          if (n < cap && AC::ShouldAddOutgoingConnection(U, B, A, *g))
            props[n++] = CompactEdge(B, A).Bits;
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

static __global__ void k_widen_u16(const uint16_t *in, size_t n, uint32_t *out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = in[i];
}

static __global__ void k_level_hist(const uint16_t *level, size_t n, uint32_t *hist) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    atomicAdd(hist + level[i], 1u);
}

// ranges[L] = first index whose (sorted) key is >= L, for L in [0, nr).
static __global__ void k_level_ranges(const uint32_t *keys, size_t m, uint32_t *ranges, int nr) {
  const int L = blockIdx.x * blockDim.x + threadIdx.x;
  if (L >= nr) return;
  size_t lo = 0, hi = m;
  while (lo < hi) {
    const size_t mid = (lo + hi) / 2;
    if ((keys[mid] & 0xFFFFu) < (uint32_t)L) lo = mid + 1;
    else hi = mid;
  }
  ranges[L] = (uint32_t)lo;
}

// Traits the fused single-layer sweep serves: Pipeline, DefaultForwardPass
// with HebbianTraceUpdate, no other hook, float Weight and Trace fields.
// Traits without structural hooks: every DoStep launches the same kernels.
template <class T> constexpr bool fixed_structure() {
  return std::is_same_v<typename T::PruneUnit, NoPruneUnit> &&
         std::is_same_v<typename T::PruneConn, NoPruneConn> &&
         std::is_same_v<typename T::AddUnit, NoAddUnit> &&
         std::is_same_v<typename T::AddConn, NoAddConn>;
}

template <class T> struct IsHebbianTrace : std::false_type {};
template <float D, float R> struct IsHebbianTrace<HebbianTraceUpdate<D, R>> : std::true_type {};
template <class T> constexpr bool fused_hebbian_traits() {
  using CA = ConnAllocFor<T>;
  constexpr size_t w = CA::template IndexOf<WeightTag>(), e = CA::template IndexOf<TraceTag>();
  if constexpr (w >= CA::NumFields || e >= CA::NumFields) {
    return false;
  } else {
    return T::Model == Propagation::Pipeline &&
           std::is_same_v<typename T::ForwardPass, DefaultForwardPass> &&
           IsHebbianTrace<typename T::UpdateConn>::value &&
           std::is_same_v<typename T::BackwardPass, NoBackwardPass> &&
           std::is_same_v<typename T::Loss, NoLoss> &&
           std::is_same_v<typename T::UpdateUnit, NoUpdateUnit> &&
           std::is_same_v<typename T::PruneUnit, NoPruneUnit> &&
           std::is_same_v<typename T::PruneConn, NoPruneConn> &&
           std::is_same_v<typename T::AddUnit, NoAddUnit> &&
           std::is_same_v<typename T::AddConn, NoAddConn> &&
           std::is_same_v<typename T::ResetGlobal, NoResetGlobalState> &&
           std::is_same_v<typename CA::template FieldTypeAt<w>, float> &&
           std::is_same_v<typename CA::template FieldTypeAt<e>, float>;
  }
}

// mm[0] = min over ToId, mm[1] = max over FromId (caller initialises
// mm = {UINT32_MAX, 0}).
static __global__ void k_any_set(const uint8_t *v, size_t m, uint32_t *flag) {
  uint32_t any = 0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < m; i += (size_t)gridDim.x * blockDim.x)
    any |= v[i];
  if (__syncthreads_or(any != 0) && threadIdx.x == 0) atomicOr(flag, 1u);
}

static __global__ void k_to_min_from_max(const uint32_t *to, const uint32_t *from, size_t m,
                                         uint32_t *mm) {
  uint32_t lo = 0xFFFFFFFFu, hi = 0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < m;
       i += (size_t)gridDim.x * blockDim.x) {
    lo = min(lo, to[i]);
    hi = max(hi, from[i]);
  }
  atomicMin(mm, lo);
  atomicMax(mm + 1, hi);
}

// 1 when the connections are stored destination-major (ToId non-decreasing
// over all connections), else 0 (flag initialised to 1 by the caller).
static __global__ void k_check_dst_major(const uint32_t *to, size_t m, uint32_t *flag) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i + 1 < m;
       i += (size_t)gridDim.x * blockDim.x)
    if (to[i + 1] < to[i]) *flag = 0;
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
  using UnitAllocator = UnitAllocFor<Traits>;
  using ConnAllocator = ConnAllocFor<Traits>;
  using UView = typename UnitAllocator::View;
  using CView = typename ConnAllocator::View;

  static_assert(std::is_trivially_copyable_v<GlobalState>, "global state is copied to the GPU");

  template <typename... Builders>
    requires(sizeof...(Builders) > 0 &&
             (LayerBuilder<Builders, UnitAllocator, ConnAllocator> && ...))
  Network(size_t InputDim, Builders... Layers) : Network(InputDim, NoUnitInit{}, Layers...) {}

  template <typename InputInit, typename... Builders>
    requires(std::is_invocable_v<InputInit, UnitAllocator &, size_t> && sizeof...(Builders) > 0 &&
             (LayerBuilder<Builders, UnitAllocator, ConnAllocator> && ...))
  Network(size_t InputDim, InputInit Init, Builders... Layers)
      : NumInput(InputDim), UA(kCapacity), CA(kCapacity) {
    for (size_t I = 0; I < InputDim; ++I) Init(UA, UA.Allocate());
    UnitRange Prev{0, InputDim};
    ((Prev = Layers(UA, CA, Prev)), ...);
    OutputRange = Prev;
    cuda_check(cudaGetDevice(&Device), "device");
    cuda_check(cudaDeviceGetAttribute(&NumSMs, cudaDevAttrMultiProcessorCount, Device), "device");
    UA.Link({&Network::FetchUnitField, this});
    CA.Link({&Network::FetchConnField, this});
    cuda_check(cudaMalloc(&d_g, sizeof(GlobalState) > 0 ? sizeof(GlobalState) : 1), "globals");
    cuda_check(cudaMemcpy(d_g, &HostG, sizeof(GlobalState), cudaMemcpyHostToDevice), "globals");
    BeginDevice();
    // As the reference's constructor: Topological networks recompute the
    // unit levels and sort the connections by source level.
    if constexpr (Traits::Model == Propagation::Topological) SortConnectionsByLevel();
    EndDevice(true, true);
  }

  Network(size_t InputDim, size_t OutputDim = 1) : Network(InputDim, FullyConnected<>{OutputDim}) {}

  ~Network() { Release(); }
  Network(const Network &) = delete;
  Network &operator=(const Network &) = delete;

  size_t GetStep() const { return Step; }

  void DoForwardPass(std::span<const float> Inputs) {
    BeginDevice();
    UploadInputs(Inputs);
    const size_t n = UA.Size(), m = CA.Size();
    constexpr bool topo = Traits::Model == Propagation::Topological;
    if constexpr (topo) {
      if (NeedsResort) SortConnectionsByLevel();
    }
    if (IndexStale) RebuildIndex();
    if constexpr (!detail::read_only_globals<Traits>()) {
      detail::k_fwd_seq<Traits><<<1, 1, 0, Stream>>>(UV(), CV(), d_g, NumInput, n, m, d_ranges,
                                                      NumLevels, topo);
    } else if constexpr (topo) {
      if (n)
        cuda_check(cudaMemcpyAsync(d_cursor, d_in_ptr, n * sizeof(uint32_t),
                                   cudaMemcpyDeviceToDevice, Stream),
                   "cursor");
      for (int L = 1; L <= NumLevels; ++L) {
        detail::k_fwd_acc_level<Traits><<<detail::blocks(n), 256, 0, Stream>>>(
            UV(), CV(), d_g, d_in_ptr, d_in_conn, d_cursor, n, L);
        detail::k_fwd_apply<Traits><<<detail::blocks(n), 256, 0, Stream>>>(
            UV(), d_g, NumInput, n, L, MseTargets, OutputRange.Begin, OutputRange.End);
      }
    } else {
      using Acc = typename FP::Accumulator;
      if (DstMajor && std::is_trivially_copyable_v<Acc> && sizeof(Acc) <= 16) {
        const unsigned grid = (unsigned)std::min<size_t>(
            std::max<size_t>(1, (n + 32 * detail::kTileWarps - 1) / (32 * detail::kTileWarps)),
            (size_t)NumSMs * 8);
        detail::k_fwd_acc_tiled<Traits><<<grid, detail::kTileWarps * 32, 0, Stream>>>(
            UV(), CV(), d_g, d_in_ptr, n);
      } else {
        detail::k_fwd_acc<Traits><<<detail::blocks(n), 256, 0, Stream>>>(UV(), CV(), d_g,
                                                                          d_in_ptr, d_in_conn, n);
      }
      detail::k_fwd_apply<Traits><<<detail::blocks(n), 256, 0, Stream>>>(
          UV(), d_g, NumInput, n, -1, MseTargets, OutputRange.Begin, OutputRange.End);
    }
    cuda_check(cudaGetLastError(), "forward pass");
    EndDevice(true, true);
    ++Step;
  }

  void DoCalculateLoss(std::span<const float> Targets) {
    if constexpr (!std::is_same_v<typename Traits::Loss, NoLoss>) {
      if (Targets.empty()) return;
      BeginDevice();
      UploadTargets(Targets);
      if constexpr (std::is_same_v<typename Traits::Loss, MSELoss>) {
        if (Targets.size() >= OutputRange.Size()) {
          const size_t k = OutputRange.Size();
          if (k)
            detail::k_loss_mse<<<detail::blocks(k), 256, 0, Stream>>>(UV(), OutputRange.Begin, k,
                                                                       d_targets);
          cuda_check(cudaGetLastError(), "loss");
          EndDevice(true, false);
          return;
        }
      }
      detail::k_loss<Traits><<<1, 1, 0, Stream>>>(UV(), d_g, OutputRange, d_targets,
                                                  Targets.size());
      cuda_check(cudaGetLastError(), "loss");
      EndDevice(true, false);
    }
  }

  void DoBackwardPass() {
    if constexpr (!std::is_same_v<BP, NoBackwardPass>) {
      BeginDevice();
      if (IndexStale) RebuildIndex();
      const size_t n = UA.Size(), m = CA.Size();
      constexpr bool topo = Traits::Model == Propagation::Topological;
      if constexpr (!detail::read_only_globals<Traits>()) {
        detail::k_bwd_seq<Traits><<<1, 1, 0, Stream>>>(UV(), CV(), d_g, NumInput, n, m, d_ranges,
                                                        NumLevels, topo);
      } else if constexpr (topo) {
        for (int L = NumLevels; L >= 1; --L) {
          detail::k_bwd_acc<Traits><<<detail::blocks(n), 256, 0, Stream>>>(
              UV(), CV(), d_g, d_out_ptr, d_out_conn, n, L);
          detail::k_bwd_apply<Traits><<<detail::blocks(n), 256, 0, Stream>>>(UV(), d_g, NumInput,
                                                                             n, L);
        }
      } else {
        detail::k_bwd_acc<Traits><<<detail::blocks(n), 256, 0, Stream>>>(
            UV(), CV(), d_g, d_out_ptr, d_out_conn, n, -1);
        detail::k_bwd_apply<Traits><<<detail::blocks(n), 256, 0, Stream>>>(UV(), d_g, 0, n, -1);
      }
      cuda_check(cudaGetLastError(), "backward pass");
      EndDevice(true, true);
    }
  }

  void DoResetGlobalState() {
    if constexpr (!std::is_same_v<typename Traits::ResetGlobal, NoResetGlobalState>) {
      BeginDevice();
      detail::k_reset<Traits><<<1, 1, 0, Stream>>>(d_g);
      cuda_check(cudaGetLastError(), "reset");
    }
  }

  void DoUpdateUnitState() {
    if constexpr (!std::is_same_v<typename Traits::UpdateUnit, NoUpdateUnit>) {
      BeginDevice();
      constexpr bool seq = !detail::read_only_globals<Traits>();
      const size_t n = UA.Size();
      detail::k_update_unit<Traits><<<seq ? 1 : detail::blocks(n), 256, 0, Stream>>>(UV(), d_g, n,
                                                                                    seq);
      cuda_check(cudaGetLastError(), "unit update");
      EndDevice(true, false);
    }
  }

  void DoUpdateConnectionState() {
    if constexpr (!std::is_same_v<typename Traits::UpdateConn, NoUpdateConn>) {
      BeginDevice();
      constexpr bool seq = detail::sequential_conn_update<Traits>();
      const size_t n = CA.Size();
      const unsigned grid = seq ? 1 : std::min<unsigned>(detail::blocks(n), 4096);
      detail::k_update_conn<Traits, true><<<grid, 256, 0, Stream>>>(UV(), CV(), d_g, n, seq);
      detail::k_update_conn<Traits, false><<<grid, 256, 0, Stream>>>(UV(), CV(), d_g, n, seq);
      cuda_check(cudaGetLastError(), "connection update");
      EndDevice(true, true);
    }
  }

  void DoPruneUnits() {
    if constexpr (!std::is_same_v<typename Traits::PruneUnit, NoPruneUnit>) {
      const size_t n = UA.Size();
      if constexpr (detail::device_structure<Traits>()) {
        BeginDevice();
        detail::k_prune_units<Traits><<<kSeq ? 1 : detail::blocks(n), 256, 0, Stream>>>(
            UV(), d_g, n, kSeq);
        cuda_check(cudaGetLastError(), "prune units");
        EndDevice(true, false);
      } else {
        // The reference's loop (plastix.hpp:257-267) on the host copy.
        PullGlobals();
        for (size_t I = 0; I < n; ++I)
          GetField<PrunedTag>(UA, I) = Traits::PruneUnit::ShouldPrune(UA, I, HostG);
        PushGlobals();
      }
    }
  }

  void DoPruneConnections() {
    if constexpr (!std::is_same_v<typename Traits::PruneUnit, NoPruneUnit> ||
                  !std::is_same_v<typename Traits::PruneConn, NoPruneConn>) {
      BeginDevice();
      const size_t m = CA.Size();
      const unsigned grid = kSeq ? 1 : std::min<unsigned>(detail::blocks(m), 4096);
      detail::k_prune_conns<Traits><<<grid, 256, 0, Stream>>>(UV(), CV(), d_g, m, kSeq);
      cuda_check(cudaGetLastError(), "prune connections");
      EndDevice(false, true);
    }
  }

  // DoAddUnits (reference plastix.hpp:300-319) on the host copy: units are
  // allocated and initialised by the policy there, then uploaded (with every
  // unit field) before the next device step.
  void DoAddUnits() {
    if constexpr (!std::is_same_v<typename Traits::AddUnit, NoAddUnit>) {
      using AP = typename Traits::AddUnit;
      PullGlobals();
      const size_t N = UA.Size();
      for (size_t I = 0; I < N; ++I) {
        const std::optional<int16_t> Offset = AP::AddUnit(UA, I, HostG);
        if (!Offset.has_value()) continue;
        const int32_t Base = GetLevel(UA, I);
        const int32_t NewLevel = std::clamp(Base + static_cast<int32_t>(*Offset), int32_t{1},
                                            static_cast<int32_t>(MaxLevels - 1));
        const size_t NewId = UA.Allocate();
        if (NewId == static_cast<size_t>(-1)) break;
        GetLevel(UA, NewId) = static_cast<uint16_t>(NewLevel);
        AP::InitUnit(UA, NewId, I, HostG);
      }
      PushGlobals();
    }
  }

  // DoAddConnections (reference plastix.hpp:320-435): units bucketed by level
  // (phase 0), the level-pair window enumerated in the reference's order
  // (phase 1) -- on the device with DeviceStructure, else on the host copy --,
  // then the proposals sorted and deduplicated on the device (phases 2-3) and
  // committed in that order through InitConnection.
  void DoAddConnections() {
    if constexpr (!std::is_same_v<typename Traits::AddConn, NoAddConn>) {
      if constexpr (detail::device_structure<Traits>()) AddConnectionsOnDevice();
      else AddConnectionsOnHost();
    }
  }

  void DoStep(std::span<const float> Inputs, std::span<const float> Targets = {}) {
    if constexpr (detail::fused_hebbian_traits<Traits>()) {
      if (FusedStep(Inputs)) return;
    }
    if constexpr (detail::fixed_structure<Traits>()) {
      if (UseSmallStep && SmallStep(Inputs, Targets)) return;
      if (UseGraphs && GraphStep(Inputs, Targets)) return;
      StepBody(Inputs, Targets);
      if (UseGraphs) EagerKey = StepKey(Targets);
    } else {
      StepBody(Inputs, Targets);
    }
  }

  // Replays of DoStep as a CUDA graph (on by default): a network whose traits
  // have no structural hooks launches the same kernels every step, so after
  // one ordinary step with the same device buffers the step is captured once
  // and then launched as one graph -- only the input and target uploads stay
  // outside it. Any change of a device buffer, the level count or the number
  // of targets falls back to an ordinary step and a new capture.
  void SetGraphReplay(bool On) { UseGraphs = On; }

  // Small networks (up to 4,096 units and 65,536 connections, read-only
  // globals, parallel connection updates): DoStep is one kernel of one CTA
  // that runs every pass in order (on by default; before graph replay).
  void SetSingleKernelStep(bool On) { UseSmallStep = On; }

  void StepBody(std::span<const float> Inputs, std::span<const float> Targets) {
    // MSELoss rides in the forward pass's Apply epilogue (Pipeline, parallel
    // passes): no separate loss launch, no second read of the outputs.
    constexpr bool mse_in_apply = std::is_same_v<typename Traits::Loss, MSELoss> &&
                                  Traits::Model == Propagation::Pipeline &&
                                  detail::read_only_globals<Traits>();
    if (mse_in_apply && !Targets.empty() && Targets.size() >= OutputRange.Size() &&
        OutputRange.Begin >= NumInput) {
      MseTargets = UploadTargets(Targets);
      DoForwardPass(Inputs);
      MseTargets = nullptr;
    } else {
      DoForwardPass(Inputs);
      DoCalculateLoss(Targets);
    }
    DoBackwardPass();
    DoUpdateUnitState();
    DoUpdateConnectionState();
    DoPruneUnits();
    DoPruneConnections();
    DoAddUnits();
    DoAddConnections();
    if constexpr (Traits::Model == Propagation::Topological)
      if (NeedsResort) {
        BeginDevice();
        SortConnectionsByLevel();
        EndDevice(true, true);
      }
    DoResetGlobalState();
  }

  // Activations of the output units (waits for the device).
  std::span<const float> GetOutput() const {
    const uint64_t act = uint64_t(1) << core::kActivation;
    if (!(UA.StaleMask() & act)) {  // the host copy is current
      const float *p = static_cast<const float *>(UA.field_data(core::kActivation));
      return {p + OutputRange.Begin, OutputRange.Size()};
    }
    // into a pinned buffer owned by the network (valid until the next call)
    const size_t k = OutputRange.Size();
    if (OutCap < k) {
      cuda_check(cudaStreamSynchronize(Stream), "output");
      if (OutHost) cudaFreeHost(OutHost);
      OutHost = nullptr;
      cuda_check(cudaMallocHost(reinterpret_cast<void **>(&OutHost), k * sizeof(float)), "output");
      OutCap = k;
    }
    if (k)
      cuda_check(cudaMemcpyAsync(OutHost,
                                 static_cast<const float *>(d_uf[core::kActivation]) +
                                     OutputRange.Begin,
                                 k * sizeof(float), cudaMemcpyDeviceToHost, Stream),
                 "output");
    cuda_check(cudaStreamSynchronize(Stream), "output");
    return {OutHost, k};
  }

  // The coherent host copies (see the header comment).
  UnitAllocator &GetUnitAlloc() { return UA; }
  ConnAllocator &GetConnAlloc() { return CA; }

  GlobalState GetGlobals() {
    PullGlobals();
    return HostG;
  }
  void SetGlobals(const GlobalState &g) {
    HostG = g;
    PushGlobals();
  }
  void SetStream(cudaStream_t s) {
    cuda_check(cudaStreamSynchronize(Stream), "stream");
    if (OwnStream && s != OwnStream) {
      cudaStreamDestroy(OwnStream);
      OwnStream = nullptr;
    }
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
    UA.FetchAll();
    CA.FetchAll();
    PullGlobals();
    CheckpointHeader H = Header();
    FILE *F = std::fopen(Path.c_str(), "wb");
    if (!F) throw std::runtime_error("cannot write " + Path);
    bool ok = std::fwrite(&H, sizeof(H), 1, F) == 1;
    ok = ok && WriteFieldSizes<UnitAllocator>(F) && WriteFieldSizes<ConnAllocator>(F);
    for (size_t i = 0; ok && i < UnitAllocator::NumFields; ++i)
      ok = WriteAll(F, UA.field_data(i), UA.Size() * UnitAllocator::field_bytes(i));
    for (size_t i = 0; ok && i < ConnAllocator::NumFields; ++i)
      ok = WriteAll(F, CA.field_data(i), CA.Size() * ConnAllocator::field_bytes(i));
    ok = ok && WriteAll(F, &HostG, sizeof(HostG));
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
    // The host copies now hold the whole state: nothing is stale, everything
    // goes to the device (re-allocated at the loaded sizes).
    UA.ClearAllStale();
    CA.ClearAllStale();
    ForceUpload();
    SetGlobals(G);
    NumInput = H.NumInput;
    OutputRange = UnitRange(H.OutBegin, H.OutEnd);
    Step = H.Step;
    NumLevels = H.NumLevels;
    NeedsResort = (H.Flags & 1u) != 0;
    BeginDevice();
    if constexpr (Traits::Model == Propagation::Topological) ComputeLevelRanges();
  }

 private:
  static constexpr bool kSeq = detail::sequential_structure<Traits>();
  static constexpr size_t kCapacity = size_t(1) << 40;

  struct CheckpointHeader {
    char Magic[8];
    uint64_t NumInput, Step, Units, Conns, OutBegin, OutEnd;
    int32_t NumLevels;
    uint32_t Flags;  // bit 0: a level re-sort is pending
    uint32_t UnitFields, ConnFields, GlobalBytes, Reserved;
  };
  CheckpointHeader Header() const {
    CheckpointHeader H{};
    std::memcpy(H.Magic, "PLXCKPT2", 8);
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
  uint16_t *LevelPtr() const { return static_cast<uint16_t *>(d_uf[core::kLevel]); }
  uint32_t *FromPtr() const { return static_cast<uint32_t *>(d_cf[core::kFromId]); }
  uint32_t *ToPtr() const { return static_cast<uint32_t *>(d_cf[core::kToId]); }
  uint8_t *DeadPtr() const { return static_cast<uint8_t *>(d_cf[core::kDead]); }
  uint16_t *SrcLevelPtr() const { return static_cast<uint16_t *>(d_cf[core::kSrcLevel]); }

  // ---- coherence of the host copies ---------------------------------------
  static void FetchUnitField(void *owner, size_t I) {
    auto *N = static_cast<Network *>(owner);
    N->InputsToField();
    N->DownloadField(N->UA, N->d_uf, N->DevUnits, I);
  }
  static void FetchConnField(void *owner, size_t I) {
    auto *N = static_cast<Network *>(owner);
    N->FieldsFromSlots();
    N->DownloadField(N->CA, N->d_cf, N->DevConns, I);
  }
  template <class A>
  void DownloadField(A &a, const std::vector<void *> &d, size_t dev_count, size_t I) {
    cuda_check(cudaStreamSynchronize(Stream), "download");
    if (dev_count == static_cast<size_t>(-1)) return;  // no device copy yet
    const size_t k = std::min(a.Size(), dev_count);
    if (k)
      cuda_check(cudaMemcpy(a.field_data(I), d[I], k * A::field_bytes(I), cudaMemcpyDeviceToHost),
                 "field download");
  }
  // Brings the device copies up to date with the host: fields the host
  // touched are uploaded; when the host changed the number of entities
  // (AddUnit, host-side AddConn, Load) the device arrays are re-made from
  // the (completed) host copy.
  template <class A>
  bool SyncAlloc(A &a, std::vector<void *> &d, size_t &dev_count) {
    const size_t n = a.Size();
    bool changed = false;
    if (n != dev_count || d.empty()) {
      a.FetchAll();
      cuda_check(cudaStreamSynchronize(Stream), "resize");
      for (void *p : d) cudaFree(p);
      d.assign(A::NumFields, nullptr);
      for (size_t i = 0; i < A::NumFields; ++i) {
        cuda_check(cudaMalloc(&d[i], std::max<size_t>(1, n) * A::field_bytes(i)), "field");
        if (n)
          cuda_check(cudaMemcpy(d[i], a.field_data(i), n * A::field_bytes(i),
                                cudaMemcpyHostToDevice),
                     "field upload");
      }
      dev_count = n;
      a.ClearDirty();
      return true;
    }
    const uint64_t dirty = a.DirtyMask();
    if (dirty) {
      for (size_t i = 0; i < A::NumFields; ++i)
        if (((dirty >> i) & 1u) && n)
          cuda_check(cudaMemcpyAsync(d[i], a.field_data(i), n * A::field_bytes(i),
                                     cudaMemcpyHostToDevice, Stream),
                     "field upload");
      // pageable host memory: the copies are staged before the calls return
      a.ClearDirty();
      changed = true;
    }
    return changed;
  }
  // Called before device work: host edits reach the device, and an edit of
  // the connection topology invalidates the connection index.
  void BeginDevice(bool fused_step = false) {
    if (!fused_step) {
      FieldsFromSlots();
      InputsToField();
    }
    const uint64_t cdirty = CA.DirtyMask();
    if (cdirty) Fused.Ready = false;  // the slot copies no longer match
    const bool units_resized = UA.Size() != DevUnits;
    const bool conns_resized = CA.Size() != DevConns;
    SyncAlloc(UA, d_uf, DevUnits);
    SyncAlloc(CA, d_cf, DevConns);
    constexpr uint64_t topo_fields = (uint64_t(1) << core::kFromId) | (uint64_t(1) << core::kToId) |
                                     (uint64_t(1) << core::kDead) |
                                     (uint64_t(1) << core::kSrcLevel);
    if (units_resized || conns_resized || (cdirty & topo_fields)) IndexStale = true;
  }
  // Called after device work that may have changed the unit / connection
  // fields: the host copies of those fields are stale.
  void EndDevice(bool units, bool conns) {
    if (units) UA.MarkStale(UnitAllocator::AllFields());
    if (conns) {
      CA.MarkStale(ConnAllocator::AllFields());
      Fused.Ready = false;  // the reference-order fields may now be newer
    }
  }
  void ForceUpload() {
    DevUnits = DevConns = static_cast<size_t>(-1);
    IndexStale = true;
  }
  void PullGlobals() {
    cuda_check(cudaMemcpyAsync(&HostG, d_g, sizeof(GlobalState), cudaMemcpyDeviceToHost, Stream),
               "globals");
    cuda_check(cudaStreamSynchronize(Stream), "globals");
  }
  void PushGlobals() {
    cuda_check(cudaMemcpyAsync(d_g, &HostG, sizeof(GlobalState), cudaMemcpyHostToDevice, Stream),
               "globals");
    cuda_check(cudaStreamSynchronize(Stream), "globals");
  }

  // ---- levels, index ---------------------------------------------------------

  // SortConnectionsByLevel (reference plastix.hpp:539-579) on the device:
  // RecomputeLevels, SrcLevel = Level[FromId], stable radix sort on the
  // 16-bit key, Gather of every connection field; NumLevels = highest
  // SrcLevel + 1, level ranges for the one-thread passes.
  void SortConnectionsByLevel() {
    const size_t n = UA.Size(), m = CA.Size();
    plx_ctx *ctx = PlxCtx();
    const size_t lb = plx_recompute_levels_scratch_bytes(n, m);
    plx_check(plx_recompute_levels(ctx, (uint32_t)n, (uint32_t)NumInput, m, FromPtr(), ToPtr(),
                                   DeadPtr(), LevelPtr(), nullptr, Buf<uint8_t>(13, lb), lb),
              "plx_recompute_levels");
    NeedsResort = false;
    UA.MarkStale(uint64_t(1) << core::kLevel);
    if (m == 0) {
      NumLevels = 0;
      ComputeLevelRanges();
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
    CA.MarkStale(ConnAllocator::AllFields());
    NumLevels = (int)(last & 0xFFFFu) + 1;
    IndexStale = true;
    ComputeLevelRanges();
  }

  // ranges[L] (L in [0, NumLevels + 2)) = first connection whose SrcLevel is
  // >= L, from the sorted SrcLevel keys (the reference's Ranges table).
  void ComputeLevelRanges() {
    const int nr = NumLevels + 2;
    d_ranges = Buf<uint32_t>(14, nr);
    const size_t m = CA.Size();
    if (m == 0 || NumLevels == 0) {
      cuda_check(cudaMemsetAsync(d_ranges, 0, nr * sizeof(uint32_t), Stream), "ranges");
      return;
    }
    uint32_t *keys = Buf<uint32_t>(1, m);
    detail::k_widen_u16<<<detail::blocks(m), 256, 0, Stream>>>(SrcLevelPtr(), m, keys);
    detail::k_level_ranges<<<(nr + 255) / 256, 256, 0, Stream>>>(keys, m, d_ranges, nr);
    cuda_check(cudaGetLastError(), "ranges");
  }

  // Incoming connection lists per destination (stored order) and outgoing per
  // source (ascending index), as CSR arrays on the device: stable radix sorts
  // of ToId and FromId, row offsets from the sorted keys.
  void RebuildIndex() {
    const size_t n = UA.Size(), m = CA.Size();
    cuda_check(cudaStreamSynchronize(Stream), "index");
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
    // Destination-major storage (ToId non-decreasing) enables the tiled
    // forward accumulation.
    uint32_t *flag = Buf<uint32_t>(15, 1);
    const uint32_t one = 1;
    cuda_check(cudaMemcpyAsync(flag, &one, 4, cudaMemcpyHostToDevice, Stream), "index");
    detail::k_check_dst_major<<<std::min<unsigned>(detail::blocks(m), 4096), 256, 0, Stream>>>(
        ToPtr(), m, flag);
    uint32_t dm = 0;
    cuda_check(cudaMemcpyAsync(&dm, flag, 4, cudaMemcpyDeviceToHost, Stream), "index");
    cuda_check(cudaStreamSynchronize(Stream), "index");
    DstMajor = dm != 0;
    Fused.Ready = false;
    Fused.Eligible = false;
    if constexpr (detail::fused_hebbian_traits<Traits>()) {
      // one layer: every source an input unit, every destination not
      uint32_t *mm = Buf<uint32_t>(15, 2);
      const uint32_t init[2] = {0xFFFFFFFFu, 0u};
      cuda_check(cudaMemcpyAsync(mm, init, 8, cudaMemcpyHostToDevice, Stream), "index");
      detail::k_to_min_from_max<<<std::min<unsigned>(detail::blocks(m), 1024), 256, 0, Stream>>>(
          ToPtr(), FromPtr(), m, mm);
      uint32_t got[2] = {0, 0};
      cuda_check(cudaMemcpyAsync(got, mm, 8, cudaMemcpyDeviceToHost, Stream), "index");
      cuda_check(cudaStreamSynchronize(Stream), "index");
      Fused.Eligible = DstMajor && got[0] >= NumInput && got[1] < NumInput && n > NumInput;
    }
    uint32_t *keys_out = Buf<uint32_t>(2, m);
    const uint32_t bits = BitsFor(n);
    RadixSort(m, ToPtr(), keys_out, d_in_conn, bits);
    plx_check(plx_csr_row_ptr(ctx, keys_out, m, 0, (uint32_t)n, d_in_ptr), "plx_csr_row_ptr");
    RadixSort(m, FromPtr(), keys_out, d_out_conn, bits);
    plx_check(plx_csr_row_ptr(ctx, keys_out, m, 0, (uint32_t)n, d_out_ptr), "plx_csr_row_ptr");
  }

  // ---- DoAddConnections ----------------------------------------------------

  // The level-pair window of phase 1 in the reference's order: the initial
  // window [0, min(N, highest)] as pairs La <= Lb, then each new right level
  // R with every level of [R - N, R].
  template <class F> static void ForEachLevelPair(uint32_t highest, F &&f) {
    constexpr uint32_t N = Traits::Neighbourhood;
    const uint32_t init_right = std::min<uint32_t>(N, highest);
    for (uint32_t La = 0; La <= init_right; ++La)
      for (uint32_t Lb = La; Lb <= init_right; ++Lb) f(La, Lb);
    for (uint32_t R = N + 1; R <= highest; ++R)
      for (uint32_t W = R - N; W <= R; ++W) f(W, R);
  }

  // Sorts and deduplicates `n_props` proposals (device) and returns the
  // unique ones in ascending CompactEdge order (device, `k` entries).
  uint64_t *SortUnique(uint64_t *props, uint64_t n_props, uint64_t &k) {
    uint64_t *uniq = Buf<uint64_t>(9, n_props), *ucnt = Buf<uint64_t>(10, 1);
    const size_t sb = plx_sort_unique_u64_scratch_bytes(n_props);
    plx_check(plx_sort_unique_u64(PlxCtx(), n_props, props, uniq, ucnt, Buf<uint8_t>(11, sb), sb),
              "plx_sort_unique_u64");
    cuda_check(cudaMemcpyAsync(&k, ucnt, 8, cudaMemcpyDeviceToHost, Stream), "unique");
    cuda_check(cudaStreamSynchronize(Stream), "unique");
    return uniq;
  }

  // Phase 0 and 1 on the host copy with the host global state, exactly the
  // reference's loops (predicates may use host-only facilities); phases 2-3
  // sort and deduplicate on the device; the commit runs InitConnection on
  // the host copy, and the new connections are uploaded before the next
  // device step.
  void AddConnectionsOnHost() {
    using AC = typename Traits::AddConn;
    const size_t n = UA.Size();
    if (n == 0) return;
    PullGlobals();
    std::vector<uint32_t> off;
    uint32_t highest = 0;
    for (size_t I = 0; I < n; ++I) highest = std::max<uint32_t>(highest, GetLevel(UA, I));
    off.assign(highest + 2, 0);
    for (size_t I = 0; I < n; ++I) ++off[GetLevel(UA, I) + 1];
    for (uint32_t L = 0; L <= highest; ++L) off[L + 1] += off[L];
    std::vector<uint32_t> ubl(n), pos(off.begin(), off.end() - 1);
    for (size_t I = 0; I < n; ++I) ubl[pos[GetLevel(UA, I)]++] = (uint32_t)I;
    std::vector<uint64_t> props;
    const uint64_t cap = ProposalCap;
    ForEachLevelPair(highest, [&](uint32_t La, uint32_t Lb) {
      for (uint32_t Ai = off[La]; Ai < off[La + 1]; ++Ai) {
        const uint32_t U = ubl[Ai];
        for (uint32_t Bi = off[Lb]; Bi < off[Lb + 1]; ++Bi) {
          const uint32_t V = ubl[Bi];
          if (U == V) continue;
          if (props.size() < cap && AC::ShouldAddIncomingConnection(UA, U, V, HostG))
            props.push_back(CompactEdge(V, U).Bits);
          if (props.size() < cap && AC::ShouldAddOutgoingConnection(UA, U, V, HostG))
            props.push_back(CompactEdge(U, V).Bits);
          if (La != Lb) {
            if (props.size() < cap && AC::ShouldAddIncomingConnection(UA, V, U, HostG))
              props.push_back(CompactEdge(U, V).Bits);
            if (props.size() < cap && AC::ShouldAddOutgoingConnection(UA, V, U, HostG))
              props.push_back(CompactEdge(V, U).Bits);
          }
        }
      }
    });
    if (props.empty()) {
      PushGlobals();
      return;
    }
    uint64_t *d_props = Buf<uint64_t>(5, props.size());
    cuda_check(cudaMemcpyAsync(d_props, props.data(), props.size() * 8, cudaMemcpyHostToDevice,
                               Stream),
               "proposals");
    uint64_t k = 0;
    const uint64_t *uniq = SortUnique(d_props, props.size(), k);
    std::vector<uint64_t> edges(k);
    if (k)
      cuda_check(cudaMemcpy(edges.data(), uniq, k * 8, cudaMemcpyDeviceToHost), "unique");
    const size_t before = CA.Size();
    for (const uint64_t b : edges) {
      const CompactEdge E{(uint32_t)b, (uint32_t)(b >> 32)};
      const size_t C = CA.Allocate();
      if (C == static_cast<size_t>(-1)) break;
      GetField<FromIdTag>(CA, C) = E.From();
      GetField<ToIdTag>(CA, C) = E.To();
      GetField<SrcLevelTag>(CA, C) = GetLevel(UA, E.From());
      AC::InitConnection(UA, E.From(), E.To(), CA, C, HostG);
    }
    PushGlobals();
    if (CA.Size() > before) {
      NeedsResort = Traits::Model == Propagation::Topological;
      IndexStale = true;
    }
  }

  // Phases 0-1 on the device: level histogram + stable radix sort (units by
  // level), the level-pair window, k_propose (count pass, per-chunk scan,
  // ordered write pass) or k_propose_seq; then sort/unique and k_commit_conns.
  void AddConnectionsOnDevice() {
    BeginDevice();
    const size_t n = UA.Size();
    if (n == 0) return;
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
    std::vector<detail::LevelPair> pairs;
    uint64_t total = 0;
    ForEachLevelPair(highest, [&](uint32_t La, uint32_t Lb) {
      const uint32_t na = off[La + 1] - off[La], nb = off[Lb + 1] - off[Lb];
      if (!na || !nb) return;
      pairs.push_back({total, off[La], na, off[Lb], nb, La == Lb ? 1u : 0u});
      total += (uint64_t)na * nb;
    });
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
    uint64_t k = 0;
    const uint64_t *uniq = SortUnique(props, n_props, k);
    if (k == 0) return;
    const size_t m0 = CA.Size();
    GrowConnections(k);
    detail::k_commit_conns<Traits><<<kSeq ? 1 : detail::blocks(k), 256, 0, Stream>>>(
        UV(), CV(), d_g, uniq, k, m0, kSeq);
    cuda_check(cudaGetLastError(), "commit");
    EndDevice(false, true);
    NeedsResort = Traits::Model == Propagation::Topological;
    IndexStale = true;
  }

  // Appends k zeroed connections (device arrays and the host copy's count).
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
    CA.AllocateMany(k);
    DevConns = m + k;
  }

  const float *UploadTargets(std::span<const float> Targets) {
    if (Capturing) return d_targets;  // uploaded before each replay
    if (Targets.size() > TargetCap) {
      cuda_check(cudaStreamSynchronize(Stream), "targets");
      if (d_targets) cudaFree(d_targets);
      d_targets = nullptr;
      cuda_check(cudaMalloc(&d_targets, Targets.size() * sizeof(float)), "targets");
      TargetCap = Targets.size();
    }
    if (!Targets.empty())
      StagedUpload(d_targets, Targets.data(), Targets.size() * sizeof(float), TargetStage);
    return d_targets;
  }
  const float *MseTargets = nullptr;  // set while DoStep runs MSELoss in the Apply

  // Input activations to the device (skipped while a step is being captured:
  // graph replays upload them before each launch).
  void UploadInputs(std::span<const float> Inputs) {
    const size_t k = std::min(Inputs.size(), NumInput);
    if (!k || Capturing) return;
    StagedUpload(d_uf[core::kActivation], Inputs.data(), k * sizeof(float), InStage);
  }
  struct Staging {
    void *Host = nullptr;
    size_t Bytes = 0;
    cudaEvent_t Done = nullptr;
  };
  struct StagingPair {
    Staging B[2];
    int Next = 0;
  };
  // Host -> device through two pinned staging buffers used in turn: the
  // transfer is asynchronous at pinned-memory speed, the host copy of the
  // next call overlaps the device work of this one, and a buffer is reused
  // only once the transfers that read it have completed. Large transfers go
  // in 1 MiB pieces, each sent while the next is copied into the buffer.
  void StagedUpload(void *dst, const void *src_host, size_t bytes, StagingPair &pair) {
    StagedUpload(dst, src_host, bytes, pair, Stream);
  }
  void StagedUpload(void *dst, const void *src_host, size_t bytes, StagingPair &pair,
                    cudaStream_t on) {
    Staging &b = pair.B[pair.Next];
    pair.Next ^= 1;
    if (b.Bytes < bytes) {
      if (b.Host) {
        cuda_check(cudaEventSynchronize(b.Done), "upload");
        cudaFreeHost(b.Host);
        b.Host = nullptr;
        b.Bytes = 0;
      }
      cuda_check(cudaMallocHost(&b.Host, std::max<size_t>(bytes, 256)), "upload");
      b.Bytes = std::max<size_t>(bytes, 256);
      if (!b.Done) cuda_check(cudaEventCreateWithFlags(&b.Done, cudaEventDisableTiming), "upload");
    } else {
      cuda_check(cudaEventSynchronize(b.Done), "upload");
    }
    constexpr size_t piece = size_t(1) << 20;
    auto *src = static_cast<const char *>(src_host);
    auto *host = static_cast<char *>(b.Host);
    auto *dev = static_cast<char *>(dst);
    for (size_t off = 0; off < bytes; off += piece) {
      const size_t len = std::min(piece, bytes - off);
      std::memcpy(host + off, src + off, len);
      cuda_check(cudaMemcpyAsync(dev + off, host + off, len, cudaMemcpyHostToDevice, on),
                 "upload");
    }
    cuda_check(cudaEventRecord(b.Done, on), "upload");
  }
  StagingPair InStage, TargetStage;

  // ---- DoStep as a CUDA graph -------------------------------------------------
  // Everything a captured step depends on besides the field contents: device
  // buffers, sizes, the level count, the index layout, the number of targets.
  std::vector<uintptr_t> StepKey(std::span<const float> Targets) const {
    std::vector<uintptr_t> k;
    for (void *p : d_uf) k.push_back(reinterpret_cast<uintptr_t>(p));
    for (void *p : d_cf) k.push_back(reinterpret_cast<uintptr_t>(p));
    for (const void *p : {(const void *)d_g, (const void *)d_in_ptr, (const void *)d_out_ptr,
                          (const void *)d_in_conn, (const void *)d_out_conn, (const void *)d_cursor,
                          (const void *)d_ranges, (const void *)d_targets})
      k.push_back(reinterpret_cast<uintptr_t>(p));
    for (void *p : Scratch) k.push_back(reinterpret_cast<uintptr_t>(p));
    for (size_t v : {UA.Size(), CA.Size(), (size_t)NumLevels, (size_t)DstMajor, Targets.size(),
                     NumInput})
      k.push_back(v);
    return k;
  }

  bool SmallStep(std::span<const float> Inputs, std::span<const float> Targets) {
    if constexpr (!detail::read_only_globals<Traits>() ||
                  detail::sequential_conn_update<Traits>()) {
      return false;
    } else {
      const size_t n = UA.Size(), m = CA.Size();
      if (n > detail::kSmallUnits || m > detail::kSmallConns) return false;
      BeginDevice();
      if (IndexStale || NeedsResort) return false;
      UploadInputs(Inputs);
      detail::SmallStepArgs a{};
      a.in_ptr = d_in_ptr;
      a.in_conn = d_in_conn;
      a.out_ptr = d_out_ptr;
      a.out_conn = d_out_conn;
      a.cur = d_cursor;
      a.n_input = NumInput;
      a.n = n;
      a.m = m;
      a.levels = NumLevels;
      a.out = OutputRange;
      using L = typename Traits::Loss;
      if constexpr (!std::is_same_v<L, NoLoss>) {
        if (!Targets.empty()) {
          const float *t = UploadTargets(Targets);
          const bool mse = std::is_same_v<L, MSELoss> && Targets.size() >= OutputRange.Size();
          if (mse && Traits::Model == Propagation::Pipeline && OutputRange.Begin >= NumInput) {
            a.mse = t;  // in the Apply epilogue, as StepBody does
          } else {
            a.loss_t = t;
            a.n_t = Targets.size();
            a.loss_kind = mse ? 1 : 2;
          }
        }
      }
      detail::k_step_small<Traits><<<1, detail::kSmallThreads, 0, Stream>>>(UV(), CV(), d_g, a);
      cuda_check(cudaGetLastError(), "step");
      EndDevice(true, true);
      ++Step;
      return true;
    }
  }

  bool GraphStep(std::span<const float> Inputs, std::span<const float> Targets) {
    BeginDevice();
    if (IndexStale || NeedsResort) return false;
    const std::vector<uintptr_t> key = StepKey(Targets);
    if (!(GraphExec && key == GraphKey)) {
      if (key != EagerKey) return false;  // one ordinary step with these buffers first
      if (!CaptureStep(Targets)) {
        UseGraphs = false;
        return false;
      }
      GraphKey = key;
    }
    UploadInputs(Inputs);
    if constexpr (!std::is_same_v<typename Traits::Loss, NoLoss>)
      if (!Targets.empty()) UploadTargets(Targets);
    cuda_check(cudaGraphLaunch(GraphExec, Stream), "graph launch");
    EndDevice(true, true);
    ++Step;
    return true;
  }

  // Captures StepBody (without its uploads) on the network's stream; false,
  // with nothing left behind, if the capture or the instantiation fails.
  bool CaptureStep(std::span<const float> Targets) {
    if (!Stream) {  // the legacy default stream cannot be captured
      cudaStream_t s = nullptr;
      cuda_check(cudaStreamCreateWithFlags(&s, cudaStreamDefault), "stream");
      SetStream(s);
      OwnStream = s;
    }
    if (GraphExec) cudaGraphExecDestroy(GraphExec);
    GraphExec = nullptr;
    if (cudaStreamBeginCapture(Stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    const size_t step0 = Step;
    bool ok = true;
    Capturing = true;
    try {
      StepBody({}, Targets);
    } catch (...) {
      ok = false;
    }
    Capturing = false;
    Step = step0;
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(Stream, &g);
    if (ok && e == cudaSuccess && g) ok = cudaGraphInstantiate(&GraphExec, g, 0) == cudaSuccess;
    else ok = false;
    if (g) cudaGraphDestroy(g);
    if (!ok) {
      GraphExec = nullptr;
      cudaGetLastError();
    }
    return ok;
  }

  bool UseGraphs = true, UseSmallStep = true, Capturing = false;
  cudaGraphExec_t GraphExec = nullptr;
  std::vector<uintptr_t> GraphKey, EagerKey;
  cudaStream_t OwnStream = nullptr;

  // ---- the fused single-layer step (HebbianTraceUpdate traits) -------------
  // The layer is re-laid once into warp-sliced rows (plx_sliced_*); each
  // DoStep is then one plx_sweep_forward_hebbian_sliced launch, bit-exact
  // with the generic passes. Weight and Trace live in slot order while
  // steps run; they are unpacked into the reference-order fields when
  // anything else -- a host read, another Do* step -- needs them, and host
  // edits or other steps invalidate the slot copies (re-packed on the next
  // fused step).
  struct FusedState {
    bool Eligible = false, Ready = false, SlotsNewer = false, AnyDead = true;
    // double-buffered inputs of the fused step (UploadInputsAside)
    float *In[2] = {nullptr, nullptr};
    cudaEvent_t InReady[2] = {nullptr, nullptr}, Swept[2] = {nullptr, nullptr};
    cudaStream_t Copy = nullptr;
    int InNext = 0, InCur = -1;
    plx_sliced Sl{};
    // slot-order FromId, Dead, Weight, Trace; lane lengths, row offsets,
    // slice offsets, lane rows, slot -> connection permutation
    void *Mem[9] = {};
    size_t Bytes[9] = {};
  };
  template <class T> T *FusedBuf(int slot, size_t count) {
    const size_t bytes = std::max<size_t>(count, 4) * sizeof(T);
    if (Fused.Bytes[slot] < bytes) {
      cuda_check(cudaStreamSynchronize(Stream), "fused");
      if (Fused.Mem[slot]) cudaFree(Fused.Mem[slot]);
      cuda_check(cudaMalloc(&Fused.Mem[slot], bytes), "fused");
      Fused.Bytes[slot] = bytes;
    }
    return static_cast<T *>(Fused.Mem[slot]);
  }
  static constexpr size_t kW = ConnAllocator::template IndexOf<WeightTag>();
  static constexpr size_t kE = ConnAllocator::template IndexOf<TraceTag>();

  // A full input vector of the fused step goes to one of two device buffers
  // of its own, on a copy stream, so that its transfer overlaps the previous
  // step's sweep; the sweep gathers from that buffer. A buffer is refilled
  // only after the sweep that read it (event). The input units' Activation
  // field is brought up to date from the buffer when anything else needs it
  // (InputsToField).
  int UploadInputsAside(std::span<const float> Inputs) {
    const size_t bytes = NumInput * sizeof(float);
    if (!Fused.Copy) {
      cuda_check(cudaStreamCreateWithFlags(&Fused.Copy, cudaStreamNonBlocking), "inputs");
      for (int b = 0; b < 2; ++b) {
        cuda_check(cudaMalloc(&Fused.In[b], std::max<size_t>(bytes, 16)), "inputs");
        cuda_check(cudaEventCreateWithFlags(&Fused.InReady[b], cudaEventDisableTiming), "inputs");
        cuda_check(cudaEventCreateWithFlags(&Fused.Swept[b], cudaEventDisableTiming), "inputs");
      }
      // the copy stream starts behind everything already queued on Stream
      cuda_check(cudaEventRecord(Fused.Swept[0], Stream), "inputs");
      cuda_check(cudaEventRecord(Fused.Swept[1], Stream), "inputs");
    }
    const int b = Fused.InNext;
    Fused.InNext ^= 1;
    cuda_check(cudaStreamWaitEvent(Fused.Copy, Fused.Swept[b], 0), "inputs");
    StagedUpload(Fused.In[b], Inputs.data(), bytes, InStage, Fused.Copy);
    cuda_check(cudaEventRecord(Fused.InReady[b], Fused.Copy), "inputs");
    cuda_check(cudaStreamWaitEvent(Stream, Fused.InReady[b], 0), "inputs");
    return b;
  }

  // The last fused step's inputs into the Activation field of the input units.
  void InputsToField() {
    if constexpr (detail::fused_hebbian_traits<Traits>()) {
      if (Fused.InCur < 0) return;
      const int b = Fused.InCur;
      Fused.InCur = -1;
      cuda_check(cudaMemcpyAsync(d_uf[core::kActivation], Fused.In[b], NumInput * sizeof(float),
                                 cudaMemcpyDeviceToDevice, Stream),
                 "inputs");
    }
  }

  void FieldsFromSlots() {
    if constexpr (detail::fused_hebbian_traits<Traits>()) {
      if (!Fused.SlotsNewer) return;
      Fused.SlotsNewer = false;
      plx_ctx *ctx = PlxCtx();
      plx_check(plx_sliced_unpack(ctx, &Fused.Sl, Fused.Mem[2], d_cf[kW], 4), "plx_sliced_unpack");
      plx_check(plx_sliced_unpack(ctx, &Fused.Sl, Fused.Mem[3], d_cf[kE], 4), "plx_sliced_unpack");
    }
  }

  void BuildFused() {
    const size_t n = UA.Size(), m = CA.Size();
    const uint32_t rows = (uint32_t)(n - NumInput);
    plx_ctx *ctx = PlxCtx();
    uint32_t *row_ptr = FusedBuf<uint32_t>(5, rows + 1);
    plx_check(plx_csr_row_ptr(ctx, ToPtr(), m, (uint32_t)NumInput, rows, row_ptr),
              "plx_csr_row_ptr");
    const uint32_t ns = plx_sliced_n_slices(rows);
    const size_t sb = plx_sliced_plan_scratch_bytes(rows);
    plx_check(plx_sliced_plan(ctx, row_ptr, rows, m, &Fused.Sl, FusedBuf<uint64_t>(6, ns + 1),
                              FusedBuf<uint32_t>(7, (size_t)ns * 32),
                              FusedBuf<uint32_t>(4, (size_t)ns * 32), Buf<uint8_t>(8, sb), sb),
              "plx_sliced_plan");
    const size_t slots = Fused.Sl.n_slots;
    plx_check(plx_sliced_perm(ctx, &Fused.Sl, row_ptr, FusedBuf<uint32_t>(8, slots)),
              "plx_sliced_perm");
    uint32_t *from = FusedBuf<uint32_t>(0, slots);
    uint8_t *dead = FusedBuf<uint8_t>(1, slots);
    float *w = FusedBuf<float>(2, slots), *e = FusedBuf<float>(3, slots);
    if (slots) {
      plx_check(plx_sliced_pack(ctx, &Fused.Sl, FromPtr(), from, 4), "plx_sliced_pack");
      plx_check(plx_sliced_pack(ctx, &Fused.Sl, DeadPtr(), dead, 1), "plx_sliced_pack");
      plx_check(plx_sliced_pack(ctx, &Fused.Sl, d_cf[kW], w, 4), "plx_sliced_pack");
      plx_check(plx_sliced_pack(ctx, &Fused.Sl, d_cf[kE], e, 4), "plx_sliced_pack");
    }
    // the dead-aware kernel only while some connection is dead
    uint32_t *flag = Buf<uint32_t>(15, 2);
    cuda_check(cudaMemsetAsync(flag, 0, 4, Stream), "fused");
    detail::k_any_set<<<std::min<unsigned>(detail::blocks(m), 1024), 256, 0, Stream>>>(DeadPtr(),
                                                                                       m, flag);
    uint32_t any = 0;
    cuda_check(cudaMemcpyAsync(&any, flag, 4, cudaMemcpyDeviceToHost, Stream), "fused");
    cuda_check(cudaStreamSynchronize(Stream), "fused");
    Fused.AnyDead = any != 0;
    Fused.Ready = true;
    Fused.SlotsNewer = false;
  }

  // One DoStep as a single fused sweep; false when the network is not (or no
  // longer) a single destination-major layer fed by input units.
  bool FusedStep(std::span<const float> Inputs) {
    if (!Fused.SlotsNewer) BeginDevice(true);
    else if (UA.DirtyMask() || CA.DirtyMask() || UA.Size() != DevUnits || CA.Size() != DevConns) {
      FieldsFromSlots();  // host edits since the last step: go through the fields
      BeginDevice(true);
    }
    if (IndexStale) RebuildIndex();
    if (!Fused.Eligible) return false;
    if (!Fused.Ready) BuildFused();
    using U = typename Traits::UpdateConn;
    float *act = static_cast<float *>(d_uf[core::kActivation]);
    const float *src = act;
    int slot = -1;
    if (Inputs.size() >= NumInput) {
      slot = UploadInputsAside(Inputs);
      src = Fused.In[slot];
    } else {
      InputsToField();
      UploadInputs(Inputs);
    }
    plx_check(plx_sweep_forward_hebbian_sliced(
                  PlxCtx(), &Fused.Sl, static_cast<uint32_t *>(Fused.Mem[0]),
                  Fused.AnyDead ? static_cast<uint8_t *>(Fused.Mem[1]) : nullptr, src,
                  (uint32_t)NumInput, static_cast<float *>(Fused.Mem[2]),
                  static_cast<float *>(Fused.Mem[3]), U::kDecay, U::kRate, act + NumInput,
                  nullptr, 0, 0, 0),
              "plx_sweep_forward_hebbian_sliced");
    if (slot >= 0) {
      cuda_check(cudaEventRecord(Fused.Swept[slot], Stream), "inputs");
      Fused.InCur = slot;
    }
    Fused.SlotsNewer = true;
    UA.MarkStale(UnitAllocator::AllFields());
    CA.MarkStale(ConnAllocator::AllFields());
    ++Step;
    return true;
  }

  void Release() {
    if (Stream) cudaStreamSynchronize(Stream);
    else cudaDeviceSynchronize();
    if (GraphExec) cudaGraphExecDestroy(GraphExec);
    GraphExec = nullptr;
    if (OwnStream) cudaStreamDestroy(OwnStream);
    OwnStream = nullptr;
    for (void *p : Fused.Mem)
      if (p) cudaFree(p);
    if (Fused.Copy) {
      cudaStreamSynchronize(Fused.Copy);
      cudaStreamDestroy(Fused.Copy);
      for (int b = 0; b < 2; ++b) {
        cudaFree(Fused.In[b]);
        cudaEventDestroy(Fused.InReady[b]);
        cudaEventDestroy(Fused.Swept[b]);
      }
    }
    if (OutHost) cudaFreeHost(OutHost);
    OutHost = nullptr;
    for (StagingPair *pair : {&InStage, &TargetStage})
      for (Staging &b : pair->B) {
        if (b.Host) cudaFreeHost(b.Host);
        if (b.Done) cudaEventDestroy(b.Done);
        b = Staging{};
      }
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
  mutable UnitAllocator UA;
  mutable ConnAllocator CA;
  GlobalState HostG{};
  int NumLevels = 0;
  size_t Step = 0;
  int Device = 0;
  std::vector<void *> d_uf, d_cf;
  size_t DevUnits = static_cast<size_t>(-1), DevConns = static_cast<size_t>(-1);
  GlobalState *d_g = nullptr;
  uint32_t *d_in_ptr = nullptr, *d_out_ptr = nullptr, *d_in_conn = nullptr, *d_out_conn = nullptr;
  uint32_t *d_cursor = nullptr, *d_ranges = nullptr;
  float *d_targets = nullptr;
  size_t TargetCap = 0;
  bool NeedsResort = false, IndexStale = true, DstMajor = false;
  FusedState Fused;
  int NumSMs = 148;
  uint64_t ProposalCap = uint64_t(1) << 26;
  cudaStream_t Stream = nullptr;
  plx_ctx *Ctx = nullptr;
  void *Scratch[16] = {};
  size_t ScratchBytes[16] = {};
  mutable float *OutHost = nullptr;
  mutable size_t OutCap = 0;
};

}  // namespace plastix
