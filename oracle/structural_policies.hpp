// structural_policies.hpp -- TEST INFRASTRUCTURE ONLY. Side-effect-free
// structural policies (prune units, prune connections, add connections) for
// the structural parity test, written once and compiled twice: against the
// reference's headers in oracle/ref_harness.cpp and against this
// repository's device Network in tests/cpp/network_structural.cu. Both sides
// name the same plastix:: accessors, so the two networks follow the same rules.
#pragma once
#ifndef PLASTIX_HD
#define PLASTIX_HD
#endif
#include <cmath>
#include <cstddef>
#include <cstdint>

namespace structural_test {

struct Globals {
  uint32_t Step = 0;
};

PLASTIX_HD inline uint32_t mix(uint32_t a, uint32_t b, uint32_t s) {
  uint32_t h = a * 0x9E3779B1u ^ b * 0x85EBCA77u ^ s * 0xC2B2AE3Du;
  h ^= h >> 15;
  h *= 0x2C1B3C6Du;
  h ^= h >> 12;
  return h;
}

// w * act summed, activation clamped to [-4, 4].
struct ClampForward {
  using Accumulator = float;
  PLASTIX_HD static float Map(auto &U, size_t, size_t Src, auto &C, size_t Id, auto &) {
    return plastix::GetWeight(C, Id) * plastix::GetActivation(U, Src);
  }
  PLASTIX_HD static float Combine(float A, float B) { return A + B; }
  PLASTIX_HD static void Apply(auto &U, size_t Id, auto &, float Acc) {
    plastix::GetActivation(U, Id) = Acc < -4.0f ? -4.0f : (Acc > 4.0f ? 4.0f : Acc);
  }
};

struct Hebbian {
  PLASTIX_HD static void UpdateIncomingConnection(auto &U, size_t Dst, size_t Src, auto &C,
                                                  size_t Id, auto &) {
    plastix::GetWeight(C, Id) +=
        0.01f * plastix::GetActivation(U, Src) * plastix::GetActivation(U, Dst);
  }
  PLASTIX_HD static void UpdateOutgoingConnection(auto &, size_t, size_t, auto &, size_t,
                                                  auto &) {}
};

// Unit 9 is pruned during the second step (its connections die).
struct PruneOneUnit {
  PLASTIX_HD static bool ShouldPrune(auto &, size_t Id, Globals &G) {
    return G.Step == 1 && Id == 9;
  }
};

struct PruneSmallWeights {
  PLASTIX_HD static bool ShouldPrune(auto &, size_t, size_t, auto &C, size_t Id, Globals &) {
    return std::fabs(plastix::GetWeight(C, Id)) < 0.02f;
  }
};

// Hash-chosen proposals, a weight that depends on both endpoints. Two-way
// (Forward false): any pair, into input units too, so cycles appear and units
// fall out of the level order. Forward: only from a lower to a higher unit
// id (units are numbered layer by layer), so the network stays acyclic.
template <uint32_t PIn, uint32_t POut, bool Forward> struct HashAdd {
  PLASTIX_HD static bool ShouldAddIncomingConnection(auto &, size_t Self, size_t Cand,
                                                     Globals &G) {
    if (Forward && Cand >= Self) return false;
    return mix((uint32_t)Self, (uint32_t)Cand, G.Step) % PIn == 0;
  }
  PLASTIX_HD static bool ShouldAddOutgoingConnection(auto &, size_t Self, size_t Cand,
                                                     Globals &G) {
    if (Forward && Self >= Cand) return false;
    return mix((uint32_t)Cand, (uint32_t)Self, G.Step + 7u) % POut == 0;
  }
  PLASTIX_HD static void InitConnection(auto &, size_t F, size_t T, auto &C, size_t Id,
                                        Globals &) {
    plastix::GetWeight(C, Id) = 0.05f * (float)((F * 7 + T * 3) % 11) - 0.25f;
  }
};

struct StepCounter {
  PLASTIX_HD static void Reset(Globals &G) { G.Step += 1; }
};

template <uint32_t PIn, uint32_t POut, bool Forward>
struct Traits : plastix::DefaultNetworkTraits<Globals> {
  using ForwardPass = ClampForward;
  using UpdateConn = Hebbian;
  using PruneUnit = PruneOneUnit;
  using PruneConn = PruneSmallWeights;
  using AddConn = HashAdd<PIn, POut, Forward>;
  using ResetGlobal = StepCounter;
};

// The two configurations: a small network (4 -> 6 -> 3) with frequent
// two-way proposals, a medium one (32 -> 200 -> 50) with rarer forward
// proposals over many more unit pairs.
using SmallTraits = Traits<23, 29, false>;
using MediumTraits = Traits<97, 101, true>;

}  // namespace structural_test
