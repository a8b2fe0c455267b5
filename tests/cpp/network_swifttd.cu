// The SwiftTD learner through the device Network<Traits>: one linear value
// unit over N features, the ten per-feature values as connection fields, the
// TD(lambda) step with meta-learned step sizes split over Loss /
// UpdateIncomingConnection (phase 1, reductions into the globals) /
// UpdateOutgoingConnection (phase 2) / ResetGlobal -- the rule set of the
// reference's swifttd example, written here with PLASTIX_HD policies. The
// per-connection hooks add into the globals, so the traits ask for the
// sequential connection update.
//
// usage: network_swifttd <in_dir>  (features.bin steps x n, rewards.bin, n in argv[2])
// prints V per step and the final W and Beta as hex floats.
#include <plastix/plastix.hpp>

#include <cmath>
#include <cstdio>
#include <fstream>
#include <string>
#include <vector>

namespace {

struct Z {};
struct Zd {};
struct Dw {};
struct H {};
struct HOld {};
struct HTemp {};
struct ZBar {};
struct P {};
struct Beta {};

struct Globals {
  float Gamma = 1.0f, Lambda = 0.9f, Eta = 0.05f, EtaMin = 1e-7f, Decay = 0.999f, Meta = 1e-3f;
  float V = 0.0f, VOld = 0.0f, Delta = 0.0f, VDeltaPrev = 0.0f, VDelta = 0.0f, Tau = 0.0f,
        B = 0.0f;
};

struct Init {
  void operator()(auto &CA, auto Id) const {
    plastix::GetField<Beta>(CA, Id) = std::log(0.05f);
  }
};

struct Forward {
  using Accumulator = float;
  PLASTIX_HD static float Map(auto &U, size_t, size_t Src, auto &C, size_t Id, auto &) {
    return plastix::GetWeight(C, Id) * plastix::GetActivation(U, Src);
  }
  PLASTIX_HD static float Combine(float A, float B) { return A + B; }
  PLASTIX_HD static void Apply(auto &U, size_t Id, auto &G, float Acc) {
    plastix::GetActivation(U, Id) = Acc;
    G.V = Acc;
  }
};

struct Loss {
  PLASTIX_HD static void CalculateLoss(auto &, plastix::UnitRange, std::span<const float> T,
                                       auto &G) {
    G.Delta = T[0] + G.Gamma * G.V - G.VOld;
    G.VDeltaPrev = G.VDelta;
    G.VDelta = 0.0f;
    G.Tau = 0.0f;
    G.B = 0.0f;
  }
};

struct Update {
  PLASTIX_HD static void UpdateIncomingConnection(auto &U, size_t, size_t Src, auto &C, size_t Id,
                                                  auto &G) {
    using plastix::GetField;
    const float F = plastix::GetActivation(U, Src);
    float &w = plastix::GetWeight(C, Id), &z = GetField<Z>(C, Id), &zd = GetField<Zd>(C, Id);
    float &dw = GetField<Dw>(C, Id), &h = GetField<H>(C, Id), &ho = GetField<HOld>(C, Id);
    float &ht = GetField<HTemp>(C, Id), &zb = GetField<ZBar>(C, Id), &p = GetField<P>(C, Id);
    float &be = GetField<Beta>(C, Id);
    dw = G.Delta * z - zd * G.VDeltaPrev;
    w += dw;
    be += G.Meta / std::exp(be) * (G.Delta - G.VDeltaPrev) * p;
    float eb = std::exp(be);
    if (eb > G.Eta || std::isinf(eb)) {
      be = std::log(G.Eta);
      eb = G.Eta;
    }
    if (eb < G.EtaMin) {
      be = std::log(G.EtaMin);
      eb = G.EtaMin;
    }
    ho = h;
    h = ht + G.Delta * zb - zd * G.VDeltaPrev;
    ht = h;
    zd = 0.0f;
    const float td = G.Gamma * G.Lambda;
    z *= td;
    p *= td;
    zb *= td;
    G.Tau += eb * F * F;
    G.B += z * F;
  }
  PLASTIX_HD static void UpdateOutgoingConnection(auto &U, size_t Src, size_t, auto &C, size_t Id,
                                                  auto &G) {
    using plastix::GetField;
    const float F = plastix::GetActivation(U, Src);
    float &z = GetField<Z>(C, Id), &zd = GetField<Zd>(C, Id), &dw = GetField<Dw>(C, Id);
    float &h = GetField<H>(C, Id), &ho = GetField<HOld>(C, Id), &ht = GetField<HTemp>(C, Id);
    float &zb = GetField<ZBar>(C, Id), &p = GetField<P>(C, Id), &be = GetField<Beta>(C, Id);
    G.VDelta += dw * F;
    float mult = 1.0f;
    if (G.Tau > 0.0f && G.Eta / G.Tau < 1.0f) mult = G.Eta / G.Tau;
    zd = mult * std::exp(be) * F;
    z += zd * (1.0f - G.B);
    p += ho * F;
    zb += zd * (1.0f - G.B - zb * F);
    ht = h - ho * F * (z - zd) - h * zd * F;
    if (G.Tau > G.Eta) {
      ht = 0.0f;
      h = 0.0f;
      ho = 0.0f;
      zb = 0.0f;
      be += std::log(G.Decay) * F * F;
    }
  }
};

struct ResetV {
  PLASTIX_HD static void Reset(auto &G) { G.VOld = G.V; }
};

struct Traits : plastix::DefaultNetworkTraits<Globals> {
  using ForwardPass = Forward;
  using Loss = ::Loss;
  using UpdateConn = Update;
  using ResetGlobal = ResetV;
  using ExtraConnFields = plastix::ConnFieldList<
      plastix::alloc::SOAField<plastix::WeightTag, float>, plastix::alloc::SOAField<Z, float>,
      plastix::alloc::SOAField<Zd, float>, plastix::alloc::SOAField<Dw, float>,
      plastix::alloc::SOAField<H, float>, plastix::alloc::SOAField<HOld, float>,
      plastix::alloc::SOAField<HTemp, float>, plastix::alloc::SOAField<ZBar, float>,
      plastix::alloc::SOAField<P, float>, plastix::alloc::SOAField<Beta, float>>;
  static constexpr bool SequentialConnectionUpdate = true;  // hooks add into globals
};

}  // namespace

int main(int argc, char **argv) {
  const std::string dir = argv[1];
  const size_t n = std::stoul(argv[2]);
  std::ifstream rf(dir + "/rewards.bin", std::ios::binary | std::ios::ate);
  const size_t steps = (size_t)rf.tellg() / 4;
  rf.seekg(0);
  std::vector<float> rewards(steps), feats(steps * n);
  rf.read(reinterpret_cast<char *>(rewards.data()), (std::streamsize)(steps * 4));
  std::ifstream ff(dir + "/features.bin", std::ios::binary);
  ff.read(reinterpret_cast<char *>(feats.data()), (std::streamsize)(feats.size() * 4));
  plastix::Network<Traits> Net(n, plastix::FullyConnected{1, Init{}});
  for (size_t s = 0; s < steps; ++s) {
    const float r[1] = {rewards[s]};
    Net.DoStep(std::span<const float>(feats.data() + s * n, n), std::span<const float>(r, 1));
    std::printf("v %a\n", (double)Net.GetOutput()[0]);
  }
  auto &C = Net.GetConnAlloc();
  for (size_t c = 0; c < n; ++c) std::printf("w %a\n", (double)plastix::GetWeight(C, c));
  for (size_t c = 0; c < n; ++c) std::printf("b %a\n", (double)plastix::GetField<Beta>(C, c));
  return 0;
}
