// The XOR MLP through the device Network<Traits> (include/plastix/plastix.hpp):
// sigmoid units in Topological propagation, MSE loss, backward pass into a
// per-unit gradient field, gradient-descent connection update -- the rule set
// of the reference's mlp-xor example, written here with PLASTIX_HD policies.
// Prints the initial and final weights and the final predictions, one value
// per line as hex floats, for the test to compare with the reference.
#include <plastix/plastix.hpp>

#include <cmath>
#include <cstdio>
#include <string>

namespace {

struct GradTag {};
constexpr float kRate = 0.5f;

struct SigmoidForward {
  using Accumulator = float;
  PLASTIX_HD static float Map(auto &U, size_t, size_t Src, auto &C, size_t Id, auto &) {
    return plastix::GetWeight(C, Id) * plastix::GetActivation(U, Src);
  }
  PLASTIX_HD static float Combine(float A, float B) { return A + B; }
  PLASTIX_HD static void Apply(auto &U, size_t Id, auto &, float Acc) {
    plastix::GetActivation(U, Id) = 1.0f / (1.0f + std::exp(-Acc));
  }
};

struct SigmoidBackward {
  using Accumulator = float;
  PLASTIX_HD static float Map(auto &U, size_t, size_t To, auto &C, size_t Id, auto &) {
    return plastix::GetWeight(C, Id) * plastix::GetField<GradTag>(U, To);
  }
  PLASTIX_HD static float Combine(float A, float B) { return A + B; }
  PLASTIX_HD static void Apply(auto &U, size_t Id, auto &, float Acc) {
    const float A = plastix::GetActivation(U, Id);
    plastix::GetField<GradTag>(U, Id) = Acc * A * (1.0f - A);
  }
};

struct GradientStep {
  PLASTIX_HD static void UpdateIncomingConnection(auto &U, size_t Dst, size_t Src, auto &C,
                                                  size_t Id, auto &) {
    plastix::GetWeight(C, Id) -= kRate * plastix::GetField<GradTag>(U, Dst) *
                                 plastix::GetActivation(U, Src);
  }
  PLASTIX_HD static void UpdateOutgoingConnection(auto &, size_t, size_t, auto &, size_t,
                                                  auto &) {}
};

struct Traits : plastix::DefaultNetworkTraits<> {
  using ForwardPass = SigmoidForward;
  using BackwardPass = SigmoidBackward;
  using Loss = plastix::MSELoss;
  using UpdateConn = GradientStep;
  using ExtraUnitFields = plastix::UnitFieldList<plastix::alloc::SOAField<GradTag, float>>;
};

void dump(const char *name, float v) { std::printf("%s %a\n", name, (double)v); }

}  // namespace

int main(int argc, char **argv) {
  const int epochs = argc > 1 ? std::stoi(argv[1]) : 200;
  plastix::Network<Traits> Net(2, plastix::FullyConnected{8, plastix::RandomUniformWeight{1234}},
                               plastix::FullyConnected{1, plastix::RandomUniformWeight{1234}});
  auto &C0 = Net.GetConnAlloc();
  for (size_t c = 0; c < C0.Size(); ++c) dump("w0", plastix::GetWeight(C0, c));
  const float In[4][2] = {{0, 0}, {0, 1}, {1, 0}, {1, 1}};
  const float Tg[4] = {0, 1, 1, 0};
  for (int e = 0; e < epochs; ++e)
    for (int s = 0; s < 4; ++s) {
      const float t[1] = {Tg[s]};
      Net.DoStep(std::span<const float>(In[s], 2), std::span<const float>(t, 1));
    }
  auto &C1 = Net.GetConnAlloc();
  for (size_t c = 0; c < C1.Size(); ++c) dump("w", plastix::GetWeight(C1, c));
  for (int s = 0; s < 4; ++s) {
    Net.DoForwardPass(std::span<const float>(In[s], 2));
    dump("p", Net.GetOutput()[0]);
  }
  return 0;
}
