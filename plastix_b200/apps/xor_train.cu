// The XOR MLP training run (2 inputs -> 8 sigmoid hidden -> 1 sigmoid output,
// MSE loss, backward pass, gradient descent at rate 0.5, four DoSteps per
// epoch, each followed by GetOutput -- the mlp-xor example's loop) written
// against the reference's C++ API. The same source builds two ways:
//   * with nvcc against this repository's headers: the device Network, whose
//     DoStep runs as one kernel of one CTA (argument "single", the default
//     for a network this small), replays a captured CUDA graph ("graph") or
//     launches every kernel of the step ("eager");
//   * with a host C++ compiler against the reference's own headers: the
//     reference's CPU implementation (the baseline of the benchmark).
// Usage: xor_train <epochs> [single|graph|eager]
// Prints one JSON object: training wall time (host clock around the epoch
// loop only), steps, the last epoch's loss and whether all four XOR cases
// are classified correctly afterwards.
#ifndef PLASTIX_HD
#define PLASTIX_HD
#endif
#include <plastix/plastix.hpp>

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <span>

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

struct XorTraits : plastix::DefaultNetworkTraits<> {
  using ForwardPass = SigmoidForward;
  using BackwardPass = SigmoidBackward;
  using Loss = plastix::MSELoss;
  using UpdateConn = GradientStep;
  using ExtraUnitFields = plastix::UnitFieldList<plastix::alloc::SOAField<GradTag, float>>;
};

}  // namespace

int main(int argc, char **argv) {
  const long epochs = argc > 1 ? std::atol(argv[1]) : 5000;
  const char *mode = argc > 2 ? argv[2] : "single";
  plastix::Network<XorTraits> Net(2, plastix::FullyConnected{8, plastix::RandomUniformWeight{1234}},
                                  plastix::FullyConnected{1, plastix::RandomUniformWeight{1234}});
#ifdef __CUDACC__
  Net.SetSingleKernelStep(std::strcmp(mode, "single") == 0);
  Net.SetGraphReplay(std::strcmp(mode, "graph") == 0);
  const char *impl = std::strcmp(mode, "single") == 0  ? "device, one kernel per step"
                     : std::strcmp(mode, "graph") == 0 ? "device, graph replay"
                                                       : "device, every pass launched";
#else
  (void)mode;
  const char *impl = "reference (host)";
#endif
  const float In[4][2] = {{0, 0}, {0, 1}, {1, 0}, {1, 1}};
  const float Tg[4] = {0, 1, 1, 0};
  float loss = 0.0f;
  const auto t0 = std::chrono::steady_clock::now();
  for (long e = 0; e < epochs; ++e) {
    loss = 0.0f;
    for (int s = 0; s < 4; ++s) {
      const float t[1] = {Tg[s]};
      Net.DoStep(std::span<const float>(In[s], 2), std::span<const float>(t, 1));
      const float d = Net.GetOutput()[0] - Tg[s];
      loss += 0.5f * d * d;
    }
  }
  const double secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  bool ok = true;
  for (int s = 0; s < 4; ++s) {
    Net.DoForwardPass(std::span<const float>(In[s], 2));
    ok = ok && ((Net.GetOutput()[0] > 0.5f) == (Tg[s] > 0.5f));
  }
  std::printf("{\"impl\": \"%s\", \"train_s\": %.6f, \"steps\": %ld, \"final_loss\": %.6e, "
              "\"pass\": %s}\n",
              impl, secs, 4 * epochs, (double)loss, ok ? "true" : "false");
  return ok ? 0 : 1;
}
