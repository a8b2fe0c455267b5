// MSELoss and the ways DoStep runs inside the device Network<Traits>: the
// library's MSELoss runs in the forward pass's Apply epilogue under DoStep
// (Pipeline) and as a parallel per-output kernel under DoCalculateLoss; a
// user loss with the same body is not recognised and runs as the generic
// one-thread loss hook; DoStep runs as one kernel of one CTA (small
// networks), as a replayed CUDA graph, or launching every pass. All of them
// must leave every weight, activation, gradient and backward accumulator
// equal bit for bit. The network: 3 inputs -> 48 sigmoid hidden -> 20 sigmoid
// outputs, backward pass and gradient step, 40 DoSteps on seeded inputs and
// targets, in both propagation models. Prints "ok" or the mismatches; the
// exit code is the number of mismatching variants.
#include <plastix/plastix.hpp>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

namespace {

struct GradTag {};
constexpr float kRate = 0.25f;

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

// The same rule as plastix::MSELoss, as a user policy.
struct UserMSE {
  PLASTIX_HD static void CalculateLoss(auto &U, plastix::UnitRange Outputs,
                                       std::span<const float> Targets, auto &) {
    size_t I = 0;
    for (size_t Id = Outputs.Begin; Id < Outputs.End; ++Id)
      plastix::GetBackwardAcc(U, Id) = plastix::GetActivation(U, Id) - Targets[I++];
  }
};

template <class LossT, plastix::Propagation M> struct Traits : plastix::DefaultNetworkTraits<> {
  using ForwardPass = SigmoidForward;
  using BackwardPass = SigmoidBackward;
  using Loss = LossT;
  using UpdateConn = GradientStep;
  using ExtraUnitFields = plastix::UnitFieldList<plastix::alloc::SOAField<GradTag, float>>;
  static constexpr plastix::Propagation Model = M;
};

constexpr int kIn = 3, kHidden = 48, kOut = 20, kSteps = 40;

struct Snapshot {
  std::vector<float> w, act, grad, bwd;
};

enum Mode { kSplit, kSingleKernel, kGraph, kEager };

// kSplit: the step as separate Do* calls (DoCalculateLoss on its own);
// kSingleKernel: DoStep as one kernel (the default for a network this
// small); kGraph: DoStep replayed as a captured CUDA graph; kEager: DoStep
// launching every pass.
template <class T> Snapshot run(Mode mode) {
  plastix::Network<T> Net(kIn, plastix::FullyConnected{kHidden, plastix::RandomUniformWeight{7}},
                          plastix::FullyConnected{kOut, plastix::RandomUniformWeight{8}});
  Net.SetSingleKernelStep(mode == kSingleKernel);
  Net.SetGraphReplay(mode == kGraph);
  const bool split = mode == kSplit;
  uint32_t h = 12345u;
  auto next = [&h] {
    h = h * 1664525u + 1013904223u;
    return (float)(h >> 8) * (1.0f / 16777216.0f);
  };
  float in[kIn], tg[kOut];
  for (int s = 0; s < kSteps; ++s) {
    for (float &v : in) v = next();
    for (float &v : tg) v = next();
    const std::span<const float> I(in, kIn), Tg(tg, kOut);
    if (split) {
      Net.DoForwardPass(I);
      Net.DoCalculateLoss(Tg);
      Net.DoBackwardPass();
      Net.DoUpdateUnitState();
      Net.DoUpdateConnectionState();
    } else {
      Net.DoStep(I, Tg);
    }
  }
  Snapshot S;
  auto &C = Net.GetConnAlloc();
  for (size_t c = 0; c < C.Size(); ++c) S.w.push_back(plastix::GetWeight(C, c));
  auto &U = Net.GetUnitAlloc();
  for (size_t i = 0; i < U.Size(); ++i) {
    S.act.push_back(plastix::GetActivation(U, i));
    S.grad.push_back(plastix::GetField<GradTag>(U, i));
    S.bwd.push_back(plastix::GetBackwardAcc(U, i));
  }
  return S;
}

bool same(const std::vector<float> &a, const std::vector<float> &b) {
  return a.size() == b.size() && std::memcmp(a.data(), b.data(), a.size() * 4) == 0;
}

int compare(const char *what, const Snapshot &a, const Snapshot &b) {
  const bool ok = same(a.w, b.w) && same(a.act, b.act) && same(a.grad, b.grad) &&
                  same(a.bwd, b.bwd);
  if (!ok) std::printf("mismatch %s\n", what);
  return ok ? 0 : 1;
}

}  // namespace

int main() {
  using plastix::MSELoss;
  using plastix::Propagation;
  int bad = 0;
  const char *names[] = {"split Do* calls", "single-kernel DoStep", "graph-replayed DoStep",
                         "eager DoStep"};
  auto check = [&](const char *model, const Snapshot &want, const Snapshot &got, const char *loss,
                   int mode) {
    char what[160];
    std::snprintf(what, sizeof what, "%s, %s loss, %s", model, loss, names[mode]);
    bad += compare(what, got, want);
  };
  {
    const Snapshot want = run<Traits<UserMSE, Propagation::Pipeline>>(kSplit);
    for (int m : {kSplit, kSingleKernel, kGraph, kEager}) {
      check("pipeline", want, run<Traits<MSELoss, Propagation::Pipeline>>(Mode(m)), "library", m);
      check("pipeline", want, run<Traits<UserMSE, Propagation::Pipeline>>(Mode(m)), "user", m);
    }
  }
  {
    const Snapshot want = run<Traits<UserMSE, Propagation::Topological>>(kSplit);
    for (int m : {kSplit, kSingleKernel, kGraph, kEager}) {
      check("topological", want, run<Traits<MSELoss, Propagation::Topological>>(Mode(m)),
            "library", m);
      check("topological", want, run<Traits<UserMSE, Propagation::Topological>>(Mode(m)), "user",
            m);
    }
  }
  if (!bad) std::printf("ok\n");
  return bad;
}
