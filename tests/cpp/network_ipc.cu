// Streaming iPC (3 inputs -> 16 tanh hidden -> 1 output, Pipeline
// propagation) through the device Network<Traits>: forward with
// eps = x - mu, backward into a bottom-up field, Hebbian weight update, the
// pre-step and value-node update done on the host through GetUnitAlloc() --
// the rule set and step order of the reference's ipc-multilayer example,
// written here with PLASTIX_HD policies.
//
// usage: network_ipc <in_dir>   (reads w0.bin, x0.bin, inputs.bin, targets.bin)
// prints final weights, value nodes and errors as hex floats.
#include <plastix/plastix.hpp>

#include <cmath>
#include <cstdio>
#include <fstream>
#include <string>
#include <vector>

namespace {

struct ValueTag {};
struct ErrTag {};
struct BottomUpTag {};
constexpr size_t kIn = 3, kHidden = 16, kHiddenBegin = kIn, kHiddenEnd = kIn + kHidden;
constexpr float kAlpha = 0.005f, kGamma = 0.1f;

PLASTIX_HD inline float act_deriv(float x) {
  const float t = std::tanh(x);
  return 1.0f - t * t;
}

struct Forward {
  using Accumulator = float;
  PLASTIX_HD static float Map(auto &U, size_t, size_t Src, auto &C, size_t Id, auto &) {
    return plastix::GetWeight(C, Id) * plastix::GetActivation(U, Src);
  }
  PLASTIX_HD static float Combine(float A, float B) { return A + B; }
  PLASTIX_HD static void Apply(auto &U, size_t Id, auto &, float Mu) {
    plastix::GetField<ErrTag>(U, Id) = plastix::GetField<ValueTag>(U, Id) - Mu;
  }
};

struct Backward {
  using Accumulator = float;
  PLASTIX_HD static float Map(auto &U, size_t, size_t To, auto &C, size_t Id, auto &) {
    return plastix::GetWeight(C, Id) * plastix::GetField<ErrTag>(U, To);
  }
  PLASTIX_HD static float Combine(float A, float B) { return A + B; }
  PLASTIX_HD static void Apply(auto &U, size_t Id, auto &, float Acc) {
    if (Id >= kHiddenBegin && Id < kHiddenEnd)
      plastix::GetField<BottomUpTag>(U, Id) = act_deriv(plastix::GetField<ValueTag>(U, Id)) * Acc;
  }
};

struct Hebbian {
  PLASTIX_HD static void UpdateIncomingConnection(auto &U, size_t Dst, size_t Src, auto &C,
                                                  size_t Id, auto &) {
    const float x = plastix::GetField<ValueTag>(U, Src);
    const float fx = Src < kIn ? x : std::tanh(x);
    plastix::GetWeight(C, Id) += kAlpha * plastix::GetField<ErrTag>(U, Dst) * fx;
  }
  PLASTIX_HD static void UpdateOutgoingConnection(auto &, size_t, size_t, auto &, size_t,
                                                  auto &) {}
};

struct Traits : plastix::DefaultNetworkTraits<> {
  using ForwardPass = Forward;
  using BackwardPass = Backward;
  using UpdateConn = Hebbian;
  using ExtraUnitFields =
      plastix::UnitFieldList<plastix::alloc::SOAField<ValueTag, float>,
                             plastix::alloc::SOAField<ErrTag, float>,
                             plastix::alloc::SOAField<BottomUpTag, float>>;
  static constexpr plastix::Propagation Model = plastix::Propagation::Pipeline;
};

std::vector<float> read_f32(const std::string &p, size_t n) {
  std::vector<float> v(n);
  std::ifstream f(p, std::ios::binary);
  f.read(reinterpret_cast<char *>(v.data()), (std::streamsize)(n * 4));
  if (!f) throw std::runtime_error("cannot read " + p);
  return v;
}

}  // namespace

int main(int argc, char **argv) {
  const std::string dir = argc > 1 ? argv[1] : ".";
  plastix::Network<Traits> Net(kIn, plastix::FullyConnected<>{kHidden},
                               plastix::FullyConnected<>{1});
  const size_t n_conn = kIn * kHidden + kHidden, n_units = kIn + kHidden + 1;
  auto w0 = read_f32(dir + "/w0.bin", n_conn);
  auto x0 = read_f32(dir + "/x0.bin", n_units);
  std::ifstream tf(dir + "/targets.bin", std::ios::binary | std::ios::ate);
  const size_t steps = (size_t)tf.tellg() / 4;
  auto inputs = read_f32(dir + "/inputs.bin", steps * kIn);
  auto targets = read_f32(dir + "/targets.bin", steps);
  {
    auto &C = Net.GetConnAlloc();
    for (size_t c = 0; c < n_conn; ++c) plastix::GetWeight(C, c) = w0[c];
    auto &U = Net.GetUnitAlloc();
    for (size_t i = 0; i < n_units; ++i) plastix::GetField<ValueTag>(U, i) = x0[i];
  }
  for (size_t t = 0; t < steps; ++t) {
    const float *in = inputs.data() + t * kIn;
    auto &U = Net.GetUnitAlloc();
    for (size_t i = 0; i < kIn; ++i) plastix::GetField<ValueTag>(U, i) = in[i];
    plastix::GetField<ValueTag>(U, n_units - 1) = targets[t];
    for (size_t i = kIn; i < n_units; ++i) {  // pre-step: Activation = f(x)
      const float x = plastix::GetField<ValueTag>(U, i);
      plastix::GetActivation(U, i) = (i >= kHiddenBegin && i < kHiddenEnd) ? std::tanh(x) : x;
    }
    Net.DoForwardPass(std::span<const float>(in, kIn));
    Net.DoBackwardPass();
    Net.DoUpdateConnectionState();
    auto &U2 = Net.GetUnitAlloc();  // value-node update of the hidden units
    for (size_t i = kHiddenBegin; i < kHiddenEnd; ++i) {
      const float e = plastix::GetField<ErrTag>(U2, i), bu = plastix::GetField<BottomUpTag>(U2, i);
      plastix::GetField<ValueTag>(U2, i) += kGamma * (-e + bu);
      plastix::GetField<BottomUpTag>(U2, i) = 0.0f;
    }
  }
  auto &C = Net.GetConnAlloc();
  for (size_t c = 0; c < n_conn; ++c) std::printf("w %a\n", (double)plastix::GetWeight(C, c));
  auto &U = Net.GetUnitAlloc();
  for (size_t i = 0; i < n_units; ++i) std::printf("x %a\n", (double)plastix::GetField<ValueTag>(U, i));
  for (size_t i = 0; i < n_units; ++i) std::printf("e %a\n", (double)plastix::GetField<ErrTag>(U, i));
  return 0;
}
