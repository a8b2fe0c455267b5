// Structural parity program: the pure prune / add-connection policies of
// oracle/structural_policies.hpp on the device Network (Topological), the
// same network and inputs as the reference run that made the fixture.
// Usage: network_structural <variant> <n_in> <h1> <h2> <seed> <steps> <dir>
//        [resume_at]
// Variants 0 (small) and 1 (medium) use the traits as written: the global
// state is not declared read-only, so the hooks that receive it run in one
// device thread, and the structural decisions run on the host copy.
// Variants 2 and 3 are the same networks with DeviceStructure and
// ReadOnlyGlobalState: parallel passes, and pruning predicates and
// connection proposals enumerated on the device.
// Reads <dir>/inputs.bin (steps x n_in floats); writes outputs.bin and the
// final connections (from, to, dead, src_level, w) and units (level, act).
// With resume_at, the network is saved before that step and the run goes on
// in a newly built network loaded from the checkpoint.
#include <plastix/plastix.hpp>

#include "../../oracle/structural_policies.hpp"

#include <cstdio>
#include <cstdlib>
#include <memory>
#include <string>
#include <vector>

namespace {

template <class Base> struct OnDevice : Base {
  static constexpr bool DeviceStructure = true;
  static constexpr bool ReadOnlyGlobalState = true;  // only ResetGlobal writes it
};

template <class T> void put(const std::string &dir, const char *name, const std::vector<T> &v) {
  FILE *f = std::fopen((dir + "/" + name).c_str(), "wb");
  if (!f) std::exit(3);
  if (!v.empty()) std::fwrite(v.data(), sizeof(T), v.size(), f);
  std::fclose(f);
}

template <class Tr> int run(uint32_t n_in, uint32_t h1, uint32_t h2, uint32_t seed, int steps,
                            const std::string &dir, int resume_at) {
  std::vector<float> x((size_t)steps * n_in);
  FILE *f = std::fopen((dir + "/inputs.bin").c_str(), "rb");
  if (!f || std::fread(x.data(), 4, x.size(), f) != x.size()) return 2;
  std::fclose(f);
  auto make = [&] {
    return std::make_unique<plastix::Network<Tr>>(
        n_in, plastix::FullyConnected{h1, plastix::RandomUniformWeight{seed, -0.3f, 0.3f}},
        plastix::FullyConnected{h2, plastix::RandomUniformWeight{seed + 1, -0.3f, 0.3f}});
  };
  auto net = make();
  std::vector<float> outs;
  for (int s = 0; s < steps; ++s) {
    if (s == resume_at) {
      // checkpoint, then continue in a freshly built network from the file
      net->Save(dir + "/ckpt.bin");
      net = make();
      net->Load(dir + "/ckpt.bin");
    }
    net->DoStep(std::span<const float>(x.data() + (size_t)s * n_in, n_in));
    auto o = net->GetOutput();
    outs.insert(outs.end(), o.begin(), o.end());
  }
  auto &N = *net;
  auto &CA = N.GetConnAlloc();
  auto &UA = N.GetUnitAlloc();
  const size_t m = CA.Size(), n = UA.Size();
  std::vector<uint32_t> from(m), to(m);
  std::vector<uint8_t> dead(m);
  std::vector<uint16_t> sl(m), level(n);
  std::vector<float> w(m), act(n);
  for (size_t c = 0; c < m; ++c) {
    from[c] = plastix::GetField<plastix::FromIdTag>(CA, c);
    to[c] = plastix::GetField<plastix::ToIdTag>(CA, c);
    dead[c] = plastix::GetField<plastix::DeadTag>(CA, c) ? 1 : 0;
    sl[c] = plastix::GetField<plastix::SrcLevelTag>(CA, c);
    w[c] = plastix::GetWeight(CA, c);
  }
  for (size_t i = 0; i < n; ++i) {
    level[i] = plastix::GetLevel(UA, i);
    act[i] = plastix::GetActivation(UA, i);
  }
  put(dir, "outputs.bin", outs);
  put(dir, "from.bin", from);
  put(dir, "to.bin", to);
  put(dir, "dead.bin", dead);
  put(dir, "src_level.bin", sl);
  put(dir, "w.bin", w);
  put(dir, "level.bin", level);
  put(dir, "act.bin", act);
  return 0;
}

}  // namespace

int main(int argc, char **argv) {
  if (argc != 8 && argc != 9) return 1;
  const int resume_at = argc == 9 ? std::atoi(argv[8]) : -1;
  const int variant = std::atoi(argv[1]);
  const uint32_t n_in = std::atoi(argv[2]), h1 = std::atoi(argv[3]), h2 = std::atoi(argv[4]);
  const uint32_t seed = std::atoi(argv[5]);
  const int steps = std::atoi(argv[6]);
  try {
    using namespace structural_test;
    switch (variant) {
      case 0: return run<SmallTraits>(n_in, h1, h2, seed, steps, argv[7], resume_at);
      case 1: return run<MediumTraits>(n_in, h1, h2, seed, steps, argv[7], resume_at);
      case 2: return run<OnDevice<SmallTraits>>(n_in, h1, h2, seed, steps, argv[7], resume_at);
      case 3: return run<OnDevice<MediumTraits>>(n_in, h1, h2, seed, steps, argv[7], resume_at);
      default: return 1;
    }
  } catch (const std::exception &e) {
    std::fprintf(stderr, "%s\n", e.what());
    return 4;
  }
}
