// The single-layer sweep (forward sum + Hebbian trace update) written against
// the reference's C++ API -- plastix::Network<Traits> with PLASTIX_HD
// policies -- and stepped with DoStep, the call a user of the header library
// makes. Used by the benchmark (workload "api": the reference API's own path
// on the GPU, timed end to end with host inputs and outputs) and by the
// parity test (small layers against the oracle).
//
// Usage:
//   network_sweep bench <n_src> <n_dst> <n_edges> <seed> <steps> <warmup> [generic|fused]
//     prints one JSON object: device ms per DoStep (CUDA events on the
//     network's stream) and end-to-end ms per step (DoStep from a host
//     input vector + GetOutput, host clock), construction time.
//   network_sweep check <dir> <steps> [generic|fused]
//     reads n_src n_dst n_edges (u64 x3), from, to (u32), weight, act (f32)
//     from <dir>/layer.bin, runs <steps> DoSteps, writes out.bin (final
//     destination activations), w.bin and e.bin (weights and traces in the
//     given connection order).
//   network_sweep check-edit <dir> <steps> [generic|fused]
//     as check, and after the first step reads trace n/3 on the host, adds
//     0.25 to weight 0 and -0.5 to weight n/2 and marks connections n/5 and
//     n/7 dead, through GetConnAlloc().
// The last argument picks the traits: "generic" (default) spells the rule
// out as a user hook; "fused" uses plastix::HebbianTraceUpdate, which DoStep
// runs as one fused sliced sweep.
#include <plastix/plastix.hpp>

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <type_traits>
#include <vector>

namespace {

struct TraceTag {};

// The Hebbian trace rule of the benchmark layer: e' = 0.9 e + pre * post,
// w' = w + 1e-3 e' (each product and sum rounded separately).
struct HebbianTrace {
  PLASTIX_HD static void UpdateIncomingConnection(auto &U, size_t Dst, size_t Src, auto &C,
                                                  size_t Id, auto &) {
    float &E = plastix::GetField<TraceTag>(C, Id);
    E = 0.9f * E + plastix::GetActivation(U, Src) * plastix::GetActivation(U, Dst);
    plastix::GetWeight(C, Id) += 1e-3f * E;
  }
  PLASTIX_HD static void UpdateOutgoingConnection(auto &, size_t, size_t, auto &, size_t,
                                                  auto &) {}
};

// Policies written out by the user: DoStep runs the generic device passes
// (tiled forward accumulation, then the per-connection update hook).
struct SweepTraits : plastix::DefaultNetworkTraits<> {
  using UpdateConn = HebbianTrace;
  using ExtraConnFields =
      plastix::ConnFieldList<plastix::alloc::SOAField<plastix::WeightTag, float>,
                             plastix::alloc::SOAField<TraceTag, float>>;
  static constexpr plastix::Propagation Model = plastix::Propagation::Pipeline;
};

// The same rule through the library's HebbianTraceUpdate policy: DoStep
// recognises it and runs the single fused sliced sweep.
struct FusedSweepTraits : plastix::DefaultNetworkTraits<> {
  using UpdateConn = plastix::HebbianTraceUpdate<0.9f, 1e-3f>;
  using ExtraConnFields =
      plastix::ConnFieldList<plastix::alloc::SOAField<plastix::WeightTag, float>,
                             plastix::alloc::SOAField<plastix::TraceTag, float>>;
  static constexpr plastix::Propagation Model = plastix::Propagation::Pipeline;
};
static_assert(plastix::detail::fused_hebbian_traits<FusedSweepTraits>());
static_assert(!plastix::detail::fused_hebbian_traits<SweepTraits>());

template <class Traits> using TraceOf =
    std::conditional_t<std::is_same_v<Traits, FusedSweepTraits>, plastix::TraceTag, TraceTag>;

// A LayerBuilder that appends n_dst units and the given destination-sorted
// connections (from: source unit ids, to: destination index in [0, n_dst)).
struct GivenConnections {
  const std::vector<uint32_t> *From, *To;
  const std::vector<float> *W;
  size_t NumUnits;
  template <class UA, class CA> plastix::UnitRange operator()(UA &U, CA &C, plastix::UnitRange Prev) const {
    const uint16_t Lvl = plastix::GetLevel(U, Prev.Begin) + 1;
    const plastix::UnitRange Units = U.AllocateMany(NumUnits);
    for (size_t I = Units.Begin; I < Units.End; ++I) plastix::GetLevel(U, I) = Lvl;
    const size_t n = From->size();
    C.AllocateMany(n);
    auto *f = C.template GetArrayFor<plastix::FromIdTag>();
    auto *t = C.template GetArrayFor<plastix::ToIdTag>();
    auto *w = C.template GetArrayFor<plastix::WeightTag>();
    for (size_t i = 0; i < n; ++i) {
      f[i] = (*From)[i];
      t[i] = (uint32_t)(Units.Begin + (*To)[i]);
      w[i] = (*W)[i];
    }
    return Units;
  }
};

uint64_t mix64(uint64_t x) {  // SplitMix64 finaliser
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// Seeded synthetic layer of the benchmark's shape: uniform random (src, dst)
// pairs counting-sorted by dst (stable), w ~ N(0, 0.05^2) (Box-Muller), act ~
// U(0, 1).
void make_layer(uint64_t n_src, uint64_t n_dst, uint64_t n, uint64_t seed,
                std::vector<uint32_t> &from, std::vector<uint32_t> &to, std::vector<float> &w,
                std::vector<float> &act) {
  std::vector<uint32_t> src(n), dst(n), count(n_dst + 1, 0);
  for (uint64_t i = 0; i < n; ++i) {
    const uint64_t h = mix64(seed * 0x100000001B3ull + i);
    src[i] = (uint32_t)(((h & 0xFFFFFFFFull) * n_src) >> 32);
    dst[i] = (uint32_t)(((h >> 32) * n_dst) >> 32);
    ++count[dst[i] + 1];
  }
  for (uint64_t d = 0; d < n_dst; ++d) count[d + 1] += count[d];
  from.assign(n, 0);
  to.assign(n, 0);
  for (uint64_t i = 0; i < n; ++i) {
    const uint32_t p = count[dst[i]]++;
    from[p] = src[i];
    to[p] = dst[i];
  }
  w.resize(n);
  for (uint64_t i = 0; i < n; ++i) {
    const uint64_t h = mix64(seed ^ (0xA5A5A5A5ull + i));
    const double u1 = ((h >> 11) + 1) * (1.0 / 9007199254740993.0);
    const double u2 = (mix64(h) >> 11) * (1.0 / 9007199254740992.0);
    w[i] = (float)(0.05 * std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
  }
  act.resize(n_src);
  for (uint64_t i = 0; i < n_src; ++i) act[i] = (float)((mix64(seed + 7 + i) >> 40) * (1.0 / 16777216.0));
}

template <class T> bool read_vec(FILE *f, std::vector<T> &v, size_t n) {
  v.resize(n);
  return n == 0 || std::fread(v.data(), sizeof(T), n, f) == n;
}
template <class T> void write_vec(const std::string &path, const std::vector<T> &v) {
  FILE *f = std::fopen(path.c_str(), "wb");
  if (!f) std::exit(3);
  if (!v.empty()) std::fwrite(v.data(), sizeof(T), v.size(), f);
  std::fclose(f);
}

template <class Traits> int check(const std::string &dir, int steps, bool edit) {
  FILE *f = std::fopen((dir + "/layer.bin").c_str(), "rb");
  if (!f) return 2;
  uint64_t hdr[3];
  if (std::fread(hdr, 8, 3, f) != 3) return 2;
  const uint64_t n_src = hdr[0], n_dst = hdr[1], n = hdr[2];
  std::vector<uint32_t> from, to;
  std::vector<float> w, act;
  if (!read_vec(f, from, n) || !read_vec(f, to, n) || !read_vec(f, w, n) || !read_vec(f, act, n_src))
    return 2;
  std::fclose(f);
  plastix::Network<Traits> Net(n_src, GivenConnections{&from, &to, &w, n_dst});
  std::span<const float> out;
  for (int s = 0; s < steps; ++s) {
    Net.DoStep(act);
    out = Net.GetOutput();
    if (edit && s == 0 && n) {
      // host edits between steps: read a trace, bump two weights
      auto &C = Net.GetConnAlloc();
      volatile float probe = plastix::GetField<TraceOf<Traits>>(C, n / 3);
      (void)probe;
      plastix::GetWeight(C, 0) += 0.25f;
      plastix::GetWeight(C, n / 2) -= 0.5f;
      // and two connections die (skipped by both passes from now on)
      plastix::GetField<plastix::DeadTag>(C, n / 5) = true;
      plastix::GetField<plastix::DeadTag>(C, n / 7) = true;
    }
  }
  std::vector<float> o(out.begin(), out.end());
  // the input units hold the last step's inputs (the fused route keeps them
  // in a buffer of its own until the unit fields are read)
  auto &U = Net.GetUnitAlloc();
  for (uint64_t i = 0; i < n_src; ++i)
    if (plastix::GetActivation(U, i) != act[i]) return 5;
  auto &C = Net.GetConnAlloc();
  std::vector<float> wo(n), eo(n);
  for (uint64_t i = 0; i < n; ++i) {
    wo[i] = plastix::GetWeight(C, i);
    eo[i] = plastix::GetField<TraceOf<Traits>>(C, i);
  }
  write_vec(dir + "/out.bin", o);
  write_vec(dir + "/w.bin", wo);
  write_vec(dir + "/e.bin", eo);
  return 0;
}

template <class Traits>
int bench(uint64_t n_src, uint64_t n_dst, uint64_t n, uint64_t seed, int steps, int warmup) {
  std::vector<uint32_t> from, to;
  std::vector<float> w, act;
  make_layer(n_src, n_dst, n, seed, from, to, w, act);
  const auto t0 = std::chrono::steady_clock::now();
  plastix::Network<Traits> Net(n_src, GivenConnections{&from, &to, &w, n_dst});
  cudaStream_t stream;
  plastix::cuda_check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
  Net.SetStream(stream);
  for (int i = 0; i < warmup; ++i) {
    Net.DoStep(act);
    Net.GetOutput();
  }
  plastix::cuda_check(cudaStreamSynchronize(stream), "warmup");
  const double build_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  std::printf("timed-region-begins\n");  // lets a caller sample clocks over the timed loops only
  std::fflush(stdout);
  // device time of DoStep (events on the network's stream)
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0, stream);
  for (int i = 0; i < steps; ++i) Net.DoStep(act);
  cudaEventRecord(e1, stream);
  plastix::cuda_check(cudaEventSynchronize(e1), "timed");
  float dev_ms = 0;
  cudaEventElapsedTime(&dev_ms, e0, e1);
  // end to end: each step's inputs come from the host vector and its outputs
  // are read back with GetOutput (a synchronising device-to-host copy)
  double checksum = 0;
  const auto h0 = std::chrono::steady_clock::now();
  for (int i = 0; i < steps; ++i) {
    Net.DoStep(act);
    auto out = Net.GetOutput();
    checksum += out[i % out.size()];
  }
  const double e2e_ms =
      std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - h0).count();
  std::printf("{\"device_ms_per_step\": %.6f, \"e2e_ms_per_step\": %.6f, \"steps\": %d, "
              "\"n_edges\": %llu, \"build_s\": %.2f, \"checksum\": \"%.6e\"}\n",
              dev_ms / steps, e2e_ms / steps, steps, (unsigned long long)n, build_s, checksum);
  return 0;
}

}  // namespace

int main(int argc, char **argv) {
  try {
    const std::string mode = argc > 1 ? argv[1] : "";
    const bool fused = std::string(argv[argc - 1]) == "fused";
    const int args = argc - (fused || std::string(argv[argc - 1]) == "generic");
    if (args == 8 && mode == "bench") {
      const uint64_t a = std::strtoull(argv[2], nullptr, 10), b = std::strtoull(argv[3], nullptr, 10),
                     c = std::strtoull(argv[4], nullptr, 10), d = std::strtoull(argv[5], nullptr, 10);
      return fused ? bench<FusedSweepTraits>(a, b, c, d, std::atoi(argv[6]), std::atoi(argv[7]))
                   : bench<SweepTraits>(a, b, c, d, std::atoi(argv[6]), std::atoi(argv[7]));
    }
    if (args == 4 && (mode == "check" || mode == "check-edit")) {
      const bool edit = mode == "check-edit";
      return fused ? check<FusedSweepTraits>(argv[2], std::atoi(argv[3]), edit)
                   : check<SweepTraits>(argv[2], std::atoi(argv[3]), edit);
    }
  } catch (const std::exception &e) {
    std::fprintf(stderr, "%s\n", e.what());
    return 4;
  }
  std::fprintf(stderr, "usage: network_sweep bench|check ...\n");
  return 1;
}
