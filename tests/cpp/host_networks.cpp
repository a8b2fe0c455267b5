// C++ host program over plastix_b200.hpp: steps the single-layer trace
// network and the SwiftTD network on the device and writes their results as
// raw little-endian arrays for the test to compare with the oracle.
//
// usage: host_networks <out_dir> <n_src> <n_dst> <n_edges> <sweeps> <td_n> <td_steps>
// inputs are read from <out_dir>/in_*.bin (written by the test).
#include <cstdio>
#include <fstream>
#include <string>
#include <vector>

#include "plastix_b200.hpp"

template <class T>
static std::vector<T> read_bin(const std::string& path, size_t n) {
  std::vector<T> v(n);
  std::ifstream f(path, std::ios::binary);
  f.read(reinterpret_cast<char*>(v.data()), (std::streamsize)(n * sizeof(T)));
  if (!f) throw std::runtime_error("cannot read " + path);
  return v;
}

template <class T>
static void write_bin(const std::string& path, const std::vector<T>& v) {
  std::ofstream f(path, std::ios::binary);
  f.write(reinterpret_cast<const char*>(v.data()), (std::streamsize)(v.size() * sizeof(T)));
}

int main(int argc, char** argv) {
  if (argc != 8) {
    std::fprintf(stderr, "usage: %s out n_src n_dst n_edges sweeps td_n td_steps\n", argv[0]);
    return 2;
  }
  const std::string dir = argv[1];
  const uint32_t n_src = std::stoul(argv[2]), n_dst = std::stoul(argv[3]);
  const size_t n = std::stoull(argv[4]);
  const int sweeps = std::stoi(argv[5]);
  const uint32_t td_n = std::stoul(argv[6]);
  const int td_steps = std::stoi(argv[7]);
  try {
    plastix_b200::Context ctx(0);
    auto from = read_bin<uint32_t>(dir + "/in_from.bin", n);
    auto to = read_bin<uint32_t>(dir + "/in_to.bin", n);
    auto w = read_bin<float>(dir + "/in_w.bin", n);
    auto act = read_bin<float>(dir + "/in_act.bin", n_src);
    plastix_b200::HebbianLayerNetwork net(ctx, n_src, n_dst, from, to, w, 0.9f, 1e-3f);
    for (int s = 0; s < sweeps; ++s) net.DoStep(act);
    write_bin(dir + "/out_act.bin", net.GetOutput());
    write_bin(dir + "/out_w.bin", net.GetWeights());
    write_bin(dir + "/out_e.bin", net.GetTraces());

    plastix_b200::SwiftTDNetwork td(ctx, td_n, td_n, {});
    auto offs = read_bin<uint32_t>(dir + "/in_td_offs.bin", td_steps + 1);
    auto idx = read_bin<uint32_t>(dir + "/in_td_idx.bin", offs[td_steps]);
    auto rw = read_bin<float>(dir + "/in_td_rw.bin", td_steps);
    std::vector<float> vs;
    for (int s = 0; s < td_steps; ++s) {
      td.DoStep(std::span<const uint32_t>(idx.data() + offs[s], offs[s + 1] - offs[s]), rw[s]);
      vs.push_back(td.GetOutput());
    }
    write_bin(dir + "/out_td_v.bin", vs);
    write_bin(dir + "/out_td_w.bin", td.GetField(0));
    std::printf("ok %zu %zu\n", net.GetStep(), td.GetStep());
  } catch (const std::exception& e) {
    std::fprintf(stderr, "error: %s\n", e.what());
    return 1;
  }
  return 0;
}
