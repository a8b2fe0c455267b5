// Drives the reference's XOR MLP example (examples/mlp-xor/mlp_xor.cpp),
// compiled unchanged in this translation unit with its main() renamed, so its
// own policies (SigmoidForwardPass, SigmoidBackwardPass, GradientDescentConn,
// MSELoss; Topological propagation) run on the reference Network.
// TEST INFRASTRUCTURE ONLY (oracle side); built by oracle/build.py.
#define main plx_ref_mlp_example_main
#include "mlp_xor.cpp"
#undef main

#include <cstdint>
#include <cstring>

// Builds MlpNetwork(n_in, FullyConnected{n_hidden, RandomUniformWeight{seed}},
// FullyConnected{1, RandomUniformWeight{seed}}) and trains it for `epochs`
// epochs of n_patterns DoSteps (mlp_xor.cpp:93-101). Outputs: the initial and
// final weights (connection order) and the final prediction per pattern
// (DoForwardPass + GetOutput, mlp_xor.cpp:110-113). inputs: n_patterns x
// n_in, targets: n_patterns. Returns the connection count, or -1.
extern "C" int64_t ref_mlp_run(uint32_t n_in, uint32_t n_hidden, uint32_t seed,
                               uint32_t epochs, uint32_t n_patterns,
                               const float *inputs, const float *targets,
                               float *w_init, float *w_final, float *preds,
                               uint64_t max_conn) {
  MlpNetwork Net(n_in, plastix::FullyConnected{n_hidden, plastix::RandomUniformWeight{seed}},
                 plastix::FullyConnected{1, plastix::RandomUniformWeight{seed}});
  auto &CA = Net.GetConnAlloc();
  if (CA.Size() > max_conn) return -1;
  for (size_t C = 0; C < CA.Size(); ++C) w_init[C] = plastix::GetWeight(CA, C);
  for (uint32_t E = 0; E < epochs; ++E)
    for (uint32_t S = 0; S < n_patterns; ++S) {
      float Tgt[1] = {targets[S]};
      Net.DoStep(std::span<const float>(inputs + (size_t)S * n_in, n_in),
                 std::span<const float>(Tgt, 1));
    }
  for (size_t C = 0; C < CA.Size(); ++C) w_final[C] = plastix::GetWeight(CA, C);
  for (uint32_t S = 0; S < n_patterns; ++S) {
    Net.DoForwardPass(std::span<const float>(inputs + (size_t)S * n_in, n_in));
    preds[S] = Net.GetOutput()[0];
  }
  return (int64_t)CA.Size();
}
