// Drives the reference's streaming iPC example
// (examples/ipc-multilayer/ipc_multilayer.cpp), compiled unchanged in this
// translation unit with its main() renamed: its own policies and its own
// iPCStep (pre-step, DoForwardPass, DoBackwardPass, DoUpdateConnectionState,
// value-node update) on the reference Network, at the example's shape
// (3 inputs -> 16 tanh hidden -> 1 output, Pipeline propagation).
// TEST INFRASTRUCTURE ONLY (oracle side); built by oracle/build.py.
#define main plx_ref_ipc_example_main
#include "ipc_multilayer.cpp"
#undef main

#include <cstdint>

// w: connection weights in and out (connection order of the example's
// FullyConnected layers); x: ValueNode of all 20 units in and out. Each step
// clamps the inputs and the output value node as the example does
// (ipc_multilayer.cpp:299-304) and runs iPCStep. err_out: ErrorTag after the
// last step. Returns the connection count, or -1.
extern "C" int64_t ref_ipc_run(uint32_t steps, const float *inputs, const float *targets,
                               float *w, float *x, float *err_out, uint64_t max_conn) {
  iPCNet Net(NumInputs, FC{HiddenSize}, FC{OutputSize});
  auto &CA = Net.GetConnAlloc();
  auto &U = Net.GetUnitAlloc();
  if (CA.Size() > max_conn) return -1;
  for (size_t C = 0; C < CA.Size(); ++C) plastix::GetWeight(CA, C) = w[C];
  for (size_t I = 0; I < U.Size(); ++I) plastix::GetField<ValueNodeTag>(U, I) = x[I];
  for (uint32_t T = 0; T < steps; ++T) {
    const float *In = inputs + (size_t)T * NumInputs;
    for (size_t I = 0; I < NumInputs; ++I) plastix::GetField<ValueNodeTag>(U, I) = In[I];
    plastix::GetField<ValueNodeTag>(U, OutputBegin) = targets[T];
    iPCStep(Net, std::span<const float>(In, NumInputs));
  }
  for (size_t C = 0; C < CA.Size(); ++C) w[C] = plastix::GetWeight(CA, C);
  for (size_t I = 0; I < U.Size(); ++I) {
    x[I] = plastix::GetField<ValueNodeTag>(U, I);
    err_out[I] = plastix::GetField<ErrorTag>(U, I);
  }
  return (int64_t)CA.Size();
}
