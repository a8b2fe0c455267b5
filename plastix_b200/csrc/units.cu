// Per-unit steps that sit between the connection sweeps of the example
// networks: the iPC value-node update and pre-step, and MSE loss folded into
// the sigmoid backward Apply of the output units. One thread per unit,
// elementwise, same evaluation order as the reference with separate roundings.
#include "common.cuh"

namespace plx {
namespace {

// examples/ipc-multilayer/ipc_multilayer.cpp:239-245 (x += Gamma * (-Eps +
// BU); BU = 0) followed by the pre-step of the next iPC step (:220-228, here
// for hidden units: Activation = tanh(x)). mode 0 runs the pre-step alone.
__global__ void k_ipc_value_update(uint64_t n, float* __restrict__ x,
                                   const float* __restrict__ eps, float* __restrict__ bu,
                                   float gamma, float* __restrict__ act, int mode) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    float xv = x[i];
    if (mode) {
      xv = __fadd_rn(xv, __fmul_rn(gamma, __fadd_rn(-eps[i], bu[i])));
      x[i] = xv;
      bu[i] = 0.0f;
    }
    act[i] = tanhf(xv);
  }
}

// MSELoss (include/plastix/traits.hpp:185-193: BackwardAcc = pred - target)
// then the sigmoid backward Apply of the output units
// (examples/mlp-xor/mlp_xor.cpp:43-46: grad = acc * a * (1 - a)).
__global__ void k_mse_sigmoid_grad(uint64_t n, const float* __restrict__ act,
                                   const float* __restrict__ target,
                                   float* __restrict__ grad) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const float a = act[i];
    const float acc = __fsub_rn(a, target[i]);
    grad[i] = __fmul_rn(__fmul_rn(acc, a), __fsub_rn(1.0f, a));
  }
}

unsigned grid_for(const plx_ctx* ctx, uint64_t n) {
  return (unsigned)std::max<uint64_t>(
      1, std::min<uint64_t>((n + 255) / 256, 8ull * (uint64_t)ctx->num_sms));
}

}  // namespace
}  // namespace plx

using namespace plx;

extern "C" int plx_ipc_value_update(plx_ctx* ctx, uint64_t n, float* x, const float* eps,
                                    float* bu, float gamma, float* act, int mode) {
  PLX_CHECK_ARG(ctx && x && act, "ctx, x and act are required");
  PLX_CHECK_ARG(!mode || (eps && bu), "the update needs eps and bu");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  if (n == 0) return PLX_OK;
  k_ipc_value_update<<<grid_for(ctx, n), 256, 0, ctx->stream>>>(n, x, eps, bu, gamma, act,
                                                                 mode);
  PLX_LAUNCH_CHECK("k_ipc_value_update");
  return PLX_OK;
}

extern "C" int plx_mse_sigmoid_grad(plx_ctx* ctx, uint64_t n, const float* act,
                                    const float* target, float* grad) {
  PLX_CHECK_ARG(ctx && act && target && grad, "ctx, act, target and grad are required");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  if (n == 0) return PLX_OK;
  k_mse_sigmoid_grad<<<grid_for(ctx, n), 256, 0, ctx->stream>>>(n, act, target, grad);
  PLX_LAUNCH_CHECK("k_mse_sigmoid_grad");
  return PLX_OK;
}
