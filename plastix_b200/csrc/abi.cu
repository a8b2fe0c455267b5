// Context, error reporting and version entry points of the C ABI.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace plx {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  return set_error(PLX_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e),
                   cudaGetErrorString(e));
}

}  // namespace plx

using namespace plx;

extern "C" const char* plx_version(void) { return "0.1.0"; }

extern "C" const char* plx_last_error(void) { return g_last_error; }

extern "C" int plx_ctx_create(int device, void* stream, plx_ctx** out) {
  PLX_CHECK_ARG(out, "out is required");
  *out = nullptr;
  int n = 0;
  PLX_TRY_CUDA(cudaGetDeviceCount(&n));
  PLX_CHECK_ARG(device >= 0 && device < n, "device %d out of range (%d devices)",
                device, n);
  PLX_TRY_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  PLX_TRY_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return set_error(PLX_ERR_UNSUPPORTED,
                     "device %d is sm_%d%d; this library is built for sm_100a only",
                     device, prop.major, prop.minor);
  plx_ctx* c = new plx_ctx();
  c->device = device;
  c->stream = static_cast<cudaStream_t>(stream);
  c->num_sms = prop.multiProcessorCount;
  cudaError_t e = cudaMalloc(&c->d_status, 64);
  if (e == cudaSuccess) e = cudaMemset(c->d_status, 0, 64);
  c->d_queue = reinterpret_cast<uint32_t*>(c->d_status + 4);
  if (e != cudaSuccess) {
    cudaFree(c->d_status);
    delete c;
    return check_cuda(e, "allocating the status word");
  }
  *out = c;
  return PLX_OK;
}

int ctx_counters(plx_ctx* ctx, size_t n, uint32_t** out) {
  if (ctx->counters_cap < n) {
    PLX_TRY_CUDA(cudaStreamSynchronize(ctx->stream));
    if (ctx->d_counters) PLX_TRY_CUDA(cudaFree(ctx->d_counters));
    ctx->d_counters = nullptr;
    ctx->counters_cap = 0;
    PLX_TRY_CUDA(cudaMalloc(&ctx->d_counters, n * sizeof(uint32_t)));
    ctx->counters_cap = n;
  }
  *out = ctx->d_counters;
  return PLX_OK;
}

extern "C" int plx_ctx_destroy(plx_ctx* ctx) {
  if (!ctx) return PLX_OK;
  cudaSetDevice(ctx->device);
  if (ctx->d_counters) cudaFree(ctx->d_counters);
  cudaError_t e = cudaFree(ctx->d_status);
  delete ctx;
  if (e != cudaSuccess) return check_cuda(e, "cudaFree(status)");
  return PLX_OK;
}

extern "C" int plx_ctx_set_stream(plx_ctx* ctx, void* stream) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  ctx->stream = static_cast<cudaStream_t>(stream);
  return PLX_OK;
}

extern "C" int plx_ctx_set_timeout_ns(plx_ctx* ctx, uint64_t timeout_ns) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  PLX_CHECK_ARG(timeout_ns > 0, "timeout must be positive");
  ctx->timeout_ns = timeout_ns;
  return PLX_OK;
}

extern "C" int plx_ctx_num_sms(plx_ctx* ctx, int* out) {
  PLX_CHECK_ARG(ctx && out, "ctx and out are required");
  *out = ctx->num_sms;
  return PLX_OK;
}

extern "C" int plx_ctx_sync(plx_ctx* ctx) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  int32_t st = 0;
  PLX_TRY_CUDA(cudaMemcpyAsync(&st, ctx->d_status, sizeof(st),
                               cudaMemcpyDeviceToHost, ctx->stream));
  PLX_TRY_CUDA(cudaStreamSynchronize(ctx->stream));
  if (st != kStatusOk) {
    PLX_TRY_CUDA(cudaMemsetAsync(ctx->d_status, 0, sizeof(int32_t), ctx->stream));
    PLX_TRY_CUDA(cudaStreamSynchronize(ctx->stream));
    if (st == kStatusTimeout)
      return set_error(PLX_ERR_TIMEOUT, "a bounded device-side wait expired");
    if (st == kStatusBadIndex)
      return set_error(PLX_ERR_ARG, "a connection referenced a unit id outside "
                                    "the activation array");
    if (st == kStatusBadPlan)
      return set_error(PLX_ERR_ARG, "a sweep was given an invalid plan");
    return set_error(PLX_ERR_ARG, "device status %d", st);
  }
  return PLX_OK;
}
