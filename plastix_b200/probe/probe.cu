// Measurement kernels for the memory ceiling of the connection sweep, built
// into their own library (libplastix_probe.so, loaded by the benchmark's
// `ceiling` workload only). They are not part of any reference path: they
// time the two pieces of the sweep's traffic that no fold order can remove,
// so that the sweep's own time can be read against them.
//
//   int plx_probe_gather(plx_ctx* ctx, const float* x, uint32_t n_x,
//                        uint64_t n_gathers, float* sink, uint64_t* done);
//     about n_gathers random 4-byte loads from x (n_x a power of two) with
//     the sweep's L2 policy; the exact count goes to *done (host) and the
//     loaded values are summed into *sink (device).
//   int plx_probe_sweep_nofold(plx_ctx* ctx, uint64_t n, const uint32_t* from_id,
//                              const float* act, uint32_t n_act, const float* w_in,
//                              const float* e_in, float decay, float rate,
//                              float* w_out, float* e_out);
//     n a multiple of 4, arrays 16-byte aligned.
//   plx_probe_gather        random 4-byte gathers from an L2-resident array
//                           (the act[FromId] loads), nothing else;
//   plx_probe_sweep_nofold  the sweep's streams and gathers without the row
//                           folds: per connection FromId, Weight and Trace
//                           loads, the gather, and the Weight and Trace
//                           stores, with the sweep's L2 policies.
#include "common.cuh"

namespace plx {
namespace {

__device__ __forceinline__ uint32_t probe_hash(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352dU;
  x ^= x >> 15;
  x *= 0x846ca68bU;
  x ^= x >> 16;
  return x;
}

__global__ void __launch_bounds__(256) k_probe_gather(const float* __restrict__ x, uint32_t mask,
                                                      uint32_t per_thread, float* __restrict__ out) {
  const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
  const uint64_t pol = l2_policy_evict_last();
  float acc = 0.0f;
  for (uint32_t i = 0; i < per_thread; i += 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = ld_keep_f32(x + (probe_hash(t * per_thread + i + j) & mask), pol);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc += v[j];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
  if ((threadIdx.x & 31u) == 0) atomicAdd(out, acc);
}

// Four consecutive connections per thread and step, four steps in flight.
__global__ void __launch_bounds__(256) k_probe_sweep_nofold(
    uint64_t n4, const uint32_t* __restrict__ src, const float* __restrict__ act, uint32_t len1,
    const float* __restrict__ w_in, const float* __restrict__ e_in, float decay, float rate,
    float* __restrict__ w_out, float* __restrict__ e_out) {
  constexpr int kB = 4;
  const uint64_t pf = l2_policy_evict_first(), pl = l2_policy_evict_last();
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t g0 = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; g0 < n4; g0 += stride * kB) {
    uint4 I[kB], W[kB], E[kB];
#pragma unroll
    for (int h = 0; h < kB; ++h) {
      const uint64_t g = g0 + h * stride;
      if (g < n4) {
        I[h] = ld_stream_v4(src + 4 * g, pf);
        W[h] = ld_stream_v4(w_in + 4 * g, pf);
        E[h] = ld_stream_v4(e_in + 4 * g, pf);
      }
    }
    float X[kB][4];
#pragma unroll
    for (int h = 0; h < kB; ++h) {
      const uint32_t ii[4] = {I[h].x, I[h].y, I[h].z, I[h].w};
#pragma unroll
      for (int c = 0; c < 4; ++c) X[h][c] = ld_keep_f32(act + min(ii[c], len1), pl);
    }
#pragma unroll
    for (int h = 0; h < kB; ++h) {
      const uint64_t g = g0 + h * stride;
      if (g >= n4) continue;
      const float ww[4] = {__uint_as_float(W[h].x), __uint_as_float(W[h].y),
                           __uint_as_float(W[h].z), __uint_as_float(W[h].w)};
      const float ee[4] = {__uint_as_float(E[h].x), __uint_as_float(E[h].y),
                           __uint_as_float(E[h].z), __uint_as_float(E[h].w)};
      float wo[4], eo[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float p = __fmul_rn(ww[c], X[h][c]);
        eo[c] = __fadd_rn(__fmul_rn(decay, ee[c]), __fmul_rn(X[h][c], p));
        wo[c] = __fadd_rn(ww[c], __fmul_rn(rate, eo[c]));
      }
      st_stream_v4(w_out + 4 * g, make_float4(wo[0], wo[1], wo[2], wo[3]), pf);
      st_stream_v4(e_out + 4 * g, make_float4(eo[0], eo[1], eo[2], eo[3]), pf);
    }
  }
}

}  // namespace
}  // namespace plx

using namespace plx;

extern "C" int plx_probe_gather(plx_ctx* ctx, const float* x, uint32_t n_x, uint64_t n_gathers,
                                float* sink, uint64_t* done) {
  PLX_CHECK_ARG(ctx && x && sink && done, "ctx, x, sink and done are required");
  PLX_CHECK_ARG(n_x && (n_x & (n_x - 1)) == 0, "n_x must be a power of two");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  const uint32_t grid = 4u * (uint32_t)ctx->num_sms, threads = grid * 256u;
  uint64_t per = (n_gathers + threads - 1) / threads;
  per = (per + 7) & ~7ull;
  PLX_CHECK_ARG(per < (1ull << 32) / threads, "n_gathers too large");
  *done = per * threads;
  PLX_TRY_CUDA(cudaMemsetAsync(sink, 0, sizeof(float), ctx->stream));
  k_probe_gather<<<grid, 256, 0, ctx->stream>>>(x, n_x - 1, (uint32_t)per, sink);
  PLX_LAUNCH_CHECK("k_probe_gather");
  return PLX_OK;
}

extern "C" int plx_probe_sweep_nofold(plx_ctx* ctx, uint64_t n, const uint32_t* from_id,
                                      const float* act, uint32_t n_act, const float* w_in,
                                      const float* e_in, float decay, float rate, float* w_out,
                                      float* e_out) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  PLX_CHECK_ARG(n % 4 == 0, "n must be a multiple of 4");
  PLX_CHECK_ARG(n == 0 || (from_id && act && n_act && w_in && e_in && w_out && e_out),
                "arrays are required");
  PLX_CHECK_ARG(aligned16(from_id) && aligned16(w_in) && aligned16(e_in) && aligned16(w_out) &&
                    aligned16(e_out),
                "connection arrays must be 16-byte aligned");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  if (n == 0) return PLX_OK;
  const uint32_t grid = 4u * (uint32_t)ctx->num_sms;
  k_probe_sweep_nofold<<<grid, 256, 0, ctx->stream>>>(n / 4, from_id, act, n_act - 1, w_in, e_in,
                                                      decay, rate, w_out, e_out);
  PLX_LAUNCH_CHECK("k_probe_sweep_nofold");
  return PLX_OK;
}
