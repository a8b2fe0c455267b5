// Connection proposals: sort 64-bit (To << 32 | From) keys and keep the
// first of every run of equal keys -- the sort and unique commit of
// DoAddConnections phases 2-3 (include/plastix/plastix.hpp:411-433), where
// the reference std::sorts CompactEdge bits and skips repeats.
//
// Two stable LSD stages of the u32 radix sort (low half, then high half)
// give the sorting permutation; flags mark the first key of each run, and
// order-preserving compaction writes the unique keys and their count. All
// integer work, bit-exact.
#include "common.cuh"

namespace plx {
namespace {

__global__ void k_split_u64(const uint64_t* __restrict__ keys, uint64_t n,
                            uint32_t* __restrict__ lo, uint32_t* __restrict__ hi) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t k = keys[i];
    lo[i] = (uint32_t)k;
    hi[i] = (uint32_t)(k >> 32);
  }
}

// out[i] = src[perm[i]]
__global__ void k_take_u32(const uint32_t* __restrict__ src, const uint32_t* __restrict__ perm,
                           uint64_t n, uint32_t* __restrict__ out) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = src[perm[i]];
}

// sorted[i] = keys[p1[p2[i]]]
__global__ void k_compose_u64(const uint64_t* __restrict__ keys, const uint32_t* __restrict__ p1,
                              const uint32_t* __restrict__ p2, uint64_t n,
                              uint64_t* __restrict__ sorted) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    sorted[i] = keys[p1[p2[i]]];
}

__global__ void k_run_heads(const uint64_t* __restrict__ sorted, uint64_t n,
                            uint8_t* __restrict__ flags) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    // The reference starts its "previous key" at UINT64_MAX, so a run of the
    // all-ones key at the front is skipped too (plastix.hpp:419-422).
    flags[i] = sorted[i] != (i == 0 ? ~0ull : sorted[i - 1]) ? 1 : 0;
}

size_t al(size_t x) { return (x + 255) & ~size_t(255); }

unsigned grid_for(const plx_ctx* ctx, uint64_t n) {
  return (unsigned)std::max<uint64_t>(
      1, std::min<uint64_t>((n + 255) / 256, 8ull * (uint64_t)ctx->num_sms));
}

}  // namespace
}  // namespace plx

using namespace plx;

extern "C" size_t plx_sort_unique_u64_scratch_bytes(uint64_t n) {
  const size_t a = al(4 * n);
  return 6 * a + al(8 * n) + al(n) + std::max(plx_radix_sort_scratch_bytes(n),
                                              plx_compact_scratch_bytes(n));
}

extern "C" int plx_sort_unique_u64(plx_ctx* ctx, uint64_t n, const uint64_t* keys,
                                   uint64_t* out, uint64_t* count_out, void* scratch,
                                   size_t scratch_bytes) {
  PLX_CHECK_ARG(ctx && count_out, "ctx and count_out are required");
  PLX_CHECK_ARG(n == 0 || (keys && out), "keys and out are required");
  PLX_CHECK_ARG(n < (1ull << 30), "n must be < 2^30");
  PLX_CHECK_ARG(scratch && scratch_bytes >= plx_sort_unique_u64_scratch_bytes(n),
                "scratch too small");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  if (n == 0) {
    PLX_TRY_CUDA(cudaMemsetAsync(count_out, 0, sizeof(uint64_t), ctx->stream));
    return PLX_OK;
  }
  char* s = static_cast<char*>(scratch);
  const size_t a = al(4 * n);
  uint32_t* lo = reinterpret_cast<uint32_t*>(s);
  uint32_t* hi = reinterpret_cast<uint32_t*>(s + a);
  uint32_t* tmp = reinterpret_cast<uint32_t*>(s + 2 * a);
  uint32_t* p1 = reinterpret_cast<uint32_t*>(s + 3 * a);
  uint32_t* hi2 = reinterpret_cast<uint32_t*>(s + 4 * a);
  uint32_t* p2 = reinterpret_cast<uint32_t*>(s + 5 * a);
  uint64_t* sorted = reinterpret_cast<uint64_t*>(s + 6 * a);
  uint8_t* flags = reinterpret_cast<uint8_t*>(s + 6 * a + al(8 * n));
  void* work = s + 6 * a + al(8 * n) + al(n);
  const size_t work_bytes = scratch_bytes - (6 * a + al(8 * n) + al(n));
  const unsigned g = grid_for(ctx, n);
  k_split_u64<<<g, 256, 0, ctx->stream>>>(keys, n, lo, hi);
  PLX_LAUNCH_CHECK("k_split_u64");
  if (int rc = plx_radix_sort_u32(ctx, n, lo, tmp, p1, 0, 32, work, work_bytes)) return rc;
  k_take_u32<<<g, 256, 0, ctx->stream>>>(hi, p1, n, hi2);
  PLX_LAUNCH_CHECK("k_take_u32");
  if (int rc = plx_radix_sort_u32(ctx, n, hi2, tmp, p2, 0, 32, work, work_bytes)) return rc;
  k_compose_u64<<<g, 256, 0, ctx->stream>>>(keys, p1, p2, n, sorted);
  PLX_LAUNCH_CHECK("k_compose_u64");
  k_run_heads<<<g, 256, 0, ctx->stream>>>(sorted, n, flags);
  PLX_LAUNCH_CHECK("k_run_heads");
  plx_field f{sorted, out, 8, 0};
  return plx_compact(ctx, n, PLX_KEEP_FLAGS, flags, 0.0f, &f, 1, nullptr, count_out, work,
                     work_bytes);
}
