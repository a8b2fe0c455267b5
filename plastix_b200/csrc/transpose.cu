// Source-major connection order for the backward sweep (K2).
//
// The reference's DoBackwardPass folds BackwardAcc[FromId] over the
// connections in DESCENDING index order in Pipeline mode
// (include/plastix/plastix.hpp:193-203) and in ascending index order within
// each SrcLevel range in Topological mode (plastix.hpp:172-181). A stable sort
// of the connections by FromId puts each source's connections together in
// ascending index order; reversing each source's run gives the Pipeline
// order. The backward pass is then the forward sweep kernel (a left fold per
// row, then Apply) run over this order, with the destination unit as the
// gathered side: it is bit-exact for rows up to PLX_SEQ_ROW_MAX connections,
// like the forward sweep.
//
// plx_transpose produces the permutation and the row offsets; plx_gather
// applies the permutation to ToId / Weight (and any other field).
#include "common.cuh"

namespace plx {
namespace {

// keys[j] = from_id[j] - src_base for sources in range, n_src otherwise (sorts
// after every source and is excluded from the rows).
__global__ void k_transpose_keys(const uint32_t* __restrict__ from_id, uint64_t n,
                                 uint32_t src_base, uint32_t n_src,
                                 uint32_t* __restrict__ keys) {
  for (uint64_t j = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; j < n;
       j += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t k = from_id[j] - src_base;
    keys[j] = k < n_src ? k : n_src;
  }
}

// row_ptr[r] = first position whose sorted key is >= r, r in [0, n_src].
__global__ void k_transpose_rows(const uint32_t* __restrict__ keys, uint64_t n, uint32_t n_src,
                                 uint32_t* __restrict__ row_ptr) {
  const uint64_t r = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (r > n_src) return;
  uint64_t lo = 0, hi = n;
  while (lo < hi) {
    const uint64_t mid = (lo + hi) >> 1;
    if (keys[mid] < r) lo = mid + 1;
    else hi = mid;
  }
  row_ptr[r] = (uint32_t)lo;
}

// out[p] = perm[rs + re - 1 - p] within each row [rs, re); positions past the
// last row (connections from other units) keep their order.
__global__ void k_transpose_reverse(const uint32_t* __restrict__ keys,
                                    const uint32_t* __restrict__ perm,
                                    const uint32_t* __restrict__ row_ptr, uint64_t n,
                                    uint32_t n_src, uint32_t* __restrict__ out) {
  for (uint64_t p = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; p < n;
       p += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t r = keys[p];
    uint64_t q = p;
    if (r < n_src) q = (uint64_t)row_ptr[r] + row_ptr[r + 1] - 1 - p;
    out[p] = perm[q];
  }
}

uint32_t bits_for(uint32_t n_src) {
  uint32_t b = 0;
  while (b < 32 && (uint64_t(1) << b) <= n_src) ++b;  // keys go up to n_src
  return b;
}

}  // namespace
}  // namespace plx

using namespace plx;

extern "C" size_t plx_transpose_scratch_bytes(uint64_t n) {
  const size_t pad = 256;
  return 2 * ((4 * n + pad - 1) / pad * pad) + plx_radix_sort_scratch_bytes(n);
}

extern "C" int plx_transpose(plx_ctx* ctx, uint64_t n, const uint32_t* from_id,
                             uint32_t src_base, uint32_t n_src, int reverse,
                             uint32_t* keys_out, uint32_t* perm_out, uint32_t* row_ptr_out,
                             void* scratch, size_t scratch_bytes) {
  PLX_CHECK_ARG(ctx && row_ptr_out, "ctx and row_ptr_out are required");
  PLX_CHECK_ARG(n == 0 || (from_id && keys_out && perm_out),
                "from_id, keys_out and perm_out are required");
  PLX_CHECK_ARG(n < (1ull << 30), "n must be < 2^30 (transpose per block of connections)");
  PLX_CHECK_ARG(n_src < 0xFFFFFFFFu, "n_src too large");
  PLX_CHECK_ARG(scratch && scratch_bytes >= plx_transpose_scratch_bytes(n),
                "scratch too small: need %zu bytes", plx_transpose_scratch_bytes(n));
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  const size_t slab = (4 * n + 255) / 256 * 256;
  char* s = static_cast<char*>(scratch);
  uint32_t* keys = reinterpret_cast<uint32_t*>(s);
  uint32_t* perm_tmp = reinterpret_cast<uint32_t*>(s + slab);
  void* radix = s + 2 * slab;
  const size_t radix_bytes = scratch_bytes - 2 * slab;
  const unsigned grid = (unsigned)std::max<uint64_t>(
      1, std::min<uint64_t>((n + 255) / 256, 8ull * (uint64_t)ctx->num_sms));
  if (n) {
    k_transpose_keys<<<grid, 256, 0, ctx->stream>>>(from_id, n, src_base, n_src, keys);
    PLX_LAUNCH_CHECK("k_transpose_keys");
    if (int rc = plx_radix_sort_u32(ctx, n, keys, keys_out, reverse ? perm_tmp : perm_out, 0,
                                    bits_for(n_src), radix, radix_bytes))
      return rc;
  }
  k_transpose_rows<<<(unsigned)((n_src + 1 + 255) / 256), 256, 0, ctx->stream>>>(
      keys_out, n, n_src, row_ptr_out);
  PLX_LAUNCH_CHECK("k_transpose_rows");
  if (n && reverse) {
    k_transpose_reverse<<<grid, 256, 0, ctx->stream>>>(keys_out, perm_tmp, row_ptr_out, n,
                                                       n_src, perm_out);
    PLX_LAUNCH_CHECK("k_transpose_reverse");
  }
  return PLX_OK;
}
