// Stable sort of keys whose leading part is already sorted: the re-sort of
// connections by destination after a structural step, where compaction has
// kept the survivors in destination order and only the regrown connections
// at the end are unordered.
//
// The result is the stable sort of all n keys (by bits [begin, end)), equal
// to plx_radix_sort_u32's output bit for bit: the unordered tail is sorted by
// the radix sort (stable), then the two sorted runs are merged, taking the
// prefix's key first on equal keys -- every prefix element precedes every
// tail element in the input, so that is exactly the stable order. The radix
// passes touch only the tail (the regrown share, 16 % of the connections in
// the structural workload); the merge reads and writes every key once.
//
// Merge: merge-path partitions of kMT outputs per CTA (one binary search per
// partition over the two runs), then each CTA stages its share of both runs
// in shared memory and each thread merges four consecutive outputs after a
// binary search of its own diagonal in shared memory; outputs are written as
// 16-byte vectors.
#include "common.cuh"

namespace plx {
namespace {

constexpr int kMThreads = 512;
constexpr int kMItems = 4;
constexpr int kMT = kMThreads * kMItems;  // outputs per CTA

struct MergeArgs {
  const uint32_t* a;       // sorted prefix keys (input order = original index)
  uint64_t na;
  const uint32_t* b;       // sorted tail keys
  const uint32_t* b_perm;  // tail position of each sorted tail key
  uint64_t nb;
  uint32_t shift, mask;
  uint64_t* split;         // prefix elements before each CTA's first output
  uint32_t* keys_out;
  uint32_t* perm_out;
};

__device__ __forceinline__ uint32_t digit(uint32_t k, uint32_t shift, uint32_t mask) {
  return (k >> shift) & mask;
}

// split[c] = number of prefix elements among the first c * kMT outputs.
__global__ void k_merge_split(MergeArgs m, uint64_t n_parts) {
  const uint64_t c = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (c > n_parts) return;
  const uint64_t d = min(c * (uint64_t)kMT, m.na + m.nb);
  uint64_t lo = d > m.nb ? d - m.nb : 0, hi = min(d, m.na);
  while (lo < hi) {
    const uint64_t mid = (lo + hi) / 2;
    // prefix element mid goes before tail element d - mid - 1 when <=
    if (digit(__ldg(m.a + mid), m.shift, m.mask) <=
        digit(__ldg(m.b + (d - mid - 1)), m.shift, m.mask))
      lo = mid + 1;
    else
      hi = mid;
  }
  m.split[c] = lo;
}

__global__ void __launch_bounds__(kMThreads) k_merge(MergeArgs m) {
  __shared__ uint32_t s_keys[kMT];  // this CTA's prefix keys, then its tail keys
  const uint64_t n = m.na + m.nb;
  const uint64_t o0 = blockIdx.x * (uint64_t)kMT;
  const uint64_t o1 = min(o0 + kMT, n);
  const uint64_t a0 = m.split[blockIdx.x], a1 = m.split[blockIdx.x + 1];
  const uint64_t b0 = o0 - a0, b1 = o1 - a1;
  const uint32_t la = (uint32_t)(a1 - a0), lb = (uint32_t)(b1 - b0);
  for (uint32_t i = threadIdx.x; i < la; i += kMThreads) s_keys[i] = __ldg(m.a + a0 + i);
  for (uint32_t i = threadIdx.x; i < lb; i += kMThreads) s_keys[la + i] = __ldg(m.b + b0 + i);
  __syncthreads();
  const uint32_t* sa = s_keys;
  const uint32_t* sb = s_keys + la;
  const uint32_t d = threadIdx.x * kMItems;
  if (d >= la + lb) return;
  uint32_t lo = d > lb ? d - lb : 0, hi = min(d, la);
  while (lo < hi) {
    const uint32_t mid = (lo + hi) / 2;
    if (digit(sa[mid], m.shift, m.mask) <= digit(sb[d - mid - 1], m.shift, m.mask)) lo = mid + 1;
    else hi = mid;
  }
  uint32_t i = lo, j = d - lo;
  uint32_t key[kMItems], perm[kMItems];
  const uint32_t cnt = min((uint32_t)kMItems, la + lb - d);
#pragma unroll
  for (int k = 0; k < kMItems; ++k) {
    if ((uint32_t)k >= cnt) break;
    const bool take_a = j >= lb || (i < la && digit(sa[i], m.shift, m.mask) <=
                                                  digit(sb[j], m.shift, m.mask));
    if (take_a) {
      key[k] = sa[i];
      perm[k] = (uint32_t)(a0 + i);
      ++i;
    } else {
      key[k] = sb[j];
      perm[k] = (uint32_t)m.na + __ldg(m.b_perm + b0 + j);
      ++j;
    }
  }
  const uint64_t o = o0 + d;
  if (cnt == kMItems && (o & 3u) == 0) {
    *reinterpret_cast<uint4*>(m.keys_out + o) = make_uint4(key[0], key[1], key[2], key[3]);
    *reinterpret_cast<uint4*>(m.perm_out + o) = make_uint4(perm[0], perm[1], perm[2], perm[3]);
  } else {
    for (uint32_t k = 0; k < cnt; ++k) {
      m.keys_out[o + k] = key[k];
      m.perm_out[o + k] = perm[k];
    }
  }
}

// The whole input is the sorted prefix: keys copied, identity permutation.
__global__ void k_copy_identity(const uint32_t* __restrict__ keys_in, uint64_t n,
                                uint32_t* __restrict__ keys_out, uint32_t* __restrict__ perm_out) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    keys_out[i] = keys_in[i];
    perm_out[i] = (uint32_t)i;
  }
}

size_t round256(size_t b) { return (b + 255) & ~size_t(255); }

}  // namespace
}  // namespace plx

using namespace plx;

extern "C" size_t plx_sort_tail_scratch_bytes(uint64_t n) {
  const uint64_t parts = (n + kMT - 1) / kMT + 2;
  return plx_radix_sort_scratch_bytes(n) + 2 * round256(n * 4) + round256(parts * 8);
}

extern "C" int plx_sort_tail_u32(plx_ctx* ctx, uint64_t n, const uint64_t* n_sorted,
                                 const uint32_t* keys_in, uint32_t* keys_out, uint32_t* perm_out,
                                 uint32_t begin_bit, uint32_t end_bit, void* scratch,
                                 size_t scratch_bytes) {
  PLX_CHECK_ARG(ctx && n_sorted, "ctx and n_sorted are required");
  PLX_CHECK_ARG(n == 0 || (keys_in && keys_out && perm_out),
                "keys_in, keys_out and perm_out are required");
  PLX_CHECK_ARG(n < (1ull << 30), "n must be < 2^30");
  PLX_CHECK_ARG(begin_bit <= end_bit && end_bit <= 32, "bad bit range [%u, %u)", begin_bit,
                end_bit);
  PLX_CHECK_ARG(keys_in != keys_out, "keys_out must not alias keys_in");
  PLX_CHECK_ARG(aligned16(keys_out) && aligned16(perm_out),
                "keys_out and perm_out must be 16-byte aligned");
  PLX_CHECK_ARG(scratch && scratch_bytes >= plx_sort_tail_scratch_bytes(n),
                "scratch too small: need %zu bytes", plx_sort_tail_scratch_bytes(n));
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  if (n == 0) return PLX_OK;
  uint64_t na = 0;  // the prefix length lives in device memory (a compaction's count)
  PLX_TRY_CUDA(cudaMemcpyAsync(&na, n_sorted, sizeof(na), cudaMemcpyDeviceToHost, ctx->stream));
  PLX_TRY_CUDA(cudaStreamSynchronize(ctx->stream));
  PLX_CHECK_ARG(na <= n, "*n_sorted = %llu exceeds n = %llu", (unsigned long long)na,
                (unsigned long long)n);
  const uint64_t nb = n - na;
  const size_t rb = plx_radix_sort_scratch_bytes(n);
  if (na == 0)
    return plx_radix_sort_u32(ctx, n, keys_in, keys_out, perm_out, begin_bit, end_bit, scratch,
                              rb);
  if (nb == 0) {
    const unsigned g = (unsigned)std::min<uint64_t>((n + 255) / 256, 8ull * ctx->num_sms);
    k_copy_identity<<<g, 256, 0, ctx->stream>>>(keys_in, n, keys_out, perm_out);
    PLX_LAUNCH_CHECK("k_copy_identity");
    return PLX_OK;
  }
  char* s = static_cast<char*>(scratch);
  uint32_t* b_keys = reinterpret_cast<uint32_t*>(s + rb);
  uint32_t* b_perm = reinterpret_cast<uint32_t*>(s + rb + round256(n * 4));
  uint64_t* split = reinterpret_cast<uint64_t*>(s + rb + 2 * round256(n * 4));
  if (int rc = plx_radix_sort_u32(ctx, nb, keys_in + na, b_keys, b_perm, begin_bit, end_bit,
                                  scratch, rb))
    return rc;
  MergeArgs m{};
  m.a = keys_in;
  m.na = na;
  m.b = b_keys;
  m.b_perm = b_perm;
  m.nb = nb;
  m.shift = begin_bit;
  const uint32_t bits = end_bit - begin_bit;
  m.mask = bits >= 32 ? 0xFFFFFFFFu : ((1u << bits) - 1u);
  if (bits == 0) m.shift = 0;
  m.split = split;
  m.keys_out = keys_out;
  m.perm_out = perm_out;
  const uint64_t parts = (n + kMT - 1) / kMT;
  k_merge_split<<<(unsigned)((parts + 1 + 255) / 256), 256, 0, ctx->stream>>>(m, parts);
  PLX_LAUNCH_CHECK("k_merge_split");
  k_merge<<<(unsigned)parts, kMThreads, 0, ctx->stream>>>(m);
  PLX_LAUNCH_CHECK("k_merge");
  return PLX_OK;
}
