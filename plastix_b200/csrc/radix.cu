// K4: stable LSD radix sort (onesweep: one read and one write of the keys and
// values per 8-bit digit, decoupled lookback across tiles for the per-digit
// offsets) of u32 keys with a u32 payload, producing the sorted keys and the
// sorting permutation. plx_gather applies the permutation to the connection
// fields.
//
// Replaces, for connections re-sorted by destination after structural change,
// the reference's std::sort of CompactEdge bits (include/plastix/plastix.hpp
// :411-415) and its stable counting sort by SrcLevel + Gather
// (plastix.hpp:553-577, alloc.hpp:145-156). LSD radix sort is stable, so the
// output equals a stable sort by key: unique, and checked bit for bit.
//
// Per pass and tile (256 threads x 16 keys; warp w owns 512 consecutive keys,
// element order = (warp, item, lane)):
//   * each warp ranks its keys by digit with __match_any_sync and warp-private
//     shared digit counters (no block barrier per item), keeping the element
//     order (stable); per-digit warp bases come from one scan over the warps;
//   * the tile publishes its 256 digit counts, each thread looks back over
//     the predecessors of its digit, eight status words per step (relaxed
//     loads: a status word carries its own flag and value; bounded spin), and
//     publishes the prefix;
//   * keys are re-ordered by digit in shared memory and written out in
//     digit runs (coalesced).
#include "common.cuh"

namespace plx {

constexpr int kRT = 256;
constexpr int kRItems = 16;
constexpr int kRTile = kRT * kRItems;
constexpr int kRWarps = kRT / 32;
constexpr uint32_t kRFlagA = 1u << 30;
constexpr uint32_t kRFlagP = 2u << 30;
constexpr uint32_t kRValMask = (1u << 30) - 1;
constexpr int kRLook = 8;  // most predecessor status words loaded per look-back step

// Status words carry their flag and value in one 32-bit word and publish
// nothing else, so relaxed (non-fencing) accesses suffice.
__device__ __forceinline__ void st_status_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_status_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Histograms of every pass's digit over all keys (one read of the keys).
__global__ void __launch_bounds__(256) k_radix_hist(const uint32_t* __restrict__ keys,
                                                    uint64_t n, uint32_t begin_bit,
                                                    uint32_t end_bit, uint32_t passes,
                                                    uint32_t* __restrict__ hist) {
  __shared__ uint32_t s_h[4][256];
  for (uint32_t i = threadIdx.x; i < 4 * 256; i += blockDim.x) (&s_h[0][0])[i] = 0;
  __syncthreads();
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t k = __ldg(keys + i);
    for (uint32_t p = 0; p < passes; ++p) {
      const uint32_t sh = begin_bit + 8 * p;
      const uint32_t bits = min(8u, end_bit - sh);
      atomicAdd(&s_h[p][(k >> sh) & ((1u << bits) - 1u)], 1u);
    }
  }
  __syncthreads();
  for (uint32_t p = 0; p < passes; ++p)
    for (uint32_t d = threadIdx.x; d < 256; d += blockDim.x)
      if (s_h[p][d]) atomicAdd(&hist[p * 256 + d], s_h[p][d]);
}

// In place: hist[p][d] -> exclusive prefix over digits (global digit starts).
__global__ void k_radix_scan(uint32_t* hist, uint32_t passes) {
  __shared__ uint32_t s[256];
  const uint32_t p = blockIdx.x, d = threadIdx.x;
  if (p >= passes) return;
  const uint32_t v = hist[p * 256 + d];
  s[d] = v;
  __syncthreads();
  for (uint32_t o = 1; o < 256; o <<= 1) {
    const uint32_t t = d >= o ? s[d - o] : 0u;
    __syncthreads();
    s[d] += t;
    __syncthreads();
  }
  hist[p * 256 + d] = s[d] - v;
}

struct RadixPassArgs {
  const uint32_t* keys_in;
  const uint32_t* vals_in;  // null on the first pass: values are the indices
  uint32_t* keys_out;
  uint32_t* vals_out;
  uint64_t n;
  uint32_t shift;
  uint32_t mask;
  const uint32_t* digit_start;  // [256] global start of each digit
  uint32_t* status;             // [tiles][256], zeroed
  uint32_t* ticket;             // zeroed
  int32_t* dstatus;
  uint64_t timeout_ns;
  uint32_t ahead;  // tiles resident at once: the tile this far ahead is prefetched
};

// Asks L2 for the 16-byte-aligned part of [p, p + bytes).
__device__ __forceinline__ void prefetch_range(const void* p, uint64_t bytes) {
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(p);
  const uintptr_t lo = (a0 + 15) & ~uintptr_t(15), hi = (a0 + bytes) & ~uintptr_t(15);
  if (hi > lo) prefetch_l2_bulk(reinterpret_cast<const void*>(lo), (uint32_t)(hi - lo));
}

__global__ void __launch_bounds__(kRT, 4) k_radix_pass(RadixPassArgs a) {
  __shared__ uint32_t s_keys[kRTile];
  __shared__ uint32_t s_vals[kRTile];
  __shared__ uint32_t s_wcnt[kRWarps][256];  // per-warp digit counts, then warp bases
  __shared__ uint32_t s_run[256];
  __shared__ uint32_t s_local[256];
  __shared__ uint32_t s_gbase[256];
  __shared__ uint32_t s_wsum[kRWarps];
  __shared__ uint32_t s_tile;
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  if (tid == 0) s_tile = atomicAdd(a.ticket, 1u);
  for (uint32_t w = 0; w < kRWarps; ++w) s_wcnt[w][tid] = 0;
  __syncthreads();
  const uint64_t tile = s_tile;
  const uint64_t base = tile * kRTile;
  const uint32_t lt = (1u << lane) - 1u;
  // The tile one resident wave ahead starts after this one: bring its keys
  // and values into L2 now so its loads hit there.
  if (tid < 2) {
    const uint64_t b2 = (tile + a.ahead) * kRTile;
    if (b2 < a.n) {
      const uint64_t cnt = min((uint64_t)kRTile, a.n - b2);
      if (tid == 0) prefetch_range(a.keys_in + b2, cnt * 4);
      else if (a.vals_in) prefetch_range(a.vals_in + b2, cnt * 4);
    }
  }

  // Warp w owns tile elements [w * 512, (w + 1) * 512): item j of lane l is
  // element w * 512 + j * 32 + l, so element order is (warp, item, lane) and
  // every load is a coalesced 128-byte row.
  constexpr uint32_t kWarpSpan = kRItems * 32;
  uint32_t key[kRItems], val[kRItems], rank[kRItems];
#pragma unroll
  for (int j = 0; j < kRItems; ++j) {
    const uint64_t e = base + (uint64_t)warp * kWarpSpan + (uint64_t)j * 32 + lane;
    const bool ok = e < a.n;
    key[j] = ok ? a.keys_in[e] : 0u;
    val[j] = ok ? (a.vals_in ? a.vals_in[e] : (uint32_t)e) : 0u;
  }
  // Rank within the warp: lanes with the same digit are matched, counts kept
  // per warp in shared memory -- no block-wide barrier per item.
  uint32_t* wc = s_wcnt[warp];
#pragma unroll
  for (int j = 0; j < kRItems; ++j) {
    const uint64_t e = base + (uint64_t)warp * kWarpSpan + (uint64_t)j * 32 + lane;
    const bool ok = e < a.n;
    const uint32_t d = (key[j] >> a.shift) & a.mask;
    const uint32_t peers = __match_any_sync(0xffffffffu, ok ? d : 0x100u);
    const uint32_t lrank = __popc(peers & lt);
    const uint32_t before = ok ? wc[d] : 0u;
    __syncwarp();
    if (ok && lrank == 0) wc[d] = before + __popc(peers);
    __syncwarp();
    rank[j] = before + lrank;
  }
  __syncthreads();
  {  // digit tid: per-warp counts -> exclusive per-warp bases; tile count
    uint32_t run = 0;
#pragma unroll
    for (int w = 0; w < kRWarps; ++w) {
      const uint32_t c = s_wcnt[w][tid];
      s_wcnt[w][tid] = run;
      run += c;
    }
    s_run[tid] = run;
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kRItems; ++j) {
    const uint32_t d = (key[j] >> a.shift) & a.mask;
    rank[j] += wc[d];
  }
  // Tile digit counts: s_run. Publish, look back, publish prefix.
  const uint32_t cnt = s_run[tid];
  uint32_t* st = a.status + tile * 256;
  bool ok = true;
  uint32_t prefix = 0;
  if (tile == 0) {
    st_status_u32(&st[tid], kRFlagP | cnt);
  } else {
    st_status_u32(&st[tid], kRFlagA | cnt);
    // Look back kRLook predecessors per step (independent loads in flight),
    // consuming them in order: aggregates add up until the first
    // inclusive prefix; a predecessor not yet published is read again.
    int64_t p = (int64_t)tile - 1;
    const uint64_t t0 = global_timer_ns();
    uint32_t spin = 0;
    bool done = false;
    while (!done && p >= 0) {
      uint32_t sv[kRLook];
#pragma unroll
      for (int i = 0; i < kRLook; ++i)
        sv[i] = p - i >= 0 ? ld_status_u32(a.status + (uint64_t)(p - i) * 256 + tid) : 0u;
      int used = 0;
#pragma unroll
      for (int i = 0; i < kRLook; ++i) {
        if (done || used != i) continue;
        if (sv[i] & kRFlagP) {
          prefix += sv[i] & kRValMask;
          done = true;
        } else if (sv[i] & kRFlagA) {
          prefix += sv[i] & kRValMask;
          ++used;
        }
      }
      if (done) break;
      p -= used;
      if (used == 0 && (++spin & 255u) == 0 && global_timer_ns() - t0 > a.timeout_ns) {
        ok = false;
        break;
      }
    }
    st_status_u32(&st[tid], kRFlagP | (prefix + cnt));
  }
  if (!ok) record_status(a.dstatus, kStatusTimeout);
  s_gbase[tid] = a.digit_start[tid] + prefix;
  // local exclusive scan of the tile's digit counts: warp scans by shuffle,
  // then the eight warp totals
  uint32_t incl = cnt;
#pragma unroll
  for (uint32_t o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) s_wsum[warp] = incl;
  __syncthreads();
  uint32_t wbase = 0;
#pragma unroll
  for (int w = 0; w < kRWarps; ++w) wbase += (uint32_t)w < warp ? s_wsum[w] : 0u;
  s_local[tid] = wbase + incl - cnt;
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kRItems; ++j) {
    const uint64_t e = base + (uint64_t)warp * kWarpSpan + (uint64_t)j * 32 + lane;
    if (e < a.n) {
      const uint32_t d = (key[j] >> a.shift) & a.mask;
      const uint32_t pos = s_local[d] + rank[j];
      s_keys[pos] = key[j];
      s_vals[pos] = val[j];
    }
  }
  __syncthreads();
  const uint32_t valid = (uint32_t)min((uint64_t)kRTile, a.n - base);
  for (uint32_t p = tid; p < valid; p += kRT) {
    const uint32_t k = s_keys[p];
    const uint32_t d = (k >> a.shift) & a.mask;
    const uint64_t out = (uint64_t)s_gbase[d] + (p - s_local[d]);
    a.keys_out[out] = k;
    a.vals_out[out] = s_vals[p];
  }
}

struct RadixScratch {
  uint32_t* hist;    // [4][256]
  uint32_t* ticket;  // [4]
  uint32_t* status;  // [tiles][256]
  uint32_t* k_alt;   // [n]
  uint32_t* v_alt;   // [n]
};

static RadixScratch carve(void* scratch, uint64_t n) {
  char* p = static_cast<char*>(scratch);
  const uint64_t tiles = (n + kRTile - 1) / kRTile + 1;
  RadixScratch s;
  s.hist = reinterpret_cast<uint32_t*>(p);
  s.ticket = reinterpret_cast<uint32_t*>(p + 4096);
  s.status = reinterpret_cast<uint32_t*>(p + 4096 + 256);
  char* q = p + 4096 + 256 + ((tiles * 1024 + 255) & ~255ull);
  s.k_alt = reinterpret_cast<uint32_t*>(q);
  s.v_alt = reinterpret_cast<uint32_t*>(q + ((n * 4 + 255) & ~255ull));
  return s;
}

}  // namespace plx

using namespace plx;

extern "C" size_t plx_radix_sort_scratch_bytes(uint64_t n) {
  const uint64_t tiles = (n + kRTile - 1) / kRTile + 1;
  return (size_t)(4096 + 256 + ((tiles * 1024 + 255) & ~255ull) +
                  2 * ((n * 4 + 255) & ~255ull));
}

extern "C" int plx_radix_sort_u32(plx_ctx* ctx, uint64_t n, const uint32_t* keys_in,
                                  uint32_t* keys_out, uint32_t* perm_out,
                                  uint32_t begin_bit, uint32_t end_bit,
                                  void* scratch, size_t scratch_bytes) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  PLX_CHECK_ARG(n == 0 || (keys_in && keys_out && perm_out),
                "keys_in, keys_out and perm_out are required");
  PLX_CHECK_ARG(n < (1ull << 30), "n must be < 2^30 (per-tile digit offsets are 30-bit)");
  PLX_CHECK_ARG(begin_bit <= end_bit && end_bit <= 32, "bad bit range [%u, %u)",
                begin_bit, end_bit);
  PLX_CHECK_ARG(keys_in != keys_out, "keys_out must not alias keys_in");
  PLX_CHECK_ARG(scratch && scratch_bytes >= plx_radix_sort_scratch_bytes(n),
                "scratch too small: need %zu bytes", plx_radix_sort_scratch_bytes(n));
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  if (n == 0) return PLX_OK;
  const uint32_t passes = (end_bit - begin_bit + 7) / 8;
  RadixScratch s = carve(scratch, n);
  const uint64_t tiles = (n + kRTile - 1) / kRTile;
  PLX_TRY_CUDA(cudaMemsetAsync(s.hist, 0, 4096 + 256, ctx->stream));
  const uint64_t hb = std::min<uint64_t>((n + 255) / 256, 4ull * ctx->num_sms);
  if (passes) {
    k_radix_hist<<<(unsigned)hb, 256, 0, ctx->stream>>>(keys_in, n, begin_bit, end_bit,
                                                        passes, s.hist);
    PLX_LAUNCH_CHECK("k_radix_hist");
    k_radix_scan<<<passes, 256, 0, ctx->stream>>>(s.hist, passes);
    PLX_LAUNCH_CHECK("k_radix_scan");
  }
  // Ping-pong so that the last pass lands in keys_out / perm_out.
  const uint32_t np = passes ? passes : 1;
  const uint32_t* kin = keys_in;
  const uint32_t* vin = nullptr;
  for (uint32_t p = 0; p < np; ++p) {
    const bool to_user = ((np - 1 - p) & 1u) == 0;
    uint32_t* kout = to_user ? keys_out : s.k_alt;
    uint32_t* vout = to_user ? perm_out : s.v_alt;
    PLX_TRY_CUDA(cudaMemsetAsync(s.status, 0, tiles * 1024, ctx->stream));
    PLX_TRY_CUDA(cudaMemsetAsync(s.ticket + p, 0, 4, ctx->stream));
    RadixPassArgs a{};
    a.keys_in = kin;
    a.vals_in = vin;
    a.keys_out = kout;
    a.vals_out = vout;
    a.n = n;
    a.shift = passes ? begin_bit + 8 * p : 0;
    const uint32_t bits = passes ? std::min(8u, end_bit - (begin_bit + 8 * p)) : 0;
    a.mask = (1u << bits) - 1u;
    a.digit_start = s.hist + (passes ? p * 256 : 0);
    a.status = s.status;
    a.ticket = s.ticket + p;
    a.dstatus = ctx->d_status;
    a.timeout_ns = ctx->timeout_ns;
    a.ahead = 4u * (uint32_t)ctx->num_sms;
    k_radix_pass<<<(unsigned)tiles, kRT, 0, ctx->stream>>>(a);
    PLX_LAUNCH_CHECK("k_radix_pass");
    kin = kout;
    vin = vout;
  }
  return PLX_OK;
}
