// K3: order-preserving stream compaction of the connection SoA with a
// single-pass decoupled-lookback scan, plus the device Gather and the seeded
// regrowth used by the structural-plasticity step.
//
// Reference: the reference never removes connections; DoPruneConnections
// (include/plastix/plastix.hpp:280-297) only sets Dead. Compaction is defined
// as the reference's SOAAllocator::Gather (include/plastix/alloc.hpp:145-156)
// applied to the increasing list of surviving ids, so the output is unique
// and checked bit for bit.
//
// Each CTA takes the next tile of 4096 connections from an atomic ticket (so
// every predecessor tile is already running), evaluates the keep predicate,
// counts survivors with warp ballots, publishes its count, looks back over
// its predecessors' published counts/prefixes (bounded spin), publishes its
// inclusive prefix, and scatters the survivors of every field in order.
#include "common.cuh"

namespace plx {

constexpr int kCT = 256;            // threads per CTA
constexpr int kCItems = 16;         // items per thread
constexpr int kCTile = kCT * kCItems;
constexpr uint32_t kMaxFields = PLX_MAX_FIELDS;

constexpr uint64_t kFlagA = 1ull << 62;  // aggregate published
constexpr uint64_t kFlagP = 2ull << 62;  // inclusive prefix published
constexpr uint64_t kValMask = (1ull << 62) - 1;

struct FieldDesc {
  const void* src;
  void* dst;
  uint32_t bytes;
  uint32_t flags;
};

struct CompactArgs {
  uint64_t n;
  int keep_kind;
  const void* keep_src;
  float threshold;
  uint32_t n_fields;
  FieldDesc f[kMaxFields];
  uint32_t* perm_out;
  uint64_t* count_out;
  uint64_t* status;   // one word per tile, zeroed
  uint32_t* ticket;   // zeroed
  int32_t* dstatus;
  uint64_t timeout_ns;
};

// A status word holds its flag and value together and publishes nothing else,
// so relaxed (non-fencing) accesses suffice.
__device__ __forceinline__ void st_status_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_status_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool keep_pred(const CompactArgs& a, uint64_t e) {
  switch (a.keep_kind) {
    case PLX_KEEP_FLAGS:
      return static_cast<const uint8_t*>(a.keep_src)[e] != 0;
    case PLX_KEEP_NOT_DEAD:
      return static_cast<const uint8_t*>(a.keep_src)[e] == 0;
    default: {  // PLX_KEEP_ABS_GE: prune when |v| < threshold
      const float v = static_cast<const float*>(a.keep_src)[e];
      return !(fabsf(v) < a.threshold);
    }
  }
}

__device__ __forceinline__ uint64_t load_elem(const FieldDesc& f, uint64_t from) {
  switch (f.bytes) {
    case 1: return static_cast<const uint8_t*>(f.src)[from];
    case 2: return static_cast<const uint16_t*>(f.src)[from];
    case 4: return static_cast<const uint32_t*>(f.src)[from];
    default: return static_cast<const uint64_t*>(f.src)[from];
  }
}

__device__ __forceinline__ void store_elem(const FieldDesc& f, uint64_t to, uint64_t v) {
  switch (f.bytes) {
    case 1: {
      uint8_t b = (uint8_t)v;
      if (f.flags & PLX_FIELD_INC_SAT_U8) b = b == 255 ? 255 : (uint8_t)(b + 1);
      static_cast<uint8_t*>(f.dst)[to] = b;
      break;
    }
    case 2: static_cast<uint16_t*>(f.dst)[to] = (uint16_t)v; break;
    case 4: static_cast<uint32_t*>(f.dst)[to] = (uint32_t)v; break;
    default: static_cast<uint64_t*>(f.dst)[to] = v; break;
  }
}

__device__ __forceinline__ void copy_elem(const FieldDesc& f, uint64_t from,
                                          uint64_t to) {
  switch (f.bytes) {
    case 1: {
      uint8_t v = static_cast<const uint8_t*>(f.src)[from];
      if (f.flags & PLX_FIELD_INC_SAT_U8) v = v == 255 ? 255 : (uint8_t)(v + 1);
      static_cast<uint8_t*>(f.dst)[to] = v;
      break;
    }
    case 2:
      static_cast<uint16_t*>(f.dst)[to] = static_cast<const uint16_t*>(f.src)[from];
      break;
    case 4:
      static_cast<uint32_t*>(f.dst)[to] = static_cast<const uint32_t*>(f.src)[from];
      break;
    default:
      static_cast<uint64_t*>(f.dst)[to] = static_cast<const uint64_t*>(f.src)[from];
      break;
  }
}

__global__ void __launch_bounds__(kCT) k_compact(CompactArgs a) {
  __shared__ uint32_t s_tile;
  __shared__ uint32_t s_cnt[kCItems * (kCT / 32)];  // [item][warp], then prefixes
  __shared__ uint64_t s_prefix;
  __shared__ uint32_t s_total;
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  if (tid == 0) s_tile = atomicAdd(a.ticket, 1u);
  __syncthreads();
  const uint64_t tile = s_tile;
  const uint64_t base = tile * kCTile;
  // The fields are copied only after the lookback; ask for the tile's ranges
  // in L2 now so those copies do not wait on DRAM.
  if (tid < a.n_fields && base < a.n) {
    const FieldDesc& fd = a.f[tid];
    const uint64_t cnt = min((uint64_t)kCTile, a.n - base);
    const uintptr_t p0 = reinterpret_cast<uintptr_t>(fd.src) + base * fd.bytes;
    const uintptr_t lo = (p0 + 15) & ~uintptr_t(15);              // inside the range
    const uintptr_t hi = (p0 + cnt * fd.bytes) & ~uintptr_t(15);
    if (hi > lo) prefetch_l2_bulk(reinterpret_cast<const void*>(lo), (uint32_t)(hi - lo));
  }

  uint32_t masks[kCItems];
#pragma unroll
  for (int j = 0; j < kCItems; ++j) {
    const uint64_t e = base + (uint64_t)j * kCT + tid;
    const bool k = e < a.n && keep_pred(a, e);
    masks[j] = __ballot_sync(0xffffffffu, k);
    if (lane == 0) s_cnt[j * (kCT / 32) + warp] = __popc(masks[j]);
  }
  __syncthreads();
  if (warp == 0) {
    // exclusive scan of the 128 counts in element order (item-major, warp)
    constexpr int kPer = kCItems * (kCT / 32) / 32;  // 4 per lane
    uint32_t v[kPer], s = 0;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      v[i] = s_cnt[lane * kPer + i];
      s += v[i];
    }
    uint32_t incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= (uint32_t)o) incl += t;
    }
    uint32_t run = incl - s;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      s_cnt[lane * kPer + i] = run;
      run += v[i];
    }
    if (lane == 31) s_total = incl;
  }
  __syncthreads();
  if (warp == 0) {
    // Warp-cooperative lookback: lane l reads predecessor p - l, so 32 status
    // words are in flight per step; values are consumed in order up to the
    // first inclusive prefix, or up to the first predecessor not yet
    // published (read again in the next step).
    const uint64_t agg = s_total;
    uint64_t prefix = 0;
    bool ok = true;
    if (tile == 0) {
      if (lane == 0) st_status_u64(&a.status[0], kFlagP | agg);
    } else {
      if (lane == 0) st_status_u64(&a.status[tile], kFlagA | agg);
      int64_t p = (int64_t)tile - 1;
      const uint64_t t0 = __shfl_sync(0xffffffffu, global_timer_ns(), 0);
      uint32_t spin = 0;
      for (;;) {
        const int64_t q = p - (int64_t)lane;
        const uint64_t sv = q >= 0 ? ld_status_u64(&a.status[q]) : 0ull;
        const uint32_t m_p = __ballot_sync(0xffffffffu, (sv & kFlagP) != 0);
        const uint32_t m_v = __ballot_sync(0xffffffffu, (sv & (kFlagA | kFlagP)) != 0);
        const int first_inv = ~m_v ? __ffs(~m_v) - 1 : 32;
        const int first_p = m_p ? __ffs(m_p) - 1 : 32;
        const bool done = first_p < first_inv;
        const int take = done ? first_p + 1 : first_inv;
        uint64_t v = (int)lane < take ? (sv & kValMask) : 0ull;
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        prefix += v;
        if (done) break;
        p -= take;
        if (take == 0 && (++spin & 255u) == 0) {
          const uint64_t now = __shfl_sync(0xffffffffu, global_timer_ns(), 0);
          if (now - t0 > a.timeout_ns) {
            ok = false;
            break;
          }
        }
      }
      if (lane == 0) st_status_u64(&a.status[tile], kFlagP | (prefix + agg));
    }
    if (lane == 0) {
      if (!ok) record_status(a.dstatus, kStatusTimeout);
      s_prefix = prefix;
      const uint64_t n_tiles = (a.n + kCTile - 1) / kCTile;
      if (tile == n_tiles - 1 || a.n == 0) *a.count_out = prefix + agg;
    }
  }
  __syncthreads();
  const uint64_t prefix = s_prefix;
  const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
  for (int j = 0; j < kCItems; ++j) {
    if (!((masks[j] >> lane) & 1u)) continue;
    const uint64_t e = base + (uint64_t)j * kCT + tid;
    const uint64_t pos = prefix + s_cnt[j * (kCT / 32) + warp] + __popc(masks[j] & lt);
    // fields four at a time: the group's loads are issued before its stores
    for (uint32_t f0 = 0; f0 < a.n_fields; f0 += 4) {
      uint64_t v[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (f0 + q < a.n_fields) v[q] = load_elem(a.f[f0 + q], e);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (f0 + q < a.n_fields) store_elem(a.f[f0 + q], pos, v[q]);
    }
    if (a.perm_out) a.perm_out[pos] = (uint32_t)e;
  }
}

// dst[i] = src[perm[i]] for every field (SOAAllocator::Gather, alloc.hpp:145-156).
struct GatherArgs {
  uint64_t n;
  const uint32_t* perm;
  uint32_t n_fields;
  FieldDesc f[kMaxFields];
};

__global__ void __launch_bounds__(256) k_gather(GatherArgs a) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < a.n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t p = __ldg(a.perm + i);
    for (uint32_t f = 0; f < a.n_fields; ++f) copy_elem(a.f[f], p, i);
  }
}

// Seeded regrowth: connections [count, n) get fresh (src, dst) pairs, weight
// 0 and age 0. Connection i of the regrown block uses
//   h = mix64(mix64(seed) + step_base + (i - count))
//   src = src_base + ((h & 0xffffffff) * n_src >> 32)
//   dst = dst_base + ((h >> 32) * n_dst >> 32)
// with mix64 the SplitMix64 finaliser (Steele, Lea, Flood 2014).
__host__ __device__ inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

struct RegrowArgs {
  uint64_t n;
  const uint64_t* count;  // survivors (device)
  uint32_t* from_id;
  uint32_t* to_id;
  float* weight;
  uint8_t* age;
  uint32_t src_base, n_src, dst_base, n_dst;
  uint64_t seed, step_base;
};

__global__ void k_regrow(RegrowArgs a) {
  const uint64_t m = *a.count;
  const uint64_t key = mix64(a.seed) + a.step_base;
  for (uint64_t i = m + blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < a.n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t h = mix64(key + (i - m));
    a.from_id[i] = a.src_base + (uint32_t)(((h & 0xffffffffull) * a.n_src) >> 32);
    a.to_id[i] = a.dst_base + (uint32_t)(((h >> 32) * a.n_dst) >> 32);
    if (a.weight) a.weight[i] = 0.0f;
    if (a.age) a.age[i] = 0;
  }
}

static int fill_fields(FieldDesc* out, const plx_field* in, uint32_t n_fields,
                       uint64_t n) {
  PLX_CHECK_ARG(n_fields <= kMaxFields, "at most %u fields", kMaxFields);
  PLX_CHECK_ARG(n == 0 || n_fields == 0 || in, "fields are required");
  for (uint32_t i = 0; i < n_fields; ++i) {
    const uint32_t b = in[i].elem_bytes;
    PLX_CHECK_ARG(b == 1 || b == 2 || b == 4 || b == 8, "field %u: elem_bytes %u", i, b);
    PLX_CHECK_ARG(n == 0 || (in[i].src && in[i].dst), "field %u: src and dst required", i);
    PLX_CHECK_ARG(!(in[i].flags & PLX_FIELD_INC_SAT_U8) || b == 1,
                  "field %u: PLX_FIELD_INC_SAT_U8 needs a 1-byte field", i);
    out[i] = FieldDesc{in[i].src, in[i].dst, b, in[i].flags};
  }
  return PLX_OK;
}

}  // namespace plx

using namespace plx;

extern "C" size_t plx_compact_scratch_bytes(uint64_t n) {
  const uint64_t tiles = (n + kCTile - 1) / kCTile + 1;
  return (size_t)(tiles * 8 + 256);
}

extern "C" int plx_compact(plx_ctx* ctx, uint64_t n, int keep_kind,
                           const void* keep_src, float threshold,
                           const plx_field* fields, uint32_t n_fields,
                           uint32_t* perm_out, uint64_t* count_out,
                           void* scratch, size_t scratch_bytes) {
  PLX_CHECK_ARG(ctx && count_out, "ctx and count_out are required");
  PLX_CHECK_ARG(keep_kind == PLX_KEEP_FLAGS || keep_kind == PLX_KEEP_NOT_DEAD ||
                    keep_kind == PLX_KEEP_ABS_GE,
                "unknown keep_kind %d", keep_kind);
  PLX_CHECK_ARG(n == 0 || keep_src, "keep_src is required");
  PLX_CHECK_ARG(n < (1ull << 32), "n must be < 2^32");
  PLX_CHECK_ARG(scratch && scratch_bytes >= plx_compact_scratch_bytes(n),
                "scratch too small: need %zu bytes", plx_compact_scratch_bytes(n));
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  CompactArgs a{};
  if (int rc = fill_fields(a.f, fields, n_fields, n)) return rc;
  a.n = n;
  a.keep_kind = keep_kind;
  a.keep_src = keep_src;
  a.threshold = threshold;
  a.n_fields = n_fields;
  a.perm_out = perm_out;
  a.count_out = count_out;
  const uint64_t tiles = (n + kCTile - 1) / kCTile;
  a.ticket = static_cast<uint32_t*>(scratch);
  a.status = reinterpret_cast<uint64_t*>(static_cast<char*>(scratch) + 256);
  a.dstatus = ctx->d_status;
  a.timeout_ns = ctx->timeout_ns;
  PLX_TRY_CUDA(cudaMemsetAsync(scratch, 0, 256 + tiles * 8, ctx->stream));
  const unsigned grid = (unsigned)(tiles ? tiles : 1);
  k_compact<<<grid, kCT, 0, ctx->stream>>>(a);
  PLX_LAUNCH_CHECK("k_compact");
  return PLX_OK;
}

extern "C" int plx_gather(plx_ctx* ctx, uint64_t n, const uint32_t* perm,
                          const plx_field* fields, uint32_t n_fields) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  PLX_CHECK_ARG(n == 0 || perm, "perm is required");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  GatherArgs a{};
  if (int rc = fill_fields(a.f, fields, n_fields, n)) return rc;
  for (uint32_t i = 0; i < n_fields; ++i)
    PLX_CHECK_ARG(!(fields[i].flags & PLX_FIELD_INC_SAT_U8),
                  "plx_gather copies fields unchanged");
  a.n = n;
  a.perm = perm;
  a.n_fields = n_fields;
  if (n == 0) return PLX_OK;
  const uint64_t blocks = std::min<uint64_t>((n + 255) / 256, 16ull * ctx->num_sms);
  k_gather<<<(unsigned)blocks, 256, 0, ctx->stream>>>(a);
  PLX_LAUNCH_CHECK("k_gather");
  return PLX_OK;
}

extern "C" int plx_regrow(plx_ctx* ctx, uint64_t n, const uint64_t* count,
                          uint32_t* from_id, uint32_t* to_id, float* weight,
                          uint8_t* age, uint32_t src_base, uint32_t n_src,
                          uint32_t dst_base, uint32_t n_dst, uint64_t seed,
                          uint64_t step_base) {
  PLX_CHECK_ARG(ctx && count && from_id && to_id, "ctx, count, from_id, to_id required");
  PLX_CHECK_ARG(n_src > 0 && n_dst > 0, "n_src and n_dst must be positive");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  RegrowArgs a{n, count, from_id, to_id, weight, age, src_base, n_src, dst_base, n_dst,
               seed, step_base};
  if (n == 0) return PLX_OK;
  const uint64_t blocks = std::min<uint64_t>((n + 255) / 256, 8ull * ctx->num_sms);
  k_regrow<<<(unsigned)blocks, 256, 0, ctx->stream>>>(a);
  PLX_LAUNCH_CHECK("k_regrow");
  return PLX_OK;
}

// ---------------------------------------------------------------------------
// Compaction that allocates nothing.
//
// For callers that cannot allocate device memory at the point where they
// compact: code running inside a region where an allocation would break the
// caller's guarantees (a real-time step loop with a fixed memory budget, a
// host framework that owns every device allocation through its own pool and
// forbids libraries from calling cudaMalloc). The scratch lives in the static
// array below, which every GPU that loads this library holds until exit.
// ---------------------------------------------------------------------------
#include <mutex>

namespace plx {

constexpr uint64_t kNoAllocMaxN = 1ull << 28;             // 268,435,456 connections
constexpr uint64_t kNoAllocTiles = kNoAllocMaxN / kCTile;  // 65,536 tiles
constexpr size_t kNoAllocBytes = 256 + kNoAllocTiles * 8;  // 512 KiB + 256 B
constexpr int kNoAllocMaxDevices = 64;

// [0, 4): tile ticket; [4, 8): device status word; [256, ...): tile status.
static __device__ __align__(256) unsigned char g_compact_scratch[kNoAllocBytes];

struct NoAllocSlot {
  std::once_flag once;
  unsigned char* ptr = nullptr;
  cudaError_t err = cudaSuccess;
};
static NoAllocSlot g_noalloc_slots[kNoAllocMaxDevices];

// A bounded wait that expired leaves the count at UINT64_MAX.
__global__ void k_compact_noalloc_finish(const int32_t* status, uint64_t* count_out) {
  if (*status != kStatusOk) *count_out = ~0ull;
}

}  // namespace plx

extern "C" int plx_compact_noalloc(void* stream, uint64_t n, int keep_kind,
                                   const void* keep_src, float threshold,
                                   const plx_field* fields, uint32_t n_fields,
                                   uint32_t* perm_out, uint64_t* count_out) {
  PLX_CHECK_ARG(count_out, "count_out is required");
  PLX_CHECK_ARG(keep_kind == PLX_KEEP_FLAGS || keep_kind == PLX_KEEP_NOT_DEAD ||
                    keep_kind == PLX_KEEP_ABS_GE,
                "unknown keep_kind %d", keep_kind);
  PLX_CHECK_ARG(n == 0 || keep_src, "keep_src is required");
  PLX_CHECK_ARG(n <= kNoAllocMaxN,
                "n = %llu exceeds the no-allocation limit of %llu connections; "
                "use plx_compact with caller-provided scratch",
                (unsigned long long)n, (unsigned long long)kNoAllocMaxN);
  int dev = 0;
  PLX_TRY_CUDA(cudaGetDevice(&dev));
  PLX_CHECK_ARG(dev >= 0 && dev < kNoAllocMaxDevices, "device %d out of range", dev);
  NoAllocSlot& slot = g_noalloc_slots[dev];
  // Once per device, with that device current: the device address of the
  // static scratch (its host-side name is only a stand-in for the symbol).
  std::call_once(slot.once, [&slot] {
    slot.err = cudaGetSymbolAddress(reinterpret_cast<void**>(&slot.ptr), g_compact_scratch);
  });
  if (slot.err != cudaSuccess) return check_cuda(slot.err, "cudaGetSymbolAddress");
  CompactArgs a{};
  if (int rc = fill_fields(a.f, fields, n_fields, n)) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint64_t tiles = (n + kCTile - 1) / kCTile;
  a.n = n;
  a.keep_kind = keep_kind;
  a.keep_src = keep_src;
  a.threshold = threshold;
  a.n_fields = n_fields;
  a.perm_out = perm_out;
  a.count_out = count_out;
  a.ticket = reinterpret_cast<uint32_t*>(slot.ptr);
  a.dstatus = reinterpret_cast<int32_t*>(slot.ptr + 4);
  a.status = reinterpret_cast<uint64_t*>(slot.ptr + 256);
  a.timeout_ns = 2000000000ull;
  // The array keeps the previous call's contents: clear ticket, status word
  // and the tile words this call uses.
  PLX_TRY_CUDA(cudaMemsetAsync(slot.ptr, 0, 256 + tiles * 8, s));
  k_compact<<<(unsigned)(tiles ? tiles : 1), kCT, 0, s>>>(a);
  PLX_LAUNCH_CHECK("k_compact");
  k_compact_noalloc_finish<<<1, 1, 0, s>>>(a.dstatus, count_out);
  PLX_LAUNCH_CHECK("k_compact_noalloc_finish");
  return PLX_OK;
}
