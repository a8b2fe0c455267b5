// Unit levels on the device: RecomputeLevels (include/plastix/plastix.hpp:
// 466-537), the level-parallel Kahn pass the Topological model runs before it
// re-sorts the connections by source level (:539-579).
//
// Reference semantics kept exactly:
//   * levels of non-input units are reset to 0; nothing else happens when the
//     network has no connections (:470-474);
//   * in-degrees and outgoing lists count live connections only (:488-493,
//     :507-512);
//   * round L starts from frontier L (round 0: the input units, :515-517); each
//     live outgoing connection of a frontier unit decrements its target's
//     in-degree, and the decrement that reaches 0 gives the target level L+1
//     (as uint16) and puts it into frontier L+1 (:523-531);
//   * rounds run until a frontier is empty.
// A target reaches 0 in round L exactly when its remaining in-degree c before
// the round satisfies 1 <= c <= d, d being the round's decrements of it, so the
// result does not depend on the order within a round: each round runs fully
// in parallel (atomicSub returning 1 is the reference's `--InDegree == 0`,
// wrap-around included), and only the order of units inside a frontier --
// which the reference never exposes -- differs.
//
// Design (B200): counting and scatter kernels build the outgoing lists (CUB
// exclusive scan for the offsets); one cooperative persistent kernel then runs
// every round, a warp per frontier unit, with warp-aggregated appends to the
// next frontier and a grid barrier between rounds whose wait is bounded (a
// barrier that runs out records PLX_ERR_TIMEOUT and every block returns).
#include <cub/device/device_scan.cuh>

#include "common.cuh"

namespace plx {
namespace {

constexpr uint32_t kFullMask = 0xFFFFFFFFu;

size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

size_t lv_scan_temp(uint64_t n_items) {
  size_t t = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, t, (const uint32_t*)nullptr, (uint32_t*)nullptr,
                                (int64_t)n_items);
  return t;
}

unsigned grid_for(const plx_ctx* ctx, uint64_t n) {
  return (unsigned)std::max<uint64_t>(
      1, std::min<uint64_t>((n + 255) / 256, 8ull * (uint64_t)ctx->num_sms));
}

// Scratch words after the arrays: frontier sizes (three, rotating), barrier
// arrival count and generation, the number of rounds run.
struct LvCounters {
  uint32_t size[3];
  uint32_t arrive;
  uint32_t gen;
  uint32_t rounds;
};

struct LvScratch {
  uint32_t* in_deg;    // [n_units]
  uint32_t* out_off;   // [n_units + 1]
  uint32_t* cursor;    // [n_units + 1] out-degrees, then write cursors
  uint32_t* out_to;    // [n_conns] target of each live outgoing connection
  uint32_t* front[2];  // [n_units] each
  LvCounters* cnt;
  void* temp;
  size_t temp_bytes;
};

LvScratch lv_layout(void* base, uint64_t n_units, uint64_t n_conns) {
  char* p = static_cast<char*>(base);
  LvScratch s;
  s.in_deg = reinterpret_cast<uint32_t*>(p);
  p += al256(4 * n_units);
  s.out_off = reinterpret_cast<uint32_t*>(p);
  p += al256(4 * (n_units + 1));
  s.cursor = reinterpret_cast<uint32_t*>(p);
  p += al256(4 * (n_units + 1));
  s.out_to = reinterpret_cast<uint32_t*>(p);
  p += al256(4 * std::max<uint64_t>(n_conns, 1));
  s.front[0] = reinterpret_cast<uint32_t*>(p);
  p += al256(4 * std::max<uint64_t>(n_units, 1));
  s.front[1] = reinterpret_cast<uint32_t*>(p);
  p += al256(4 * std::max<uint64_t>(n_units, 1));
  s.cnt = reinterpret_cast<LvCounters*>(p);
  p += 256;
  s.temp = p;
  s.temp_bytes = lv_scan_temp(n_units + 1);
  return s;
}

size_t lv_bytes(uint64_t n_units, uint64_t n_conns) {
  return 3 * al256(4 * (n_units + 1)) + al256(4 * std::max<uint64_t>(n_conns, 1)) +
         2 * al256(4 * std::max<uint64_t>(n_units, 1)) + 256 + lv_scan_temp(n_units + 1) + 256;
}

__device__ __forceinline__ bool lv_live(const uint8_t* dead, uint64_t c) {
  return dead == nullptr || dead[c] == 0;
}

// Levels of non-input units to 0; frontier 0 = the input units.
__global__ void k_lv_reset(uint16_t* __restrict__ level, uint32_t n_units, uint32_t n_input,
                           uint32_t* __restrict__ front0) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n_units;
       i += gridDim.x * blockDim.x) {
    if (i >= n_input) level[i] = 0;
    else front0[i] = i;
  }
}

// Out-degree by FromId (into cursor), in-degree by ToId, live connections.
__global__ void k_lv_degrees(const uint32_t* __restrict__ from_id,
                             const uint32_t* __restrict__ to_id, const uint8_t* __restrict__ dead,
                             uint64_t n_conns, uint32_t n_units, uint32_t* __restrict__ out_deg,
                             uint32_t* __restrict__ in_deg, int32_t* status) {
  bool bad = false;
  for (uint64_t c = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; c < n_conns;
       c += (uint64_t)gridDim.x * blockDim.x) {
    if (!lv_live(dead, c)) continue;
    const uint32_t f = from_id[c], t = to_id[c];
    if (f >= n_units || t >= n_units) {
      bad = true;
      continue;
    }
    atomicAdd(out_deg + f, 1u);
    atomicAdd(in_deg + t, 1u);
  }
  if (bad) record_status(status, kStatusBadIndex);
}

// Outgoing lists: the target of every live connection under its source.
__global__ void k_lv_scatter(const uint32_t* __restrict__ from_id,
                             const uint32_t* __restrict__ to_id, const uint8_t* __restrict__ dead,
                             uint64_t n_conns, uint32_t n_units, uint32_t* __restrict__ cursor,
                             uint32_t* __restrict__ out_to) {
  for (uint64_t c = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; c < n_conns;
       c += (uint64_t)gridDim.x * blockDim.x) {
    if (!lv_live(dead, c)) continue;
    const uint32_t f = from_id[c], t = to_id[c];
    if (f >= n_units || t >= n_units) continue;
    out_to[atomicAdd(cursor + f, 1u)] = t;
  }
}

// Grid barrier for a cooperative launch; false when the wait ran past
// timeout_ns (the caller records the status and returns).
__device__ bool lv_grid_barrier(LvCounters* cnt, uint64_t timeout_ns) {
  __syncthreads();
  bool ok = true;
  if (threadIdx.x == 0) {
    volatile uint32_t* gen = &cnt->gen;
    const uint32_t g = *gen;
    __threadfence();
    if (atomicAdd(&cnt->arrive, 1u) == gridDim.x - 1) {
      cnt->arrive = 0;
      __threadfence();
      atomicAdd(&cnt->gen, 1u);
    } else {
      const uint64_t t0 = global_timer_ns();
      for (uint32_t spin = 0; *gen == g; ++spin) {
        if ((spin & 63u) == 63u && global_timer_ns() - t0 > timeout_ns) {
          ok = false;
          break;
        }
      }
    }
    __threadfence();
  }
  return __syncthreads_and(ok) != 0;
}

// Every round of the level-parallel Kahn pass.
__global__ void __launch_bounds__(256) k_lv_rounds(
    const uint32_t* __restrict__ out_off, const uint32_t* __restrict__ out_to,
    uint32_t* __restrict__ in_deg, uint16_t* __restrict__ level, uint32_t* front0,
    uint32_t* front1, LvCounters* cnt, uint32_t* rounds_out, int32_t* status,
    uint64_t timeout_ns) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t n_warps = (gridDim.x * blockDim.x) >> 5;
  uint32_t L = 0;
  for (;; ++L) {
    volatile uint32_t* sizes = cnt->size;
    const uint32_t sz = sizes[L % 3];
    if (sz == 0) break;
    const uint32_t* cur = (L & 1u) ? front1 : front0;
    uint32_t* nxt = (L & 1u) ? front0 : front1;
    uint32_t* nsz = &cnt->size[(L + 1) % 3];
    if (blockIdx.x == 0 && threadIdx.x == 0) cnt->size[(L + 2) % 3] = 0;  // read in round L-1
    const uint16_t lv = (uint16_t)(L + 1u);
    for (uint32_t f = warp; f < sz; f += n_warps) {
      const uint32_t u = cur[f];
      const uint32_t e1 = out_off[u + 1];
      for (uint32_t e = out_off[u] + lane; e < e1; e += 32) {
        const uint32_t t = out_to[e];
        const bool fire = atomicSub(in_deg + t, 1u) == 1u;
        const uint32_t act = __activemask();
        const uint32_t m = __ballot_sync(act, fire);
        if (m) {
          const uint32_t leader = __ffs(m) - 1;
          uint32_t base = 0;
          if (lane == leader) base = atomicAdd(nsz, (uint32_t)__popc(m));
          base = __shfl_sync(act, base, leader);
          if (fire) {
            level[t] = lv;
            nxt[base + __popc(m & ((1u << lane) - 1u))] = t;
          }
        }
      }
    }
    if (!lv_grid_barrier(cnt, timeout_ns)) {
      if (threadIdx.x == 0) record_status(status, kStatusTimeout);
      return;
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && rounds_out) *rounds_out = L;
}

// src_level[c] = level[from_id[c]] (SortConnectionsByLevel, plastix.hpp:546-549).
__global__ void k_src_levels(const uint32_t* __restrict__ from_id, uint64_t n,
                             const uint16_t* __restrict__ level, uint32_t n_units,
                             uint16_t* __restrict__ src_level, int32_t* status) {
  bool bad = false;
  for (uint64_t c = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; c < n;
       c += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t f = from_id[c];
    bad |= f >= n_units;
    src_level[c] = f < n_units ? level[f] : (uint16_t)0;
  }
  if (bad) record_status(status, kStatusBadIndex);
}

}  // namespace
}  // namespace plx

using namespace plx;

extern "C" size_t plx_recompute_levels_scratch_bytes(uint64_t n_units, uint64_t n_conns) {
  return lv_bytes(n_units, n_conns);
}

extern "C" int plx_recompute_levels(plx_ctx* ctx, uint32_t n_units, uint32_t n_input,
                                    uint64_t n_conns, const uint32_t* from_id,
                                    const uint32_t* to_id, const uint8_t* dead,
                                    uint16_t* level, uint32_t* rounds_out, void* scratch,
                                    size_t scratch_bytes) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  PLX_CHECK_ARG(n_input <= n_units, "n_input must be <= n_units");
  PLX_CHECK_ARG(n_units == 0 || level, "level is required");
  PLX_CHECK_ARG(n_conns == 0 || (from_id && to_id), "from_id and to_id are required");
  PLX_CHECK_ARG(n_conns < 0xFFFFFFFFull, "n_conns must be < 2^32 - 1");
  PLX_CHECK_ARG(n_units < 0xFFFFFFFFu, "n_units must be < 2^32 - 1");
  PLX_CHECK_ARG(scratch && scratch_bytes >= lv_bytes(n_units, n_conns), "scratch too small");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  cudaStream_t st = ctx->stream;
  const LvScratch s = lv_layout(scratch, n_units, n_conns);
  if (n_units == 0 || n_conns == 0) {
    // No BFS: only the reset of non-input levels (plastix.hpp:470-474).
    if (n_units)
      k_lv_reset<<<grid_for(ctx, n_units), 256, 0, st>>>(level, n_units, n_input, s.front[0]);
    PLX_LAUNCH_CHECK("k_lv_reset");
    if (rounds_out) PLX_TRY_CUDA(cudaMemsetAsync(rounds_out, 0, sizeof(uint32_t), st));
    return PLX_OK;
  }
  PLX_TRY_CUDA(cudaMemsetAsync(s.in_deg, 0, 4ull * n_units, st));
  PLX_TRY_CUDA(cudaMemsetAsync(s.cursor, 0, 4ull * (n_units + 1), st));
  k_lv_reset<<<grid_for(ctx, n_units), 256, 0, st>>>(level, n_units, n_input, s.front[0]);
  PLX_LAUNCH_CHECK("k_lv_reset");
  k_lv_degrees<<<grid_for(ctx, n_conns), 256, 0, st>>>(from_id, to_id, dead, n_conns, n_units,
                                                       s.cursor, s.in_deg, ctx->d_status);
  PLX_LAUNCH_CHECK("k_lv_degrees");
  size_t tb = s.temp_bytes;
  PLX_TRY_CUDA(cub::DeviceScan::ExclusiveSum(s.temp, tb, s.cursor, s.out_off,
                                             (int64_t)n_units + 1, st));
  PLX_TRY_CUDA(cudaMemcpyAsync(s.cursor, s.out_off, 4ull * n_units, cudaMemcpyDeviceToDevice, st));
  k_lv_scatter<<<grid_for(ctx, n_conns), 256, 0, st>>>(from_id, to_id, dead, n_conns, n_units,
                                                       s.cursor, s.out_to);
  PLX_LAUNCH_CHECK("k_lv_scatter");
  LvCounters init{};
  init.size[0] = n_input;
  PLX_TRY_CUDA(cudaMemcpyAsync(s.cnt, &init, sizeof(init), cudaMemcpyHostToDevice, st));
  int per_sm = 0;
  PLX_TRY_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_lv_rounds, 256, 0));
  if (per_sm < 1) per_sm = 1;
  per_sm = std::min(per_sm, 4);
  unsigned grid = (unsigned)(ctx->num_sms * per_sm);
  const uint64_t want = ((uint64_t)n_units + 7) / 8;  // a warp per frontier unit
  if (want < grid) grid = (unsigned)std::max<uint64_t>(want, 1);
  const uint32_t* out_off = s.out_off;
  const uint32_t* out_to = s.out_to;
  uint32_t* in_deg = s.in_deg;
  uint32_t* f0 = s.front[0];
  uint32_t* f1 = s.front[1];
  LvCounters* cnt = s.cnt;
  int32_t* status = ctx->d_status;
  uint64_t timeout = ctx->timeout_ns;
  void* args[] = {(void*)&out_off, (void*)&out_to, (void*)&in_deg, (void*)&level, (void*)&f0,
                  (void*)&f1,      (void*)&cnt,    (void*)&rounds_out, (void*)&status,
                  (void*)&timeout};
  PLX_TRY_CUDA(cudaLaunchCooperativeKernel((const void*)k_lv_rounds, dim3(grid), dim3(256), args,
                                           0, st));
  return PLX_OK;
}

extern "C" int plx_src_levels(plx_ctx* ctx, uint64_t n_conns, const uint32_t* from_id,
                              const uint16_t* level, uint32_t n_units, uint16_t* src_level) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  PLX_CHECK_ARG(n_conns == 0 || (from_id && level && src_level),
                "from_id, level and src_level are required");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  if (n_conns == 0) return PLX_OK;
  k_src_levels<<<grid_for(ctx, n_conns), 256, 0, ctx->stream>>>(from_id, n_conns, level,
                                                                 n_units, src_level,
                                                                 ctx->d_status);
  PLX_LAUNCH_CHECK("k_src_levels");
  return PLX_OK;
}
