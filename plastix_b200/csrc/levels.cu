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
// Design (B200): one cooperative persistent kernel runs every round after an
// in-degree count. The first kEdgeRounds rounds are edge-centric: a pass over
// the live connections that takes those whose source is in the current
// frontier (round 0: the input units; later: units whose `reached` round is
// L), with no outgoing lists at all -- a shallow graph (the structural
// configuration has two non-empty rounds) never builds them. A deeper graph
// then builds the outgoing lists inside the same kernel (out-degree count,
// block scan, scatter) and continues frontier-centric: each warp takes 32
// frontier units and deals their outgoing connections out one per lane. Units
// reaching in-degree 0 are buffered per warp in shared memory and appended to
// the next frontier a buffer at a time. Grid barriers separate the phases;
// their waits are bounded (a barrier that runs out records PLX_ERR_TIMEOUT and
// every block returns). A unit's `reached` round is written once, to L+1,
// during round L, so the membership test for round L never races with it.
#include <algorithm>

#include <cub/block/block_reduce.cuh>
#include <cub/block/block_scan.cuh>
#include "common.cuh"

namespace plx {
namespace {

constexpr uint32_t kFullMask = 0xFFFFFFFFu;
constexpr uint32_t kLvBuf = 256;  // per-warp buffer of next-frontier units

size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

__host__ __device__ inline uint64_t min_u64(uint64_t x, uint64_t y) { return x < y ? x : y; }

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

constexpr uint32_t kEdgeRounds = 2;    // edge-centric rounds before lists are built
constexpr uint32_t kMaxLvBlocks = 4096;  // per-block sums of the in-kernel scan
constexpr uint32_t kNotReached = 0xFFFFFFFFu;

struct LvScratch {
  uint32_t* in_deg;      // [n_units]
  uint32_t* reached;     // [n_units] round in which the unit joined a frontier
  uint32_t* out_off;     // [n_units + 1]
  uint32_t* cursor;      // [n_units + 1] out-degrees, then write cursors
  uint32_t* out_to;      // [n_conns] target of each live outgoing connection
  uint32_t* front[2];    // [n_units] each
  uint32_t* block_sums;  // [kMaxLvBlocks]
  LvCounters* cnt;
};

LvScratch lv_layout(void* base, uint64_t n_units, uint64_t n_conns) {
  char* p = static_cast<char*>(base);
  const size_t u = al256(4 * std::max<uint64_t>(n_units + 1, 1));
  LvScratch s;
  s.in_deg = reinterpret_cast<uint32_t*>(p);
  p += u;
  s.reached = reinterpret_cast<uint32_t*>(p);
  p += u;
  s.out_off = reinterpret_cast<uint32_t*>(p);
  p += u;
  s.cursor = reinterpret_cast<uint32_t*>(p);
  p += u;
  s.front[0] = reinterpret_cast<uint32_t*>(p);
  p += u;
  s.front[1] = reinterpret_cast<uint32_t*>(p);
  p += u;
  s.out_to = reinterpret_cast<uint32_t*>(p);
  p += al256(4 * std::max<uint64_t>(n_conns, 1));
  s.block_sums = reinterpret_cast<uint32_t*>(p);
  p += 4 * kMaxLvBlocks;
  s.cnt = reinterpret_cast<LvCounters*>(p);
  return s;
}

size_t lv_bytes(uint64_t n_units, uint64_t n_conns) {
  return 6 * al256(4 * std::max<uint64_t>(n_units + 1, 1)) +
         al256(4 * std::max<uint64_t>(n_conns, 1)) + 4 * kMaxLvBlocks + 256;
}

__device__ __forceinline__ bool lv_live(const uint8_t* dead, uint64_t c) {
  return dead == nullptr || dead[c] == 0;
}

// Levels of non-input units to 0; frontier 0 = the input units; no unit
// reached yet.
__global__ void k_lv_reset(uint16_t* __restrict__ level, uint32_t n_units, uint32_t n_input,
                           uint32_t* __restrict__ front0, uint32_t* __restrict__ reached) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n_units;
       i += gridDim.x * blockDim.x) {
    if (i >= n_input) level[i] = 0;
    else front0[i] = i;
    reached[i] = kNotReached;
  }
}

// In-degree by ToId over live connections; records bad unit ids.
__global__ void k_lv_in_degrees(const uint32_t* __restrict__ from_id,
                                const uint32_t* __restrict__ to_id,
                                const uint8_t* __restrict__ dead, uint64_t n_conns,
                                uint32_t n_units, uint32_t* __restrict__ in_deg,
                                int32_t* status) {
  bool bad = false;
  for (uint64_t c = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; c < n_conns;
       c += (uint64_t)gridDim.x * blockDim.x) {
    if (!lv_live(dead, c)) continue;
    const uint32_t f = from_id[c], t = to_id[c];
    if (f >= n_units || t >= n_units) {
      bad = true;
      continue;
    }
    atomicAdd(in_deg + t, 1u);
  }
  if (bad) record_status(status, kStatusBadIndex);
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

struct LvArgs {
  const uint32_t* from_id;
  const uint32_t* to_id;
  const uint8_t* dead;
  uint64_t n_conns;
  uint32_t n_units;
  uint32_t n_input;
  uint32_t* in_deg;
  uint32_t* reached;
  uint16_t* level;
  uint32_t* front[2];
  uint32_t* out_off;
  uint32_t* cursor;  // zeroed before the launch
  uint32_t* out_to;
  uint32_t* block_sums;
  LvCounters* cnt;
  uint32_t* rounds_out;
  int32_t* status;
  uint64_t timeout_ns;
};

using LvBlockScan = cub::BlockScan<uint32_t, 256>;
using LvBlockReduce = cub::BlockReduce<uint32_t, 256>;

// Outgoing lists inside the cooperative kernel: out-degrees, an exclusive
// scan over n_units + 1 counts (per-block sums, then each block scans its
// contiguous chunk), and the scatter of every live connection's target.
__device__ bool lv_build_lists(const LvArgs& a) {
  __shared__ union {
    typename LvBlockScan::TempStorage scan;
    typename LvBlockReduce::TempStorage reduce;
  } tmp;
  __shared__ uint32_t s_total;
  const uint64_t tid = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  const uint64_t nthreads = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t c = tid; c < a.n_conns; c += nthreads) {
    if (!lv_live(a.dead, c)) continue;
    const uint32_t f = a.from_id[c], t = a.to_id[c];
    if (f < a.n_units && t < a.n_units) atomicAdd(a.cursor + f, 1u);
  }
  if (!lv_grid_barrier(a.cnt, a.timeout_ns)) return false;
  const uint64_t n = (uint64_t)a.n_units + 1;  // cursor[n_units] is 0
  const uint64_t chunk = (n + gridDim.x - 1) / gridDim.x;
  const uint64_t c0 = min_u64(blockIdx.x * chunk, n), c1 = min_u64(c0 + chunk, n);
  uint32_t part = 0;
  for (uint64_t i = c0 + threadIdx.x; i < c1; i += blockDim.x) part += a.cursor[i];
  part = LvBlockReduce(tmp.reduce).Sum(part);
  if (threadIdx.x == 0) a.block_sums[blockIdx.x] = part;
  if (!lv_grid_barrier(a.cnt, a.timeout_ns)) return false;
  uint32_t off = 0;
  for (uint32_t b = threadIdx.x; b < blockIdx.x; b += blockDim.x) off += a.block_sums[b];
  __syncthreads();
  off = LvBlockReduce(tmp.reduce).Sum(off);
  if (threadIdx.x == 0) s_total = off;
  __syncthreads();
  uint32_t carry = s_total;
  for (uint64_t base = c0; base < c1; base += blockDim.x) {
    const uint64_t i = base + threadIdx.x;
    const uint32_t v = i < c1 ? a.cursor[i] : 0u;
    uint32_t ex, tile;
    __syncthreads();
    LvBlockScan(tmp.scan).ExclusiveSum(v, ex, tile);
    if (i < c1) {
      a.out_off[i] = carry + ex;
      a.cursor[i] = carry + ex;
    }
    carry += tile;
  }
  if (!lv_grid_barrier(a.cnt, a.timeout_ns)) return false;
  for (uint64_t c = tid; c < a.n_conns; c += nthreads) {
    if (!lv_live(a.dead, c)) continue;
    const uint32_t f = a.from_id[c], t = a.to_id[c];
    if (f < a.n_units && t < a.n_units) a.out_to[atomicAdd(a.cursor + f, 1u)] = t;
  }
  return lv_grid_barrier(a.cnt, a.timeout_ns);
}

// Every round of the level-parallel Kahn pass.
__global__ void __launch_bounds__(256) k_lv_rounds(LvArgs a) {
  __shared__ uint32_t s_buf[8][kLvBuf];
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t n_warps = (gridDim.x * blockDim.x) >> 5;
  uint32_t* const buf = s_buf[threadIdx.x >> 5];
  bool lists = false;
  uint32_t L = 0;
  for (;; ++L) {
    volatile uint32_t* sizes = a.cnt->size;
    const uint32_t sz = sizes[L % 3];
    if (sz == 0) break;
    if (!lists && L >= kEdgeRounds) {
      if (!lv_build_lists(a)) {
        if (threadIdx.x == 0) record_status(a.status, kStatusTimeout);
        return;
      }
      lists = true;
    }
    const uint32_t* cur = a.front[L & 1u];
    uint32_t* nxt = a.front[(L & 1u) ^ 1u];
    uint32_t* nsz = &a.cnt->size[(L + 1) % 3];
    if (blockIdx.x == 0 && threadIdx.x == 0) a.cnt->size[(L + 2) % 3] = 0;  // read in round L-1
    const uint16_t lv = (uint16_t)(L + 1u);
    // Units reaching in-degree 0 collect in the warp's shared buffer and go to
    // the next frontier a buffer at a time (one atomic per flush).
    uint32_t nbuf = 0;  // warp-uniform
    auto flush = [&]() {
      __syncwarp();
      uint32_t base = 0;
      if (lane == 0) base = atomicAdd(nsz, nbuf);
      base = __shfl_sync(kFullMask, base, 0);
      for (uint32_t i = lane; i < nbuf; i += 32) nxt[base + i] = buf[i];
      __syncwarp();
      nbuf = 0;
    };
    // Decrements t's in-degree for one live connection of a frontier unit
    // (lanes with `take` false only join the warp-wide collection).
    auto visit = [&](bool take, uint32_t t) {
      bool fire = false;
      if (take) fire = atomicSub(a.in_deg + t, 1u) == 1u;
      const uint32_t m = __ballot_sync(kFullMask, fire);
      if (m) {
        if (nbuf + 32u > kLvBuf) flush();
        if (fire) {
          a.level[t] = lv;
          a.reached[t] = L + 1u;
          buf[nbuf + __popc(m & ((1u << lane) - 1u))] = t;
        }
        nbuf += (uint32_t)__popc(m);
      }
    };
    if (!lists) {
      // edge-centric: every live connection whose source is in frontier L
      for (uint64_t c0 = (uint64_t)warp * 32u; c0 < a.n_conns; c0 += (uint64_t)n_warps * 32u) {
        const uint64_t c = c0 + lane;
        bool take = false;
        uint32_t t = 0;
        if (c < a.n_conns && lv_live(a.dead, c)) {
          const uint32_t f = a.from_id[c];
          if (f < a.n_units && ((L == 0 && f < a.n_input) || a.reached[f] == L)) {
            t = a.to_id[c];
            take = t < a.n_units;
          }
        }
        visit(take, t);
      }
    } else {
      // frontier-centric: each warp takes 32 frontier units and deals their
      // outgoing connections out one per lane (degree scan + owner search)
      for (uint32_t f0 = warp * 32u; f0 < sz; f0 += n_warps * 32u) {
        const uint32_t f = f0 + lane;
        uint32_t beg = 0, deg = 0;
        if (f < sz) {
          const uint32_t u = cur[f];
          beg = a.out_off[u];
          deg = a.out_off[u + 1] - beg;
        }
        uint32_t incl = deg;
#pragma unroll
        for (uint32_t o = 1; o < 32; o <<= 1) {
          const uint32_t v = __shfl_up_sync(kFullMask, incl, o);
          if (lane >= o) incl += v;
        }
        const uint32_t excl = incl - deg;
        const uint32_t total = __shfl_sync(kFullMask, incl, 31);
        for (uint32_t j0 = 0; j0 < total; j0 += 32) {
          const uint32_t j = j0 + lane;
          // owner: the last lane whose first connection index is <= j
          uint32_t own = 0;
#pragma unroll
          for (uint32_t step = 16; step; step >>= 1) {
            const uint32_t e = __shfl_sync(kFullMask, excl, own + step);
            if (e <= j) own += step;
          }
          const uint32_t ob = __shfl_sync(kFullMask, beg, own);
          const uint32_t oe = __shfl_sync(kFullMask, excl, own);
          const bool take = j < total;
          visit(take, take ? a.out_to[ob + (j - oe)] : 0u);
        }
      }
    }
    if (nbuf) flush();
    if (!lv_grid_barrier(a.cnt, a.timeout_ns)) {
      if (threadIdx.x == 0) record_status(a.status, kStatusTimeout);
      return;
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && a.rounds_out) *a.rounds_out = L;
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
    if (n_units) {
      k_lv_reset<<<grid_for(ctx, n_units), 256, 0, st>>>(level, n_units, n_input, s.front[0],
                                                         s.reached);
      PLX_LAUNCH_CHECK("k_lv_reset");
    }
    if (rounds_out) PLX_TRY_CUDA(cudaMemsetAsync(rounds_out, 0, sizeof(uint32_t), st));
    return PLX_OK;
  }
  PLX_TRY_CUDA(cudaMemsetAsync(s.in_deg, 0, 4ull * n_units, st));
  PLX_TRY_CUDA(cudaMemsetAsync(s.cursor, 0, 4ull * (n_units + 1), st));
  k_lv_reset<<<grid_for(ctx, n_units), 256, 0, st>>>(level, n_units, n_input, s.front[0],
                                                     s.reached);
  PLX_LAUNCH_CHECK("k_lv_reset");
  k_lv_in_degrees<<<grid_for(ctx, n_conns), 256, 0, st>>>(from_id, to_id, dead, n_conns, n_units,
                                                          s.in_deg, ctx->d_status);
  PLX_LAUNCH_CHECK("k_lv_in_degrees");
  LvCounters init{};
  init.size[0] = n_input;
  PLX_TRY_CUDA(cudaMemcpyAsync(s.cnt, &init, sizeof(init), cudaMemcpyHostToDevice, st));
  int per_sm = 0;
  PLX_TRY_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_lv_rounds, 256, 0));
  if (per_sm < 1) per_sm = 1;
  per_sm = std::min(per_sm, 4);
  uint64_t grid = (uint64_t)ctx->num_sms * per_sm;
  // a warp per 32 frontier units or connections at the least
  const uint64_t want = (std::max<uint64_t>(n_units, n_conns) + 255) / 256;
  grid = std::max<uint64_t>(1, std::min<uint64_t>({grid, want, kMaxLvBlocks}));
  LvArgs a{};
  a.from_id = from_id;
  a.to_id = to_id;
  a.dead = dead;
  a.n_conns = n_conns;
  a.n_units = n_units;
  a.n_input = n_input;
  a.in_deg = s.in_deg;
  a.reached = s.reached;
  a.level = level;
  a.front[0] = s.front[0];
  a.front[1] = s.front[1];
  a.out_off = s.out_off;
  a.cursor = s.cursor;
  a.out_to = s.out_to;
  a.block_sums = s.block_sums;
  a.cnt = s.cnt;
  a.rounds_out = rounds_out;
  a.status = ctx->d_status;
  a.timeout_ns = ctx->timeout_ns;
  void* args[] = {(void*)&a};
  PLX_TRY_CUDA(cudaLaunchCooperativeKernel((const void*)k_lv_rounds, dim3((unsigned)grid),
                                           dim3(256), args, 0, st));
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
