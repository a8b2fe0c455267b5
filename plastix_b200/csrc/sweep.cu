// K1: the per-connection sweep over dst-sorted connections.
//
// Reference loops replaced (include/plastix/plastix.hpp):
//   DoForwardPass, Pipeline branch            :133-148
//   DoForwardPass, one Topological level      :112-130
//   DoUpdateConnectionState (incoming sweep)  :238-245
//
// Design (B200):
// * Rows (destination units) are classified once per connectivity by
//   plx_csr_plan: short rows (<= PLX_SEQ_ROW_MAX connections), wide rows
//   (<= 8192) and long rows.
// * Short rows are swept by k_sweep, a persistent warp-specialised kernel
//   over fixed edge tiles of S connections. A producer warp streams each
//   tile's SoA slices (FromId, Weight, [Trace], [Dead]) and the tile's slice
//   of row_ptr into a ring of shared-memory stages with 1-D bulk copies (TMA
//   engine, mbarrier transaction counts). Consumer warps then
//     A  gather act[FromId] (L2-resident) into shared memory, plus the
//        pieces of the two boundary rows that lie outside the tile (halo),
//     B  fold w*act of each short row strictly left to right (one thread per
//        row: bit-exact with the reference), run Apply, write the row output
//        and broadcast the row value to the row's connections,
//     C  apply the per-connection update in shared memory,
//   and bulk-store the updated Weight/Trace slices. A row crossing a tile
//   boundary is summed by both tiles from the halo; only the tile holding
//   its first connection writes its output, each tile updates its own part.
//   Because of that re-read, the fused variant reads w_in and writes w_out.
// * Wide rows are summed by k_wide_rows (one warp per row, coalesced
//   lane-strided fold, deterministic) and long rows by k_long_rows (one CTA
//   per row) before k_sweep; k_sweep then only updates their connections.
#include <cstdio>
#include <cstdlib>

#include "common.cuh"

namespace plx {

constexpr uint32_t kPlanG = 256;                // plan granularity (edges)
constexpr uint32_t kSeqMax = PLX_SEQ_ROW_MAX;   // short-row limit
constexpr uint32_t kLongRow = 8192;             // wide-row limit
constexpr uint32_t kHalo = kSeqMax;             // max out-of-tile piece of a short row
constexpr uint32_t kPlanMagic = 0x504C4E32u;    // "PLN2"
constexpr uint32_t kPlanHdr = 8;

// Plan layout (u32 words):
//   [0] magic (0 when row_ptr failed validation)  [1] n_blocks
//   [2] n_wide  [3] n_long  [4] n_short  [5] max_wide  [6] max_long
//   [7] longest row (connections)
//   [8 + 3b + 0]  first row f whose start >= b*kPlanG (b = n_blocks: n_rows)
//   [8 + 3b + 1]  row_ptr[f-1]: start of the last row starting before b*kPlanG
//   [8 + 3b + 2]  row_ptr[f]:   its end (0 and 0 when f == 0)
//   for b in [0, n_blocks]; then max_wide wide-row ids, then max_long
//   long-row ids.
__host__ __device__ inline uint64_t plan_blocks(uint64_t n_edges) {
  uint64_t b = (n_edges + kPlanG - 1) / kPlanG;
  return b ? b : 1;
}
__host__ __device__ inline uint64_t plan_max_wide(uint64_t n_edges) {
  return n_edges / (kSeqMax + 1) + 1;
}
__host__ __device__ inline uint64_t plan_max_long(uint64_t n_edges) {
  return n_edges / (kLongRow + 1) + 1;
}
__host__ __device__ inline uint64_t plan_wide_off(uint64_t nb) {
  return kPlanHdr + 3 * (nb + 1);
}
__host__ __device__ inline uint64_t min_u64(uint64_t x, uint64_t y) {
  return x < y ? x : y;
}

struct SweepArgs {
  const uint32_t* row_ptr;
  const uint32_t* plan;
  uint64_t n_edges;
  uint32_t n_rows;
  uint32_t act_src_len;
  const uint32_t* src;
  const float* w_in;
  float* w_out;
  const float* e_in;
  float* e_out;
  const uint8_t* dead;
  const float* act_src;
  float* act_dst;
  const float* value;
  float* err_out;
  const float* post;
  float decay;
  float rate;
  int32_t* status;
  uint64_t timeout_ns;
  const uint32_t* to_id;  // ToId field (warp fast path)
  uint32_t row_base;      // unit id of row 0
  uint32_t* queue;        // stripe work counter (warp fast path), zeroed
  uint32_t only_long;     // warp fast path: run only if the longest row > 128
  // Hand-off over peer memory: every row value is also stored to
  // peer_out[p][peer_offset + r] for each of the n_peers destination buffers
  // (this GPU's and the other GPUs' all-gather buffers, NVLink-mapped).
  uint32_t n_peers;
  uint32_t peer_offset;
  float* peer_out[PLX_MAX_PEERS];
  uint32_t no_prefetch;  // skip the next-tile L2 prefetch (large source arrays)
};

enum UpdKind : int { kUpdNone = 0, kUpdHebbTrace = 1, kUpdGrad = 2, kUpdHebb = 3, kUpdHebbT = 4 };

// ---------------------------------------------------------------------------
// Plan construction
// ---------------------------------------------------------------------------
// row_ptr[r] = first index whose ToId is >= row_base + r (ToId sorted),
// row_ptr[n_rows] = n_edges. One pass over the connections: index i owns the
// rows r with key(i-1) < r <= key(i), keys clamped to [-1, n_rows] (index
// n_edges acts as key n_rows). Each thread takes four consecutive indices
// with one 16-byte load (to_id is 16-byte aligned) plus the key before them.
constexpr int64_t kRowGapMax = 64;  // empty rows one thread of k_row_ptr stores

__device__ __forceinline__ int64_t row_key(uint32_t to, uint32_t row_base, uint32_t n_rows) {
  const int64_t k = (int64_t)to - (int64_t)row_base;
  return k < -1 ? -1 : (k > (int64_t)n_rows ? (int64_t)n_rows : k);
}

// A run of more empty rows than kRowGapMax is not stored by the thread that
// finds it (it would store the run serially); it is appended to a list of
// (first row, last row, value) runs that k_row_ptr_runs fills in parallel.
// Runs that do not fit the list are stored serially after all.
constexpr uint32_t kRowRunsCap = 4096;

__global__ void k_row_ptr(const uint32_t* __restrict__ to_id, uint64_t n_edges,
                          uint32_t row_base, uint32_t n_rows,
                          uint32_t* __restrict__ row_ptr, uint32_t* __restrict__ runs) {
  const uint64_t i0 = 4 * (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x);
  if (i0 > n_edges) return;
  int64_t k[5];  // keys of i0 - 1 .. i0 + 3
  k[0] = i0 ? row_key(__ldg(to_id + i0 - 1), row_base, n_rows) : -1;
  if (i0 + 4 <= n_edges) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(to_id + i0));
    k[1] = row_key(v.x, row_base, n_rows);
    k[2] = row_key(v.y, row_base, n_rows);
    k[3] = row_key(v.z, row_base, n_rows);
    k[4] = row_key(v.w, row_base, n_rows);
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      k[j + 1] = i0 + j < n_edges ? row_key(__ldg(to_id + i0 + j), row_base, n_rows)
                                  : (int64_t)n_rows;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint64_t i = i0 + j;
    if (i > n_edges) break;
    const int64_t hi = min(k[j + 1], (int64_t)n_rows - 1);
    bool inline_store = hi - k[j] <= kRowGapMax;
    if (!inline_store) {
      const uint32_t slot = atomicAdd(runs, 1u);
      if (slot < kRowRunsCap) {
        uint32_t* run = runs + 1 + 3 * slot;
        run[0] = (uint32_t)(k[j] + 1);
        run[1] = (uint32_t)hi;
        run[2] = (uint32_t)i;
      } else {
        inline_store = true;
      }
    }
    if (inline_store)
      for (int64_t r = k[j] + 1; r <= hi; ++r) row_ptr[r] = (uint32_t)i;
    if (i == n_edges) row_ptr[n_rows] = (uint32_t)n_edges;
  }
}

// The listed runs of empty rows: rows [first, last] all start at `value`.
// Every run is spread over the whole grid (one run can be millions of rows).
__global__ void k_row_ptr_runs(const uint32_t* __restrict__ runs, uint32_t* __restrict__ row_ptr) {
  const uint32_t n = min(runs[0], kRowRunsCap);
  const uint64_t t0 = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint32_t q = 0; q < n; ++q) {
    const uint32_t first = runs[1 + 3 * q], last = runs[2 + 3 * q], v = runs[3 + 3 * q];
    for (uint64_t r = (uint64_t)first + t0; r <= last; r += stride) row_ptr[r] = v;
  }
}

__global__ void k_plan_blocks(const uint32_t* __restrict__ row_ptr,
                              uint32_t n_rows, uint64_t n_edges,
                              uint32_t* __restrict__ plan) {
  const uint64_t nb = plan_blocks(n_edges);
  uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (b > nb) return;
  uint32_t lo = n_rows;
  if (b < nb) {
    const uint64_t key = b * kPlanG;
    lo = 0;
    uint32_t hi = n_rows;  // first row r in [0, n_rows] with start >= key
    while (lo < hi) {
      uint32_t mid = (lo + hi) >> 1;
      if ((uint64_t)__ldg(row_ptr + mid) < key) lo = mid + 1;
      else hi = mid;
    }
  }
  uint32_t* e = plan + kPlanHdr + 3 * b;
  e[0] = lo;
  e[1] = lo ? row_ptr[lo - 1] : 0u;
  e[2] = lo ? row_ptr[lo] : 0u;
}

// Validates row_ptr (monotone, row_ptr[0]==0, row_ptr[n_rows]==n_edges),
// counts short rows and lists wide and long rows (list order is irrelevant:
// each row is reduced independently). Any violation clears the magic word so
// every sweep using this plan stops and reports a bad-plan status.
__global__ void __launch_bounds__(256) k_plan_rows(const uint32_t* __restrict__ row_ptr,
                                                   uint32_t n_rows, uint64_t n_edges,
                                                   uint32_t* __restrict__ plan) {
  __shared__ uint32_t s_short[8], s_max[8];
  const uint64_t nb = plan_blocks(n_edges);
  const uint64_t max_wide = plan_max_wide(n_edges);
  const uint64_t max_long = plan_max_long(n_edges);
  uint32_t* wide = plan + plan_wide_off(nb);
  uint32_t* lng = wide + max_wide;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (row_ptr[0] != 0 || row_ptr[n_rows] != (uint32_t)n_edges) plan[0] = 0;
  }
  uint32_t n_short = 0, longest = 0;
  for (uint64_t r = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; r < n_rows;
       r += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t a = row_ptr[r], b = row_ptr[r + 1];
    if (b < a || b > n_edges) {
      plan[0] = 0;
      continue;
    }
    const uint32_t len = b - a;
    longest = max(longest, len);
    if (len <= kSeqMax) {
      ++n_short;
    } else if (len <= kLongRow) {
      const uint32_t slot = atomicAdd(&plan[2], 1u);
      if (slot < max_wide) wide[slot] = (uint32_t)r;
      else plan[0] = 0;
    } else {
      const uint32_t slot = atomicAdd(&plan[3], 1u);
      if (slot < max_long) lng[slot] = (uint32_t)r;
      else plan[0] = 0;
    }
  }
  // One atomic per block for the short-row count and the longest row.
  n_short = __reduce_add_sync(0xffffffffu, n_short);
  longest = __reduce_max_sync(0xffffffffu, longest);
  const uint32_t lane = threadIdx.x & 31u, w = threadIdx.x >> 5;
  if (lane == 0) {
    s_short[w] = n_short;
    s_max[w] = longest;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t ts = 0, tm = 0;
    for (uint32_t i = 0; i < blockDim.x / 32; ++i) {
      ts += s_short[i];
      tm = max(tm, s_max[i]);
    }
    if (ts) atomicAdd(&plan[4], ts);
    if (tm) atomicMax(&plan[7], tm);
  }
}

// ---------------------------------------------------------------------------
// Apply / update rules
// ---------------------------------------------------------------------------
template <int APPLY>
__device__ __forceinline__ float apply_row(float acc, uint32_t r,
                                           const SweepArgs& a, bool owned) {
  float v = 0.0f;
  if constexpr (apply_reads_value(APPLY)) v = __ldg(a.value + r);
  const float post = apply_value<APPLY>(acc, v);
  if (owned) {
    if constexpr (APPLY == PLX_APPLY_IPC_ERROR) a.err_out[r] = post;
    else a.act_dst[r] = post;
    for (uint32_t p = 0; p < a.n_peers; ++p) a.peer_out[p][a.peer_offset + r] = post;
  }
  return post;
}

// Value a row's connections see in the update (what Apply stored).
template <int APPLY>
__device__ __forceinline__ float stored_post(uint32_t r, const SweepArgs& a) {
  if constexpr (APPLY == PLX_APPLY_IPC_ERROR) return a.err_out[r];
  else return a.act_dst[r];
}

// Gathers act[s]; an out-of-range id reads 0 and sets `bad`.
__device__ __forceinline__ float gather_act(const SweepArgs& a, uint32_t s,
                                            bool& bad) {
  const bool ok = s < a.act_src_len;
  bad |= !ok;
  return ok ? __ldg(a.act_src + s) : 0.0f;
}

// w*act of connection k read straight from global memory.
template <bool DEAD>
__device__ __forceinline__ float global_term(const SweepArgs& a, uint32_t k,
                                             bool& bad) {
  const float w = __ldg(a.w_in + k);
  const uint32_t s = __ldg(a.src + k);
  const float p = __fmul_rn(w, gather_act(a, s, bad));
  if constexpr (DEAD) {
    if (__ldg(a.dead + k)) return 0.0f;
  }
  return p;
}

// ---------------------------------------------------------------------------
// Wide rows (kSeqMax < len <= kLongRow): one warp per row. Order: lane l folds
// connections rs+l, rs+l+32, ... left to right; then the 32 lane partials are
// folded in lane order.
// ---------------------------------------------------------------------------
template <int APPLY, bool DEAD>
__global__ void __launch_bounds__(256) k_wide_rows(SweepArgs a) {
  const uint32_t* plan = a.plan;
  if (plan[0] != kPlanMagic) return;
  const uint64_t nb = plan[1];
  const uint32_t n_wide = plan[2];
  const uint32_t* wide = plan + plan_wide_off(nb);
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t nw = (gridDim.x * blockDim.x) >> 5;
  bool bad = false;
  for (uint32_t i = gw; i < n_wide; i += nw) {
    const uint32_t r = wide[i];
    const uint32_t rs = a.row_ptr[r], re = a.row_ptr[r + 1];
    float acc = 0.0f;
    uint32_t k = rs + lane;
    for (; k + 96 < re; k += 128) {
      float p[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) p[j] = global_term<DEAD>(a, k + 32 * j, bad);
#pragma unroll
      for (int j = 0; j < 4; ++j) acc = __fadd_rn(acc, p[j]);
    }
    for (; k < re; k += 32) acc = __fadd_rn(acc, global_term<DEAD>(a, k, bad));
    float tot = 0.0f;
#pragma unroll
    for (int l = 0; l < 32; ++l) tot = __fadd_rn(tot, __shfl_sync(0xffffffffu, acc, l));
    if (lane == 0) apply_row<APPLY>(tot, r, a, true);
  }
  if (bad) record_status(a.status, kStatusBadIndex);
}

// ---------------------------------------------------------------------------
// Long rows (> kLongRow): one CTA per row. Order: thread t folds connections
// rs+t, rs+t+256, ... then thread 0 folds the 256 partials in order.
// ---------------------------------------------------------------------------
template <int APPLY, bool DEAD>
__global__ void __launch_bounds__(256) k_long_rows(SweepArgs a) {
  __shared__ float part[256];
  const uint32_t* plan = a.plan;
  if (plan[0] != kPlanMagic) return;
  const uint64_t nb = plan[1];
  const uint32_t n_long = plan[3];
  const uint32_t* lng = plan + plan_wide_off(nb) + plan_max_wide(a.n_edges);
  bool bad = false;
  for (uint32_t i = blockIdx.x; i < n_long; i += gridDim.x) {
    const uint32_t r = lng[i];
    const uint32_t rs = a.row_ptr[r], re = a.row_ptr[r + 1];
    float acc = 0.0f;
    for (uint32_t k = rs + threadIdx.x; k < re; k += blockDim.x)
      acc = __fadd_rn(acc, global_term<DEAD>(a, k, bad));
    part[threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
      float s = 0.0f;
      for (uint32_t t = 0; t < blockDim.x; ++t) s = __fadd_rn(s, part[t]);
      apply_row<APPLY>(s, r, a, true);
    }
    __syncthreads();
  }
  if (bad) record_status(a.status, kStatusBadIndex);
}

// ---------------------------------------------------------------------------
// The tile sweep
// ---------------------------------------------------------------------------
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Named barrier that also ORs a predicate across the participating threads.
__device__ __forceinline__ bool named_or(uint32_t id, uint32_t n, bool p) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.or.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)p), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

constexpr uint32_t kHaloCap = kHalo + 4;  // halo slice incl. alignment slack

// Folds buf[lo, hi) (shared memory) into acc strictly left to right, loading
// eight values ahead of the additions.
__device__ __forceinline__ float fold_range(const float* buf, uint32_t lo,
                                            uint32_t hi, float acc) {
  uint32_t q = lo;
  for (; q + 8 <= hi; q += 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = buf[q + u];
#pragma unroll
    for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, v[u]);
  }
  for (; q < hi; ++q) acc = __fadd_rn(acc, buf[q]);
  return acc;
}

// buf[lo, hi) = v, with float4 stores for the aligned middle.
__device__ __forceinline__ void fill_range(float* buf, uint32_t lo, uint32_t hi,
                                           float v) {
  uint32_t q = lo;
  for (; q < hi && (q & 3u); ++q) buf[q] = v;
  const float4 v4 = make_float4(v, v, v, v);
  for (; q + 4 <= hi; q += 4) *reinterpret_cast<float4*>(buf + q) = v4;
  for (; q < hi; ++q) buf[q] = v;
}

template <int S_, int NSTAGE_, int NCW_, bool FOLD, bool UPD, bool TRACE, bool DEAD>
struct SweepLayout {
  static constexpr int S = S_, NSTAGE = NSTAGE_, NCW = NCW_;
  static constexpr uint32_t NCT = NCW * 32;  // consumer threads
  static constexpr uint32_t NT = NCT + 32;   // + one producer warp
  // row_ptr slice capacity (u32): update sweeps target rows of >= 4
  // connections; forward sweeps also cover graphs of ~1-2 per row. Tiles with
  // more rows read row_ptr from global memory instead.
  static constexpr uint32_t RCAP = (UPD ? S / 4 : S) + 16;
  static constexpr uint32_t kWideCap = 64;   // wide rows touching one tile
  // per stage
  static constexpr uint32_t kOffW = S * 4u;
  static constexpr uint32_t kOffE = kOffW + S * 4u;
  static constexpr uint32_t kOffDead = kOffE + (TRACE ? S * 4u : 0u);
  static constexpr uint32_t kOffRp = kOffDead + (DEAD ? S : 0u);
  static constexpr uint32_t kOffHalo = kOffRp + RCAP * 4u;  // pre src,w; post src,w
  static constexpr uint32_t kStage = kOffHalo + (FOLD ? 4u * kHaloCap * 4u : 0u);
  // shared by all stages
  static constexpr uint32_t kPost = NSTAGE * kStage;
  // s_post holds the products w*act (fold input), then the row value.
  static constexpr uint32_t kHaloP = kPost + S * 4u;
  static constexpr uint32_t kWide = kHaloP + (FOLD ? 2u * kHaloCap * 4u : 0u);
  static constexpr uint32_t kMeta = kWide + kWideCap * 4u + 16u;
  static constexpr uint32_t kBar = kMeta + NSTAGE * 32u;
  static constexpr uint32_t kBytes = kBar + 2u * NSTAGE * 8u;
  static_assert(kStage % 16 == 0 && kPost % 16 == 0 && kOffHalo % 16 == 0,
                "16-byte stage alignment");
};

template <class L, bool FOLD, int APPLY, int UPD, bool TRACE, bool DEAD>
__global__ void __launch_bounds__(L::NT) k_sweep(SweepArgs a) {
  constexpr int S = L::S, NSTAGE = L::NSTAGE;
  constexpr uint32_t NCT = L::NCT;
  constexpr uint32_t kBlocksPerTile = S / kPlanG;
  constexpr uint32_t kPer = S / NCT;  // tile connections per consumer thread
  static_assert(S % kPlanG == 0, "tile must be a multiple of the plan block");
  static_assert(S % NCT == 0 && kPer <= 16, "tile/consumer ratio");
  static_assert(S >= 2 * kSeqMax, "a short row must not span a whole tile");

  extern __shared__ __align__(128) unsigned char smem[];
  float* s_post = reinterpret_cast<float*>(smem + L::kPost);
  float* s_haloP = reinterpret_cast<float*>(smem + L::kHaloP);
  uint32_t* s_wide = reinterpret_cast<uint32_t*>(smem + L::kWide);
  uint32_t* s_wide_n = s_wide + L::kWideCap;
  uint32_t* s_meta = reinterpret_cast<uint32_t*>(smem + L::kMeta);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* done = full + NSTAGE;

  const uint32_t* __restrict__ plan = a.plan;
  if (plan[0] != kPlanMagic) {
    if (threadIdx.x == 0 && blockIdx.x == 0) record_status(a.status, kStatusBadPlan);
    return;
  }
  // Launched next to k_sweep_warp for a plan whose row counts the host does
  // not know: the warp kernel does the work when there is no wide/long row.
  if (a.to_id && plan[2] == 0 && plan[3] == 0) return;
  const uint64_t nb = plan[1];
  const uint64_t n_edges = a.n_edges;
  const uint32_t n_rows = a.n_rows;
  const uint32_t n_tiles = (uint32_t)((nb + kBlocksPerTile - 1) / kBlocksPerTile);
  const uint32_t my_tiles =
      blockIdx.x < n_tiles ? (n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;

  auto stage = [&](int st) { return smem + st * L::kStage; };

  if (tid == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&done[s], 1);
    }
    mbar_init_fence();
  }
  __syncthreads();

  // ======================= producer warp ===================================
  // Streams tile i into stage i % NSTAGE once the consumers are done with the
  // tile that used the stage before; for update sweeps it also bulk-stores
  // that finished tile, so consumers never wait on stores.
  if (warp == 0) {
    if (lane != 0) return;
    bool timed_out = false;
    for (uint32_t i = 0; i < my_tiles + NSTAGE; ++i) {
      const int st = (int)(i % NSTAGE);
      unsigned char* sb = stage(st);
      if (i >= (uint32_t)NSTAGE) {
        const uint32_t j = i - NSTAGE;  // tile leaving this stage
        if (j >= my_tiles) continue;
        if (!mbar_wait_bounded(&done[st], (j / NSTAGE) & 1u, a.timeout_ns)) {
          timed_out = true;
          break;
        }
        if constexpr (UPD != kUpdNone) {
          const uint64_t js = (uint64_t)(blockIdx.x + j * gridDim.x) * S;
          const uint32_t jn4 = (uint32_t)min_u64(S, n_edges - js) & ~3u;
          if (jn4) {
            bulk_store(a.w_out + js, sb + L::kOffW, jn4 * 4u);
            if constexpr (TRACE) bulk_store(a.e_out + js, sb + L::kOffE, jn4 * 4u);
          }
          bulk_commit();
          bulk_wait_read<0>();
        }
      }
      if (i >= my_tiles) continue;
      const uint32_t t = blockIdx.x + i * gridDim.x;
      const uint64_t ts = (uint64_t)t * S;
      const uint32_t n = (uint32_t)min_u64(S, n_edges - ts);
      const uint64_t te = ts + n;
      const uint32_t b0 = t * kBlocksPerTile;
      const uint32_t b1 = (uint32_t)min_u64((uint64_t)b0 + kBlocksPerTile, nb);
      const uint32_t* P0 = plan + kPlanHdr + 3 * b0;
      const uint32_t* P1 = plan + kPlanHdr + 3 * b1;
      const uint32_t o_begin = P0[0], o_end = P1[0];
      const uint32_t rp_lo = o_begin ? o_begin - 1 : 0u;
      const uint32_t rp_a = rp_lo & ~3u;
      const uint32_t rp_cnt = o_end + 1 - rp_a;  // row_ptr[rp_a .. o_end]
      const bool rp_ok = rp_cnt <= L::RCAP;
      // Halo extents of the two boundary rows (short rows only).
      uint32_t pre_lo = (uint32_t)ts, pre_shift = 0, pre_len = 0, post_len = 0;
      if (FOLD && n > 0) {
        if (o_begin > 0 && P0[2] > ts && P0[2] - P0[1] <= kSeqMax) {
          pre_lo = P0[1] & ~3u;
          pre_shift = P0[1] - pre_lo;
          pre_len = (uint32_t)ts - P0[1];
        }
        if (o_end > o_begin && P1[2] > te && P1[2] - P1[1] <= kSeqMax)
          post_len = P1[2] - (uint32_t)te;
      }
      uint32_t* s_src = reinterpret_cast<uint32_t*>(sb);
      float* s_w = reinterpret_cast<float*>(sb + L::kOffW);
      float* s_e = reinterpret_cast<float*>(sb + L::kOffE);
      uint8_t* s_dead = sb + L::kOffDead;
      uint32_t* s_rp = reinterpret_cast<uint32_t*>(sb + L::kOffRp);
      uint32_t* h_src = reinterpret_cast<uint32_t*>(sb + L::kOffHalo);
      float* h_w = reinterpret_cast<float*>(h_src + kHaloCap);
      uint32_t* g_src = reinterpret_cast<uint32_t*>(h_w + kHaloCap);
      float* g_w = reinterpret_cast<float*>(g_src + kHaloCap);
      const uint32_t n4 = n & ~3u, n16 = n & ~15u;
      const uint32_t rp4 = rp_ok ? (rp_cnt & ~3u) : 0u;
      const uint32_t pre_cnt = pre_len ? (uint32_t)ts - pre_lo : 0u;  // multiple of 4
      const uint32_t post4 = post_len & ~3u;
      for (uint32_t k = n4; k < n; ++k) {
        s_src[k] = a.src[ts + k];
        s_w[k] = a.w_in[ts + k];
        if constexpr (TRACE) s_e[k] = a.e_in[ts + k];
      }
      if constexpr (DEAD) {
        for (uint32_t k = n16; k < n; ++k) s_dead[k] = a.dead[ts + k];
      }
      if (rp_ok)
        for (uint32_t k = rp4; k < rp_cnt; ++k) s_rp[k] = a.row_ptr[rp_a + k];
      for (uint32_t k = post4; k < post_len; ++k) {
        g_src[k] = a.src[te + k];
        g_w[k] = a.w_in[te + k];
      }
      uint32_t* m = s_meta + st * 8;
      m[0] = o_begin;
      m[1] = o_end;
      m[2] = rp_a;
      m[3] = rp_ok ? 1u : 0u;
      m[4] = pre_shift;
      m[5] = pre_len;
      m[6] = post_len;
      const uint32_t bytes = n4 * 4u * (TRACE ? 3u : 2u) + (DEAD ? n16 : 0u) +
                             rp4 * 4u + (pre_cnt + post4) * 8u;
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&full[st], bytes);
      if (n4) {
        bulk_load(s_src, a.src + ts, n4 * 4u, &full[st]);
        bulk_load(s_w, a.w_in + ts, n4 * 4u, &full[st]);
        if constexpr (TRACE) bulk_load(s_e, a.e_in + ts, n4 * 4u, &full[st]);
      }
      if constexpr (DEAD) {
        if (n16) bulk_load(s_dead, a.dead + ts, n16, &full[st]);
      }
      if (rp4) bulk_load(s_rp, a.row_ptr + rp_a, rp4 * 4u, &full[st]);
      if (pre_cnt) {
        bulk_load(h_src, a.src + pre_lo, pre_cnt * 4u, &full[st]);
        bulk_load(h_w, a.w_in + pre_lo, pre_cnt * 4u, &full[st]);
      }
      if (post4) {
        bulk_load(g_src, a.src + te, post4 * 4u, &full[st]);
        bulk_load(g_w, a.w_in + te, post4 * 4u, &full[st]);
      }
    }
    if (timed_out) record_status(a.status, kStatusTimeout);
    if constexpr (UPD != kUpdNone) bulk_wait_all<0>();
    return;
  }

  // ======================= consumer warps ==================================
  // Software pipeline: the gathers of tile i+1 are issued before tile i is
  // folded and updated, and written to shared memory after it, so their L2
  // latency overlaps the fold.
  constexpr uint32_t HMAX = (2 * kHalo + NCT - 1) / NCT;  // halo connections per thread
  const uint32_t ctid = tid - 32u;
  const uint32_t cwarp = warp - 1u;
  bool bad = false;

  struct Geo {
    uint32_t ts, n_in, te, o_begin, o_end, rp_a, pre_shift, pre_len, post_len;
    bool rp_ok, has_head;
  };
  auto rp_at = [&](int st, const Geo& g, uint32_t r) -> uint32_t {
    const uint32_t* s_rp = reinterpret_cast<const uint32_t*>(stage(st) + L::kOffRp);
    return g.rp_ok ? s_rp[r - g.rp_a] : a.row_ptr[r];
  };
  auto load_geo = [&](uint32_t i) -> Geo {
    const int st = (int)(i % NSTAGE);
    const uint32_t* m = s_meta + st * 8;
    const uint64_t ts64 = (uint64_t)(blockIdx.x + i * gridDim.x) * S;
    Geo g;
    g.ts = (uint32_t)ts64;
    g.n_in = (uint32_t)min_u64(S, n_edges - ts64);
    g.te = g.ts + g.n_in;
    g.o_begin = m[0];
    g.o_end = m[1];
    g.rp_a = m[2];
    g.rp_ok = m[3] != 0;
    g.pre_shift = m[4];
    g.pre_len = m[5];
    g.post_len = m[6];
    g.has_head = g.n_in > 0 && (g.o_begin == n_rows || rp_at(st, g, g.o_begin) > g.ts);
    return g;
  };

  // Gathers in flight (registers): the tile's connections of this thread and
  // its halo connections.
  float pav[kPer];
  float phv[HMAX];
  uint8_t phd[HMAX];

  auto issue = [&](uint32_t i) -> bool {
    const int st = (int)(i % NSTAGE);
    if (!mbar_wait_bounded(&full[st], (i / NSTAGE) & 1u, a.timeout_ns)) return false;
    const Geo g = load_geo(i);
    const unsigned char* sb = stage(st);
    const uint32_t* s_src = reinterpret_cast<const uint32_t*>(sb);
    const uint32_t* h_src = reinterpret_cast<const uint32_t*>(sb + L::kOffHalo);
    const uint32_t* g_src = h_src + 2 * kHaloCap;
    uint32_t sv[kPer];
#pragma unroll
    for (uint32_t j = 0; j < kPer; ++j) {
      const uint32_t k = ctid + j * NCT;
      sv[j] = k < g.n_in ? s_src[k] : 0u;
    }
    const uint32_t n_halo = FOLD ? g.pre_len + g.post_len : 0u;
    uint32_t hv[HMAX];
#pragma unroll
    for (uint32_t m = 0; m < HMAX; ++m) {
      const uint32_t j = ctid + m * NCT;
      hv[m] = j < n_halo ? (j < g.pre_len ? h_src[g.pre_shift + j] : g_src[j - g.pre_len]) : 0u;
    }
#pragma unroll
    for (uint32_t j = 0; j < kPer; ++j) pav[j] = gather_act(a, sv[j], bad);
#pragma unroll
    for (uint32_t m = 0; m < HMAX; ++m) {
      const uint32_t j = ctid + m * NCT;
      phv[m] = j < n_halo ? gather_act(a, hv[m], bad) : 0.0f;
      phd[m] = 0;
      if constexpr (DEAD) {
        if (j < n_halo)
          phd[m] = __ldg(a.dead + (j < g.pre_len ? g.ts - g.pre_len + j : g.te + j - g.pre_len));
      }
    }
    return true;
  };

  // Lands the gathers of tile i: act into the FromId slot, products w*act
  // into s_post, halo products into s_haloP.
  auto finish = [&](uint32_t i) {
    const int st = (int)(i % NSTAGE);
    const Geo g = load_geo(i);
    unsigned char* sb = stage(st);
    float* s_a = reinterpret_cast<float*>(sb);
    const float* s_w = reinterpret_cast<const float*>(sb + L::kOffW);
    const uint8_t* s_dead = sb + L::kOffDead;
    const float* h_w = reinterpret_cast<const float*>(sb + L::kOffHalo) + kHaloCap;
    const float* g_w = h_w + 2 * kHaloCap;
#pragma unroll
    for (uint32_t j = 0; j < kPer; ++j) {
      const uint32_t k = ctid + j * NCT;
      if (k < g.n_in) {
        float v = pav[j];
        float p = __fmul_rn(s_w[k], v);
        if constexpr (DEAD) {
          if (s_dead[k]) {
            v = 0.0f;
            p = 0.0f;
          }
        }
        s_a[k] = v;
        s_post[k] = p;
      }
    }
    const uint32_t n_halo = FOLD ? g.pre_len + g.post_len : 0u;
#pragma unroll
    for (uint32_t m = 0; m < HMAX; ++m) {
      const uint32_t j = ctid + m * NCT;
      if (j < n_halo) {
        const float w = j < g.pre_len ? h_w[g.pre_shift + j] : g_w[j - g.pre_len];
        const float p = phd[m] ? 0.0f : __fmul_rn(w, phv[m]);
        s_haloP[j < g.pre_len ? j : kHaloCap + (j - g.pre_len)] = p;
      }
    }
    if (ctid == 0) *s_wide_n = 0;
  };

  bool ok = my_tiles == 0 || issue(0);
  if (named_or(1, NCT, !ok)) {
    if (ctid == 0) record_status(a.status, kStatusTimeout);
  } else {
    if (my_tiles) finish(0);
    named_sync(1, NCT);
  }
  for (uint32_t i = 0; ok && i < my_tiles; ++i) {
    const int st = (int)(i % NSTAGE);
    const Geo g = load_geo(i);
    const uint32_t ts = g.ts, te = g.te, n_in = g.n_in;
    const bool has_next = i + 1 < my_tiles;
    const bool ok_next = !has_next || issue(i + 1);

    unsigned char* sb = stage(st);
    const float* s_a = reinterpret_cast<const float*>(sb);
    float* s_w = reinterpret_cast<float*>(sb + L::kOffW);
    float* s_e = reinterpret_cast<float*>(sb + L::kOffE);
    const uint8_t* s_dead = sb + L::kOffDead;
    const uint32_t n_items = (g.o_end - g.o_begin) + (g.has_head ? 1u : 0u);

    // ---- B: per-row fold / Apply / broadcast (rows spread over warps) ----
    for (uint32_t base = 0; base < n_items; base += NCT) {
      const uint32_t idx = base + lane * L::NCW + cwarp;
      if (idx >= n_items) continue;
      const bool head = g.has_head && idx == 0;
      const uint32_t r = g.has_head ? g.o_begin - 1 + idx : g.o_begin + idx;
      const uint32_t rs = rp_at(st, g, r), re = rp_at(st, g, r + 1);
      if (re - rs > kSeqMax) {
        if constexpr (UPD != kUpdNone) {
          const uint32_t slot = atomicAdd(s_wide_n, 1u);
          if (slot < L::kWideCap) s_wide[slot] = r;
        }
        continue;
      }
      const uint32_t lo = max(rs, ts) - ts, hi = min(re, te) - ts;
      float post;
      if constexpr (FOLD) {
        float acc = 0.0f;
        if (head) acc = fold_range(s_haloP, 0, g.pre_len, acc);
        acc = fold_range(s_post, lo, hi, acc);
        if (re > te) acc = fold_range(s_haloP + kHaloCap, 0, re - te, acc);
        post = apply_row<APPLY>(acc, r, a, !head);
      } else {
        post = __ldg(a.post + r);
      }
      if constexpr (UPD != kUpdNone) fill_range(s_post, lo, hi, post);
    }
    if (named_or(1, NCT, !ok_next)) {
      if (ctid == 0) record_status(a.status, kStatusTimeout);
      break;
    }

    if constexpr (UPD != kUpdNone) {
      // Rows summed by k_wide_rows / k_long_rows: broadcast their stored value.
      const uint32_t n_wide = min(*s_wide_n, L::kWideCap);
      for (uint32_t w = cwarp; w < n_wide; w += L::NCW) {
        const uint32_t r = s_wide[w];
        const float post = FOLD ? stored_post<APPLY>(r, a) : __ldg(a.post + r);
        const uint32_t lo = max(rp_at(st, g, r), ts) - ts;
        const uint32_t hi = min(rp_at(st, g, r + 1), te) - ts;
        for (uint32_t q = lo + lane; q < hi; q += 32) s_post[q] = post;
      }
      if (*s_wide_n > L::kWideCap && ctid == 0) record_status(a.status, kStatusBadPlan);
      named_sync(1, NCT);

      // ---- C: per-connection update in shared memory ----
#pragma unroll
      for (uint32_t j = 0; j < kPer; ++j) {
        const uint32_t k = ctid + j * NCT;
        if (k >= n_in) break;
        if constexpr (DEAD) {
          if (s_dead[k]) continue;
        }
        const float w = s_w[k], av = s_a[k], post = s_post[k];
        if constexpr (UPD == kUpdHebbTrace) {
          const float e = __fadd_rn(__fmul_rn(a.decay, s_e[k]), __fmul_rn(av, post));
          s_e[k] = e;
          s_w[k] = __fadd_rn(w, __fmul_rn(a.rate, e));
        } else if constexpr (UPD == kUpdGrad) {
          s_w[k] = __fsub_rn(w, __fmul_rn(__fmul_rn(a.rate, post), av));
        } else if constexpr (UPD == kUpdHebbT) {
          s_w[k] = __fadd_rn(w, __fmul_rn(__fmul_rn(a.rate, av), post));
        } else {
          s_w[k] = __fadd_rn(w, __fmul_rn(__fmul_rn(a.rate, post), av));
        }
      }
      // The last (n_in % 4) connections are stored here; the producer
      // bulk-stores the rest.
      const uint32_t n4 = n_in & ~3u;
      if (ctid < n_in - n4) {
        const uint32_t k = n4 + ctid;
        a.w_out[ts + k] = s_w[k];
        if constexpr (TRACE) a.e_out[ts + k] = s_e[k];
      }
      named_sync(1, NCT);
    }
    if (has_next) finish(i + 1);
    // Order this thread's shared-memory writes before the producer's bulk
    // copies (stores of this tile, loads of a later tile) into the stage.
    fence_proxy_async_smem();
    named_sync(1, NCT);
    if (ctid == 0) mbar_arrive(&done[st]);
  }
  if (bad) record_status(a.status, kStatusBadIndex);
}

// ---------------------------------------------------------------------------
// Fast path for CSRs whose rows all have at most PLX_SEQ_ROW_MAX connections
// (the plan lists no wide or long row): warp-autonomous and register
// resident, no shared memory and no CTA barrier.
//
// Warps take row-aligned stripes (the rows starting in 16 plan blocks, ~4096
// connections) from an atomic work queue and walk them in windows of 256
// connections, 8 consecutive connections per lane loaded with 128-bit loads
// (ToId, FromId, Weight, [Trace], [Dead]). Each row is folded strictly left
// to right: lanes fold their own connections, and the running sum of a row
// that spans lanes is chained from lane to lane with shuffles (one hop per
// round, as many rounds as the longest chain in the window), so the sums are
// bit-exact with the reference loop. The row that continues into the next
// window carries its running sum across; its connections' update waits in
// registers until the next window completes the row.
// ---------------------------------------------------------------------------
constexpr uint32_t kStripeBlocks = 16;
constexpr uint32_t kWin = 256;
constexpr uint32_t kNone = 0xFFFFFFFFu;
constexpr uint32_t kCont = 0xFFFFFFFEu;
constexpr uint32_t kFull = 0xFFFFFFFFu;

template <typename T>
__device__ __forceinline__ void load8(const T* base, uint32_t k0, uint64_t n, T (&v)[8]) {
  static_assert(sizeof(T) == 4, "4-byte fields");
  if ((uint64_t)k0 + 8 <= n) {
    const uint4 x = __ldg(reinterpret_cast<const uint4*>(base + k0));
    const uint4 y = __ldg(reinterpret_cast<const uint4*>(base + k0 + 4));
    const uint32_t u[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = *reinterpret_cast<const T*>(&u[j]);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (uint64_t)k0 + j < n ? base[k0 + j] : T();
  }
}

__device__ __forceinline__ void load8_u8(const uint8_t* base, uint32_t k0, uint64_t n,
                                         uint8_t (&v)[8]) {
  if ((uint64_t)k0 + 8 <= n && (k0 & 7u) == 0) {
    const uint2 x = __ldg(reinterpret_cast<const uint2*>(base + k0));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[j] = (uint8_t)(x.x >> (8 * j));
      v[j + 4] = (uint8_t)(x.y >> (8 * j));
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (uint64_t)k0 + j < n ? base[k0 + j] : (uint8_t)0;
  }
}

// Stores the elements of `mask` (8 consecutive connections from k0).
__device__ __forceinline__ void store8(float* base, uint32_t k0, uint32_t mask,
                                       const float (&v)[8]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t m = (mask >> (4 * h)) & 0xFu;
    if (m == 0xFu) {
      *reinterpret_cast<float4*>(base + k0 + 4 * h) =
          make_float4(v[4 * h], v[4 * h + 1], v[4 * h + 2], v[4 * h + 3]);
    } else if (m) {
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if ((m >> c) & 1u) base[k0 + 4 * h + c] = v[4 * h + c];
    }
  }
}

// Folds s[q0, q1) (shared memory) into acc strictly left to right: scalar
// head to the 16-byte boundary, float4 body loaded 16 vectors at a time,
// scalar tail.
__device__ __forceinline__ float fold_seg(const float* s, uint32_t q0, uint32_t q1,
                                          float acc) {
  uint32_t q = q0;
  for (; q < q1 && (q & 3u); ++q) acc = __fadd_rn(acc, s[q]);
  for (; q + 64 <= q1; q += 64) {
    float4 v[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) v[u] = *reinterpret_cast<const float4*>(s + q + 4 * u);
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      acc = __fadd_rn(acc, v[u].x);
      acc = __fadd_rn(acc, v[u].y);
      acc = __fadd_rn(acc, v[u].z);
      acc = __fadd_rn(acc, v[u].w);
    }
  }
  for (; q + 4 <= q1; q += 4) {
    const float4 v = *reinterpret_cast<const float4*>(s + q);
    acc = __fadd_rn(acc, v.x);
    acc = __fadd_rn(acc, v.y);
    acc = __fadd_rn(acc, v.z);
    acc = __fadd_rn(acc, v.w);
  }
  for (; q < q1; ++q) acc = __fadd_rn(acc, s[q]);
  return acc;
}

template <int EPL, typename T>
__device__ __forceinline__ void loadv(const T* base, uint32_t k0, uint64_t n, T (&v)[EPL]) {
  if constexpr (EPL == 8) {
    load8(base, k0, n, v);
  } else {
    static_assert(EPL == 4 && sizeof(T) == 4, "4 or 8 elements per lane");
    if ((uint64_t)k0 + 4 <= n) {
      const uint4 x = __ldg(reinterpret_cast<const uint4*>(base + k0));
      const uint32_t u[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = *reinterpret_cast<const T*>(&u[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = (uint64_t)k0 + j < n ? base[k0 + j] : T();
    }
  }
}

template <int EPL>
__device__ __forceinline__ void loadv_u8(const uint8_t* base, uint32_t k0, uint64_t n,
                                         uint8_t (&v)[EPL]) {
  if constexpr (EPL == 8) {
    load8_u8(base, k0, n, v);
  } else {
    if ((uint64_t)k0 + 4 <= n && (k0 & 3u) == 0) {
      const uint32_t x = __ldg(reinterpret_cast<const uint32_t*>(base + k0));
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = (uint8_t)(x >> (8 * j));
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = (uint64_t)k0 + j < n ? base[k0 + j] : (uint8_t)0;
    }
  }
}

template <int EPL>
__device__ __forceinline__ void storev(float* base, uint32_t k0, uint32_t mask,
                                       const float (&v)[EPL]) {
  if constexpr (EPL == 8) {
    store8(base, k0, mask, v);
  } else {
    if ((mask & 0xFu) == 0xFu) {
      *reinterpret_cast<float4*>(base + k0) = make_float4(v[0], v[1], v[2], v[3]);
    } else if (mask) {
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if ((mask >> c) & 1u) base[k0 + c] = v[c];
    }
  }
}

// Warp-tile sweep. Each warp takes a row-aligned tile (the rows that start in
// kTileBlocks consecutive plan blocks, at most kTileCap connections because
// every row has at most PLX_SEQ_ROW_MAX) from an atomic queue and runs three
// phases on it with only __syncwarp between them:
//   1  coalesced 128-bit loads of FromId/Weight (4 consecutive connections per
//      lane per step), gathers of act[FromId], products w*act and activations
//      staged in the warp's shared memory;
//   2  one lane per row folds the row's products strictly left to right
//      (bit-exact with the reference), runs Apply, writes the row output and
//      writes the row value over the row's products;
//   3  (update) coalesced reloads of Weight/Trace, trace/weight update from
//      the staged activation and row value, coalesced stores.
template <uint32_t TB, int KB, int NW, int MINB = 1>
struct WTileCfg {
  static constexpr int kMinBlocks = MINB;  // CTAs per SM the register budget targets
  static constexpr uint32_t kTileBlocks = TB;                        // plan blocks per tile
  static constexpr uint32_t kTileCap = TB * kPlanG + kSeqMax + 8;    // connections
  static constexpr uint32_t kTileVec = (kTileCap + 127) / 128;       // 4-wide steps
  static constexpr int kB = KB;            // 4-wide steps in flight per lane (phase 1)
  static constexpr int kWarpsPerCta = NW;
  static constexpr size_t smem(bool upd) {
    return (upd ? 2 : 1) * (size_t)NW * kTileVec * 128 * sizeof(float);
  }
};

template <class C, int APPLY, bool UPD, bool DEAD>
__global__ void __launch_bounds__(C::kWarpsPerCta * 32, C::kMinBlocks)
    k_sweep_wtile(SweepArgs a) {
  constexpr uint32_t kTileBlocks = C::kTileBlocks;
  constexpr uint32_t kTileVec = C::kTileVec;
  constexpr int kWarpsPerCta = C::kWarpsPerCta;
  // per warp: products, then row values; (update) staged activations
  extern __shared__ __align__(16) float s_tile[];
  constexpr uint32_t kStride = kTileVec * 128;
  const uint32_t* __restrict__ plan = a.plan;
  // Only for plans whose rows are all short (the tile kernel handles others).
  if (plan[0] != kPlanMagic || plan[2] != 0 || plan[3] != 0) return;
  const uint64_t nb = plan[1];
  const uint32_t n_tiles = (uint32_t)((nb + kTileBlocks - 1) / kTileBlocks);
  const uint32_t lane = threadIdx.x & 31u, wid = threadIdx.x >> 5;
  float* sp = s_tile + wid * kStride;
  float* sa = s_tile + (kWarpsPerCta + wid) * kStride;  // used only by update sweeps
  const uint64_t n = a.n_edges;
  const uint32_t len1 = a.act_src_len - 1u;
  const uint64_t pol_first = l2_policy_evict_first();
  const uint64_t pol_last = l2_policy_evict_last();
  bool bad = false;
  // Each warp holds two tiles: the one it works on and the next, whose
  // connection ranges (FromId, Weight, Trace, row offsets) it asks the TMA
  // unit to prefetch into L2 right away. The DRAM stream then runs ahead of
  // the warps without registers or shared memory; the warp's own loads of
  // the next tile hit L2.
  auto prefetch_tile = [&](uint32_t tp) {
    const uint32_t pb0 = tp * kTileBlocks;
    const uint32_t pb1 = (uint32_t)min_u64((uint64_t)pb0 + kTileBlocks, nb);
    const uint32_t* Q0 = plan + kPlanHdr + 3 * pb0;
    const uint32_t* Q1 = plan + kPlanHdr + 3 * pb1;
    const uint32_t plo = Q0[2] & ~3u, phi = Q1[2];
    const uint64_t end = min_u64((uint64_t)phi + 3, n) & ~3ull;  // whole 16 B, inside
    if (end > plo) {
      const uint32_t bytes = (uint32_t)(end - plo) * 4u;
      prefetch_l2_bulk(a.src + plo, bytes, pol_first);
      prefetch_l2_bulk(a.w_in + plo, bytes, pol_first);
      if constexpr (UPD) prefetch_l2_bulk(a.e_in + plo, bytes, pol_first);
    }
    const uint32_t r0 = Q0[0] & ~3u;
    const uint32_t r1 = min(Q1[0] + 4u, a.n_rows) & ~3u;  // row_ptr has n_rows + 1 entries
    if (r1 > r0) prefetch_l2_bulk(a.row_ptr + r0, (r1 - r0) * 4u);
  };
  uint32_t t_cur = 0;
  if (lane == 0) {
    t_cur = atomicAdd(a.queue, 1u);
    if (t_cur < n_tiles && !a.no_prefetch) prefetch_tile(t_cur);
  }
  t_cur = __shfl_sync(kFull, t_cur, 0);
  for (;;) {
    const uint32_t t = t_cur;
    if (t >= n_tiles) break;
    uint32_t t_nxt = 0;
    if (lane == 0) {
      t_nxt = atomicAdd(a.queue, 1u);
      if (t_nxt < n_tiles && !a.no_prefetch) prefetch_tile(t_nxt);
    }
    t_cur = __shfl_sync(kFull, t_nxt, 0);
    const uint32_t b0 = t * kTileBlocks;
    const uint32_t b1 = (uint32_t)min_u64((uint64_t)b0 + kTileBlocks, nb);
    const uint32_t* P0 = plan + kPlanHdr + 3 * b0;
    const uint32_t* P1 = plan + kPlanHdr + 3 * b1;
    const uint32_t f0 = P0[0], f1 = P1[0];
    const uint32_t lo = P0[2], hi = P1[2];  // row_ptr[f0], row_ptr[f1]
    const uint32_t base = lo & ~3u;
    const uint32_t nv = (hi - base + 127) / 128;  // 4-wide steps of the warp

    // ---- 1: stream, gather, stage (kB 4-wide steps in flight per lane) ----
    constexpr int kB = C::kB;
    for (uint32_t v0 = 0; v0 < nv; v0 += kB) {
      uint32_t sid[kB][4];
      float w[kB][4];
      uint8_t dd[kB][4];
#pragma unroll
      for (int h = 0; h < kB; ++h) {
        const uint32_t k = base + 128 * (v0 + h) + 4 * lane;
        if (v0 + h < nv) {
          if ((uint64_t)k + 4 <= n) {
            const uint4 x = ld_stream_v4(a.src + k, pol_first);
            sid[h][0] = x.x; sid[h][1] = x.y; sid[h][2] = x.z; sid[h][3] = x.w;
          } else {
            loadv<4>(a.src, k, n, sid[h]);
          }
          loadv<4>(a.w_in, k, n, w[h]);
          if constexpr (DEAD) loadv_u8<4>(a.dead, k, n, dd[h]);
        }
      }
      float av[kB][4];
      uint32_t smax = 0;
#pragma unroll
      for (int h = 0; h < kB; ++h) {
        const uint32_t k = base + 128 * (v0 + h) + 4 * lane;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const bool in = v0 + h < nv && k + c >= lo && k + c < hi;
          const uint32_t sj = in ? sid[h][c] : 0u;
          smax = max(smax, sj);
          av[h][c] = ld_keep_f32(a.act_src + min(sj, len1), pol_last);
        }
      }
      bad |= smax > len1;
#pragma unroll
      for (int h = 0; h < kB; ++h) {
        if (v0 + h >= nv) continue;
        const uint32_t k = base + 128 * (v0 + h) + 4 * lane;
        float pv[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          bool live = k + c >= lo && k + c < hi;
          if constexpr (DEAD) live = live && !dd[h][c];
          pv[c] = live ? __fmul_rn(w[h][c], av[h][c]) : 0.0f;
        }
        const uint32_t q = 128 * (v0 + h) + 4 * lane;
        *reinterpret_cast<float4*>(sp + q) = make_float4(pv[0], pv[1], pv[2], pv[3]);
        if constexpr (UPD)
          *reinterpret_cast<float4*>(sa + q) =
              make_float4(av[h][0], av[h][1], av[h][2], av[h][3]);
      }
    }
    __syncwarp();

    // ---- 2: one lane per row ----
    for (uint32_t r = f0 + lane; r < f1; r += 32) {
      const uint32_t rs = a.row_ptr[r], re = a.row_ptr[r + 1];
      const float acc = fold_seg(sp, rs - base, re - base, 0.0f);
      const float post = apply_row<APPLY>(acc, r, a, true);
      if constexpr (UPD) fill_range(sp, rs - base, re - base, post);
    }

    if constexpr (UPD) {
      __syncwarp();
      // ---- 3: per-connection update ----
#pragma unroll 4
      for (uint32_t v = 0; v < nv; ++v) {
        const uint32_t k = base + 128 * v + 4 * lane;
        const uint32_t q = 128 * v + 4 * lane;
        float w[4], e[4];
        uint8_t dd[4];
        if ((uint64_t)k + 4 <= n) {
          const uint4 xw = ld_stream_v4(a.w_in + k, pol_first);
          const uint4 xe = ld_stream_v4(a.e_in + k, pol_first);
          w[0] = __uint_as_float(xw.x); w[1] = __uint_as_float(xw.y);
          w[2] = __uint_as_float(xw.z); w[3] = __uint_as_float(xw.w);
          e[0] = __uint_as_float(xe.x); e[1] = __uint_as_float(xe.y);
          e[2] = __uint_as_float(xe.z); e[3] = __uint_as_float(xe.w);
        } else {
          loadv<4>(a.w_in, k, n, w);
          loadv<4>(a.e_in, k, n, e);
        }
        if constexpr (DEAD) loadv_u8<4>(a.dead, k, n, dd);
        const float4 av = *reinterpret_cast<const float4*>(sa + q);
        const float avv[4] = {av.x, av.y, av.z, av.w};
        const float4 ps = *reinterpret_cast<const float4*>(sp + q);
        const float pst[4] = {ps.x, ps.y, ps.z, ps.w};
        uint32_t m = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const bool in = k + c >= lo && k + c < hi;
          m |= (uint32_t)in << c;
          bool live = in;
          if constexpr (DEAD) live = live && !dd[c];
          if (live) {
            const float ne = __fadd_rn(__fmul_rn(a.decay, e[c]), __fmul_rn(avv[c], pst[c]));
            e[c] = ne;
            w[c] = __fadd_rn(w[c], __fmul_rn(a.rate, ne));
          }
        }
        if (m == 0xFu) {
          st_stream_v4(a.w_out + k, make_float4(w[0], w[1], w[2], w[3]), pol_first);
          st_stream_v4(a.e_out + k, make_float4(e[0], e[1], e[2], e[3]), pol_first);
        } else {
          storev<4>(a.w_out, k, m, w);
          storev<4>(a.e_out, k, m, e);
        }
      }
    }
    __syncwarp();  // the next tile overwrites the staged values
  }
  if (bad) record_status(a.status, kStatusBadIndex);
}

// ---------------------------------------------------------------------------
// Host launch helpers
// ---------------------------------------------------------------------------
template <class L, bool FOLD, int APPLY, int UPD, bool TRACE, bool DEAD>
int launch_tiles(plx_ctx* ctx, const SweepArgs& args) {
  auto kern = k_sweep<L, FOLD, APPLY, UPD, TRACE, DEAD>;
  PLX_TRY_CUDA(cudaFuncSetAttribute(
      kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kBytes));
  int per_sm = 0;
  PLX_TRY_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, L::NT,
                                                             L::kBytes));
  if (per_sm < 1) per_sm = 1;
  const uint64_t nb = plan_blocks(args.n_edges);
  const uint64_t n_tiles = (nb + L::S / kPlanG - 1) / (L::S / kPlanG);
  const uint64_t grid = std::min<uint64_t>(n_tiles, (uint64_t)ctx->num_sms * per_sm);
  kern<<<(unsigned)grid, L::NT, L::kBytes, ctx->stream>>>(args);
  PLX_LAUNCH_CHECK("k_sweep");
  return PLX_OK;
}

template <class C, int APPLY, bool UPD, bool DEAD>
int launch_wtile(plx_ctx* ctx, const SweepArgs& args) {
  auto kern = k_sweep_wtile<C, APPLY, UPD, DEAD>;
  const size_t smem = C::smem(UPD);
  PLX_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)smem));
  int per_sm = 0;
  PLX_TRY_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern,
                                                             C::kWarpsPerCta * 32, smem));
  if (per_sm < 1) per_sm = 1;
  const uint64_t nb = plan_blocks(args.n_edges);
  const uint64_t tiles = (nb + C::kTileBlocks - 1) / C::kTileBlocks;
  const uint64_t grid = std::min<uint64_t>((tiles + C::kWarpsPerCta - 1) / C::kWarpsPerCta,
                                           (uint64_t)ctx->num_sms * per_sm);
  PLX_TRY_CUDA(cudaMemsetAsync(ctx->d_queue, 0, sizeof(uint32_t), ctx->stream));
  SweepArgs wa = args;
  wa.queue = ctx->d_queue;
  // The next-tile L2 prefetch keeps upcoming streams resident in L2; with a
  // source array of 2^22 or more units (16 MB) it evicts the gathered
  // activations instead (measured at 64M connections: 2^23 sources
  // 0.667 ms with it, 0.527 ms without; 2^20 sources 0.474 ms with, 0.496
  // without; equal at 2^22).
  wa.no_prefetch = args.act_src_len >= (1u << 22) ? 1u : 0u;
  kern<<<(unsigned)std::max<uint64_t>(grid, 1), C::kWarpsPerCta * 32, smem, ctx->stream>>>(wa);
  PLX_LAUNCH_CHECK("k_sweep_wtile");
  return PLX_OK;
}

// The warp-tile configuration: 4 plan blocks per tile, 4 four-wide steps in
// flight per lane, 8 warps per CTA (the fastest of the tile sizes, step
// depths and CTA shapes measured on the 64M-connection sweep).
using WTileDefault = WTileCfg<4, 4, 8>;

template <int APPLY, bool UPD, bool DEAD>
int launch_warp(plx_ctx* ctx, const SweepArgs& args) {
  return launch_wtile<WTileDefault, APPLY, UPD, DEAD>(ctx, args);
}

template <bool FOLD, int APPLY, int UPD, bool TRACE, bool DEAD>
int launch_sweep(plx_ctx* ctx, const SweepArgs& args, const plx_csr* csr) {
  constexpr bool U = UPD != kUpdNone;
  // Row counts of PLX_COUNT_UNKNOWN (plans built without a host sync): the
  // row kernels read the counts from the plan on the device.
  const uint64_t max_wide = std::min<uint64_t>(plan_max_wide(args.n_edges), args.n_rows);
  const uint64_t max_long = std::min<uint64_t>(plan_max_long(args.n_edges), args.n_rows);
  const uint64_t n_wide = csr->n_wide == PLX_COUNT_UNKNOWN ? max_wide : csr->n_wide;
  const uint64_t n_long = csr->n_long == PLX_COUNT_UNKNOWN ? max_long : csr->n_long;
  if (FOLD && n_wide) {
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((n_wide + 7) / 8, 16u * ctx->num_sms);
    k_wide_rows<APPLY, DEAD><<<blocks, 256, 0, ctx->stream>>>(args);
    PLX_LAUNCH_CHECK("k_wide_rows");
  }
  if (FOLD && n_long) {
    const uint32_t blocks = (uint32_t)std::min<uint64_t>(n_long, 4u * ctx->num_sms);
    k_long_rows<APPLY, DEAD><<<blocks, 256, 0, ctx->stream>>>(args);
    PLX_LAUNCH_CHECK("k_long_rows");
  }
  // A forward-only sweep with no short row is complete after the row kernels.
  if (!U && csr->n_short == 0) return PLX_OK;
  const bool unknown = csr->n_wide == PLX_COUNT_UNKNOWN || csr->n_long == PLX_COUNT_UNKNOWN;
  const bool all_short = !unknown && csr->n_wide == 0 && csr->n_long == 0;
  if (args.to_id && (all_short || unknown) &&
      (UPD == kUpdNone || UPD == kUpdHebbTrace)) {
    if (int rc = launch_warp<APPLY, UPD == kUpdHebbTrace, DEAD>(ctx, args))
      return rc;
    if (all_short) return PLX_OK;
    // unknown counts: the tile kernel below runs only if the plan has wide rows
  }
  SweepArgs targs = args;
  if (!(args.to_id && unknown && (UPD == kUpdNone || UPD == kUpdHebbTrace))) targs.to_id = nullptr;
  // Tile kernel: 1024-connection tiles, 4 bulk-copy stages, 4 consumer warps.
  return launch_tiles<SweepLayout<1024, 4, 4, FOLD, U, TRACE, DEAD>, FOLD, APPLY, UPD, TRACE,
                      DEAD>(ctx, targs);
}

// One thread per row, connections folded left to right (the reference's
// order for every row length): for layers of a few connections per row,
// where a warp per row or a tile plan costs more than it saves.
template <int APPLY, bool DEAD>
__global__ void k_rows_fold(const uint32_t* __restrict__ row_ptr, uint32_t n_rows,
                            const uint32_t* __restrict__ src, const float* __restrict__ w,
                            const uint8_t* __restrict__ dead, const float* __restrict__ act,
                            uint32_t act_len, const float* __restrict__ value,
                            float* __restrict__ act_dst, float* __restrict__ err_out,
                            int32_t* status) {
  bool bad = false;
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < n_rows;
       r += gridDim.x * blockDim.x) {
    const uint32_t b = __ldg(row_ptr + r), e = __ldg(row_ptr + r + 1);
    float acc = 0.0f;
    for (uint32_t k = b; k < e; ++k) {
      if constexpr (DEAD)
        if (__ldg(dead + k)) continue;
      const uint32_t s = __ldg(src + k);
      const bool ok = s < act_len;
      bad |= !ok;
      acc = __fadd_rn(acc, __fmul_rn(__ldg(w + k), ok ? __ldg(act + s) : 0.0f));
    }
    float v = 0.0f;
    if constexpr (apply_reads_value(APPLY)) v = __ldg(value + r);
    const float post = apply_value<APPLY>(acc, v);
    if constexpr (APPLY == PLX_APPLY_IPC_ERROR) err_out[r] = post;
    else act_dst[r] = post;
  }
  if (bad) record_status(status, kStatusBadIndex);
}

static int validate_csr(const plx_csr* csr) {
  PLX_CHECK_ARG(csr && csr->row_ptr && csr->plan, "csr, row_ptr and plan are required");
  PLX_CHECK_ARG(aligned16(csr->row_ptr), "row_ptr must be 16-byte aligned");
  PLX_CHECK_ARG(aligned16(csr->to_id), "to_id must be 16-byte aligned");
  PLX_CHECK_ARG(csr->n_edges < 0xFFFF0000ull,
                "n_edges must be < 2^32 - 2^16 per sweep (split larger layers)");
  return PLX_OK;
}

static SweepArgs base_args(plx_ctx* ctx, const plx_csr* csr) {
  SweepArgs a{};
  a.row_ptr = csr->row_ptr;
  a.plan = csr->plan;
  a.n_edges = csr->n_edges;
  a.n_rows = csr->n_rows;
  a.status = ctx->d_status;
  a.timeout_ns = ctx->timeout_ns;
  a.to_id = csr->to_id;
  a.row_base = csr->row_base;
  return a;
}

}  // namespace plx

using namespace plx;

extern "C" int plx_csr_row_ptr(plx_ctx* ctx, const uint32_t* to_id,
                               uint64_t n_edges, uint32_t row_base,
                               uint32_t n_rows, uint32_t* row_ptr) {
  PLX_CHECK_ARG(ctx && row_ptr, "ctx and row_ptr are required");
  PLX_CHECK_ARG(n_edges == 0 || to_id, "to_id is required when n_edges > 0");
  PLX_CHECK_ARG(n_edges < 0xFFFF0000ull, "n_edges must be < 2^32 - 2^16");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  const uint64_t n = (uint64_t)n_rows + 1;
  (void)n;
  PLX_CHECK_ARG(aligned16(to_id), "to_id must be 16-byte aligned");
  const uint64_t threads = n_edges / 4 + 1;  // indices 0 .. n_edges, four per thread
  uint32_t* runs = nullptr;  // run count + kRowRunsCap (first, last, value) runs
  if (int rc = ctx_counters(ctx, 1 + 3 * (size_t)kRowRunsCap, &runs)) return rc;
  PLX_TRY_CUDA(cudaMemsetAsync(runs, 0, sizeof(uint32_t), ctx->stream));
  k_row_ptr<<<(unsigned)((threads + 255) / 256), 256, 0, ctx->stream>>>(to_id, n_edges,
                                                                        row_base, n_rows,
                                                                        row_ptr, runs);
  PLX_LAUNCH_CHECK("k_row_ptr");
  k_row_ptr_runs<<<(unsigned)ctx->num_sms, 256, 0, ctx->stream>>>(runs, row_ptr);
  PLX_LAUNCH_CHECK("k_row_ptr_runs");
  return PLX_OK;
}

extern "C" uint64_t plx_csr_plan_words(uint64_t n_edges, uint32_t n_rows) {
  (void)n_rows;
  const uint64_t nb = plan_blocks(n_edges);
  return plan_wide_off(nb) + plan_max_wide(n_edges) + plan_max_long(n_edges);
}

static int csr_plan(plx_ctx* ctx, const uint32_t* row_ptr, uint32_t n_rows,
                    uint64_t n_edges, uint32_t* plan, uint64_t plan_words,
                    plx_csr* out, bool sync);

extern "C" int plx_csr_plan(plx_ctx* ctx, const uint32_t* row_ptr,
                            uint32_t n_rows, uint64_t n_edges, uint32_t* plan,
                            uint64_t plan_words, plx_csr* out) {
  return csr_plan(ctx, row_ptr, n_rows, n_edges, plan, plan_words, out, true);
}

extern "C" int plx_csr_plan_async(plx_ctx* ctx, const uint32_t* row_ptr,
                                  uint32_t n_rows, uint64_t n_edges,
                                  uint32_t* plan, uint64_t plan_words,
                                  plx_csr* out) {
  return csr_plan(ctx, row_ptr, n_rows, n_edges, plan, plan_words, out, false);
}

// Header words are written by a kernel (no host staging) so the async variant
// needs no synchronisation.
__global__ void k_plan_header(uint32_t* plan, uint32_t nb, uint32_t max_wide,
                              uint32_t max_long) {
  plan[0] = kPlanMagic;
  plan[1] = nb;
  plan[2] = 0;
  plan[3] = 0;
  plan[4] = 0;
  plan[5] = max_wide;
  plan[6] = max_long;
  plan[7] = 0;
}

static int csr_plan(plx_ctx* ctx, const uint32_t* row_ptr, uint32_t n_rows,
                    uint64_t n_edges, uint32_t* plan, uint64_t plan_words,
                    plx_csr* out, bool sync) {
  PLX_CHECK_ARG(ctx && row_ptr && plan, "ctx, row_ptr and plan are required");
  PLX_CHECK_ARG(n_edges < 0xFFFF0000ull, "n_edges must be < 2^32 - 2^16");
  PLX_CHECK_ARG(aligned16(row_ptr), "row_ptr must be 16-byte aligned");
  const uint64_t need = plx_csr_plan_words(n_edges, n_rows);
  PLX_CHECK_ARG(plan_words >= need, "plan buffer too small: %llu words, need %llu",
                (unsigned long long)plan_words, (unsigned long long)need);
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  const uint64_t nb = plan_blocks(n_edges);
  k_plan_header<<<1, 1, 0, ctx->stream>>>(plan, (uint32_t)nb,
                                          (uint32_t)plan_max_wide(n_edges),
                                          (uint32_t)plan_max_long(n_edges));
  PLX_LAUNCH_CHECK("k_plan_header");
  k_plan_blocks<<<(unsigned)((nb + 1 + 255) / 256), 256, 0, ctx->stream>>>(
      row_ptr, n_rows, n_edges, plan);
  PLX_LAUNCH_CHECK("k_plan_blocks");
  k_plan_rows<<<(unsigned)std::max<uint64_t>(1, std::min<uint64_t>(((uint64_t)n_rows + 255) / 256,
                                                                     4ull * ctx->num_sms)),
                256, 0, ctx->stream>>>(
      row_ptr, n_rows, n_edges, plan);
  PLX_LAUNCH_CHECK("k_plan_rows");
  if (!sync) {
    if (out) {
      out->row_ptr = row_ptr;
      out->plan = plan;
      out->n_edges = n_edges;
      out->n_rows = n_rows;
      out->n_wide = PLX_COUNT_UNKNOWN;
      out->n_long = PLX_COUNT_UNKNOWN;
      out->n_short = PLX_COUNT_UNKNOWN;
      out->to_id = nullptr;
      out->row_base = 0;
      out->max_row = PLX_COUNT_UNKNOWN;
    }
    return PLX_OK;
  }
  uint32_t hdr[kPlanHdr] = {};
  PLX_TRY_CUDA(cudaMemcpyAsync(hdr, plan, sizeof(hdr), cudaMemcpyDeviceToHost,
                               ctx->stream));
  PLX_TRY_CUDA(cudaStreamSynchronize(ctx->stream));
  if (hdr[0] != kPlanMagic)
    return set_error(PLX_ERR_ARG,
                     "row_ptr is not a valid CSR index (must start at 0, be "
                     "non-decreasing and end at n_edges)");
  if (out) {
    out->row_ptr = row_ptr;
    out->plan = plan;
    out->n_edges = n_edges;
    out->n_rows = n_rows;
    out->n_wide = hdr[2];
    out->n_long = hdr[3];
    out->n_short = hdr[4];
    out->to_id = nullptr;
    out->row_base = 0;
    out->max_row = hdr[7];
  }
  return PLX_OK;
}

extern "C" int plx_sweep_forward_rows(plx_ctx* ctx, const uint32_t* row_ptr, uint32_t n_rows,
                                      const uint32_t* from_id, const float* weight,
                                      const uint8_t* dead, const float* act_src,
                                      uint32_t act_src_len, int apply_kind, float* act_dst,
                                      const float* value, float* err_out) {
  PLX_CHECK_ARG(ctx && row_ptr, "ctx and row_ptr are required");
  if (apply_kind == PLX_APPLY_IPC_ERROR)
    PLX_CHECK_ARG(value && err_out, "IPC_ERROR needs value and err_out");
  else
    PLX_CHECK_ARG(act_dst, "act_dst is required");
  if (apply_kind == PLX_APPLY_SIGMOID_GRAD || apply_kind == PLX_APPLY_TANH_GRAD)
    PLX_CHECK_ARG(value, "the gradient applies need value");
  PLX_CHECK_ARG(apply_kind >= PLX_APPLY_IDENTITY && apply_kind <= PLX_APPLY_TANH_GRAD,
                "unknown apply_kind %d", apply_kind);
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  if (n_rows == 0) return PLX_OK;
  const unsigned g = (unsigned)std::min<uint64_t>((n_rows + 255) / 256, 32ull * ctx->num_sms);
  const uint32_t len = act_src ? act_src_len : 0;
  switch (apply_kind) {
#define PLX_ROWS_CASE(K)                                                                   \
  case K:                                                                                  \
    if (dead)                                                                              \
      k_rows_fold<K, true><<<g, 256, 0, ctx->stream>>>(row_ptr, n_rows, from_id, weight,  \
                                                       dead, act_src, len, value, act_dst, \
                                                       err_out, ctx->d_status);            \
    else                                                                                   \
      k_rows_fold<K, false><<<g, 256, 0, ctx->stream>>>(row_ptr, n_rows, from_id, weight, \
                                                        dead, act_src, len, value,         \
                                                        act_dst, err_out, ctx->d_status);  \
    break;
    PLX_ROWS_CASE(PLX_APPLY_IDENTITY)
    PLX_ROWS_CASE(PLX_APPLY_SIGMOID)
    PLX_ROWS_CASE(PLX_APPLY_TANH)
    PLX_ROWS_CASE(PLX_APPLY_IPC_ERROR)
    PLX_ROWS_CASE(PLX_APPLY_SIGMOID_GRAD)
    PLX_ROWS_CASE(PLX_APPLY_TANH_GRAD)
#undef PLX_ROWS_CASE
  }
  PLX_LAUNCH_CHECK("k_rows_fold");
  return PLX_OK;
}

extern "C" int plx_sweep_forward(plx_ctx* ctx, const plx_csr* csr,
                                 const uint32_t* from_id, const float* weight,
                                 const uint8_t* dead, const float* act_src,
                                 uint32_t act_src_len, int apply_kind,
                                 float* act_dst, const float* value,
                                 float* err_out) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  if (int rc = validate_csr(csr)) return rc;
  PLX_CHECK_ARG(csr->n_edges == 0 || (from_id && weight && act_src),
                "from_id, weight and act_src are required");
  PLX_CHECK_ARG(aligned16(from_id) && aligned16(weight) && aligned16(dead),
                "connection arrays must be 16-byte aligned");
  if (apply_kind == PLX_APPLY_IPC_ERROR)
    PLX_CHECK_ARG(value && err_out, "IPC_ERROR needs value and err_out");
  else
    PLX_CHECK_ARG(act_dst, "act_dst is required");
  if (apply_kind == PLX_APPLY_SIGMOID_GRAD || apply_kind == PLX_APPLY_TANH_GRAD)
    PLX_CHECK_ARG(value, "the gradient applies need value");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  SweepArgs a = base_args(ctx, csr);
  a.src = from_id;
  a.w_in = weight;
  a.dead = dead;
  a.act_src = act_src;
  a.act_src_len = act_src_len;
  a.act_dst = act_dst;
  a.value = value;
  a.err_out = err_out;
  const bool d = dead != nullptr;
  switch (apply_kind) {
#define PLX_FWD_CASE(K)                                                       \
  case K:                                                                     \
    return d ? launch_sweep<true, K, kUpdNone, false, true>(ctx, a, csr)      \
             : launch_sweep<true, K, kUpdNone, false, false>(ctx, a, csr);
    PLX_FWD_CASE(PLX_APPLY_IDENTITY)
    PLX_FWD_CASE(PLX_APPLY_SIGMOID)
    PLX_FWD_CASE(PLX_APPLY_TANH)
    PLX_FWD_CASE(PLX_APPLY_IPC_ERROR)
    PLX_FWD_CASE(PLX_APPLY_SIGMOID_GRAD)
    PLX_FWD_CASE(PLX_APPLY_TANH_GRAD)
#undef PLX_FWD_CASE
    default:
      return set_error(PLX_ERR_ARG, "unknown apply_kind %d", apply_kind);
  }
}

extern "C" int plx_sweep_forward_hebbian(
    plx_ctx* ctx, const plx_csr* csr, const uint32_t* from_id,
    const uint8_t* dead, const float* act_src, uint32_t act_src_len,
    const float* w_in, float* w_out, const float* trace_in, float* trace_out,
    float decay, float rate, float* act_dst) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  if (int rc = validate_csr(csr)) return rc;
  PLX_CHECK_ARG(act_dst, "act_dst is required");
  PLX_CHECK_ARG(csr->n_edges == 0 ||
                    (from_id && act_src && w_in && w_out && trace_in && trace_out),
                "connection arrays and act_src are required");
  PLX_CHECK_ARG(csr->n_edges == 0 || (w_in != w_out && trace_in != trace_out),
                "the fused sweep needs distinct input and output weight/trace buffers");
  PLX_CHECK_ARG(aligned16(from_id) && aligned16(dead) && aligned16(w_in) &&
                    aligned16(w_out) && aligned16(trace_in) && aligned16(trace_out),
                "connection arrays must be 16-byte aligned");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  SweepArgs a = base_args(ctx, csr);
  a.src = from_id;
  a.dead = dead;
  a.act_src = act_src;
  a.act_src_len = act_src_len;
  a.w_in = w_in;
  a.w_out = w_out;
  a.e_in = trace_in;
  a.e_out = trace_out;
  a.decay = decay;
  a.rate = rate;
  a.act_dst = act_dst;
  return dead ? launch_sweep<true, PLX_APPLY_IDENTITY, kUpdHebbTrace, true, true>(ctx, a, csr)
              : launch_sweep<true, PLX_APPLY_IDENTITY, kUpdHebbTrace, true, false>(ctx, a, csr);
}

extern "C" int plx_sweep_forward_hebbian_gather(
    plx_ctx* ctx, const plx_csr* csr, const uint32_t* from_id, const uint8_t* dead,
    const float* act_src, uint32_t act_src_len, const float* w_in, float* w_out,
    const float* trace_in, float* trace_out, float decay, float rate, float* act_dst,
    float* const* peer_out, uint32_t n_peers, uint32_t peer_offset, uint32_t peer_len) {
  PLX_CHECK_ARG(n_peers <= PLX_MAX_PEERS, "at most %d peers", PLX_MAX_PEERS);
  PLX_CHECK_ARG(n_peers == 0 || peer_out, "peer_out is required");
  for (uint32_t p = 0; p < n_peers; ++p) PLX_CHECK_ARG(peer_out[p], "peer_out[%u] is NULL", p);
  PLX_CHECK_ARG(ctx, "ctx is required");
  if (int rc = validate_csr(csr)) return rc;
  // Every destination row r is stored to peer_out[p][peer_offset + r]: the
  // whole slice must lie inside the peer buffers (checked before any device
  // work, so a bad offset never reaches another GPU's memory).
  PLX_CHECK_ARG(n_peers == 0 || (uint64_t)peer_offset + csr->n_rows <= peer_len,
                "peer slice [%u, %llu) exceeds the peer buffers of %u floats", peer_offset,
                (unsigned long long)peer_offset + csr->n_rows, peer_len);
  PLX_CHECK_ARG(act_dst, "act_dst is required");
  PLX_CHECK_ARG(csr->n_edges == 0 ||
                    (from_id && act_src && w_in && w_out && trace_in && trace_out),
                "connection arrays and act_src are required");
  PLX_CHECK_ARG(csr->n_edges == 0 || (w_in != w_out && trace_in != trace_out),
                "the fused sweep needs distinct input and output weight/trace buffers");
  PLX_CHECK_ARG(aligned16(from_id) && aligned16(dead) && aligned16(w_in) &&
                    aligned16(w_out) && aligned16(trace_in) && aligned16(trace_out),
                "connection arrays must be 16-byte aligned");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  SweepArgs a = base_args(ctx, csr);
  a.src = from_id;
  a.dead = dead;
  a.act_src = act_src;
  a.act_src_len = act_src_len;
  a.w_in = w_in;
  a.w_out = w_out;
  a.e_in = trace_in;
  a.e_out = trace_out;
  a.decay = decay;
  a.rate = rate;
  a.act_dst = act_dst;
  a.n_peers = n_peers;
  a.peer_offset = peer_offset;
  for (uint32_t p = 0; p < n_peers; ++p) a.peer_out[p] = peer_out[p];
  return dead ? launch_sweep<true, PLX_APPLY_IDENTITY, kUpdHebbTrace, true, true>(ctx, a, csr)
              : launch_sweep<true, PLX_APPLY_IDENTITY, kUpdHebbTrace, true, false>(ctx, a, csr);
}

extern "C" int plx_sweep_update(plx_ctx* ctx, const plx_csr* csr,
                                const uint32_t* from_id, const uint8_t* dead,
                                const float* act_src, uint32_t act_src_len,
                                const float* post, int update_kind, float rate,
                                const float* w_in, float* w_out) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  if (int rc = validate_csr(csr)) return rc;
  PLX_CHECK_ARG(csr->n_edges == 0 || (from_id && act_src && post && w_in && w_out),
                "from_id, act_src, post, w_in and w_out are required");
  PLX_CHECK_ARG(aligned16(from_id) && aligned16(dead) && aligned16(w_in) &&
                    aligned16(w_out),
                "connection arrays must be 16-byte aligned");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  SweepArgs a = base_args(ctx, csr);
  a.src = from_id;
  a.dead = dead;
  a.act_src = act_src;
  a.act_src_len = act_src_len;
  a.post = post;
  a.rate = rate;
  a.w_in = w_in;
  a.w_out = w_out;
  const bool d = dead != nullptr;
  switch (update_kind) {
    case PLX_UPDATE_GRADIENT:
      return d ? launch_sweep<false, PLX_APPLY_IDENTITY, kUpdGrad, false, true>(ctx, a, csr)
               : launch_sweep<false, PLX_APPLY_IDENTITY, kUpdGrad, false, false>(ctx, a, csr);
    case PLX_UPDATE_HEBBIAN:
      return d ? launch_sweep<false, PLX_APPLY_IDENTITY, kUpdHebb, false, true>(ctx, a, csr)
               : launch_sweep<false, PLX_APPLY_IDENTITY, kUpdHebb, false, false>(ctx, a, csr);
    case PLX_UPDATE_HEBBIAN_T:
      return d ? launch_sweep<false, PLX_APPLY_IDENTITY, kUpdHebbT, false, true>(ctx, a, csr)
               : launch_sweep<false, PLX_APPLY_IDENTITY, kUpdHebbT, false, false>(ctx, a, csr);
    default:
      return set_error(PLX_ERR_ARG, "unknown update_kind %d", update_kind);
  }
}
