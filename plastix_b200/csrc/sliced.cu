// K1S: the connection sweep (forward sum + fused Hebbian trace update) over a
// warp-sliced row layout.
//
// Reference loops replaced (include/plastix/plastix.hpp): the Pipeline
// DoForwardPass (:133-148) followed by the UpdateIncomingConnection sweep of
// DoUpdateConnectionState (:238-245), for the Hebbian trace rule.
//
// Why a second layout. In the destination-sorted CSR order a warp streams
// consecutive connections, which belong to a few rows; every row's sum must
// then be folded left to right by one lane from staged products (the
// reference's order), a serial phase on top of the streaming. Here one lane
// owns one row for the whole sweep:
//
// * Rows are cut into windows of 512 consecutive rows; inside a window they
//   are ordered by length (descending, stable) and dealt 32 at a time into
//   slices, one row per lane, so the rows of a slice have nearly equal
//   lengths.
// * A slice stores its rows interleaved four connections at a time: slot
//   slice_ptr[s] + 128*g + 4*lane + c holds connection 4g + c of the lane's
//   row (c in [0, 4)); a row shorter than the slice's longest leaves padding
//   slots. Every field (FromId, Weight, Trace, Dead) is stored in this slot
//   order; perm[slot] is the reference connection index of a slot.
// * A warp sweeps a slice with coalesced 128-bit loads -- each lane reads 16
//   bytes of its own row per step -- gathers act[FromId], and folds its row
//   strictly left to right as the loads arrive (w*act with a separate
//   rounding, then the add: bit-exact with the reference). The gathered
//   activations are staged in shared memory (lane-interleaved, no bank
//   conflicts); after Apply the second pass over the slice applies the trace
//   and weight update in place from the staged activations and the row's
//   value; each lane writes its row's value to act_dst, and for the
//   multi-GPU hand-off the warp that completes a 512-row window copies the
//   window to every peer's all-gather buffer with coalesced stores.
// * Warps take slices from an atomic queue, each on its own. Measured
//   configuration (64M connections): 16 connections per lane in flight per
//   step, 4 warps per CTA, 4 CTAs per SM (shallower steps with more warps,
//   deeper steps with fewer CTAs, and Weight staged in shared memory instead
//   of read again in pass 2 were all slower).
#include <cub/device/device_scan.cuh>

#include "common.cuh"

namespace plx {
namespace {

constexpr uint32_t kSlLanes = 32;                       // rows per slice
constexpr uint32_t kSlSlicesPerWin = 16;                // slices per window
constexpr uint32_t kSlWin = kSlLanes * kSlSlicesPerWin;  // rows per window
constexpr uint32_t kSlWarps = 4;                         // warps per CTA
constexpr uint32_t kSlCapGroups = 24;  // staged groups of 4 per lane (rows of <= 96)
constexpr uint32_t kSlNone = PLX_SLICED_NONE;
constexpr uint32_t kFullMask = 0xFFFFFFFFu;

struct SlicedArgs {
  const uint64_t* slice_ptr;
  const uint32_t* lane_row;
  const uint32_t* lane_len;
  uint32_t n_slices;
  uint32_t n_rows;
  const uint32_t* src;
  const uint8_t* dead;
  const float* act_src;
  uint32_t act_src_len;
  float* w;
  float* e;
  float decay;
  float rate;
  float* act_dst;
  uint32_t* queue;
  int32_t* status;
  uint32_t* win_done;  // [n_slices / 16 rounded up] slices finished per window
  uint32_t w_first;    // pass-1 Weight loads evict-first (large source arrays)
  uint32_t n_peers;
  uint32_t peer_offset;
  float* peer_out[PLX_MAX_PEERS];
};

// ---- plan construction ------------------------------------------------------

// key[r] = window(r) << 16 | (0xFFFF - min(len(r), 0xFFFF)): a stable sort on
// it orders each window's rows by descending length.
__global__ void k_sl_keys(const uint32_t* __restrict__ row_ptr, uint32_t n_rows,
                          uint32_t* __restrict__ key) {
  const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n_rows) return;
  const uint32_t len = row_ptr[r + 1] - row_ptr[r];
  key[r] = (r / kSlWin) << 16 | (0xFFFFu - min(len, 0xFFFFu));
}

// One warp per slice: lane_row / lane_len, and the slice's slot count
// (128 per group of 4, enough groups for its longest row) into size[s].
__global__ void k_sl_lanes(const uint32_t* __restrict__ row_ptr, const uint32_t* __restrict__ order,
                           uint32_t n_rows, uint32_t n_slices, uint32_t* __restrict__ lane_row,
                           uint32_t* __restrict__ lane_len, uint64_t* __restrict__ size) {
  const uint32_t s = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const uint32_t lane = threadIdx.x & 31u;
  if (s >= n_slices) return;
  const uint32_t i = s * kSlLanes + lane;
  uint32_t row = kSlNone, len = 0;
  if (i < n_rows) {
    row = order[i];
    len = row_ptr[row + 1] - row_ptr[row];
  }
  lane_row[i] = row;
  lane_len[i] = len;
  uint32_t mx = len;
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = max(mx, __shfl_xor_sync(kFullMask, mx, o));
  if (lane == 0) size[s] = (uint64_t)((mx + 3) / 4) * 128u;
}

// perm[slot] for every slot of slice s (one warp per slice, 16-byte stores).
__global__ void k_sl_perm(const uint64_t* __restrict__ slice_ptr, const uint32_t* __restrict__ lane_row,
                          const uint32_t* __restrict__ lane_len, const uint32_t* __restrict__ row_ptr,
                          uint32_t n_slices, uint32_t* __restrict__ perm) {
  const uint32_t s = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const uint32_t lane = threadIdx.x & 31u;
  if (s >= n_slices) return;
  const uint64_t base = slice_ptr[s];
  const uint32_t groups = (uint32_t)((slice_ptr[s + 1] - base) / 128);
  const uint32_t row = lane_row[s * kSlLanes + lane], len = lane_len[s * kSlLanes + lane];
  const uint32_t first = row == kSlNone ? 0u : row_ptr[row];
  for (uint32_t g = 0; g < groups; ++g) {
    uint32_t v[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t j = 4 * g + c;
      v[c] = j < len ? first + j : kSlNone;
    }
    *reinterpret_cast<uint4*>(perm + base + 128ull * g + 4 * lane) = make_uint4(v[0], v[1], v[2], v[3]);
  }
}

// slot[i] = ref[perm[i]] (0 for padding) / ref[perm[i]] = slot[i].
template <typename T>
__global__ void k_sl_pack(const uint32_t* __restrict__ perm, uint64_t n_slots, const T* __restrict__ ref,
                          T* __restrict__ slot) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n_slots;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t p = perm[i];
    slot[i] = p == kSlNone ? T() : ref[p];
  }
}
template <typename T>
__global__ void k_sl_unpack(const uint32_t* __restrict__ perm, uint64_t n_slots, const T* __restrict__ slot,
                            T* __restrict__ ref) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n_slots;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t p = perm[i];
    if (p != kSlNone) ref[p] = slot[i];
  }
}

// ---- the sweep --------------------------------------------------------------

template <bool DEAD>
__device__ __forceinline__ uint32_t ld_dead4(const uint8_t* dead, uint64_t k) {
  if constexpr (DEAD) return __ldg(reinterpret_cast<const uint32_t*>(dead + k));
  else return 0u;
}

constexpr size_t kSlSmemBytes = (size_t)kSlWarps * kSlCapGroups * kSlLanes * 16;
constexpr int kSlStep = 4;  // groups of 4 connections per lane per step

// FromId of kSlStep groups of a lane's row (groups past the row read nothing).
__device__ __forceinline__ void load_sid(const SlicedArgs& a, uint64_t base, uint32_t lane,
                                         uint32_t g0, uint32_t my_groups, uint64_t pol,
                                         uint32_t (&sid)[kSlStep][4]) {
#pragma unroll
  for (int h = 0; h < kSlStep; ++h) {
    const uint32_t g = g0 + h;
    if (g < my_groups) {
      const uint4 x = ld_stream_v4(a.src + base + 128ull * g + 4 * lane, pol);
      sid[h][0] = x.x; sid[h][1] = x.y; sid[h][2] = x.z; sid[h][3] = x.w;
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c) sid[h][c] = 0;
    }
  }
}

// The hand-off to the other GPUs. A window's rows are contiguous
// ([512 w, 512 w + 512)) but its lanes' rows are permuted, so row values are
// not stored to the peers one lane at a time (scattered 4-byte NVLink
// writes); the warp that finishes a window's last slice instead copies the
// whole window from act_dst to every peer buffer with coalesced stores.
// Every warp makes its row values visible (fence) before it counts its slice.
__device__ __forceinline__ void push_window(const SlicedArgs& a, uint32_t s, uint32_t lane) {
  __threadfence();
  __syncwarp();
  const uint32_t win = s / kSlSlicesPerWin;
  uint32_t last = 0;
  if (lane == 0) {
    const uint32_t in_win = min(kSlSlicesPerWin, a.n_slices - win * kSlSlicesPerWin);
    last = atomicAdd(a.win_done + win, 1u) == in_win - 1;
  }
  if (!__shfl_sync(kFullMask, last, 0)) return;
  __threadfence();
  const uint32_t lo = win * kSlWin, hi = min(a.n_rows, lo + kSlWin);
  for (uint32_t r = lo + lane; r < hi; r += kSlLanes) {
    const float v = __ldcg(a.act_dst + r);
    for (uint32_t p = 0; p < a.n_peers; ++p) a.peer_out[p][a.peer_offset + r] = v;
  }
}

// Each warp takes slices one at a time from an atomic queue: no CTA-level
// barrier, so a warp never waits for the others (measured: the same passes
// inside a CTA that swept a window of slices together ran at half this rate).
template <bool DEAD>
__global__ void __launch_bounds__(kSlWarps * 32, 4) k_sweep_sliced(SlicedArgs a) {
  extern __shared__ __align__(16) float4 s_pre[];  // [warp][group][lane]
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const uint32_t len1 = a.act_src_len - 1u;
  const uint64_t pol_first = l2_policy_evict_first();
  const uint64_t pol_last = l2_policy_evict_last();
  // Weight is read again in pass 2, a few microseconds later. At normal
  // priority it stays in L2 until then; with a source array of 16 MB and
  // more, whose gathers miss L2 more often as it grows, evict-first Weight
  // lines leave the gathered array more room (measured at 32 MB: 0.460 ->
  // 0.443 ms; at 4 MB: 0.384 -> 0.402 ms, hence the switch).
  const uint64_t pol_w = a.w_first ? pol_first : l2_policy_evict_normal();
  float4(*pre)[kSlLanes] =
      reinterpret_cast<float4(*)[kSlLanes]>(s_pre + (size_t)warp * kSlCapGroups * kSlLanes);
  bool bad = false;

  for (;;) {
    uint32_t s = 0;
    if (lane == 0) s = atomicAdd(a.queue, 1u);
    s = __shfl_sync(kFullMask, s, 0);
    if (s >= a.n_slices) break;
    const uint64_t base = a.slice_ptr[s];
    const uint32_t groups = (uint32_t)((a.slice_ptr[s + 1] - base) / 128);
    const uint32_t row = a.lane_row[s * kSlLanes + lane];
    const uint32_t len = a.lane_len[s * kSlLanes + lane];
    const uint32_t my_groups = (len + 3) / 4;  // groups holding this lane's connections
    // Trace is first read in pass 2: the TMA unit brings the slice's traces
    // into L2 while pass 1 runs (measured 0.382 -> 0.379 ms at 64M).
    if (lane == 0 && groups) prefetch_l2_bulk(a.e + base, groups * 512u);
    // ---- pass 1: stream FromId/Weight, gather, fold left to right ----------
    // kSlStep groups (16 connections per lane) per step: the step's gathers
    // and Weight loads, then the next step's FromId loads, are in flight
    // together. Weight is read again in pass 2 (L2 priority: pol_w).
    float acc = 0.0f;
    uint32_t sid[kSlStep][4], sid_next[kSlStep][4];
    load_sid(a, base, lane, 0, my_groups, pol_first, sid);
    for (uint32_t g0 = 0; g0 < groups; g0 += kSlStep) {
      float av[kSlStep][4], wv[kSlStep][4];
      uint32_t dd[kSlStep];
      uint32_t smax = 0;
#pragma unroll
      for (int h = 0; h < kSlStep; ++h)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const bool in = 4 * (g0 + h) + c < len;
          const uint32_t sj = in ? sid[h][c] : 0u;
          smax = max(smax, sj);
          av[h][c] = in ? ld_keep_f32(a.act_src + min(sj, len1), pol_last) : 0.0f;
        }
      bad |= smax > len1;
#pragma unroll
      for (int h = 0; h < kSlStep; ++h) {
        const uint32_t g = g0 + h;
        const uint64_t k = base + 128ull * g + 4 * lane;
        if (g < my_groups) {
          const uint4 y = ld_stream_v4(a.w + k, pol_w);
          wv[h][0] = __uint_as_float(y.x); wv[h][1] = __uint_as_float(y.y);
          wv[h][2] = __uint_as_float(y.z); wv[h][3] = __uint_as_float(y.w);
          dd[h] = ld_dead4<DEAD>(a.dead, k);
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c) wv[h][c] = 0.0f;
          dd[h] = 0;
        }
      }
      if (g0 + kSlStep < groups)
        load_sid(a, base, lane, g0 + kSlStep, my_groups, pol_first, sid_next);
#pragma unroll
      for (int h = 0; h < kSlStep; ++h) {
        const uint32_t g = g0 + h;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          bool live = 4 * g + c < len;
          if constexpr (DEAD) live = live && ((dd[h] >> (8 * c)) & 0xFFu) == 0;
          if (live) acc = __fadd_rn(acc, __fmul_rn(wv[h][c], av[h][c]));
        }
        if (g < kSlCapGroups && g < my_groups)
          pre[g][lane] = make_float4(av[h][0], av[h][1], av[h][2], av[h][3]);
      }
#pragma unroll
      for (int h = 0; h < kSlStep; ++h)
#pragma unroll
        for (int c = 0; c < 4; ++c) sid[h][c] = sid_next[h][c];
    }
    // Apply (identity): the row's value, written by its lane
    const float post = acc;
    if (row != kSlNone) a.act_dst[row] = post;
    if (a.n_peers) push_window(a, s, lane);
    __syncwarp();
    // ---- pass 2: trace and weight update in place ----------------------------
    for (uint32_t g0 = 0; g0 < my_groups; g0 += kSlStep) {
      float w[kSlStep][4], e[kSlStep][4], pv[kSlStep][4];
      uint32_t d4[kSlStep];
#pragma unroll
      for (int h = 0; h < kSlStep; ++h) {
        const uint32_t g = g0 + h;
        const uint64_t k = base + 128ull * g + 4 * lane;
        if (g < my_groups) {
          const uint4 xw = ld_stream_v4(a.w + k, pol_first);
          const uint4 xe = ld_stream_v4(a.e + k, pol_first);
          w[h][0] = __uint_as_float(xw.x); w[h][1] = __uint_as_float(xw.y);
          w[h][2] = __uint_as_float(xw.z); w[h][3] = __uint_as_float(xw.w);
          e[h][0] = __uint_as_float(xe.x); e[h][1] = __uint_as_float(xe.y);
          e[h][2] = __uint_as_float(xe.z); e[h][3] = __uint_as_float(xe.w);
          d4[h] = ld_dead4<DEAD>(a.dead, k);
          if (g < kSlCapGroups) {
            const float4 p = pre[g][lane];
            pv[h][0] = p.x; pv[h][1] = p.y; pv[h][2] = p.z; pv[h][3] = p.w;
          } else {  // rows longer than the staging: gather again
            const uint4 x = ld_stream_v4(a.src + k, pol_first);
            const uint32_t sj[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int c = 0; c < 4; ++c)
              pv[h][c] = 4 * g + c < len ? ld_keep_f32(a.act_src + min(sj[c], len1), pol_last)
                                         : 0.0f;
          }
        }
      }
#pragma unroll
      for (int h = 0; h < kSlStep; ++h) {
        const uint32_t g = g0 + h;
        if (g >= my_groups) continue;
        const uint64_t k = base + 128ull * g + 4 * lane;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          bool live = 4 * g + c < len;
          if constexpr (DEAD) live = live && ((d4[h] >> (8 * c)) & 0xFFu) == 0;
          if (live) {
            const float ne = __fadd_rn(__fmul_rn(a.decay, e[h][c]), __fmul_rn(pv[h][c], post));
            e[h][c] = ne;
            w[h][c] = __fadd_rn(w[h][c], __fmul_rn(a.rate, ne));
          }
        }
        st_stream_v4(a.w + k, make_float4(w[h][0], w[h][1], w[h][2], w[h][3]), pol_first);
        st_stream_v4(a.e + k, make_float4(e[h][0], e[h][1], e[h][2], e[h][3]), pol_first);
      }
    }
    __syncwarp();  // the next slice overwrites the staging
  }
  if (bad) record_status(a.status, kStatusBadIndex);
}

int sl_check(const plx_sliced* sl) {
  PLX_CHECK_ARG(sl && sl->slice_ptr && sl->lane_row && sl->lane_len,
                "sliced layout: slice_ptr, lane_row and lane_len are required");
  PLX_CHECK_ARG(sl->n_slices == (sl->n_rows + kSlLanes - 1) / kSlLanes,
                "sliced layout: n_slices must be ceil(n_rows / 32)");
  return PLX_OK;
}

}  // namespace
}  // namespace plx

using namespace plx;

extern "C" uint32_t plx_sliced_n_slices(uint32_t n_rows) {
  return (n_rows + kSlLanes - 1) / kSlLanes;
}

extern "C" size_t plx_sliced_plan_scratch_bytes(uint32_t n_rows) {
  const size_t n = n_rows ? n_rows : 1;
  size_t scan = 0;
  cub::DeviceScan::InclusiveSum(nullptr, scan, (const uint64_t*)nullptr, (uint64_t*)nullptr,
                                (int)plx_sliced_n_slices(n_rows) + 1);
  return 3 * 4 * ((n + 3) & ~size_t(3)) + 8 * ((size_t)plx_sliced_n_slices(n_rows) + 2) +
         plx_radix_sort_scratch_bytes(n) + scan + 256;
}

extern "C" int plx_sliced_plan(plx_ctx* ctx, const uint32_t* row_ptr, uint32_t n_rows,
                               uint64_t n_edges, plx_sliced* out, uint64_t* slice_ptr,
                               uint32_t* lane_row, uint32_t* lane_len, void* scratch,
                               size_t scratch_bytes) {
  PLX_CHECK_ARG(ctx && out && row_ptr && slice_ptr && lane_row && lane_len && scratch,
                "ctx, row_ptr, out, slice_ptr, lane_row, lane_len and scratch are required");
  PLX_CHECK_ARG(n_rows > 0 && n_rows < (1u << 30), "n_rows must be in [1, 2^30)");
  PLX_CHECK_ARG((uint64_t)(n_rows + kSlWin - 1) / kSlWin < (1u << 16), "too many rows");
  PLX_CHECK_ARG(scratch_bytes >= plx_sliced_plan_scratch_bytes(n_rows),
                "scratch_bytes below plx_sliced_plan_scratch_bytes");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  const uint32_t n_slices = plx_sliced_n_slices(n_rows);
  const size_t nr4 = ((size_t)n_rows + 3) & ~size_t(3);
  uint8_t* p = static_cast<uint8_t*>(scratch);
  uint32_t* keys = reinterpret_cast<uint32_t*>(p);
  uint32_t* keys_sorted = keys + nr4;
  uint32_t* order = keys_sorted + nr4;
  uint64_t* size = reinterpret_cast<uint64_t*>(order + nr4);
  uint8_t* rest = reinterpret_cast<uint8_t*>(size + n_slices + 2);
  rest = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(rest) + 255) & ~uintptr_t(255));
  const size_t rs = plx_radix_sort_scratch_bytes(n_rows);
  k_sl_keys<<<(n_rows + 255) / 256, 256, 0, ctx->stream>>>(row_ptr, n_rows, keys);
  PLX_LAUNCH_CHECK("k_sl_keys");
  uint32_t win_bits = 1;
  while ((1u << win_bits) < (n_rows + kSlWin - 1) / kSlWin + 1) ++win_bits;
  if (int rc = plx_radix_sort_u32(ctx, n_rows, keys, keys_sorted, order, 0, 16 + win_bits, rest, rs))
    return rc;
  const uint32_t warps_per_block = 8;
  k_sl_lanes<<<(n_slices + warps_per_block - 1) / warps_per_block, 32 * warps_per_block, 0,
               ctx->stream>>>(row_ptr, order, n_rows, n_slices, lane_row, lane_len, size + 1);
  PLX_LAUNCH_CHECK("k_sl_lanes");
  PLX_TRY_CUDA(cudaMemsetAsync(size, 0, sizeof(uint64_t), ctx->stream));
  size_t scan_bytes = scratch_bytes - (size_t)(rest + rs - p);
  uint8_t* scan_tmp = rest + rs;
  PLX_TRY_CUDA(cub::DeviceScan::InclusiveSum(scan_tmp, scan_bytes, size, slice_ptr,
                                             (int)n_slices + 1, ctx->stream));
  uint64_t n_slots = 0;
  PLX_TRY_CUDA(cudaMemcpyAsync(&n_slots, slice_ptr + n_slices, sizeof(uint64_t),
                               cudaMemcpyDeviceToHost, ctx->stream));
  PLX_TRY_CUDA(cudaStreamSynchronize(ctx->stream));
  PLX_CHECK_ARG(n_slots < (1ull << 32), "more than 2^32 slots: split the layer");
  out->slice_ptr = slice_ptr;
  out->lane_row = lane_row;
  out->lane_len = lane_len;
  out->perm = nullptr;
  out->n_slots = n_slots;
  out->n_edges = n_edges;
  out->n_rows = n_rows;
  out->n_slices = n_slices;
  return PLX_OK;
}

extern "C" int plx_sliced_perm(plx_ctx* ctx, plx_sliced* sl, const uint32_t* row_ptr,
                               uint32_t* perm) {
  PLX_CHECK_ARG(ctx && row_ptr && perm, "ctx, row_ptr and perm are required");
  if (int rc = sl_check(sl)) return rc;
  PLX_CHECK_ARG(aligned16(perm), "perm must be 16-byte aligned");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  k_sl_perm<<<(sl->n_slices + 7) / 8, 256, 0, ctx->stream>>>(sl->slice_ptr, sl->lane_row,
                                                            sl->lane_len, row_ptr, sl->n_slices,
                                                            perm);
  PLX_LAUNCH_CHECK("k_sl_perm");
  sl->perm = perm;
  return PLX_OK;
}

template <typename F>
static int sl_dispatch(uint32_t elem_bytes, F&& f) {
  switch (elem_bytes) {
    case 1: return f(uint8_t{});
    case 2: return f(uint16_t{});
    case 4: return f(uint32_t{});
    case 8: return f(uint64_t{});
    default: return set_error(PLX_ERR_ARG, "elem_bytes must be 1, 2, 4 or 8");
  }
}

extern "C" int plx_sliced_pack(plx_ctx* ctx, const plx_sliced* sl, const void* ref, void* slot,
                               uint32_t elem_bytes) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  if (int rc = sl_check(sl)) return rc;
  if (sl->n_slots == 0) return PLX_OK;  // no connections
  PLX_CHECK_ARG(slot && (ref || sl->n_edges == 0), "ref and slot are required");
  PLX_CHECK_ARG(sl->perm, "the layout has no perm (plx_sliced_perm)");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  const unsigned grid = (unsigned)std::min<uint64_t>((sl->n_slots + 255) / 256, 8u * ctx->num_sms);
  return sl_dispatch(elem_bytes, [&](auto t) {
    using T = decltype(t);
    k_sl_pack<T><<<std::max(grid, 1u), 256, 0, ctx->stream>>>(sl->perm, sl->n_slots,
                                                               static_cast<const T*>(ref),
                                                               static_cast<T*>(slot));
    PLX_LAUNCH_CHECK("k_sl_pack");
    return PLX_OK;
  });
}

extern "C" int plx_sliced_unpack(plx_ctx* ctx, const plx_sliced* sl, const void* slot, void* ref,
                                 uint32_t elem_bytes) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  if (int rc = sl_check(sl)) return rc;
  if (sl->n_slots == 0) return PLX_OK;  // no connections
  PLX_CHECK_ARG(slot && (ref || sl->n_edges == 0), "slot and ref are required");
  PLX_CHECK_ARG(sl->perm, "the layout has no perm (plx_sliced_perm)");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  const unsigned grid = (unsigned)std::min<uint64_t>((sl->n_slots + 255) / 256, 8u * ctx->num_sms);
  return sl_dispatch(elem_bytes, [&](auto t) {
    using T = decltype(t);
    k_sl_unpack<T><<<std::max(grid, 1u), 256, 0, ctx->stream>>>(sl->perm, sl->n_slots,
                                                                 static_cast<const T*>(slot),
                                                                 static_cast<T*>(ref));
    PLX_LAUNCH_CHECK("k_sl_unpack");
    return PLX_OK;
  });
}

extern "C" int plx_sweep_forward_hebbian_sliced(plx_ctx* ctx, const plx_sliced* sl,
                                                const uint32_t* from_id, const uint8_t* dead,
                                                const float* act_src, uint32_t act_src_len,
                                                float* weight, float* trace, float decay,
                                                float rate, float* act_dst,
                                                float* const* peer_out, uint32_t n_peers,
                                                uint32_t peer_offset, uint32_t peer_len) {
  PLX_CHECK_ARG(n_peers <= PLX_MAX_PEERS, "at most %d peers", PLX_MAX_PEERS);
  PLX_CHECK_ARG(n_peers == 0 || peer_out, "peer_out is required");
  for (uint32_t p = 0; p < n_peers; ++p) PLX_CHECK_ARG(peer_out[p], "peer_out[%u] is NULL", p);
  PLX_CHECK_ARG(ctx, "ctx is required");
  if (int rc = sl_check(sl)) return rc;
  PLX_CHECK_ARG(n_peers == 0 || (uint64_t)peer_offset + sl->n_rows <= peer_len,
                "peer slice [%u, %llu) exceeds the peer buffers of %u floats", peer_offset,
                (unsigned long long)peer_offset + sl->n_rows, peer_len);
  PLX_CHECK_ARG(act_dst, "act_dst is required");
  PLX_CHECK_ARG(sl->n_slots == 0 || (from_id && weight && trace && act_src && act_src_len),
                "from_id, weight, trace and act_src are required");
  PLX_CHECK_ARG(aligned16(from_id) && aligned16(dead) && aligned16(weight) && aligned16(trace),
                "slot arrays must be 16-byte aligned");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  SlicedArgs a{};
  a.slice_ptr = sl->slice_ptr;
  a.lane_row = sl->lane_row;
  a.lane_len = sl->lane_len;
  a.n_slices = sl->n_slices;
  a.n_rows = sl->n_rows;
  a.src = from_id;
  a.dead = dead;
  a.act_src = act_src;
  a.act_src_len = act_src_len ? act_src_len : 1;
  a.w = weight;
  a.e = trace;
  a.decay = decay;
  a.rate = rate;
  a.act_dst = act_dst;
  a.queue = ctx->d_queue;
  a.status = ctx->d_status;
  a.n_peers = n_peers;
  a.w_first = act_src_len >= (1u << 22) ? 1u : 0u;
  a.peer_offset = peer_offset;
  for (uint32_t p = 0; p < n_peers; ++p) a.peer_out[p] = peer_out[p];
  auto kern = dead ? k_sweep_sliced<true> : k_sweep_sliced<false>;
  PLX_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kSlSmemBytes));
  int per_sm = 0;
  PLX_TRY_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kSlWarps * 32,
                                                             kSlSmemBytes));
  if (per_sm < 1) per_sm = 1;
  const uint32_t n_blocks = (sl->n_slices + kSlWarps - 1) / kSlWarps;
  const uint32_t grid = std::min<uint32_t>(n_blocks, (uint32_t)ctx->num_sms * per_sm);
  if (n_peers) {
    const size_t n_win = (sl->n_slices + kSlSlicesPerWin - 1) / kSlSlicesPerWin;
    if (int rc = ctx_counters(ctx, n_win, &a.win_done)) return rc;
    PLX_TRY_CUDA(cudaMemsetAsync(a.win_done, 0, n_win * sizeof(uint32_t), ctx->stream));
  }
  PLX_TRY_CUDA(cudaMemsetAsync(ctx->d_queue, 0, sizeof(uint32_t), ctx->stream));
  kern<<<std::max(grid, 1u), kSlWarps * 32, kSlSmemBytes, ctx->stream>>>(a);
  PLX_LAUNCH_CHECK("k_sweep_sliced");
  return PLX_OK;
}
