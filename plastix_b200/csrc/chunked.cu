// Chunked-source layout for long rows (hundreds to thousands of connections
// per row, e.g. the 2,048-fan-in blocks of the multilayer predictive-coding
// network).
//
// A row sweep gathers one value per connection from the source side. Random
// 4-byte gathers from global memory cost one L1TEX wavefront each, and at
// about one per clock per SM they, not HBM, bound a row sweep with 8 bytes of
// connection data per gather (~35 % of the HBM roofline). Here the gathered
// array is cut into chunks of PLX_CHUNK_SOURCES values (64 KB), and each
// connection is stored under (chunk, row) with a 16-bit offset into its chunk.
// A CTA loads one chunk into shared memory once and folds the chunk's part of
// many rows from there: shared-memory gathers instead of global ones, and 6
// bytes per connection (offset + weight) instead of 8. Per (chunk, row) the
// partial sum goes to a small array; a second kernel adds a row's partials in
// chunk order and applies the row rule. Segments are padded to multiples of
// four connections (offset PLX_CHUNK_SOURCES reads a zero) so every lane loads
// four connections with 8- and 16-byte vector loads.
//
// Order: a row's sum is the chunk-ordered sum of per-chunk sums, each a fixed
// lane-strided order: deterministic, not the reference's left fold (rows this
// long are compared at 1e-5 relative). The update kernels apply the
// per-connection rules exactly as the row sweeps do, so a weight updated here
// has the same bits as the same rule applied in any other layout.
#include <cub/device/device_scan.cuh>

#include "common.cuh"

namespace plx {
namespace {

constexpr uint32_t kChunk = PLX_CHUNK_SOURCES;
constexpr uint32_t kPad = 4;            // segment length granularity
constexpr int kCThreads = 256;          // 8 warps
constexpr int kCRowsPerWarp = 8;        // rows a warp works on together

__host__ __device__ inline uint32_t n_chunks_for(uint32_t n_src) {
  return (n_src + kChunk - 1) / kChunk;
}

uint32_t bits_for(uint64_t v) {  // bits to hold 0..v
  uint32_t b = 0;
  while (b < 32 && (uint64_t(1) << b) <= v) ++b;
  return b;
}

// ---- build -----------------------------------------------------------------
__global__ void k_chunk_keys(const uint32_t* __restrict__ gather_id,
                             const uint32_t* __restrict__ row_id, uint64_t n,
                             uint32_t src_base, uint32_t n_src, uint32_t row_base,
                             uint32_t n_rows, uint32_t* __restrict__ keys) {
  const uint64_t n_keys = (uint64_t)n_chunks_for(n_src) * n_rows;
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < n;
       e += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t s = gather_id[e] - src_base;
    const uint32_t r = row_id[e] - row_base;
    keys[e] = (s < n_src && r < n_rows) ? (uint32_t)((uint64_t)(s / kChunk) * n_rows + r)
                                         : (uint32_t)n_keys;
  }
}

// cnt[k] = first sorted position with key >= k, k in [0, n_keys].
__global__ void k_chunk_counts(const uint32_t* __restrict__ skeys, uint64_t n,
                               uint64_t n_keys, uint32_t* __restrict__ cnt) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k <= n_keys;
       k += (uint64_t)gridDim.x * blockDim.x) {
    uint64_t lo = 0, hi = n;
    while (lo < hi) {
      const uint64_t mid = (lo + hi) >> 1;
      if (skeys[mid] < k) lo = mid + 1;
      else hi = mid;
    }
    cnt[k] = (uint32_t)lo;
  }
}

__global__ void k_chunk_padlen(const uint32_t* __restrict__ cnt, uint64_t n_keys,
                               uint32_t* __restrict__ plen) {
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k <= n_keys;
       k += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t len = k < n_keys ? cnt[k + 1] - cnt[k] : 0;
    plen[k] = (len + kPad - 1) / kPad * kPad;
  }
}

__global__ void k_chunk_fill(uint16_t* __restrict__ src16, uint32_t* __restrict__ perm,
                             uint64_t n) {
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < n;
       e += (uint64_t)gridDim.x * blockDim.x) {
    src16[e] = (uint16_t)kChunk;
    perm[e] = 0xFFFFFFFFu;
  }
}

__global__ void k_chunk_scatter(const uint32_t* __restrict__ skeys,
                                const uint32_t* __restrict__ sperm,
                                const uint32_t* __restrict__ cnt,
                                const uint32_t* __restrict__ seg_ptr,
                                const uint32_t* __restrict__ gather_id, uint64_t n_keys,
                                uint32_t src_base, uint32_t n_rows,
                                uint16_t* __restrict__ src16, uint32_t* __restrict__ perm) {
  const uint64_t n_valid = cnt[n_keys];
  for (uint64_t p = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; p < n_valid;
       p += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t k = skeys[p];
    const uint32_t e = sperm[p];
    const uint64_t d = (uint64_t)seg_ptr[k] + (p - cnt[k]);
    src16[d] = (uint16_t)((gather_id[e] - src_base) % kChunk);
    perm[d] = e;
    (void)n_rows;
  }
}

__global__ void k_chunk_gather_f32(const uint32_t* __restrict__ perm, uint64_t n,
                                   const float* __restrict__ field, float* __restrict__ out) {
  for (uint64_t d = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; d < n;
       d += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t e = perm[d];
    out[d] = e == 0xFFFFFFFFu ? 0.0f : field[e];
  }
}

// ---- sweeps ----------------------------------------------------------------
struct ChunkArgs {
  const uint32_t* seg_ptr;
  const uint16_t* src;
  float* w;
  const float* gathered;  // n_src values: the chunk source
  uint32_t n_src, n_rows, n_chunks;
  uint32_t rows_per_cta;
  float* partial;         // [n_chunks][n_rows]
  const float* row_val;   // update: per-row value
  float rate;
};

// The chunk of `gathered` this CTA works on, in shared memory; slot kChunk
// (the padding offset) reads 0.
__device__ __forceinline__ void load_chunk(float* s_src, const ChunkArgs& a, uint32_t c) {
  const uint64_t base = (uint64_t)c * kChunk;
  const uint64_t left = a.n_src - base;
  const uint32_t len = left < kChunk ? (uint32_t)left : kChunk;
  for (uint32_t i = threadIdx.x; i < kChunk + 1; i += blockDim.x)
    s_src[i] = i < len ? __ldg(a.gathered + base + i) : 0.0f;
  __syncthreads();
}

// Four connections per lane per step: 8-byte offset load, 16-byte weight load.
// Offsets are clamped to the padding slot, so a damaged layout cannot read
// outside the chunk.
__device__ __forceinline__ float fold4(const float* s_src, uint2 sv, float4 wv) {
  const float g0 = s_src[min(sv.x & 0xFFFFu, kChunk)], g1 = s_src[min(sv.x >> 16, kChunk)];
  const float g2 = s_src[min(sv.y & 0xFFFFu, kChunk)], g3 = s_src[min(sv.y >> 16, kChunk)];
  float acc = __fmul_rn(wv.x, g0);
  acc = __fadd_rn(acc, __fmul_rn(wv.y, g1));
  acc = __fadd_rn(acc, __fmul_rn(wv.z, g2));
  return __fadd_rn(acc, __fmul_rn(wv.w, g3));
}

__global__ void __launch_bounds__(kCThreads) k_chunk_fold(ChunkArgs a) {
  extern __shared__ float s_src[];
  const uint32_t c = blockIdx.x;
  load_chunk(s_src, a, c);
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  const uint32_t r_lo = blockIdx.y * a.rows_per_cta;
  const uint32_t r_hi = min(a.n_rows, r_lo + a.rows_per_cta);
  const uint32_t* seg = a.seg_ptr + (uint64_t)c * a.n_rows;
  for (uint32_t r0 = r_lo + warp * kCRowsPerWarp; r0 < r_hi;
       r0 += (kCThreads / 32) * kCRowsPerWarp) {
    uint32_t beg[kCRowsPerWarp], end[kCRowsPerWarp];
    float acc[kCRowsPerWarp];
#pragma unroll
    for (int j = 0; j < kCRowsPerWarp; ++j) {
      const uint32_t r = r0 + j;
      beg[j] = r < r_hi ? seg[r] : 0;
      end[j] = r < r_hi ? seg[r + 1] : 0;
      acc[j] = 0.0f;
    }
    for (uint32_t off = 4 * lane;; off += 128) {
      bool any = false;
      uint2 sv[kCRowsPerWarp];
      float4 wv[kCRowsPerWarp];
#pragma unroll
      for (int j = 0; j < kCRowsPerWarp; ++j) {
        const uint32_t k = beg[j] + off;
        if (k < end[j]) {
          sv[j] = *reinterpret_cast<const uint2*>(a.src + k);
          wv[j] = *reinterpret_cast<const float4*>(a.w + k);
        }
      }
#pragma unroll
      for (int j = 0; j < kCRowsPerWarp; ++j) {
        const uint32_t k = beg[j] + off;
        if (k < end[j]) acc[j] = __fadd_rn(acc[j], fold4(s_src, sv[j], wv[j]));
        any |= beg[j] + off + 128 < end[j];
      }
      if (!__any_sync(0xffffffffu, any)) break;
    }
#pragma unroll
    for (int j = 0; j < kCRowsPerWarp; ++j) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
        acc[j] = __fadd_rn(acc[j], __shfl_xor_sync(0xffffffffu, acc[j], o));
      const uint32_t r = r0 + j;
      if (lane == 0 && r < r_hi) a.partial[(uint64_t)c * a.n_rows + r] = acc[j];
    }
  }
}

template <int APPLY>
__global__ void k_chunk_combine(const float* __restrict__ partial, uint32_t n_rows,
                                uint32_t n_chunks, const float* __restrict__ value,
                                float* __restrict__ out) {
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < n_rows;
       r += gridDim.x * blockDim.x) {
    float acc = 0.0f;
    for (uint32_t c = 0; c < n_chunks; ++c)
      acc = __fadd_rn(acc, partial[(uint64_t)c * n_rows + r]);
    float v = 0.0f;
    if constexpr (apply_reads_value(APPLY)) v = value[r];
    out[r] = apply_value<APPLY>(acc, v);
  }
}

// The iPC bottom-up Apply (TANH_GRAD) of a hidden layer with the value-node
// update of the same units folded into it (plx_ipc_value_update mode 1:
// x += gamma * (-eps + bu); act = tanh(x)). bu is consumed here and never
// stored: the reference zeroes it right after the update
// (ipc_multilayer.cpp:239-245). Same operations and roundings as the two
// separate kernels, so x and act are equal bit for bit.
__global__ void k_chunk_combine_ipc_value(const float* __restrict__ partial, uint32_t n_rows,
                                          uint32_t n_chunks, float* __restrict__ x,
                                          const float* __restrict__ eps, float gamma,
                                          float* __restrict__ act) {
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < n_rows;
       r += gridDim.x * blockDim.x) {
    float acc = 0.0f;
    for (uint32_t c = 0; c < n_chunks; ++c)
      acc = __fadd_rn(acc, partial[(uint64_t)c * n_rows + r]);
    const float v = x[r];
    const float bu = apply_value<PLX_APPLY_TANH_GRAD>(acc, v);
    const float xv = __fadd_rn(v, __fmul_rn(gamma, __fadd_rn(-eps[r], bu)));
    x[r] = xv;
    act[r] = tanhf(xv);
  }
}

// Per-connection update, same rules and rounding as plx_sweep_update:
//   GRADIENT:   w -= (rate * row) * g      HEBBIAN: w += (rate * row) * g
//   HEBBIAN_T:  w += (rate * g) * row
template <int KIND>
__device__ __forceinline__ float upd1(float w, float g, float rv, float rate) {
  if constexpr (KIND == PLX_UPDATE_GRADIENT) return __fsub_rn(w, __fmul_rn(__fmul_rn(rate, rv), g));
  else if constexpr (KIND == PLX_UPDATE_HEBBIAN) return __fadd_rn(w, __fmul_rn(__fmul_rn(rate, rv), g));
  else return __fadd_rn(w, __fmul_rn(__fmul_rn(rate, g), rv));
}

template <int KIND>
__global__ void __launch_bounds__(kCThreads) k_chunk_update(ChunkArgs a) {
  extern __shared__ float s_src[];
  const uint32_t c = blockIdx.x;
  load_chunk(s_src, a, c);
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  const uint32_t r_lo = blockIdx.y * a.rows_per_cta;
  const uint32_t r_hi = min(a.n_rows, r_lo + a.rows_per_cta);
  const uint32_t* seg = a.seg_ptr + (uint64_t)c * a.n_rows;
  for (uint32_t r0 = r_lo + warp * kCRowsPerWarp; r0 < r_hi;
       r0 += (kCThreads / 32) * kCRowsPerWarp) {
    uint32_t beg[kCRowsPerWarp], end[kCRowsPerWarp];
    float rv[kCRowsPerWarp];
#pragma unroll
    for (int j = 0; j < kCRowsPerWarp; ++j) {
      const uint32_t r = r0 + j;
      beg[j] = r < r_hi ? seg[r] : 0;
      end[j] = r < r_hi ? seg[r + 1] : 0;
      rv[j] = r < r_hi ? __ldg(a.row_val + r) : 0.0f;
    }
    for (uint32_t off = 4 * lane;; off += 128) {
      bool any = false;
      uint2 sv[kCRowsPerWarp];
      float4 wv[kCRowsPerWarp];
#pragma unroll
      for (int j = 0; j < kCRowsPerWarp; ++j) {
        const uint32_t k = beg[j] + off;
        if (k < end[j]) {
          sv[j] = *reinterpret_cast<const uint2*>(a.src + k);
          wv[j] = *reinterpret_cast<const float4*>(a.w + k);
        }
      }
#pragma unroll
      for (int j = 0; j < kCRowsPerWarp; ++j) {
        const uint32_t k = beg[j] + off;
        if (k < end[j]) {
          float4 o = wv[j];
          o.x = upd1<KIND>(o.x, s_src[min(sv[j].x & 0xFFFFu, kChunk)], rv[j], a.rate);
          o.y = upd1<KIND>(o.y, s_src[min(sv[j].x >> 16, kChunk)], rv[j], a.rate);
          o.z = upd1<KIND>(o.z, s_src[min(sv[j].y & 0xFFFFu, kChunk)], rv[j], a.rate);
          o.w = upd1<KIND>(o.w, s_src[min(sv[j].y >> 16, kChunk)], rv[j], a.rate);
          *reinterpret_cast<float4*>(a.w + k) = o;
        }
        any |= beg[j] + off + 128 < end[j];
      }
      if (!__any_sync(0xffffffffu, any)) break;
    }
  }
}

unsigned grid_1d(const plx_ctx* ctx, uint64_t n) {
  return (unsigned)std::max<uint64_t>(
      1, std::min<uint64_t>((n + 255) / 256, 8ull * (uint64_t)ctx->num_sms));
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

size_t scan_temp_bytes(uint64_t n_items) {
  size_t t = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, t, (const uint32_t*)nullptr, (uint32_t*)nullptr,
                                (int64_t)n_items);
  return t;
}

int check_chunked(const plx_chunked* L) {
  PLX_CHECK_ARG(L && L->seg_ptr && L->src, "layout with seg_ptr and src required");
  PLX_CHECK_ARG(L->n_chunks == n_chunks_for(L->n_src), "n_chunks does not match n_src");
  PLX_CHECK_ARG(aligned16(L->src) && aligned16(L->seg_ptr), "layout arrays must be 16-byte aligned");
  return PLX_OK;
}

dim3 sweep_grid(const plx_ctx* ctx, const plx_chunked* L, uint32_t* rows_per_cta) {
  // About 4 CTAs per SM in total, split across the chunks; each CTA covers a
  // contiguous row range of one chunk.
  const uint64_t want = 4ull * (uint64_t)ctx->num_sms;
  uint64_t slices = std::max<uint64_t>(1, want / std::max<uint32_t>(1, L->n_chunks));
  const uint64_t min_rows = (kCThreads / 32) * kCRowsPerWarp;
  uint64_t rows = (L->n_rows + slices - 1) / slices;
  rows = std::max<uint64_t>(rows, min_rows);
  slices = (L->n_rows + rows - 1) / rows;
  *rows_per_cta = (uint32_t)rows;
  return dim3(std::max<uint32_t>(1, L->n_chunks), (unsigned)std::max<uint64_t>(1, slices));
}

}  // namespace
}  // namespace plx

using namespace plx;

extern "C" uint64_t plx_chunked_max_padded(uint64_t n_edges, uint32_t n_rows, uint32_t n_src) {
  return n_edges + (uint64_t)(kPad - 1) * n_chunks_for(n_src) * n_rows;
}

extern "C" size_t plx_chunked_scratch_bytes(uint64_t n_edges, uint32_t n_rows, uint32_t n_src) {
  const uint64_t n_keys = (uint64_t)n_chunks_for(n_src) * n_rows;
  return 3 * align256(4 * n_edges) + 2 * align256(4 * (n_keys + 1)) +
         align256(scan_temp_bytes(n_keys + 1)) + plx_radix_sort_scratch_bytes(n_edges);
}

extern "C" int plx_chunked_build(plx_ctx* ctx, uint64_t n_edges, const uint32_t* gather_id,
                                 uint32_t src_base, uint32_t n_src, const uint32_t* row_id,
                                 uint32_t row_base, uint32_t n_rows, uint32_t* seg_ptr,
                                 uint16_t* src, uint32_t* perm, void* scratch,
                                 size_t scratch_bytes) {
  PLX_CHECK_ARG(ctx && seg_ptr && src && perm, "ctx, seg_ptr, src and perm are required");
  PLX_CHECK_ARG(n_edges == 0 || (gather_id && row_id), "gather_id and row_id are required");
  PLX_CHECK_ARG(n_edges < (1ull << 30), "n_edges must be < 2^30 (build per block)");
  PLX_CHECK_ARG(n_src > 0 && n_rows > 0, "n_src and n_rows must be positive");
  const uint64_t n_keys = (uint64_t)n_chunks_for(n_src) * n_rows;
  PLX_CHECK_ARG(n_keys < 0xFFFFFFFFull, "too many (chunk, row) segments");
  PLX_CHECK_ARG(plx_chunked_max_padded(n_edges, n_rows, n_src) < 0xFFFFFFFFull,
                "padded layout exceeds 32-bit offsets");
  PLX_CHECK_ARG(aligned16(src) && aligned16(seg_ptr), "seg_ptr and src must be 16-byte aligned");
  PLX_CHECK_ARG(scratch && scratch_bytes >= plx_chunked_scratch_bytes(n_edges, n_rows, n_src),
                "scratch too small");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  char* s = static_cast<char*>(scratch);
  const size_t ne = align256(4 * n_edges), nk = align256(4 * (n_keys + 1));
  uint32_t* keys = reinterpret_cast<uint32_t*>(s);
  uint32_t* skeys = reinterpret_cast<uint32_t*>(s + ne);
  uint32_t* sperm = reinterpret_cast<uint32_t*>(s + 2 * ne);
  uint32_t* cnt = reinterpret_cast<uint32_t*>(s + 3 * ne);
  uint32_t* plen = reinterpret_cast<uint32_t*>(s + 3 * ne + nk);
  size_t temp = scan_temp_bytes(n_keys + 1);
  void* temp_p = s + 3 * ne + 2 * nk;
  void* radix = s + 3 * ne + 2 * nk + align256(temp);
  const size_t radix_bytes = scratch_bytes - (3 * ne + 2 * nk + align256(temp));
  const uint64_t max_pad = plx_chunked_max_padded(n_edges, n_rows, n_src);

  k_chunk_fill<<<grid_1d(ctx, max_pad), 256, 0, ctx->stream>>>(src, perm, max_pad);
  PLX_LAUNCH_CHECK("k_chunk_fill");
  if (n_edges) {
    k_chunk_keys<<<grid_1d(ctx, n_edges), 256, 0, ctx->stream>>>(
        gather_id, row_id, n_edges, src_base, n_src, row_base, n_rows, keys);
    PLX_LAUNCH_CHECK("k_chunk_keys");
    if (int rc = plx_radix_sort_u32(ctx, n_edges, keys, skeys, sperm, 0, bits_for(n_keys),
                                    radix, radix_bytes))
      return rc;
  }
  k_chunk_counts<<<grid_1d(ctx, n_keys + 1), 256, 0, ctx->stream>>>(skeys, n_edges, n_keys,
                                                                     cnt);
  PLX_LAUNCH_CHECK("k_chunk_counts");
  k_chunk_padlen<<<grid_1d(ctx, n_keys + 1), 256, 0, ctx->stream>>>(cnt, n_keys, plen);
  PLX_LAUNCH_CHECK("k_chunk_padlen");
  PLX_TRY_CUDA(cub::DeviceScan::ExclusiveSum(temp_p, temp, plen, seg_ptr, (int64_t)(n_keys + 1),
                                             ctx->stream));
  if (n_edges) {
    k_chunk_scatter<<<grid_1d(ctx, n_edges), 256, 0, ctx->stream>>>(
        skeys, sperm, cnt, seg_ptr, gather_id, n_keys, src_base, n_rows, src, perm);
    PLX_LAUNCH_CHECK("k_chunk_scatter");
  }
  return PLX_OK;
}

extern "C" int plx_chunked_gather(plx_ctx* ctx, uint64_t n_padded, const uint32_t* perm,
                                  const float* field, float* out) {
  PLX_CHECK_ARG(ctx && (n_padded == 0 || (perm && field && out)), "arguments required");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  if (!n_padded) return PLX_OK;
  k_chunk_gather_f32<<<grid_1d(ctx, n_padded), 256, 0, ctx->stream>>>(perm, n_padded, field,
                                                                       out);
  PLX_LAUNCH_CHECK("k_chunk_gather_f32");
  return PLX_OK;
}

// The chunk partials of a row sweep (the first half of both fold entries).
static int chunk_partials(plx_ctx* ctx, const plx_chunked* L, const float* w,
                          const float* gathered, float* partial) {
  ChunkArgs a{};
  a.seg_ptr = L->seg_ptr;
  a.src = L->src;
  a.w = const_cast<float*>(w);
  a.gathered = gathered;
  a.n_src = L->n_src;
  a.n_rows = L->n_rows;
  a.n_chunks = L->n_chunks;
  a.partial = partial;
  const size_t smem = (kChunk + 1) * sizeof(float);
  static thread_local int attr_device = -1;
  if (attr_device != ctx->device) {
    PLX_TRY_CUDA(cudaFuncSetAttribute(k_chunk_fold, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
    PLX_TRY_CUDA(cudaFuncSetAttribute(k_chunk_update<PLX_UPDATE_GRADIENT>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    PLX_TRY_CUDA(cudaFuncSetAttribute(k_chunk_update<PLX_UPDATE_HEBBIAN>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    PLX_TRY_CUDA(cudaFuncSetAttribute(k_chunk_update<PLX_UPDATE_HEBBIAN_T>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_device = ctx->device;
  }
  const dim3 grid = sweep_grid(ctx, L, &a.rows_per_cta);
  k_chunk_fold<<<grid, kCThreads, smem, ctx->stream>>>(a);
  PLX_LAUNCH_CHECK("k_chunk_fold");
  return PLX_OK;
}

extern "C" int plx_chunked_fold(plx_ctx* ctx, const plx_chunked* L, const float* w,
                                const float* gathered, int apply_kind, const float* value,
                                float* out, float* partial) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  if (int rc = check_chunked(L)) return rc;
  PLX_CHECK_ARG(w && gathered && out && partial, "w, gathered, out and partial are required");
  PLX_CHECK_ARG(aligned16(w), "w must be 16-byte aligned");
  PLX_CHECK_ARG(!apply_reads_value(apply_kind) || value, "this apply needs value");
  PLX_CHECK_ARG(apply_kind >= PLX_APPLY_IDENTITY && apply_kind <= PLX_APPLY_TANH_GRAD,
                "unknown apply_kind %d", apply_kind);
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  if (int rc = chunk_partials(ctx, L, w, gathered, partial)) return rc;
  const unsigned cg = (unsigned)std::max<uint64_t>(1, (L->n_rows + 255) / 256);
  switch (apply_kind) {
#define PLX_CHUNK_APPLY(K)                                                              \
  case K:                                                                               \
    k_chunk_combine<K><<<cg, 256, 0, ctx->stream>>>(partial, L->n_rows, L->n_chunks, value, \
                                                    out);                               \
    break;
    PLX_CHUNK_APPLY(PLX_APPLY_IDENTITY)
    PLX_CHUNK_APPLY(PLX_APPLY_SIGMOID)
    PLX_CHUNK_APPLY(PLX_APPLY_TANH)
    PLX_CHUNK_APPLY(PLX_APPLY_IPC_ERROR)
    PLX_CHUNK_APPLY(PLX_APPLY_SIGMOID_GRAD)
    PLX_CHUNK_APPLY(PLX_APPLY_TANH_GRAD)
#undef PLX_CHUNK_APPLY
    default:
      return set_error(PLX_ERR_ARG, "unknown apply_kind %d", apply_kind);
  }
  PLX_LAUNCH_CHECK("k_chunk_combine");
  return PLX_OK;
}

extern "C" int plx_chunked_fold_ipc_value(plx_ctx* ctx, const plx_chunked* L, const float* w,
                                          const float* gathered, float* x, const float* eps,
                                          float gamma, float* act, float* partial) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  if (int rc = check_chunked(L)) return rc;
  PLX_CHECK_ARG(w && gathered && x && eps && act && partial,
                "w, gathered, x, eps, act and partial are required");
  PLX_CHECK_ARG(aligned16(w), "w must be 16-byte aligned");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  if (int rc = chunk_partials(ctx, L, w, gathered, partial)) return rc;
  const unsigned cg = (unsigned)std::max<uint64_t>(1, (L->n_rows + 255) / 256);
  k_chunk_combine_ipc_value<<<cg, 256, 0, ctx->stream>>>(partial, L->n_rows, L->n_chunks, x,
                                                          eps, gamma, act);
  PLX_LAUNCH_CHECK("k_chunk_combine_ipc_value");
  return PLX_OK;
}

extern "C" int plx_chunked_update(plx_ctx* ctx, const plx_chunked* L, float* w,
                                  const float* gathered, const float* row_val, int update_kind,
                                  float rate) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  if (int rc = check_chunked(L)) return rc;
  PLX_CHECK_ARG(w && gathered && row_val, "w, gathered and row_val are required");
  PLX_CHECK_ARG(aligned16(w), "w must be 16-byte aligned");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  // Shared-memory attributes are set by the first plx_chunked_fold on this
  // device; set them here too for callers that update first.
  const size_t smem = (kChunk + 1) * sizeof(float);
  PLX_TRY_CUDA(cudaFuncSetAttribute(k_chunk_update<PLX_UPDATE_GRADIENT>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  PLX_TRY_CUDA(cudaFuncSetAttribute(k_chunk_update<PLX_UPDATE_HEBBIAN>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  PLX_TRY_CUDA(cudaFuncSetAttribute(k_chunk_update<PLX_UPDATE_HEBBIAN_T>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  ChunkArgs a{};
  a.seg_ptr = L->seg_ptr;
  a.src = L->src;
  a.w = w;
  a.gathered = gathered;
  a.n_src = L->n_src;
  a.n_rows = L->n_rows;
  a.n_chunks = L->n_chunks;
  a.row_val = row_val;
  a.rate = rate;
  const dim3 grid = sweep_grid(ctx, L, &a.rows_per_cta);
  switch (update_kind) {
    case PLX_UPDATE_GRADIENT:
      k_chunk_update<PLX_UPDATE_GRADIENT><<<grid, kCThreads, smem, ctx->stream>>>(a);
      break;
    case PLX_UPDATE_HEBBIAN:
      k_chunk_update<PLX_UPDATE_HEBBIAN><<<grid, kCThreads, smem, ctx->stream>>>(a);
      break;
    case PLX_UPDATE_HEBBIAN_T:
      k_chunk_update<PLX_UPDATE_HEBBIAN_T><<<grid, kCThreads, smem, ctx->stream>>>(a);
      break;
    default:
      return set_error(PLX_ERR_ARG, "unknown update_kind %d", update_kind);
  }
  PLX_LAUNCH_CHECK("k_chunk_update");
  return PLX_OK;
}
