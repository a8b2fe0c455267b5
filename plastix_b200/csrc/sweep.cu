// K1: the per-connection sweep over dst-sorted connections.
//
// Reference loops replaced (include/plastix/plastix.hpp):
//   DoForwardPass, Pipeline branch            :133-148
//   DoForwardPass, one Topological level      :112-130
//   DoUpdateConnectionState (incoming sweep)  :238-245
//
// Design (B200): persistent CTAs walk fixed edge tiles of S connections.
// Thread 0 streams each tile's SoA slices (FromId, Weight, [Trace], [Dead])
// into a ring of shared-memory stages with 1-D bulk copies (TMA engine,
// mbarrier transaction counts), NSTAGE-2 tiles ahead of the compute. Per tile:
//   A  edge-parallel gather act[FromId] into shared memory (L2-resident),
//   B  per destination row, fold w*act strictly left to right (one thread per
//      row; rows longer than PLX_SEQ_ROW_MAX use a warp and 33-edge chunks),
//      run Apply, write the row output, broadcast the row value to its edges,
//   C  edge-parallel per-connection update in shared memory,
// and thread 0 bulk-stores the updated Weight/Trace slices.
// A row that crosses a tile boundary is summed by every tile it touches (the
// pieces outside the tile are re-read from global memory, which is why the
// fused variant reads w_in and writes w_out); only the tile that holds the
// row's first connection writes its output. Rows longer than 2048
// connections are summed beforehand by k_long_rows.
#include <cstdio>

#include "common.cuh"

namespace plx {

constexpr uint32_t kPlanG = 256;        // plan granularity (edges per block)
constexpr uint32_t kLongRow = 2048;     // rows longer than this: k_long_rows
constexpr uint32_t kWideChunk = 33;     // chunk length of the warp fold
constexpr uint32_t kMaxWideChunks = 64; // ceil(2048 / 33) <= 64
constexpr uint32_t kPlanMagic = 0x504C4E31u;  // "PLN1"

// plan layout (u32 words):
//   [0] magic (0 when row_ptr failed validation)  [1] n_blocks  [2] n_long
//   [3 .. 3+n_blocks]  first row whose start >= b*kPlanG (last = n_rows)
//   [4+n_blocks ..]    ids of rows longer than kLongRow
__host__ __device__ inline uint64_t plan_blocks(uint64_t n_edges) {
  uint64_t b = (n_edges + kPlanG - 1) / kPlanG;
  return b ? b : 1;
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
};

enum UpdKind : int { kUpdNone = 0, kUpdHebbTrace = 1, kUpdGrad = 2, kUpdHebb = 3 };

// ---------------------------------------------------------------------------
// Plan construction
// ---------------------------------------------------------------------------
__global__ void k_row_ptr(const uint32_t* __restrict__ to_id, uint64_t n_edges,
                          uint32_t row_base, uint32_t n_rows,
                          uint32_t* __restrict__ row_ptr) {
  uint64_t r = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (r > n_rows) return;
  if (r == n_rows) {
    row_ptr[r] = (uint32_t)n_edges;
    return;
  }
  const uint64_t key = (uint64_t)row_base + r;
  uint64_t lo = 0, hi = n_edges;  // first index with to_id >= key
  while (lo < hi) {
    uint64_t mid = (lo + hi) >> 1;
    if ((uint64_t)__ldg(to_id + mid) < key) lo = mid + 1;
    else hi = mid;
  }
  row_ptr[r] = (uint32_t)lo;
}

__global__ void k_plan_blocks(const uint32_t* __restrict__ row_ptr,
                              uint32_t n_rows, uint64_t n_edges,
                              uint32_t* __restrict__ plan) {
  const uint64_t nb = plan_blocks(n_edges);
  uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (b > nb) return;
  if (b == nb) {
    plan[3 + b] = n_rows;
    return;
  }
  const uint64_t key = b * kPlanG;
  uint32_t lo = 0, hi = n_rows;  // first row r in [0, n_rows] with start >= key
  while (lo < hi) {
    uint32_t mid = (lo + hi) >> 1;
    if ((uint64_t)__ldg(row_ptr + mid) < key) lo = mid + 1;
    else hi = mid;
  }
  plan[3 + b] = lo;
}

// Validates row_ptr (monotone, row_ptr[0]==0, row_ptr[n_rows]==n_edges) and
// lists the long rows. Any violation clears the magic word so that every
// sweep using this plan stops and reports a bad-plan status.
__global__ void k_plan_rows(const uint32_t* __restrict__ row_ptr,
                            uint32_t n_rows, uint64_t n_edges,
                            uint32_t* __restrict__ plan, uint64_t max_long) {
  const uint64_t nb = plan_blocks(n_edges);
  uint64_t r = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (r == 0) {
    if (row_ptr[0] != 0 || row_ptr[n_rows] != (uint32_t)n_edges) plan[0] = 0;
  }
  if (r >= n_rows) return;
  const uint32_t a = row_ptr[r], b = row_ptr[r + 1];
  if (b < a || b > n_edges) {
    plan[0] = 0;
    return;
  }
  if (b - a > kLongRow) {
    uint32_t slot = atomicAdd(&plan[2], 1u);
    if (slot < max_long) plan[4 + nb + slot] = (uint32_t)r;
    else plan[0] = 0;
  }
}

// ---------------------------------------------------------------------------
// Apply / update rules
// ---------------------------------------------------------------------------
template <int APPLY>
__device__ __forceinline__ float apply_row(float acc, uint32_t r,
                                           const SweepArgs& a, bool owned) {
  float post;
  if constexpr (APPLY == PLX_APPLY_IDENTITY) {
    post = acc;
  } else if constexpr (APPLY == PLX_APPLY_SIGMOID) {
    post = 1.0f / __fadd_rn(1.0f, expf(-acc));
  } else if constexpr (APPLY == PLX_APPLY_TANH) {
    post = tanhf(acc);
  } else {
    post = __fsub_rn(__ldg(a.value + r), acc);
  }
  if (owned) {
    if constexpr (APPLY == PLX_APPLY_IPC_ERROR) a.err_out[r] = post;
    else a.act_dst[r] = post;
  }
  return post;
}

// Value a row's connections see in the update (what Apply stored).
template <int APPLY>
__device__ __forceinline__ float stored_post(uint32_t r, const SweepArgs& a) {
  if constexpr (APPLY == PLX_APPLY_IPC_ERROR) return a.err_out[r];
  else return a.act_dst[r];
}

__device__ __forceinline__ float gather_act(const SweepArgs& a, uint32_t s) {
  if (s >= a.act_src_len) {
    record_status(a.status, kStatusBadIndex);
    return 0.0f;
  }
  return __ldg(a.act_src + s);
}

// Product of one connection read straight from global memory (pieces of a
// row outside the current tile).
template <bool DEAD>
__device__ __forceinline__ float global_term(const SweepArgs& a, uint32_t k) {
  if constexpr (DEAD) {
    if (__ldg(a.dead + k)) return 0.0f;
  }
  return __fmul_rn(__ldg(a.w_in + k), gather_act(a, __ldg(a.src + k)));
}

// ---------------------------------------------------------------------------
// Long rows (> kLongRow): one CTA per row, deterministic order: thread t folds
// connections t, t+NT, ... then thread 0 folds the NT partials in order.
// ---------------------------------------------------------------------------
template <int APPLY, bool DEAD>
__global__ void __launch_bounds__(256) k_long_rows(SweepArgs a) {
  __shared__ float part[256];
  const uint32_t* plan = a.plan;
  if (plan[0] != kPlanMagic) return;
  const uint64_t nb = plan_blocks(a.n_edges);
  const uint32_t n_long = plan[2];
  for (uint32_t i = blockIdx.x; i < n_long; i += gridDim.x) {
    const uint32_t r = plan[4 + nb + i];
    const uint32_t rs = a.row_ptr[r], re = a.row_ptr[r + 1];
    float acc = 0.0f;
    for (uint32_t k = rs + threadIdx.x; k < re; k += blockDim.x)
      acc = __fadd_rn(acc, global_term<DEAD>(a, k));
    part[threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
      float s = 0.0f;
      for (uint32_t t = 0; t < blockDim.x; ++t) s = __fadd_rn(s, part[t]);
      apply_row<APPLY>(s, r, a, true);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// The tile sweep
// ---------------------------------------------------------------------------
template <int S, int NSTAGE, int NT, bool DEAD, bool TRACE>
struct SweepSmem {
  static constexpr uint32_t kStageBytes =
      S * 4u /*src*/ + S * 4u /*w*/ + (TRACE ? S * 4u : 0u) + (DEAD ? S : 0u);
  static constexpr uint32_t kOffA = NSTAGE * kStageBytes;
  static constexpr uint32_t kOffPost = kOffA + S * 4u;
  static constexpr uint32_t kOffWide = kOffPost + S * 4u;
  static constexpr uint32_t kOffBar = kOffWide + (NT / 32) * kMaxWideChunks * 4u;
  static constexpr uint32_t kBytes = kOffBar + NSTAGE * 8u + 16u;
};

template <int S, int NSTAGE, int NT, bool FOLD, int APPLY, int UPD, bool TRACE,
          bool DEAD>
__global__ void __launch_bounds__(NT) k_sweep(SweepArgs a) {
  static_assert(S % kPlanG == 0, "tile must be a multiple of the plan block");
  static_assert(NSTAGE >= 3, "need at least 3 stages");
  constexpr int LOOK = NSTAGE - 2;
  constexpr int NWARPS = NT / 32;
  constexpr uint32_t kBlocksPerTile = S / kPlanG;
  using L = SweepSmem<S, NSTAGE, NT, DEAD, TRACE>;

  extern __shared__ __align__(128) unsigned char smem[];
  float* s_a = reinterpret_cast<float*>(smem + L::kOffA);
  float* s_post = reinterpret_cast<float*>(smem + L::kOffPost);
  float* s_wide = reinterpret_cast<float*>(smem + L::kOffWide);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);

  const uint32_t* __restrict__ plan = a.plan;
  if (plan[0] != kPlanMagic) {
    if (threadIdx.x == 0 && blockIdx.x == 0) record_status(a.status, kStatusBadPlan);
    return;
  }
  const uint64_t nb = plan[1];
  const uint64_t n_edges = a.n_edges;
  const uint32_t n_tiles = (uint32_t)((nb + kBlocksPerTile - 1) / kBlocksPerTile);
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;

  auto stage_src = [&](int st) {
    return reinterpret_cast<uint32_t*>(smem + st * L::kStageBytes);
  };
  auto stage_w = [&](int st) {
    return reinterpret_cast<float*>(smem + st * L::kStageBytes + S * 4u);
  };
  auto stage_e = [&](int st) {
    return reinterpret_cast<float*>(smem + st * L::kStageBytes + S * 8u);
  };
  auto stage_dead = [&](int st) {
    return reinterpret_cast<uint8_t*>(smem + st * L::kStageBytes + S * 8u +
                                      (TRACE ? S * 4u : 0u));
  };

  if (tid == 0) {
    for (int s = 0; s < NSTAGE; ++s) mbar_init(&bars[s], 1);
    mbar_init_fence();
  }
  __syncthreads();

  // Thread 0: stream tile `t` into stage `st`.
  auto issue = [&](uint32_t t, int st) {
    const uint64_t ts = (uint64_t)t * S;
    const uint32_t n = (uint32_t)min_u64(S, n_edges > ts ? n_edges - ts : 0);
    const uint32_t n4 = n & ~3u, n16 = n & ~15u;
    uint32_t* ssrc = stage_src(st);
    float* sw = stage_w(st);
    for (uint32_t k = n4; k < n; ++k) {
      ssrc[k] = a.src[ts + k];
      sw[k] = a.w_in[ts + k];
      if constexpr (TRACE) stage_e(st)[k] = a.e_in[ts + k];
    }
    if constexpr (DEAD) {
      for (uint32_t k = n16; k < n; ++k) stage_dead(st)[k] = a.dead[ts + k];
    }
    const uint32_t bytes =
        n4 * 4u * (TRACE ? 3u : 2u) + (DEAD ? n16 : 0u);
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&bars[st], bytes);
    if (n4) {
      bulk_load(ssrc, a.src + ts, n4 * 4u, &bars[st]);
      bulk_load(sw, a.w_in + ts, n4 * 4u, &bars[st]);
      if constexpr (TRACE) bulk_load(stage_e(st), a.e_in + ts, n4 * 4u, &bars[st]);
    }
    if constexpr (DEAD) {
      if (n16) bulk_load(stage_dead(st), a.dead + ts, n16, &bars[st]);
    }
  };

  const uint32_t my_tiles =
      blockIdx.x < n_tiles ? (n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  if (tid == 0) {
    for (uint32_t j = 0; j < (uint32_t)LOOK && j < my_tiles; ++j)
      issue(blockIdx.x + j * gridDim.x, (int)(j % NSTAGE));
  }

  for (uint32_t i = 0; i < my_tiles; ++i) {
    const uint32_t t = blockIdx.x + i * gridDim.x;
    const int st = (int)(i % NSTAGE);
    if (tid == 0 && i + LOOK < my_tiles) {
      if constexpr (UPD != kUpdNone) bulk_wait_read<1>();
      issue(t + LOOK * gridDim.x, (int)((i + LOOK) % NSTAGE));
    }

    const uint64_t ts64 = (uint64_t)t * S;
    const uint32_t ts = (uint32_t)ts64;
    const uint32_t n_in = (uint32_t)min_u64(S, n_edges > ts64 ? n_edges - ts64 : 0);
    const uint32_t te = ts + n_in;
    const uint32_t b0 = t * kBlocksPerTile;
    const uint32_t b1 = (uint32_t)min_u64((uint64_t)b0 + kBlocksPerTile, nb);
    const uint32_t o_begin = plan[3 + b0];
    const uint32_t o_end = plan[3 + b1];
    const bool has_head =
        n_in > 0 && (o_begin == a.n_rows || a.row_ptr[o_begin] > ts);
    const uint32_t n_items = (o_end - o_begin) + (has_head ? 1u : 0u);

    const bool ok = mbar_wait_bounded(&bars[st], (i / NSTAGE) & 1u, a.timeout_ns);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) record_status(a.status, kStatusTimeout);
      break;
    }

    const uint32_t* s_src = stage_src(st);
    float* s_w = stage_w(st);
    float* s_e = stage_e(st);
    const uint8_t* s_dead = stage_dead(st);

    // ---- A: gather source activations ----
    for (uint32_t k = tid; k < n_in; k += NT) {
      float v = 0.0f;
      if (!DEAD || !s_dead[k]) v = gather_act(a, s_src[k]);
      s_a[k] = v;
    }
    __syncthreads();

    // ---- B: per-row fold / Apply / broadcast ----
    auto item_row = [&](uint32_t idx) -> uint32_t {
      return has_head ? (idx == 0 ? o_begin - 1 : o_begin + idx - 1) : o_begin + idx;
    };
    // B1: rows up to PLX_SEQ_ROW_MAX, one thread each.
    for (uint32_t idx = tid; idx < n_items; idx += NT) {
      const uint32_t r = item_row(idx);
      const bool owned = !(has_head && idx == 0);
      const uint32_t rs = a.row_ptr[r], re = a.row_ptr[r + 1];
      if (re - rs > PLX_SEQ_ROW_MAX) continue;
      float post;
      if constexpr (FOLD) {
        float acc = 0.0f;
        uint32_t k = rs;
        for (; k < re && k < ts; ++k) acc = __fadd_rn(acc, global_term<DEAD>(a, k));
        const uint32_t mid_end = min(re, te);
        for (; k < mid_end; ++k) {
          const uint32_t q = k - ts;
          float p = __fmul_rn(s_w[q], s_a[q]);
          if constexpr (DEAD) p = s_dead[q] ? 0.0f : p;
          acc = __fadd_rn(acc, p);
        }
        for (; k < re; ++k) acc = __fadd_rn(acc, global_term<DEAD>(a, k));
        post = apply_row<APPLY>(acc, r, a, owned);
      } else {
        post = __ldg(a.post + r);
      }
      if constexpr (UPD != kUpdNone) {
        const uint32_t lo = max(rs, ts), hi = min(re, te);
        for (uint32_t k = lo; k < hi; ++k) s_post[k - ts] = post;
      }
    }
    // B2: longer rows, one warp each.
    for (uint32_t idx = warp; idx < n_items; idx += NWARPS) {
      const uint32_t r = item_row(idx);
      const bool owned = !(has_head && idx == 0);
      const uint32_t rs = a.row_ptr[r], re = a.row_ptr[r + 1];
      const uint32_t len = re - rs;
      if (len <= PLX_SEQ_ROW_MAX) continue;
      float post = 0.0f;
      if constexpr (FOLD) {
        if (len > kLongRow) {
          post = stored_post<APPLY>(r, a);  // written by k_long_rows
        } else {
          float* wide = s_wide + warp * kMaxWideChunks;
          const uint32_t nch = (len + kWideChunk - 1) / kWideChunk;
          for (uint32_t c = lane; c < nch; c += 32) {
            const uint32_t c0 = rs + c * kWideChunk;
            const uint32_t c1 = min(re, c0 + kWideChunk);
            float acc = 0.0f;
            for (uint32_t k = c0; k < c1; ++k) {
              float p;
              if (k >= ts && k < te) {
                const uint32_t q = k - ts;
                p = __fmul_rn(s_w[q], s_a[q]);
                if constexpr (DEAD) p = s_dead[q] ? 0.0f : p;
              } else {
                p = global_term<DEAD>(a, k);
              }
              acc = __fadd_rn(acc, p);
            }
            wide[c] = acc;
          }
          __syncwarp();
          if (lane == 0) {
            float acc = 0.0f;
            for (uint32_t c = 0; c < nch; ++c) acc = __fadd_rn(acc, wide[c]);
            post = apply_row<APPLY>(acc, r, a, owned);
          }
          post = __shfl_sync(0xffffffffu, post, 0);
          __syncwarp();
        }
      } else {
        post = __ldg(a.post + r);
      }
      if constexpr (UPD != kUpdNone) {
        const uint32_t lo = max(rs, ts), hi = min(re, te);
        for (uint32_t k = lo + lane; k < hi; k += 32) s_post[k - ts] = post;
      }
    }
    __syncthreads();

    if constexpr (UPD != kUpdNone) {
      // ---- C: per-connection update in shared memory ----
      for (uint32_t k = tid; k < n_in; k += NT) {
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
        } else {
          s_w[k] = __fadd_rn(w, __fmul_rn(__fmul_rn(a.rate, post), av));
        }
      }
      fence_proxy_async_smem();
      __syncthreads();
      const uint32_t n4 = n_in & ~3u;
      if (tid == 0) {
        if (n4) {
          bulk_store(a.w_out + ts, s_w, n4 * 4u);
          if constexpr (TRACE) bulk_store(a.e_out + ts, s_e, n4 * 4u);
        }
        bulk_commit();  // one group per tile, empty or not
      }
      for (uint32_t k = n4 + tid; k < n_in; k += NT) {
        a.w_out[ts + k] = s_w[k];
        if constexpr (TRACE) a.e_out[ts + k] = s_e[k];
      }
    }
    __syncthreads();
  }
  if constexpr (UPD != kUpdNone) {
    if (tid == 0) bulk_wait_all<0>();
  }
}

// ---------------------------------------------------------------------------
// Host launch helpers
// ---------------------------------------------------------------------------
struct TileCfg {
  static constexpr int S = 2048;
  static constexpr int NSTAGE = 4;
  static constexpr int NT = 256;
};

template <bool FOLD, int APPLY, int UPD, bool TRACE, bool DEAD>
int launch_sweep(plx_ctx* ctx, const SweepArgs& args, uint32_t n_long) {
  constexpr int S = TileCfg::S, NSTAGE = TileCfg::NSTAGE, NT = TileCfg::NT;
  using L = SweepSmem<S, NSTAGE, NT, DEAD, TRACE>;
  auto kern = k_sweep<S, NSTAGE, NT, FOLD, APPLY, UPD, TRACE, DEAD>;
  PLX_TRY_CUDA(cudaFuncSetAttribute(
      kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kBytes));
  int per_sm = 0;
  PLX_TRY_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NT,
                                                             L::kBytes));
  if (per_sm < 1) per_sm = 1;
  const uint64_t nb = plan_blocks(args.n_edges);
  const uint64_t n_tiles = (nb + S / kPlanG - 1) / (S / kPlanG);
  const uint64_t grid =
      std::min<uint64_t>(n_tiles, (uint64_t)ctx->num_sms * per_sm);
  if (FOLD && n_long) {
    // Rows longer than kLongRow are summed first.
    const uint32_t g2 = std::min<uint32_t>(n_long, 4u * ctx->num_sms);
    k_long_rows<APPLY, DEAD><<<g2, 256, 0, ctx->stream>>>(args);
    PLX_LAUNCH_CHECK("k_long_rows");
  }
  kern<<<(unsigned)grid, NT, L::kBytes, ctx->stream>>>(args);
  PLX_LAUNCH_CHECK("k_sweep");
  return PLX_OK;
}

static int validate_csr(const plx_csr* csr) {
  PLX_CHECK_ARG(csr && csr->row_ptr && csr->plan, "csr, row_ptr and plan are required");
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
  k_row_ptr<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(
      to_id, n_edges, row_base, n_rows, row_ptr);
  PLX_LAUNCH_CHECK("k_row_ptr");
  return PLX_OK;
}

extern "C" uint64_t plx_csr_plan_words(uint64_t n_edges, uint32_t n_rows) {
  (void)n_rows;
  return 4 + plan_blocks(n_edges) + n_edges / kLongRow + 1;
}

extern "C" int plx_csr_plan(plx_ctx* ctx, const uint32_t* row_ptr,
                            uint32_t n_rows, uint64_t n_edges, uint32_t* plan,
                            uint64_t plan_words, uint32_t* n_long_out) {
  PLX_CHECK_ARG(ctx && row_ptr && plan, "ctx, row_ptr and plan are required");
  PLX_CHECK_ARG(n_edges < 0xFFFF0000ull, "n_edges must be < 2^32 - 2^16");
  const uint64_t need = plx_csr_plan_words(n_edges, n_rows);
  PLX_CHECK_ARG(plan_words >= need, "plan buffer too small: %llu words, need %llu",
                (unsigned long long)plan_words, (unsigned long long)need);
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  const uint64_t nb = plan_blocks(n_edges);
  const uint32_t header[3] = {kPlanMagic, (uint32_t)nb, 0u};
  PLX_TRY_CUDA(cudaMemcpyAsync(plan, header, sizeof(header),
                               cudaMemcpyHostToDevice, ctx->stream));
  k_plan_blocks<<<(unsigned)((nb + 1 + 255) / 256), 256, 0, ctx->stream>>>(
      row_ptr, n_rows, n_edges, plan);
  PLX_LAUNCH_CHECK("k_plan_blocks");
  const uint64_t max_long = n_edges / kLongRow + 1;
  k_plan_rows<<<(unsigned)(((uint64_t)n_rows + 256) / 256), 256, 0, ctx->stream>>>(
      row_ptr, n_rows, n_edges, plan, max_long);
  PLX_LAUNCH_CHECK("k_plan_rows");
  // The header copy reads a host stack array: wait for it before returning.
  uint32_t hdr[3] = {0, 0, 0};
  PLX_TRY_CUDA(cudaMemcpyAsync(hdr, plan, sizeof(hdr), cudaMemcpyDeviceToHost,
                               ctx->stream));
  PLX_TRY_CUDA(cudaStreamSynchronize(ctx->stream));
  if (hdr[0] != kPlanMagic)
    return set_error(PLX_ERR_ARG,
                     "row_ptr is not a valid CSR index (must start at 0, be "
                     "non-decreasing and end at n_edges; at most %llu long rows)",
                     (unsigned long long)max_long);
  if (n_long_out) *n_long_out = hdr[2];
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
    return d ? launch_sweep<true, K, kUpdNone, false, true>(ctx, a, csr->n_long)           \
             : launch_sweep<true, K, kUpdNone, false, false>(ctx, a, csr->n_long);
    PLX_FWD_CASE(PLX_APPLY_IDENTITY)
    PLX_FWD_CASE(PLX_APPLY_SIGMOID)
    PLX_FWD_CASE(PLX_APPLY_TANH)
    PLX_FWD_CASE(PLX_APPLY_IPC_ERROR)
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
  PLX_CHECK_ARG(w_in != w_out && trace_in != trace_out,
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
  return dead ? launch_sweep<true, PLX_APPLY_IDENTITY, kUpdHebbTrace, true, true>(ctx, a, csr->n_long)
              : launch_sweep<true, PLX_APPLY_IDENTITY, kUpdHebbTrace, true, false>(ctx, a, csr->n_long);
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
      return d ? launch_sweep<false, PLX_APPLY_IDENTITY, kUpdGrad, false, true>(ctx, a, csr->n_long)
               : launch_sweep<false, PLX_APPLY_IDENTITY, kUpdGrad, false, false>(ctx, a, csr->n_long);
    case PLX_UPDATE_HEBBIAN:
      return d ? launch_sweep<false, PLX_APPLY_IDENTITY, kUpdHebb, false, true>(ctx, a, csr->n_long)
               : launch_sweep<false, PLX_APPLY_IDENTITY, kUpdHebb, false, false>(ctx, a, csr->n_long);
    default:
      return set_error(PLX_ERR_ARG, "unknown update_kind %d", update_kind);
  }
}
