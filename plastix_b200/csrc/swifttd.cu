// SwiftTD step on the device: TD(lambda) with per-feature meta-learned step
// sizes, one linear value unit fed by N features, every per-feature value a
// connection field in SoA (examples/swifttd/swifttd.cpp:29-209 in the
// reference; its Network::DoStep is plastix.hpp:439-455).
//
// The reference runs three dense sweeps over all N connections per step
// (forward, UpdateIncoming = phase 1, UpdateOutgoing = phase 2) and mutates
// the globals V, Tau, B and VDelta from inside the per-connection policies.
// Only active features (F != 0) contribute to those four sums, so the step is
// restructured around them:
//
//   k_td_value   over the active list: V = sum W*F (fp64, fixed tree order),
//                then Loss (Delta, VDeltaPrev) in the last block; also the
//                per-tile start offsets into the active list for k_td_dense.
//   k_td_terms   over the active list: phase 1 for the active features only,
//                to form Tau = sum exp(Beta')*F*F, B = sum Z'*F and
//                VDelta = sum DeltaW*F (fp64, fixed tree order).
//   k_td_dense   one pass over all N features: phase 1 and phase 2 fused,
//                8 fields read and 10 written with 128-bit accesses, F taken
//                from a shared-memory tile into which the tile's few active
//                features are scattered. ResetGlobal (VOld = V) at the end.
//
// Per-feature arithmetic follows the reference's evaluation order with
// separate roundings (the library is built with --fmad=false); exp/log are
// CUDA's expf/logf. The four sums are fp64 trees in a fixed order, so results
// are deterministic run to run; against the reference's sequential fp32 sums
// they agree to the rounding of those sums.
#include <cmath>

#include "common.cuh"

namespace plx {
namespace {

constexpr int kTdThreads = 256;
constexpr int kTdActivePerBlock = 1024;  // 4 active entries per thread
constexpr int kTdTile = 1024;            // features per dense tile (float4/thread)

struct TdGlobals {
  float gamma, lambda, eta, eta_min, decay, meta;
  float v, v_old, delta, v_delta_prev, v_delta, tau, b;
};
static_assert(sizeof(TdGlobals) == sizeof(plx_td_globals), "globals layout");

struct TdScratch {
  uint32_t* tickets;  // [0] value, [1] terms; zero between steps
  double* part_v;     // [blocks]
  double* part_t;     // [blocks][3]
  uint32_t* start;    // [n_tiles + 1]
};

struct TdFields {
  float* f[PLX_TD_NUM_FIELDS];
};

enum : int { W = 0, Z, ZD, DW, H, HOLD, HTEMP, ZBAR, P, BETA };

__host__ __device__ inline uint64_t td_blocks(uint64_t n_active) {
  return (n_active + kTdActivePerBlock) / kTdActivePerBlock;  // covers k = n_active
}

inline uint64_t align256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

inline uint64_t td_scratch_layout(uint64_t n_features, uint64_t max_active,
                                  uint64_t* off_v, uint64_t* off_t, uint64_t* off_s) {
  const uint64_t blocks = td_blocks(max_active);
  const uint64_t tiles = (n_features + kTdTile - 1) / kTdTile;
  uint64_t o = 256;  // tickets
  *off_v = o;
  o = align256(o + 8 * blocks);
  *off_t = o;
  o = align256(o + 24 * blocks);
  *off_s = o;
  o = align256(o + 4 * (tiles + 1));
  return o;
}

// Per-step constants every feature uses (plain copies of globals, plus the
// three logs the reference evaluates per connection).
struct TdConst {
  float delta, vdp, meta, eta, eta_min, td, log_eta, log_eta_min, log_decay;
  float mult, one_minus_b;
  bool reset;
};

__device__ __forceinline__ TdConst td_const(const TdGlobals& g) {
  TdConst c;
  c.delta = g.delta;
  c.vdp = g.v_delta_prev;
  c.meta = g.meta;
  c.eta = g.eta;
  c.eta_min = g.eta_min;
  c.td = __fmul_rn(g.gamma, g.lambda);
  c.log_eta = logf(g.eta);
  c.log_eta_min = logf(g.eta_min);
  c.log_decay = logf(g.decay);
  // swifttd.cpp:169-171: the multiplier depends only on the globals.
  c.mult = 1.0f;
  if (g.tau > 0.0f && __fdiv_rn(g.eta, g.tau) < 1.0f) c.mult = __fdiv_rn(g.eta, g.tau);
  c.one_minus_b = __fsub_rn(1.0f, g.b);
  c.reset = g.tau > g.eta;
  return c;
}

// Phase 1 for one feature (swifttd.cpp:106-150), in place. Returns
// exp(Beta') for the Tau term.
__device__ __forceinline__ float td_phase1(const TdConst& c, float& w, float& z, float& zd,
                                           float& dw, float& h, float& h_old, float& h_temp,
                                           float& z_bar, float& p, float& beta) {
  dw = __fsub_rn(__fmul_rn(c.delta, z), __fmul_rn(zd, c.vdp));
  w = __fadd_rn(w, dw);
  beta = __fadd_rn(beta, __fmul_rn(__fmul_rn(__fdiv_rn(c.meta, expf(beta)),
                                             __fsub_rn(c.delta, c.vdp)),
                                   p));
  float eb = expf(beta);
  if (eb > c.eta || isinf(eb)) {
    beta = c.log_eta;
    eb = c.eta;
  }
  if (eb < c.eta_min) {
    beta = c.log_eta_min;
    eb = c.eta_min;
  }
  h_old = h;
  h = __fsub_rn(__fadd_rn(h_temp, __fmul_rn(c.delta, z_bar)), __fmul_rn(zd, c.vdp));
  h_temp = h;
  zd = 0.0f;
  z = __fmul_rn(z, c.td);
  p = __fmul_rn(p, c.td);
  z_bar = __fmul_rn(z_bar, c.td);
  return eb;
}

// Phase 2 for one feature (swifttd.cpp:152-186), in place.
__device__ __forceinline__ void td_phase2(const TdConst& c, float f, float& z, float& zd,
                                          float& h, float& h_old, float& h_temp,
                                          float& z_bar, float& p, float& beta) {
  zd = __fmul_rn(__fmul_rn(c.mult, expf(beta)), f);
  z = __fadd_rn(z, __fmul_rn(zd, c.one_minus_b));
  p = __fadd_rn(p, __fmul_rn(h_old, f));
  z_bar = __fadd_rn(z_bar, __fmul_rn(zd, __fsub_rn(c.one_minus_b, __fmul_rn(z_bar, f))));
  h_temp = __fsub_rn(__fsub_rn(h, __fmul_rn(__fmul_rn(h_old, f), __fsub_rn(z, zd))),
                     __fmul_rn(__fmul_rn(h, zd), f));
  if (c.reset) {
    h_temp = 0.0f;
    h = 0.0f;
    h_old = 0.0f;
    z_bar = 0.0f;
    beta = __fadd_rn(beta, __fmul_rn(__fmul_rn(c.log_decay, f), f));
  }
}

// Deterministic block sum of NV doubles per thread (fixed shuffle tree, then
// warps in order). Result valid in thread 0.
template <int NV>
__device__ __forceinline__ void block_sum(double (&v)[NV], double (*s_red)[kTdThreads / 32]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[j] += __shfl_down_sync(0xffffffffu, v[j], o);
    if (lane == 0) s_red[j][warp] = v[j];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      double s = 0.0;
      for (int k = 0; k < kTdThreads / 32; ++k) s += s_red[j][k];
      v[j] = s;
    }
  }
}

// Returns true in every thread of the last block to arrive (after its partial
// is visible to that block); the last block resets the ticket.
__device__ __forceinline__ bool last_block(uint32_t* ticket) {
  __shared__ bool s_last;
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last) __threadfence();
  return s_last;
}

struct TdActiveArgs {
  uint64_t n;
  uint32_t k;  // number of active features
  const uint32_t* idx;
  const float* val;  // null: every active value is 1
  const float* reward;
  TdGlobals* g;
  float* v_out;
  TdScratch s;
  uint64_t n_tiles;
  int32_t* status;
};

__device__ __forceinline__ float active_value(const TdActiveArgs& a, uint32_t k) {
  return a.val ? a.val[k] : 1.0f;
}

__global__ void __launch_bounds__(kTdThreads) k_td_value(TdActiveArgs a, TdFields fl) {
  __shared__ double s_red[1][kTdThreads / 32];
  double part[1] = {0.0};
  const uint64_t k0 = (uint64_t)blockIdx.x * kTdActivePerBlock;
#pragma unroll
  for (int j = 0; j < kTdActivePerBlock / kTdThreads; ++j) {
    const uint64_t k = k0 + (uint64_t)j * kTdThreads + threadIdx.x;
    if (k > a.k) continue;
    // Tile start offsets: start[t] = first k with tile(idx[k]) >= t.
    uint64_t t_lo, t_hi;
    uint32_t cur = 0;
    if (k < a.k) {
      cur = a.idx[k];
      const uint32_t prev = k ? a.idx[k - 1] : 0;
      if (cur >= a.n || (k && prev >= cur)) {
        record_status(a.status, kStatusBadIndex);
        continue;
      }
      t_lo = k ? (uint64_t)prev / kTdTile + 1 : 0;
      t_hi = (uint64_t)cur / kTdTile;
    } else {
      const uint32_t prev = k ? a.idx[k - 1] : 0;
      const uint64_t pv = prev < a.n ? prev : a.n - 1;  // n >= 1
      t_lo = k ? pv / kTdTile + 1 : 0;
      t_hi = a.n_tiles;
    }
    for (uint64_t t = t_lo; t <= t_hi && t <= a.n_tiles; ++t) a.s.start[t] = (uint32_t)k;
    if (k < a.k) part[0] += (double)__fmul_rn(fl.f[W][cur], active_value(a, (uint32_t)k));
  }
  block_sum<1>(part, s_red);
  if (threadIdx.x == 0) a.s.part_v[blockIdx.x] = part[0];
  if (!last_block(&a.s.tickets[0])) return;
  if (threadIdx.x == 0) {
    double v = 0.0;
    for (uint32_t b = 0; b < gridDim.x; ++b) v += __ldcg(&a.s.part_v[b]);
    TdGlobals& g = *a.g;
    // DoForwardPass Apply (swifttd.cpp:81-84) and Loss (:90-100).
    g.v = (float)v;
    g.delta = __fsub_rn(__fadd_rn(*a.reward, __fmul_rn(g.gamma, g.v)), g.v_old);
    g.v_delta_prev = g.v_delta;
    g.v_delta = 0.0f;
    g.tau = 0.0f;
    g.b = 0.0f;
    if (a.v_out) *a.v_out = g.v;
    a.s.tickets[0] = 0;
  }
}

__global__ void __launch_bounds__(kTdThreads) k_td_terms(TdActiveArgs a, TdFields fl) {
  __shared__ double s_red[3][kTdThreads / 32];
  const TdConst c = td_const(*a.g);
  double part[3] = {0.0, 0.0, 0.0};
  const uint64_t k0 = (uint64_t)blockIdx.x * kTdActivePerBlock;
#pragma unroll
  for (int j = 0; j < kTdActivePerBlock / kTdThreads; ++j) {
    const uint64_t k = k0 + (uint64_t)j * kTdThreads + threadIdx.x;
    if (k >= a.k) continue;
    const uint32_t i = a.idx[k];
    if (i >= a.n) continue;  // recorded by k_td_value
    const float f = active_value(a, (uint32_t)k);
    float w = fl.f[W][i], z = fl.f[Z][i], zd = fl.f[ZD][i], dw, h = fl.f[H][i], h_old,
          h_temp = fl.f[HTEMP][i], z_bar = fl.f[ZBAR][i], p = fl.f[P][i],
          beta = fl.f[BETA][i];
    const float eb = td_phase1(c, w, z, zd, dw, h, h_old, h_temp, z_bar, p, beta);
    part[0] += (double)__fmul_rn(__fmul_rn(eb, f), f);  // Tau, swifttd.cpp:148
    part[1] += (double)__fmul_rn(z, f);                 // B, :149
    part[2] += (double)__fmul_rn(dw, f);                // VDelta, :167
  }
  block_sum<3>(part, s_red);
  if (threadIdx.x == 0) {
#pragma unroll
    for (int j = 0; j < 3; ++j) a.s.part_t[(uint64_t)blockIdx.x * 3 + j] = part[j];
  }
  if (!last_block(&a.s.tickets[1])) return;
  if (threadIdx.x == 0) {
    double t[3] = {0.0, 0.0, 0.0};
    for (uint32_t b = 0; b < gridDim.x; ++b)
      for (int j = 0; j < 3; ++j) t[j] += __ldcg(&a.s.part_t[(uint64_t)b * 3 + j]);
    a.g->tau = (float)t[0];
    a.g->b = (float)t[1];
    a.g->v_delta = (float)t[2];
    a.s.tickets[1] = 0;
  }
}

__device__ __forceinline__ float4 ld4(const float* p) {
  return __ldcs(reinterpret_cast<const float4*>(p));
}
__device__ __forceinline__ void st4(float* p, float4 v) {
  __stcs(reinterpret_cast<float4*>(p), v);
}

#define PLX_TD_LANE(comp)                                                          \
  do {                                                                             \
    float dw_, h_old_;                                                             \
    td_phase1(c, w.comp, z.comp, zd.comp, dw_, h.comp, h_old_, ht.comp, zb.comp,   \
              p.comp, be.comp);                                                    \
    td_phase2(c, fv.comp, z.comp, zd.comp, h.comp, h_old_, ht.comp, zb.comp,       \
              p.comp, be.comp);                                                    \
    dw.comp = dw_;                                                                 \
    ho.comp = h_old_;                                                              \
  } while (0)

__global__ void __launch_bounds__(kTdThreads) k_td_dense(TdActiveArgs a, TdFields fl) {
  __shared__ __align__(16) float s_f[kTdTile];
  const TdConst c = td_const(*a.g);
  for (uint64_t tile = blockIdx.x; tile < a.n_tiles; tile += gridDim.x) {
    const uint64_t base = tile * kTdTile;
    const uint64_t i0 = base + 4ull * threadIdx.x;
    const bool full = i0 + 4 <= a.n;
    // Issue the streaming loads before the tile's F is assembled.
    float4 w{}, z{}, zd{}, h{}, ht{}, zb{}, p{}, be{};
    if (full) {
      w = ld4(fl.f[W] + i0);
      z = ld4(fl.f[Z] + i0);
      zd = ld4(fl.f[ZD] + i0);
      h = ld4(fl.f[H] + i0);
      ht = ld4(fl.f[HTEMP] + i0);
      zb = ld4(fl.f[ZBAR] + i0);
      p = ld4(fl.f[P] + i0);
      be = ld4(fl.f[BETA] + i0);
    }
    __syncthreads();  // previous tile's s_f reads are done
    reinterpret_cast<float4*>(s_f)[threadIdx.x] = make_float4(0.f, 0.f, 0.f, 0.f);
    __syncthreads();
    const uint32_t ka = min(a.s.start[tile], a.k);
    const uint32_t kb = max(min(a.s.start[tile + 1], a.k), ka);
    for (uint32_t k = ka + threadIdx.x; k < kb; k += kTdThreads) {
      const uint64_t off = (uint64_t)a.idx[k] - base;
      if (off < kTdTile) s_f[off] = active_value(a, k);
    }
    __syncthreads();
    if (full) {
      const float4 fv = reinterpret_cast<const float4*>(s_f)[threadIdx.x];
      float4 dw, ho;
      PLX_TD_LANE(x);
      PLX_TD_LANE(y);
      PLX_TD_LANE(z);
      PLX_TD_LANE(w);
      st4(fl.f[W] + i0, w);
      st4(fl.f[Z] + i0, z);
      st4(fl.f[ZD] + i0, zd);
      st4(fl.f[DW] + i0, dw);
      st4(fl.f[H] + i0, h);
      st4(fl.f[HOLD] + i0, ho);
      st4(fl.f[HTEMP] + i0, ht);
      st4(fl.f[ZBAR] + i0, zb);
      st4(fl.f[P] + i0, p);
      st4(fl.f[BETA] + i0, be);
    } else {
      for (uint64_t i = i0; i < a.n && i < i0 + 4; ++i) {
        float* const* f = fl.f;
        float w1 = f[W][i], z1 = f[Z][i], zd1 = f[ZD][i], dw1, h1 = f[H][i], ho1,
              ht1 = f[HTEMP][i], zb1 = f[ZBAR][i], p1 = f[P][i], be1 = f[BETA][i];
        td_phase1(c, w1, z1, zd1, dw1, h1, ho1, ht1, zb1, p1, be1);
        td_phase2(c, s_f[i - base], z1, zd1, h1, ho1, ht1, zb1, p1, be1);
        f[W][i] = w1;
        f[Z][i] = z1;
        f[ZD][i] = zd1;
        f[DW][i] = dw1;
        f[H][i] = h1;
        f[HOLD][i] = ho1;
        f[HTEMP][i] = ht1;
        f[ZBAR][i] = zb1;
        f[P][i] = p1;
        f[BETA][i] = be1;
      }
    }
  }
  // ResetGlobal (swifttd.cpp:189-191). No block of this kernel reads V or VOld.
  if (blockIdx.x == 0 && threadIdx.x == 0) a.g->v_old = a.g->v;
}
#undef PLX_TD_LANE

}  // namespace
}  // namespace plx

using namespace plx;

extern "C" uint64_t plx_swifttd_scratch_bytes(uint64_t n_features, uint32_t max_active) {
  uint64_t ov, ot, os;
  return td_scratch_layout(n_features, max_active, &ov, &ot, &os);
}

extern "C" int plx_swifttd_step(plx_ctx* ctx, uint64_t n_features,
                                float* const* fields, const uint32_t* active_idx,
                                const float* active_val, uint32_t n_active,
                                const float* reward, plx_td_globals* globals,
                                float* v_out, void* scratch, uint64_t scratch_bytes) {
  PLX_CHECK_ARG(ctx && fields && reward && globals && scratch,
                "ctx, fields, reward, globals and scratch are required");
  PLX_CHECK_ARG(n_features > 0 && n_features <= 0xFFFFFFFFull,
                "n_features must be in [1, 2^32 - 1]");
  PLX_CHECK_ARG(n_active <= n_features, "more active features than features");
  PLX_CHECK_ARG(n_active == 0 || active_idx, "active_idx is required when n_active > 0");
  TdFields fl;
  for (int j = 0; j < PLX_TD_NUM_FIELDS; ++j) {
    PLX_CHECK_ARG(fields[j] && aligned16(fields[j]),
                  "field %d must be a non-null 16-byte-aligned device pointer", j);
    fl.f[j] = fields[j];
  }
  PLX_CHECK_ARG(aligned16(scratch), "scratch must be 16-byte aligned");
  uint64_t ov, ot, os;
  const uint64_t need = td_scratch_layout(n_features, n_active, &ov, &ot, &os);
  PLX_CHECK_ARG(scratch_bytes >= need, "scratch is %llu bytes, %llu needed",
                (unsigned long long)scratch_bytes, (unsigned long long)need);
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  char* s = static_cast<char*>(scratch);
  TdActiveArgs a;
  a.n = n_features;
  a.k = n_active;
  a.idx = active_idx;
  a.val = active_val;
  a.reward = reward;
  a.g = reinterpret_cast<TdGlobals*>(globals);
  a.v_out = v_out;
  a.s.tickets = reinterpret_cast<uint32_t*>(s);
  a.s.part_v = reinterpret_cast<double*>(s + ov);
  a.s.part_t = reinterpret_cast<double*>(s + ot);
  a.s.start = reinterpret_cast<uint32_t*>(s + os);
  a.n_tiles = (n_features + kTdTile - 1) / kTdTile;
  a.status = ctx->d_status;
  const unsigned blocks = (unsigned)td_blocks(n_active);
  k_td_value<<<blocks, kTdThreads, 0, ctx->stream>>>(a, fl);
  PLX_LAUNCH_CHECK("k_td_value");
  k_td_terms<<<blocks, kTdThreads, 0, ctx->stream>>>(a, fl);
  PLX_LAUNCH_CHECK("k_td_terms");
  const unsigned dense =
      (unsigned)std::min<uint64_t>(a.n_tiles, 8ull * (uint64_t)ctx->num_sms);
  k_td_dense<<<dense, kTdThreads, 0, ctx->stream>>>(a, fl);
  PLX_LAUNCH_CHECK("k_td_dense");
  return PLX_OK;
}
